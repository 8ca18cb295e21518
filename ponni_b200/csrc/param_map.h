// Device-side parameter updates: where every trainable parameter lives in the
// planned device images, and the kernels that rewrite them in place.
//
// A planned model holds each trainable parameter in up to three device
// images: the packed parameter array (model dtype, read by the tile and
// narrow kernels and the device API), the resident tensor-core image (fp32
// bias, 16-bit weights or, for fp32 models, the three bf16 parts of each
// weight in swizzled K-major layout) and the streamed tensor-core image.  The
// planner records one ParamRec per (parameter, image location) while it
// writes the images; a parameter update then converts each new value to the
// model dtype and re-encodes it into every location with one kernel, so a
// weight change costs a scatter of the parameters instead of a re-plan and a
// re-upload of every image.
//
// Reference counterparts: the generated model's set_parameters (convert,
// scatter into the parameter storage, refresh the fp16 mirror;
// src/generator/kokkos_nn/emitter.py:1826-1866), parameters_are_finite
// (:1868-1880) and parameters_synchronized (:1882-1895).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace ponni_b200 {

enum ParamImage : uint8_t { PIMG_PACKED = 0, PIMG_TC = 1, PIMG_TS = 2, PIMG_COUNT = 3 };

enum ParamEnc : uint8_t {
  PENC_MODEL = 0,   // the canonical value in the model dtype
  PENC_F32 = 1,     // float(canonical) (tensor-core bias)
  PENC_SPLIT0 = 2,  // bf16 part q of the exact three-way split of an fp32
  PENC_SPLIT1 = 3,  //   value: w = b0 + b1 + b2, b0 = bf16(w), b1 = bf16(w - b0),
  PENC_SPLIT2 = 4,  //   b2 = bf16(w - b0 - b1)
};

struct ParamRec {
  uint32_t src;  // trainable parameter index (tuple order)
  uint32_t dst;  // byte offset in the image
  uint8_t img;   // ParamImage
  uint8_t enc;   // ParamEnc
  uint16_t pad;
};

// Host-side recorder filled by the planner.  `ranges` lists the canonical
// parameter arrays of the trainable layers; `add` translates a pointer into
// one of them to its trainable index (pointers into non-trainable layers are
// fixed values and are not recorded).
struct ParamMap {
  struct Range {
    const unsigned char* begin;
    const unsigned char* end;
    int64_t base;
  };
  std::vector<Range> ranges;
  size_t esz = 4;
  std::vector<ParamRec> recs;
  int hint = 0;
  bool overflow = false;  // an offset beyond 32 bits: device updates unavailable

  void clear() {
    ranges.clear();
    recs.clear();
    hint = 0;
    overflow = false;
  }
  void add(const unsigned char* p, ParamImage img, ParamEnc enc, size_t dst) {
    if (dst > 0xffffffffull) overflow = true;
    const int n = (int)ranges.size();
    for (int t = 0; t < n; ++t) {
      const Range& r = ranges[(hint + t) % n];
      if (p >= r.begin && p < r.end) {
        hint = (hint + t) % n;
        if (r.base + (p - r.begin) / (ptrdiff_t)esz > 0xffffffffll) overflow = true;
        recs.push_back(ParamRec{(uint32_t)(r.base + (p - r.begin) / (ptrdiff_t)esz), (uint32_t)dst, img, enc, 0});
        return;
      }
    }
  }
};

// Device side of a model's map (owned by the model, uploaded on first use).
struct ParamMapDev {
  ParamRec* recs = nullptr;         // sorted by (image, dst)
  uint32_t* packed_of = nullptr;    // trainable index -> element offset in the packed image
  int* counts = nullptr;            // [0] mismatches, [1] non-finite values
  void* staging = nullptr;          // source values of host updates (device)
  void* pinned = nullptr;           // pinned host staging of host updates
  cudaEvent_t pinned_free = nullptr;  // recorded after the copy out of `pinned`
  cudaEvent_t done = nullptr;         // orders the model stream after updates on another stream
  std::vector<uint32_t> packed_of_host;  // host copy of packed_of
  int64_t n_recs = 0;
  int64_t n_trainable = 0;
  size_t staging_bytes = 0;
};

// Scatter: for every record, image[dst] = enc(model dtype(src[rec.src])).
// src_dtype / model_dtype: 0 fp32, 1 fp64, 2 fp16, 3 bf16.
cudaError_t launch_param_scatter(const ParamMapDev& d, const void* src, int src_dtype, int model_dtype,
                                 void* const images[PIMG_COUNT], cudaStream_t s);
// Gather: dst[i] = convert(packed[packed_of[i]]) for every trainable i.
cudaError_t launch_param_gather(const ParamMapDev& d, const void* packed, void* dst, int dst_dtype,
                                int model_dtype, cudaStream_t s);
// Count records whose image bytes differ from the encoding of the packed
// value (counts[0]) and trainable values that are not finite (counts[1]).
cudaError_t launch_param_check(const ParamMapDev& d, int model_dtype, void* const images[PIMG_COUNT],
                               cudaStream_t s);

}  // namespace ponni_b200
