// Kernels of the device-side parameter update (param_map.h).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "param_map.h"

namespace ponni_b200 {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ double load_any(const void* p, int64_t i, int dt) {
  switch (dt) {
    case 0: return (double)static_cast<const float*>(p)[i];
    case 1: return static_cast<const double*>(p)[i];
    case 2: return (double)__half2float(static_cast<const __half*>(p)[i]);
    default: return (double)__bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  }
}

// The model's canonical value of a source value: the same conversion as the
// host's store_scalar (fp64 kept, everything else through fp32).
struct Canon {
  double v;     // canonical value
  uint64_t b;   // its bytes in the model dtype (low bytes)
};

__device__ __forceinline__ Canon canon(double v, int mdt) {
  Canon c;
  switch (mdt) {
    case 0: {
      const float f = (float)v;
      c.v = f;
      c.b = __float_as_uint(f);
      break;
    }
    case 1:
      c.v = v;
      c.b = (uint64_t)__double_as_longlong(v);
      break;
    case 2: {
      const __half h = __float2half_rn((float)v);
      c.v = __half2float(h);
      c.b = __half_as_ushort(h);
      break;
    }
    default: {
      const __nv_bfloat16 h = __float2bfloat16_rn((float)v);
      c.v = __bfloat162float(h);
      c.b = __bfloat16_as_ushort(h);
      break;
    }
  }
  return c;
}

__device__ __forceinline__ int model_bytes(int mdt) { return mdt == 1 ? 8 : mdt == 0 ? 4 : 2; }

// Bytes and size of one encoded location.
__device__ __forceinline__ uint64_t encode(const Canon& c, int enc, int mdt, int* nbytes) {
  switch (enc) {
    case PENC_MODEL: *nbytes = model_bytes(mdt); return c.b;
    case PENC_F32: *nbytes = 4; return __float_as_uint((float)c.v);
    default: {
      const float w = (float)c.v;
      const __nv_bfloat16 b0 = __float2bfloat16_rn(w);
      const float r = w - __bfloat162float(b0);
      const __nv_bfloat16 b1 = __float2bfloat16_rn(r);
      const __nv_bfloat16 b2 = __float2bfloat16_rn(r - __bfloat162float(b1));
      *nbytes = 2;
      return enc == PENC_SPLIT0 ? __bfloat16_as_ushort(b0)
             : enc == PENC_SPLIT1 ? __bfloat16_as_ushort(b1)
                                  : __bfloat16_as_ushort(b2);
    }
  }
}

__device__ __forceinline__ void store_bytes(unsigned char* p, uint64_t v, int n) {
  switch (n) {
    case 8: *reinterpret_cast<unsigned long long*>(p) = v; break;
    case 4: *reinterpret_cast<uint32_t*>(p) = (uint32_t)v; break;
    default: *reinterpret_cast<uint16_t*>(p) = (uint16_t)v; break;
  }
}

__device__ __forceinline__ uint64_t load_bytes(const unsigned char* p, int n) {
  switch (n) {
    case 8: return *reinterpret_cast<const unsigned long long*>(p);
    case 4: return *reinterpret_cast<const uint32_t*>(p);
    default: return *reinterpret_cast<const uint16_t*>(p);
  }
}

struct Images {
  unsigned char* p[PIMG_COUNT];
};

__global__ void __launch_bounds__(kThreads) param_scatter_kernel(const ParamRec* __restrict__ recs, int64_t n,
                                                                 const void* __restrict__ src, int sdt, int mdt,
                                                                 Images img) {
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const ParamRec r = recs[i];
    unsigned char* base = img.p[r.img];
    if (!base) continue;
    const Canon c = canon(load_any(src, r.src, sdt), mdt);
    int nb;
    const uint64_t v = encode(c, r.enc, mdt, &nb);
    store_bytes(base + r.dst, v, nb);
  }
}

__global__ void __launch_bounds__(kThreads) param_gather_kernel(const uint32_t* __restrict__ packed_of, int64_t n,
                                                                const void* __restrict__ packed, void* dst, int ddt,
                                                                int mdt) {
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const double v = load_any(packed, packed_of[i], mdt);
    switch (ddt) {
      case 0: static_cast<float*>(dst)[i] = (float)v; break;
      case 1: static_cast<double*>(dst)[i] = v; break;
      case 2: static_cast<__half*>(dst)[i] = __float2half_rn((float)v); break;
      default: static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn((float)v); break;
    }
  }
}

__global__ void __launch_bounds__(kThreads) param_check_kernel(const ParamRec* __restrict__ recs, int64_t n,
                                                               const uint32_t* __restrict__ packed_of, int mdt,
                                                               Images img, int* counts) {
  int mism = 0, nonfinite = 0;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const ParamRec r = recs[i];
    const unsigned char* base = img.p[r.img];
    if (!base) continue;
    const double v = load_any(img.p[PIMG_PACKED], packed_of[r.src], mdt);
    if (r.img == PIMG_PACKED) {
      if (!isfinite(v)) ++nonfinite;
      continue;
    }
    const Canon c = canon(v, mdt);
    int nb;
    const uint64_t want = encode(c, r.enc, mdt, &nb);
    if (load_bytes(base + r.dst, nb) != want) ++mism;
  }
  if (mism) atomicAdd(&counts[0], mism);
  if (nonfinite) atomicAdd(&counts[1], nonfinite);
}

int grid_for(int64_t n) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n + kThreads - 1) / kThreads;
  return (int)(want < 8LL * sms ? (want > 0 ? want : 1) : 8LL * sms);
}

Images to_images(void* const images[PIMG_COUNT]) {
  Images m;
  for (int i = 0; i < PIMG_COUNT; ++i) m.p[i] = static_cast<unsigned char*>(images[i]);
  return m;
}

}  // namespace

cudaError_t launch_param_scatter(const ParamMapDev& d, const void* src, int src_dtype, int model_dtype,
                                 void* const images[PIMG_COUNT], cudaStream_t s) {
  if (d.n_recs == 0) return cudaSuccess;
  param_scatter_kernel<<<grid_for(d.n_recs), kThreads, 0, s>>>(d.recs, d.n_recs, src, src_dtype, model_dtype,
                                                                to_images(images));
  return cudaGetLastError();
}

cudaError_t launch_param_gather(const ParamMapDev& d, const void* packed, void* dst, int dst_dtype, int model_dtype,
                                cudaStream_t s) {
  if (d.n_trainable == 0) return cudaSuccess;
  param_gather_kernel<<<grid_for(d.n_trainable), kThreads, 0, s>>>(d.packed_of, d.n_trainable, packed, dst,
                                                                    dst_dtype, model_dtype);
  return cudaGetLastError();
}

cudaError_t launch_param_check(const ParamMapDev& d, int model_dtype, void* const images[PIMG_COUNT],
                               cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(d.counts, 0, 2 * sizeof(int), s);
  if (e != cudaSuccess || d.n_recs == 0) return e;
  param_check_kernel<<<grid_for(d.n_recs), kThreads, 0, s>>>(d.recs, d.n_recs, d.packed_of, model_dtype,
                                                              to_images(images), d.counts);
  return cudaGetLastError();
}

}  // namespace ponni_b200
