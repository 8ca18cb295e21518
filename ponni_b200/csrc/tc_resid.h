// Tensor-core kernel for dense chains with LayerNorm and residual barriers
// (tc_resid.cu), fp32 models on the exact three-way bf16 split, weights
// streamed from L2.
//
// PONNI's residual blocks (Save_State, LayerNorm, Matvec, Bias, GELU, Matvec,
// Bias, Binop_Add; reference src/layers/ponni_Save_State.h:58-67,
// ponni_LayerNorm.h:77-99, ponni_Binop_Add.h:58-68, traversal
// src/ponni_Inference.h:416-555) are lowered to one "dense job" per Matvec
// whose epilogue runs every layer up to the next Matvec, in tuple order:
// element-wise operations (Bias, activations, Binop_Add of a saved state,
// Save_State) on 32-column chunks of the accumulator, and at most one
// LayerNorm, a whole-row operation whose four 32-column chunks exchange
// partial sums.
// Batch columns sit on the TMEM lanes, so one row of a tile is one sample.
//
// Work unit ("job"): one Matvec for one tile of 128 batch columns,
// D[128 x N<=128] = A[128 x K<=128] * W[K x N], A and W split exactly into
// bf16 parts (x = x0 + x1 + x2) and the six products of order <= 2
// accumulated in TMEM, the five small ones first: the tensor core's fp32
// accumulation truncates, and summing the small products before the
// dominant x0*w0 ones keeps their truncation relative to their own size.
// The weights stream through a two-stage shared-memory ring in chunks of one
// part of one K block of 64 (N rows x 128 B): per layer parts 2 and 1 of
// each K block, then the part-0 chunks, held until the x0*w0 products.  Two
// tiles are in flight per CTA and their jobs alternate Matvec by Matvec, so
// one tile's epilogue overlaps the other's MMAs.  A single saved state lives
// in TMEM next to its tile's accumulators (128 columns per slot); models with
// two keep them in a per-CTA global scratch area (L2-resident: 64 KB per
// tile slot and saved state).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

struct ponni_b200_model;

namespace ponni_b200 {

constexpr int kTrMaxLayers = 16;                // Matvecs
constexpr int kTrMaxOps = 96;                   // epilogue operations of all Matvecs
constexpr int kTrMaxN = 128;                    // width limit (accumulator columns of one job)
constexpr int kTrMaxSaved = 2;                  // distinct Save_State indices
constexpr int kTrChunkBytes = kTrMaxN * 128;    // ring stage: up to 128 rows x 128 B
constexpr int kTrStages = 2;
constexpr int kTrSlots = 2;                     // tiles in flight per CTA
constexpr int kTrEpiWarps = 16;                 // epilogue warps: 4 TMEM lane quarters x 4 column quarters
constexpr int kTrProducerWarp = kTrEpiWarps;
constexpr int kTrMmaWarp = kTrEpiWarps + 1;
constexpr int kTrThreads = (kTrEpiWarps + 2) * 32;
constexpr uint32_t kTrSlotTmem = 256;           // TMEM columns per slot: accumulators + saved state
constexpr uint32_t kTrAccCols = 128;            // accumulator columns of a job (its main groups)
constexpr uint32_t kTrPartBytes = 2 * 128 * 128;  // one operand part: 2 K blocks x 128 rows x 128 B
constexpr int kTrMaxParts = 3;

// Epilogue operations (tuple order after each Matvec).
enum TrOpKind : int32_t {
  TR_BIAS = 1,  // v += b[f]                        (off: float[128] in the image)
  TR_ACT = 2,   // v = activation(kind)(v)          (arg: ponni_b200 layer kind)
  TR_ADD = 3,   // v += saved[arg][f]               (Binop_Add)
  TR_SAVE = 4,  // saved[arg][f] = v                (Save_State)
  TR_LN = 5,    // LayerNorm over the row           (off: gamma float[128], beta at off + 512; s0 = eps)
};

struct TrOp {
  int32_t kind;
  int32_t arg;
  int32_t flags;
  float s0, s1;
  uint32_t off;
};

struct TrLayer {
  int32_t nin, nout;     // true widths
  int32_t k_pad, n_pad;  // K and N rounded to 16
  int32_t kblk;          // K blocks of 64
  int32_t nsteps;        // UMMA K steps of 16
  int32_t group_steps;   // K steps per accumulator group (4: one K block, or all)
  int32_t groups;        // accumulator groups (1 or 2); the five smaller products go into group 0
  int32_t op_first;      // epilogue operations [op_first, op_first + n_ops)
  int32_t n_ops;
  int32_t ln;            // index (within the layer's operations) of its LayerNorm, or -1
  uint32_t idesc;        // UMMA instruction descriptor
  uint64_t w_off;        // byte offset of the layer's first weight chunk in the image
};

struct TrProgram {
  int32_t n_layers;
  int32_t dtype;          // ponni_b200_dtype (0: fp32 on the bf16 split)
  int32_t nin, nout;
  int32_t nparts;         // 3 (fp32 split) or 1
  int32_t n_saved;        // saved-state slots used
  uint32_t smem_bytes;    // dynamic shared memory requested
  uint64_t image_bytes;   // weight chunks + float vectors
  int32_t saved_tmem;     // 1: the (single) saved state lives in TMEM beside the accumulators
  uint64_t scratch_per_cta;  // bytes of saved-state scratch per CTA (0 with saved_tmem)
  TrLayer layers[kTrMaxLayers];
  TrOp ops[kTrMaxOps];
};

// Plan the kernel for `m`: false (with the reason in `why`) when the model is
// not a chain this kernel supports.  Builds the chunked, pre-swizzled,
// pre-split weight image; `rec` (optional) receives the image location of
// every trainable parameter.
struct ParamMap;
bool tr_plan(const ponni_b200_model* m, TrProgram& p, std::vector<unsigned char>& image, std::string& why,
             ParamMap* rec = nullptr);

// `scratch`: grid x p.scratch_per_cta bytes of device memory.
cudaError_t launch_tr_forward(const TrProgram& p, const void* image, void* scratch, const void* in, int64_t in_ld,
                              void* out, int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream);

}  // namespace ponni_b200
