// Program of the tensor-core (tcgen05) dense-chain kernel, shared by the host
// packer (tc_plan.cu) and the kernel (tc_kernel.cu).
//
// A dense chain is Matvec [Bias] [activation] repeated, PONNI's fused dense
// blocks (reference src/ponni_Inference.h:416-444) without barriers.  Each
// layer is one UMMA chain D[M=128 batch rows, N=features] +=
// A[M, K=in features] * B[N, K]^T with the fp32 accumulator in TMEM.
//
// Shared-memory operand layouts (128-byte swizzle, "SW128"):
//  * K-major (weights B, and the activations A of layers >= 1): rows of 128 B
//    holding 128/esz consecutive K elements; 8-row groups 1024 B apart (SBO);
//    K beyond one row lives in the next "K block" of rows x 128 B; 16-byte
//    chunk c of row r is stored at chunk position c ^ (r % 8).
//  * MN-major (the layer-0 activations of 16-bit models, copied straight from
//    the batch-contiguous input): atoms of 8 k-rows x 128 B (64 batch
//    columns); atoms along M 1024 B apart (LBO), along K 2048 B apart (SBO).
// All operands are 16-bit (fp16 / bf16); fp32 models split every operand
// x exactly into three bf16 parts x = b0 + b1 + b2.
#pragma once
#include <stdint.h>

namespace ponni_b200 {

constexpr int kTcMaxLayers = 16;
constexpr int kTcMaxSlots = 8;      // tiles in flight per CTA (TcProgram::slots = 1..8; 5..8 for 16-bit models)
constexpr int kTcMaxThreads = 1024; // slots x slot_threads (fp32 split models: at most 512)
// Threads of one slot (TcProgram::slot_threads): 128 = 4 warps, one per TMEM
// lane quarter, each thread walking all accumulator columns of its lane; or
// 256 = 8 warps, 4 lane quarters x 2 column halves (used with <= 2 slots).
constexpr int kTcM = 128;        // batch rows per tile (UMMA M)

struct TcLayer {
  int32_t nin, nout;     // true widths
  int32_t k_pad;         // K rounded to the UMMA K step (8 tf32 / 16 f16/bf16)
  int32_t n_pad;         // N rounded to 16 (UMMA N for M=128)
  int32_t act, act_flags;
  float s0, s1;          // activation scalars
  int32_t has_bias;      // the epilogue adds float bias[n_pad] (fp32 split models)
  uint32_t bias_off;     // byte offset of that float bias in the staged image
  int32_t bias_mma;      // 16-bit models: the bias enters the accumulator through one extra UMMA
                         // (A = a column of ones, B = the bias block at bias_off)
  uint32_t w_off[3];     // byte offsets of the K-major B operand parts (1, or 3 for split fp32)
  uint32_t idesc;        // UMMA instruction descriptor (A K-major)
  uint32_t idesc_mn;     // same with A MN-major (layer 0)
  int32_t groups;        // fp32 accumulators summed in the epilogue (split models: main ones + one correction)
  int32_t group_steps;   // consecutive K steps per (main) accumulator
};

struct TcProgram {
  int32_t n_layers;
  int32_t dtype;         // ponni_b200_dtype (0 f32 -> bf16 3-way split, 2 f16, 3 bf16)
  int32_t nin, nout;
  int32_t nparts;        // operand parts: 3 (fp32 split into bf16 b0+b1+b2) or 1
  uint32_t image_bytes;  // staged parameter image (multiple of 16)
  uint32_t ones_off;     // 16-bit models with a bias: byte offset of the ones block (A of the bias UMMA)
  uint32_t zero_off;     //   and of the zero block that the second K half of every bias UMMA operand reads
  uint32_t a_bytes;      // one activation operand buffer (one part)
  uint32_t stage_bytes;  // one input staging buffer (one per slot)
  uint32_t slot_bytes;   // shared memory of one slot: parts x a_bytes + stage_bytes
  uint32_t slot_cols;    // TMEM columns of one tile slot (max over layers of groups * n_pad)
  uint32_t tmem_cols;    // allocated TMEM columns: power of two >= slots * slot_cols
  int32_t slots;         // tile slots per CTA (1..8); the CTA runs slots * slot_threads threads
  int32_t slot_threads;  // 128 or 256
  uint32_t smem_bytes;   // total dynamic shared memory requested (incl. 1 KB alignment slack,
                         // mbarriers, the TMEM address and a copy of the layer table)
  TcLayer layers[kTcMaxLayers];
};

}  // namespace ponni_b200
