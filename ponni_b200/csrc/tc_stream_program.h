// Program of the streamed-weights tensor-core kernel (tc_stream.cu), shared
// by the host planner (ts_plan in tc_plan.cu), the kernel body
// (tc_stream_body.cuh) and its model-specialised build; device-safe (no host
// headers).
#pragma once
#include <stdint.h>

namespace ponni_b200 {

constexpr int kTsMaxLayers = 16;
constexpr int kTsMaxN = 256;                    // layer width limit = accumulator columns of one job
constexpr int kTsBlockK = 64;                   // K elements of one streamed chunk
constexpr int kTsChunkBytes = kTsMaxN * 128;    // ring stage: up to 256 rows x 128 B
constexpr int kTsSlots = 2;                     // tiles in flight per CTA
constexpr int kTsEpiWarps = 16;                 // two groups (one per slot) of 8 warps
constexpr int kTsGroupWarps = kTsEpiWarps / kTsSlots;  // 4 TMEM lane quarters x 2 column halves
constexpr int kTsGroupThreads = kTsGroupWarps * 32;
constexpr int kTsColsPerWarp = kTsMaxN / 2;     // accumulator columns per warp and job
constexpr int kTsProducerWarp = kTsEpiWarps;
constexpr int kTsMmaWarp = kTsEpiWarps + 1;
constexpr int kTsLoaderWarp = kTsEpiWarps + 2;       // input tiles through the tensor memory accelerator
constexpr int kTsThreads = (kTsEpiWarps + 3) * 32;  // + producer, MMA and loader warps
constexpr int kTsMaxStages = 8;
constexpr int kTsBarBytes = 320;                // mbarriers, TMEM address and abort flag, then the layer table

struct TsLayer {
  int32_t nin, nout;
  int32_t k_pad, n_pad;  // K rounded to 16, N rounded to 16
  int32_t kblk;          // K chunks of 64
  int32_t act, act_flags;
  float s0, s1;
  int32_t has_bias;
  uint32_t bias_off;     // byte offset of float bias[round_up(n_pad, 32)] in the image
  uint64_t w_off;        // byte offset of chunk kb = 0; chunk kb at + kb * kTsChunkBytes (n_pad rows x 128 B)
};

struct TsProgram {
  int32_t n_layers;
  int32_t dtype;          // ponni_b200_dtype: 2 f16, 3 bf16
  int32_t nin, nout;
  int32_t fast_act;       // SiLU / sigmoid / tanh through the hardware approximations (fp32 accumulation mode)
  uint32_t a_bytes;       // one tile's activation operand buffer (also holds its MN-major input stage)
  uint32_t stage_bytes;   // MN-major layer-0 input stage (inside the operand buffer)
  uint32_t ring_stages;   // weight ring stages of kTsChunkBytes (pair mode: of kTsChunkBytes / 2)
  int32_t pair;           // clusters of two CTAs sharing M = 256 MMAs (cta_group::2)
  uint32_t smem_bytes;    // dynamic shared memory requested
  uint64_t image_bytes;   // weight chunks + biases
  TsLayer layers[kTsMaxLayers];
};

}  // namespace ponni_b200
