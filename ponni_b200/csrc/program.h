// Lowered execution program shared by the host planner (model.cu) and the
// fused tile kernel (tile_kernel.cu).
//
// PONNI's template executor walks the layer tuple per sample and fuses each
// dense layer with the pointwise layers that follow it
// (reference src/ponni_Inference.h:56-70 fused_dense_block_end, :416-444
// apply_fused_epilogue / compute_fused_dense_block, :454-555
// traverse_mixed_batch_parallel).  Here the same walk is done once on the host
// and produces a list of steps over on-chip buffers: every step reads and
// writes shared-memory tiles [width][BT] holding BT batch columns, so no
// intermediate state ever reaches HBM.
#pragma once
#include <stdint.h>

#include "epi_kinds.h"

namespace ponni_b200 {

constexpr int kMaxSteps = 64;
constexpr int kMaxEpilogue = 96;
constexpr int kMaxBuffers = 16;
constexpr int kThreads = 256;  // threads per CTA of the tile kernel
constexpr int kTO = 8;         // output features per thread micro-tile
constexpr int kTB = 4;         // batch columns per thread micro-tile

enum StepKind : int32_t {
  STEP_DENSE = 0,      // out[o][c] = epi( init + sum_k W[k][o] * in[k][c] )
  STEP_POINTWISE = 1,  // in place: x[f][c] = epi(x[f][c]) (pointwise run not after a dense)
  STEP_LAYERNORM = 2,  // in place, per column
  STEP_MINMAXNORM = 3, // in place, per column
  STEP_SOFTMAX = 4,    // in place, per column
  STEP_LOGSOFTMAX = 5, // in place, per column
  STEP_COPY = 6,       // Save_State: dst[f][c] = src[f][c]
  STEP_ADD = 7,        // Binop_Add: src[f][c] += aux[f][c]
  STEP_CONCAT = 8,     // Binop_Concatenate: dst = [src ; aux] or [aux ; src]
};

// Dense flags.
constexpr int32_t DENSE_INIT_BIAS = 0x1;    // accumulator starts at bias (Projection_Add order)
constexpr int32_t DENSE_ADD_RESIDUAL = 0x2; // out = res[o][c] + acc (Projection_Add)
constexpr int32_t DENSE_TO_GLOBAL = 0x4;    // final block: write the caller's output
constexpr int32_t DENSE_FAST_EPI = 0x8;     // epilogue is [Bias?][activation?]: fast path
constexpr int32_t DENSE_HALF_FMA = 0x10;    // 16-bit: one fused multiply-add per product (generated arithmetic)
constexpr int32_t CONCAT_AFTER = 0x4;
constexpr int32_t LN_WELFORD = 0x20;        // LayerNorm of the generated model (Welford; 16-bit: in float)

struct EpiDesc {
  int32_t kind;
  int32_t flags;     // bit 0x2: GELU approximate
  double s0, s1, s2; // already rounded to the model dtype
  int64_t p_off;     // EPI_BIAS: element offset of b[] in the packed parameter buffer
};

struct StepDesc {
  int32_t kind;
  int32_t flags;
  int32_t nin, nout;     // feature widths
  int32_t src, dst, aux; // buffer ids (-1 = none / global output)
  int32_t epi_first, n_epi;
  int32_t nout_pad;      // dense: packed weight row length (multiple of kTO)
  int32_t fast_act;      // DENSE_FAST_EPI: activation kind (EPI_NONE if none)
  int32_t fast_act_flags;
  int64_t w_off;         // dense: packed W[k][nout_pad]; LN: gamma; element offsets
  int64_t b_off;         // dense INIT_BIAS bias; LN: beta
  int64_t fast_bias_off; // DENSE_FAST_EPI: bias offset, or -1
  double s0, s1, s2;     // LN: eps; MinMax: out_min, out_max, eps; fast act scalars s0/s1
};

struct Program {
  int32_t n_steps;
  int32_t n_epi;
  int32_t bt;            // batch columns per tile (multiple of 32)
  int32_t n_buffers;
  int32_t in_buf;        // buffer receiving the input tile (double-buffered: in_buf, in_buf2)
  int32_t in_buf2;
  int32_t final_buf;     // buffer holding the result when the last step is not a dense step
  int32_t nin, nout;     // model input/output widths
  int32_t params_in_smem;   // 1: the packed parameters are staged in shared memory
  int32_t param_smem_off;   // element offset of the staged parameters
  int32_t n_params;         // packed parameter elements
  int32_t buf_off[kMaxBuffers];   // element offsets in dynamic shared memory
  int32_t buf_width[kMaxBuffers];
  StepDesc steps[kMaxSteps];
  EpiDesc epi[kMaxEpilogue];
};

}  // namespace ponni_b200
