// Tensor-core dense-chain kernel with the weights streamed from HBM/L2
// (tc_stream.cu), for 16-bit chains whose weights exceed shared memory
// (the 64->256x5->32 bf16 network: 573 KB of weights).
//
// Work unit ("job"): one layer for one tile of 128 batch columns,
// D[128 x N<=256] = A[128 x K] * B[N x K]^T, with B streamed in chunks of
// K = 64 (one 128-byte swizzle block: N rows x 128 B <= 32 KB) through a
// ring of shared-memory stages.  Two tiles are in flight per CTA and their
// jobs alternate layer by layer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "tc_stream_program.h"

struct ponni_b200_model;

namespace ponni_b200 {

// Plan the streamed kernel for a Matvec[Bias][activation] chain of a 16-bit
// model; builds the chunked, pre-swizzled weight image.  False with `why`
// when not eligible.
// `rec` (optional) receives the image location of every trainable parameter.
struct ParamMap;
bool ts_plan(const ponni_b200_model* m, TsProgram& p, std::vector<unsigned char>& image, std::string& why,
             ParamMap* rec = nullptr);

cudaError_t launch_ts_forward(const TsProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                              int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream);

// Model-specialised build of the same kernel (narrow_jit.cpp): the body of
// tc_stream_body.cuh compiled with NVRTC, the epilogue's layer loop unrolled
// with every layer's widths, bias flag and activation as compile-time
// constants.  Parameters stay in the device image.  False with `why` when
// NVRTC or the toolkit headers are unavailable, or in CTA-pair mode.
bool ts_jit_build(const TsProgram& p, const void** kernel, std::string* why);
// Launch of `kernel` from ts_jit_build (single-CTA form), same arguments as
// launch_ts_forward.
cudaError_t launch_ts_forward_jit(const void* kernel, const TsProgram& p, const void* image, const void* in,
                                  int64_t in_ld, void* out, int64_t out_ld, int64_t batch, int grid, int* err,
                                  cudaStream_t stream);

}  // namespace ponni_b200
