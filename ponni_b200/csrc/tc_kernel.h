// Host entry point of the tensor-core dense-chain kernel (tc_kernel.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "tc_program.h"

namespace ponni_b200 {

// `image`: device copy of the packed parameter image (TcProgram::image_bytes);
// `err`: device int set to a nonzero code when a bounded wait gives up.
cudaError_t launch_tc_forward(const TcProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                              int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream);

// Model-specialised build of the same kernel (narrow_jit.cpp): the body of
// tc_kernel_body.cuh compiled with NVRTC for this program's layer structure
// (layer count, widths, accumulator groups, activations, bias flags as
// compile-time constants).  Parameters stay in the device image, so parameter
// updates need no recompilation.  False with `why` when NVRTC or the toolkit
// headers are unavailable (the generic kernel then runs).
bool tc_jit_build(const TcProgram& p, const void** kernel, std::string* why);
cudaError_t launch_tc_forward_jit(const void* kernel, const TcProgram& p, const void* image, const void* in,
                                  int64_t in_ld, void* out, int64_t out_ld, int64_t batch, int grid, int* err,
                                  cudaStream_t stream);

}  // namespace ponni_b200
