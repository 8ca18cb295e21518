// Host entry point of the tensor-core dense-chain kernel (tc_kernel.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "tc_program.h"

namespace ponni_b200 {

// `image`: device copy of the packed parameter image (TcProgram::image_bytes);
// `err`: device int set to a nonzero code when a bounded wait gives up.
cudaError_t launch_tc_forward(const TcProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                              int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream);

}  // namespace ponni_b200
