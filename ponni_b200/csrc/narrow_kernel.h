// Host entry points of the narrow-chain streaming kernel (narrow_kernel.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "program.h"

namespace ponni_b200 {

// True when the program is a chain of dense and pointwise steps at most 32
// wide; *maxw receives the widest width.
bool narrow_eligible(const Program& p, int* maxw);

cudaError_t launch_narrow_forward(int dtype, const Program& p, int maxw, const void* params, const void* in,
                                  int64_t in_ld, void* out, int64_t out_ld, int64_t batch, int num_sms,
                                  cudaStream_t stream);

}  // namespace ponni_b200
