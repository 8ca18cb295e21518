// Host entry points of the fused tile kernel (tile_kernel.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "program.h"

namespace ponni_b200 {

// dtype: 0 f32, 1 f64, 2 f16, 3 bf16 (ponni_b200_dtype).
cudaError_t launch_tile_forward(int dtype, const Program& p, const void* params, const void* in,
                                int64_t in_ld, void* out, int64_t out_ld, int64_t batch, int grid,
                                size_t smem, cudaStream_t stream);
// Resident CTAs per SM for `smem` bytes of dynamic shared memory (0 = does not fit).
int tile_forward_occupancy(int dtype, size_t smem);

}  // namespace ponni_b200
