// Host entry points of the narrow-chain streaming kernel (narrow_kernel.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "program.h"

namespace ponni_b200 {

// True when the program is a chain of dense and pointwise steps at most 32
// wide whose weights fit shared memory; *maxw receives the widest width.
// dtype: 0 fp32, 1 fp64, 2 fp16, 3 bf16.
bool narrow_eligible(int dtype, const Program& p, int* maxw);

// Launch configuration, fixed when the model is planned.
struct NarrowLaunch {
  int dtype = 0;
  int maxw = 0;       // register width bound of the instantiation (4, 8, 16, 32)
  int cols = 1;       // batch columns per thread
  int smem = 0;       // dynamic shared memory bytes
  int stage_off = 0;  // staging rows (byte offset and size; size 0 = none)
  int stage_size = 0;
  int grid = 0;       // persistent grid: SMs x resident CTAs
};

// Choose the instantiation and grid for a narrow-eligible program (on the
// current device).
cudaError_t narrow_prepare(int dtype, const Program& p, int maxw, int num_sms, NarrowLaunch* L);

// prog_dev: the same Program in device memory.
cudaError_t launch_narrow_forward(const NarrowLaunch& L, const Program* prog_dev, const void* params, const void* in,
                                  int64_t in_ld, void* out, int64_t out_ld, int64_t batch, cudaStream_t stream);

}  // namespace ponni_b200
