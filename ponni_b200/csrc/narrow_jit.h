// Model-specialised narrow-chain kernel, generated and compiled at plan time.
//
// The reference ships a generator (src/generator/kokkos_nn) that emits
// straight-line per-model inference code.  The B200 counterpart for narrow
// chains (every width <= 32): the planner writes a CUDA kernel whose layer
// widths, step sequence and epilogue operations are compile-time constants,
// compiles it with NVRTC for sm_100a and loads it with cudaLibraryLoadData.
// The weights are not baked in: they travel as a __grid_constant__ kernel
// parameter read at static offsets (constant-bank operands), so changing the
// weights reuses the compiled kernel, and so do models of the same structure.
// When NVRTC is unavailable or the parameters exceed the kernel-parameter
// space, the generic narrow kernel (narrow_kernel.cu) runs instead.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "program.h"

namespace ponni_b200 {

struct NarrowJit {
  const void* kernel = nullptr;      // cudaKernel_t of the compiled kernel
  int cols = 1;                      // batch columns per thread
  int elem = 4;                      // storage element bytes
  int grid = 0;                      // persistent grid (SMs x resident CTAs)
  std::vector<unsigned char> params; // parameter block in the compute type
};

// The generated CUDA source for a narrow-eligible program (exposed for tests
// and diagnostics); dtype 0 fp32, 1 fp64, 2 fp16, 3 bf16.
std::string narrow_jit_source(int dtype, const Program& p, int maxw, int* cols);

// Build (or fetch from the process-wide cache) the kernel of this program and
// convert the packed parameters (model dtype) to the kernel's parameter block.
// Returns false with *why set when the generic kernel has to be used.
bool narrow_jit_build(int dtype, const Program& p, int maxw, const std::vector<unsigned char>& packed, int num_sms,
                      NarrowJit* J, std::string* why);

// Re-derive the kernel's parameter block from new packed parameters (the
// compiled kernel is kept).
void narrow_jit_refresh(int dtype, const Program& p, const std::vector<unsigned char>& packed, NarrowJit* J);

cudaError_t narrow_jit_launch(const NarrowJit& J, const void* in, int64_t in_ld, void* out, int64_t out_ld,
                              int64_t batch, cudaStream_t stream);

}  // namespace ponni_b200
