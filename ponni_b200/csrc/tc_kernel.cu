// Tensor-core dense-chain kernel for sm_100a (tcgen05 UMMA + TMEM).
//
// One persistent CTA per SM with up to four thread groups, each owning one
// tile slot, so that the slots' epilogues overlap the others' MMAs.  Per batch tile of 128
// columns:
//   input  : cp.async (16 B, zero-filled tail) of the batch-contiguous input
//            rows into a staging tile, prefetched one tile ahead into a
//            second buffer; 16-bit models stage it as an MN-major SW128
//            operand and use it for layer 0 directly, fp32 models stage it
//            row-major and split it into K-major bf16 operand parts;
//   layer l: thread 0 issues the UMMA chain D[128 x N] = A[128 x K] B[N x K]^T
//            (tcgen05.mma, fp32 accumulator in TMEM) and commits it to an
//            mbarrier; all threads wait (bounded), then each warp reads its 32
//            TMEM lanes (= 32 batch columns) with tcgen05.ld, applies bias and
//            activation in fp32 (the reference's fused epilogue,
//            src/ponni_Inference.h:416-444) and writes the next layer's
//            K-major operand to shared memory, or the caller's output for the
//            last layer (coalesced: a warp writes 32 consecutive columns).
// Weights and biases are staged once per CTA (the packed image built on the
// host is byte-for-byte the swizzled operand layout).
//
// Arithmetic:
//   fp32 models: every operand x is split exactly into three bfloat16 parts
//     x = b0 + b1 + b2 (b0 = bf16(x), b1 = bf16(x - b0), b2 = x - b0 - b1;
//     8 + 8 + 8 significand bits cover fp32's 24) and D accumulates the six
//     products whose parts sum to order <= 2 (a1B1, a0B2, a2B0, a0B1, a1B0,
//     a0B0, smallest first); the three dropped products are below 2^-24
//     relative.  Six bf16 MMAs cost the same tensor time as three TF32 ones
//     and, unlike a two-way TF32 split (22 bits), represent the operands
//     exactly, so the result is fp32-accurate;
//   fp16/bf16 models: operands in the model type, fp32 accumulation, states
//     rounded to the model type where the reference stores them.
//
// Every wait is bounded: on timeout the kernel records an error code in
// `err`, stops issuing work, frees its TMEM and returns.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "device_math.cuh"
#include "tc_common.cuh"
#include "tc_kernel.h"

PONNI_B200_SKIP_ARRIVE_FLAG(tc)

#include "tc_kernel_body.cuh"  // (after the flag: the wait-test build's body reads it)

namespace ponni_b200 {
namespace {
using namespace tc;

template <class T, int TPS>
__global__ void __launch_bounds__(TPS == 128 && sizeof(T) == 2 ? kTcMaxThreads : kTcMaxThreads / 2, 1)
    tc_forward_kernel(const __grid_constant__ TcProgram p, const unsigned char* __restrict__ image,
                      const T* __restrict__ in, int64_t in_ld, T* __restrict__ out, int64_t out_ld, int64_t batch,
                      int in_vec, int* __restrict__ err) {
  tck::tc_forward_body<T, TPS, tck::RuntimeShape>(p, image, in, in_ld, out, out_ld, batch, in_vec, err);
}

template <class T, int TPS>
cudaError_t launch_tps(const TcProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                       int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  auto kern = tc_forward_kernel<T, TPS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
  if (e != cudaSuccess) return e;
  const bool vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && ((in_ld * (int64_t)sizeof(T)) % 16 == 0);
  kern<<<grid, p.slots * TPS, p.smem_bytes, stream>>>(p, static_cast<const unsigned char*>(image),
                                                     static_cast<const T*>(in), in_ld, static_cast<T*>(out), out_ld,
                                                     batch, vec ? 1 : 0, err);
  return cudaGetLastError();
}

template <class T>
cudaError_t launch_impl(const TcProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                        int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  if (p.slot_threads == 128) return launch_tps<T, 128>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
  return launch_tps<T, 256>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
}

}  // namespace

cudaError_t launch_tc_forward(const TcProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                              int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  switch (p.dtype) {
    case 0: return launch_impl<float>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
    case 2: return launch_impl<__half>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
    case 3: return launch_impl<__nv_bfloat16>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ponni_b200
