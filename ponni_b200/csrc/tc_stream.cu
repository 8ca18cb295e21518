// Tensor-core dense-chain kernel with streamed weights (sm_100a, tcgen05).
//
// For 16-bit Matvec[Bias][activation] chains whose weights do not fit in
// shared memory next to the operand tiles (e.g. 64->256x5->32 bf16: 573 KB).
// One persistent CTA per SM, warp-specialised:
//   producer (warp 16, one thread): streams the pre-swizzled weight chunks of
//     every job, in job order, from global memory (L2-resident: every CTA
//     reads the same image) into a ring of shared-memory stages with 1-D bulk
//     copies (cp.async.bulk, completion counted in bytes on the stage's
//     "full" mbarrier; no multicast);
//   MMA issuer (warp 17, issue loop run by the whole warp, one elected lane
//     issues): per job (one layer of one tile)
//     issues D[128 x N<=256] += A[128 x K] * B[N x K]^T chunk by chunk
//     (tcgen05.mma kind::f16, fp32 accumulator in the slot's 256 TMEM
//     columns), frees each ring stage with tcgen05.commit and signals the
//     finished job on the slot's "acc full" mbarrier;
//   epilogue (warps 0-15: two groups of 8, one per tile slot, each 4 TMEM
//     lane quarters x 2 column halves): per job of its slot,
//     tcgen05.ld of the accumulator, bias, activation (reference fused
//     epilogue, src/ponni_Inference.h:416-444), and the next layer's K-major
//     operand, written in place into the slot's operand buffer (the job's
//     MMAs have completed), or the caller's output; each column half then
//     signals its own mbarrier.  They also stage each tile's input (cp.async,
//     the MN-major layer-0 operand, in the same buffer) once the slot's last
//     layer has consumed the buffer.
// Pair mode (the default; clusters of two CTAs on two SMs): the even CTA
// issues M = 256 MMAs (tcgen05 cta_group::2) over both CTAs' tiles, each
// CTA streams only half of every weight chunk (N / 2 rows) into its own
// ring, and the odd CTA's MMA warp relays the arrival of its half; this
// halves the weight bytes staged and the MMA instructions issued per SM.
// Two tiles (slots) are in flight and their jobs alternate layer by layer,
// so one slot's epilogue runs while the tensor core works on the other's;
// the two epilogue groups run independently, which keeps the MUFU unit fed
// while the other group loads accumulators or stores operands.
//
// In this fp32-accumulation mode SiLU, sigmoid and tanh use the hardware
// tanh approximation (sigmoid(x) = (1 + tanh(x/2)) / 2), one MUFU operation
// per value, whose error is below one unit of the 16-bit model type.
//
// Every wait is bounded; a role that gives up raises a shared abort flag
// (the others see it and leave), records an error code, and the CTA drains
// its bulk copies and MMAs before it frees TMEM and returns.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include "device_math.cuh"
#include "tc_common.cuh"
#include "tc_stream.h"

PONNI_B200_SKIP_ARRIVE_FLAG(ts)

#include "tc_stream_body.cuh"  // (after the flag: the wait-test build's body reads it)

namespace ponni_b200 {
namespace {
using namespace tsk;

template <class T, bool PAIR>
__global__ void __launch_bounds__(kTsThreads, 1)
    ts_forward_kernel(const __grid_constant__ TsProgram p, const unsigned char* __restrict__ image,
                      const T* __restrict__ in, int64_t in_ld, T* __restrict__ out, int64_t out_ld, int64_t batch,
                      int in_vec, const __grid_constant__ CUtensorMap in_map, int in_tma, int* __restrict__ err) {
  ts_forward_body<T, PAIR, TsRuntimeShape>(p, image, in, in_ld, out, out_ld, batch, in_vec, in_map, in_tma, err);
}

bool getenv_flag_off(const char* name) {
  const char* v = getenv(name);
  return v && atoi(v) == 0;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      f = nullptr;
    }
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// Tensor map of the caller's input [nin features x batch columns] (row
// stride in_ld elements) with boxes of 64 columns x k0 features and 128-byte
// swizzle; features nin..k0 and columns past the batch read as zeros.
// False when the input does not meet the copy engine's alignment rules (base
// and row stride multiples of 16 bytes) or the entry point is missing; the
// kernel then stages its tiles with cp.async.
template <class T>
bool make_input_map(CUtensorMap& map, const void* in, int64_t in_ld, int nin, int k0, int64_t batch) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc || getenv_flag_off("PONNI_B200_TS_TMA")) return false;
  if (reinterpret_cast<uintptr_t>(in) % 16 != 0 || (in_ld * 2) % 16 != 0 || k0 > 256 || batch < 1) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)batch, (cuuint64_t)nin};
  const cuuint64_t strides[1] = {(cuuint64_t)in_ld * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)k0};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  return enc(&map, dt, 2, const_cast<void*>(in), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <class T>
cudaError_t launch_impl(const TsProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                        int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  const bool vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && ((in_ld * (int64_t)sizeof(T)) % 16 == 0);
  const unsigned char* img = static_cast<const unsigned char*>(image);
  const T* x = static_cast<const T*>(in);
  T* y = static_cast<T*>(out);
  if (!p.pair) {
    auto kern = ts_forward_kernel<T, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
    if (e != cudaSuccess) return e;
    CUtensorMap map;
    std::memset(&map, 0, sizeof map);
    const bool tma = make_input_map<T>(map, in, in_ld, p.nin, p.layers[0].k_pad, batch);
    kern<<<grid, kTsThreads, p.smem_bytes, stream>>>(p, img, x, in_ld, y, out_ld, batch, vec ? 1 : 0, map,
                                                     tma ? 1 : 0, err);
    return cudaGetLastError();
  }
  // Clusters of two CTAs; the grid is a whole number of pairs, at most one
  // pair per pair of tiles.
  auto kern = ts_forward_kernel<T, true>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
  if (e != cudaSuccess) return e;
  const int64_t ntiles = (batch + kTcM - 1) / kTcM;
  const int64_t pairs = std::max<int64_t>(1, std::min<int64_t>(grid / 2, (ntiles + 1) / 2));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kTsThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CUtensorMap map;  // pair mode stages its tiles with cp.async
  std::memset(&map, 0, sizeof map);
  return cudaLaunchKernelEx(&cfg, kern, p, img, x, in_ld, y, out_ld, batch, vec ? 1 : 0, map, 0, err);
}

}  // namespace

cudaError_t launch_ts_forward(const TsProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                              int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  switch (p.dtype) {
    case 2: return launch_impl<__half>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
    case 3: return launch_impl<__nv_bfloat16>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_ts_forward_jit(const void* kernel, const TsProgram& p, const void* image, const void* in,
                                  int64_t in_ld, void* out, int64_t out_ld, int64_t batch, int grid, int* err,
                                  cudaStream_t stream) {
  if (p.pair || (p.dtype != 2 && p.dtype != 3)) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
  if (e != cudaSuccess) return e;
  int vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && ((in_ld * 2) % 16 == 0);
  CUtensorMap map;
  std::memset(&map, 0, sizeof map);
  int tma = (p.dtype == 2 ? make_input_map<__half>(map, in, in_ld, p.nin, p.layers[0].k_pad, batch)
                          : make_input_map<__nv_bfloat16>(map, in, in_ld, p.nin, p.layers[0].k_pad, batch))
                ? 1
                : 0;
  long long a_in_ld = in_ld, a_out_ld = out_ld, a_batch = batch;
  TsProgram prog = p;
  void* args[] = {&prog, const_cast<void**>(&image), const_cast<void**>(&in), &a_in_ld, &out, &a_out_ld, &a_batch,
                  &vec, &map, &tma, &err};
  return cudaLaunchKernel(kernel, dim3(grid), dim3(kTsThreads), args, p.smem_bytes, stream);
}

}  // namespace ponni_b200
