// Host-buffer forward pipeline and the synthetic input generator.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "model.h"

using namespace ponni_b200;

namespace {

// Counter-based generator: a splitmix64-style finaliser over
// (seed, row, column), so any GPU can regenerate any column of any shard and
// the 1-GPU and N-GPU runs see identical inputs.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
  z = (z ^ (z >> 27)) * UINT64_C(0x94d049bb133111eb);
  return z ^ (z >> 31);
}

__device__ __forceinline__ double unit_open(uint64_t h) {  // (0, 1)
  return ((double)(h >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

template <class T> __device__ __forceinline__ T from_double(double v);
template <> __device__ __forceinline__ float from_double<float>(double v) { return (float)v; }
template <> __device__ __forceinline__ double from_double<double>(double v) { return v; }
template <> __device__ __forceinline__ __half from_double<__half>(double v) { return __float2half_rn((float)v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_double<__nv_bfloat16>(double v) {
  return __float2bfloat16_rn((float)v);
}

template <class T>
__global__ void fill_kernel(T* out, int64_t rows, int64_t cols, int64_t ld, int64_t col0, uint64_t seed, int dist,
                            double lo, double hi) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const uint64_t key = mix64(seed ^ mix64(((uint64_t)r << 40) ^ (uint64_t)(col0 + c)));
    const double u1 = unit_open(key);
    double v;
    if (dist == 0) {  // Box-Muller
      const double u2 = unit_open(mix64(key + UINT64_C(0x9e3779b97f4a7c15)));
      v = sqrt(-2.0 * log(u1)) * cospi(2.0 * u2);
    } else {
      v = lo + (hi - lo) * u1;
    }
    out[r * ld + c] = from_double<T>(v);
  }
}

ponni_b200_status cuda_status(ponni_b200_model* m, cudaError_t e, const char* what) {
  return pb_fail(m, PONNI_B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

ponni_b200_status ponni_b200_fill_synthetic(ponni_b200_dtype dtype, void* ptr, int64_t rows, int64_t cols, int64_t ld,
                                            int64_t col0, uint64_t seed, int dist, double lo, double hi,
                                            void* stream) {
  if (!ptr || rows < 0 || cols < 0 || ld < cols) return PONNI_B200_ERR_INVALID_ARGUMENT;
  if (rows == 0 || cols == 0) return PONNI_B200_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t total = rows * cols;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  switch (dtype) {
    case PONNI_B200_F32:
      fill_kernel<float><<<blocks, 256, 0, s>>>((float*)ptr, rows, cols, ld, col0, seed, dist, lo, hi);
      break;
    case PONNI_B200_F64:
      fill_kernel<double><<<blocks, 256, 0, s>>>((double*)ptr, rows, cols, ld, col0, seed, dist, lo, hi);
      break;
    case PONNI_B200_F16:
      fill_kernel<__half><<<blocks, 256, 0, s>>>((__half*)ptr, rows, cols, ld, col0, seed, dist, lo, hi);
      break;
    case PONNI_B200_BF16:
      fill_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((__nv_bfloat16*)ptr, rows, cols, ld, col0, seed, dist, lo, hi);
      break;
    default: return PONNI_B200_ERR_INVALID_ARGUMENT;
  }
  return cudaGetLastError() == cudaSuccess ? PONNI_B200_OK : PONNI_B200_ERR_CUDA;
}

// Host-memory forward: column chunks alternate between two streams, each with
// its own device staging slot, so the H2D copy of one chunk, the kernel of
// the previous one and the D2H copy of the one before overlap (the copy
// engines of each direction and the SMs work concurrently).
ponni_b200_status ponni_b200_forward_host(ponni_b200_model* m, const void* input, int64_t in_ld, void* output,
                                          int64_t out_ld, int64_t batch) {
  if (!m) return PONNI_B200_ERR_INVALID_ARGUMENT;
  if (batch <= 0) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "Inference requires a nonzero batch size");
  if (!input || !output) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "input/output pointer is NULL");
  if (in_ld < batch || out_ld < batch)
    return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "row stride smaller than the batch size");
  DeviceGuard guard(m->device);
  ponni_b200_status st = pb_plan(m);
  if (st) return st;
  cudaError_t e = cudaSuccess;
  if (!m->copy_stream) {
    e = cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_status(m, e, "cudaStreamCreate");
  }
  const size_t esz = dtype_bytes(m->dtype);
  const int nin = ponni_b200_num_inputs(m), nout = ponni_b200_num_outputs(m);
  const size_t col_bytes = (size_t)(nin + nout) * esz;
  int64_t chunk = (int64_t)((size_t)64 << 20) / (int64_t)col_bytes;
  chunk = std::max<int64_t>(128, chunk / 128 * 128);
  chunk = std::min<int64_t>(chunk, (batch + 127) / 128 * 128);
  const size_t slot_bytes = (size_t)chunk * col_bytes;
  if (m->stage_bytes < 2 * slot_bytes) {
    if (m->stage_dev) {
      cudaStreamSynchronize(m->stream);
      cudaStreamSynchronize(m->copy_stream);
      cudaFree(m->stage_dev);
    }
    m->stage_dev = nullptr;
    m->stage_bytes = 0;
    e = cudaMalloc(&m->stage_dev, 2 * slot_bytes);
    if (e != cudaSuccess) return cuda_status(m, e, "cudaMalloc(staging)");
    m->stage_bytes = 2 * slot_bytes;
  }
  cudaStream_t streams[2] = {m->stream, m->copy_stream};
  // Work queued by the caller on the model stream comes first.
  cudaEvent_t ev;
  cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  cudaEventRecord(ev, m->stream);
  cudaStreamWaitEvent(m->copy_stream, ev, 0);
  int idx = 0;
  for (int64_t c0 = 0; c0 < batch; c0 += chunk, idx ^= 1) {
    const int64_t n = std::min(chunk, batch - c0);
    cudaStream_t s = streams[idx];
    unsigned char* din = static_cast<unsigned char*>(m->stage_dev) + idx * slot_bytes;
    unsigned char* dout = din + (size_t)nin * chunk * esz;
    e = cudaMemcpy2DAsync(din, (size_t)chunk * esz, static_cast<const unsigned char*>(input) + c0 * esz,
                          (size_t)in_ld * esz, (size_t)n * esz, nin, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) break;
    st = ponni_b200_forward(m, din, chunk, dout, chunk, n, s);
    if (st) break;
    e = cudaMemcpy2DAsync(static_cast<unsigned char*>(output) + c0 * esz, (size_t)out_ld * esz, dout,
                          (size_t)chunk * esz, (size_t)n * esz, nout, cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) break;
  }
  cudaError_t e1 = cudaStreamSynchronize(streams[0]);
  cudaError_t e2 = cudaStreamSynchronize(streams[1]);
  cudaEventDestroy(ev);
  if (st) return st;
  if (e == cudaSuccess) e = e1 != cudaSuccess ? e1 : e2;
  if (e != cudaSuccess) return cuda_status(m, e, "forward_host");
  return pb_check_device_error(m);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Host-buffer forward without any device allocation.
//
// Some callers cannot allocate device memory while they run inference: an
// application that hands all of its GPU memory to its own pool or allocator
// at start-up, a process whose allocation budget is fixed before a
// time-stepping loop begins, or code where a cudaMalloc would synchronise
// the device at the wrong moment.  For them this entry point stages the
// host input and output in a static device array that the library holds for
// the life of the process (on every GPU that loads it), instead of the
// cudaMalloc'd staging of ponni_b200_forward_host.
namespace {

constexpr size_t kStaticStageBytes = (size_t)64 << 20;  // 64 MiB per GPU
static __device__ __align__(256) unsigned char g_static_stage[kStaticStageBytes];

// Device address of g_static_stage, looked up at set-up once per device
// (with that device current) and kept with the CUDA context it belongs to:
// if the application has since reset the device (a new primary context),
// the address is looked up again instead of reusing a stale one.
constexpr int kMaxDevices = 64;
struct StageAddress {
  void* ctx = nullptr;
  void* ptr = nullptr;
};
StageAddress g_static_stage_addr[kMaxDevices];
std::mutex g_static_stage_mutex;

// The current driver context (cuCtxGetCurrent through the runtime's entry
// point query, so the library needs no link against the driver library).
void* current_context() {
  typedef int (*CtxGetCurrent)(void**);
  static CtxGetCurrent fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      f = nullptr;
    }
    return reinterpret_cast<CtxGetCurrent>(f);
  }();
  void* ctx = nullptr;
  if (fn && fn(&ctx) != 0) ctx = nullptr;
  return ctx;
}

cudaError_t static_stage_address(int device, void** out) {
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_static_stage_mutex);
  StageAddress& a = g_static_stage_addr[device];
  void* ctx = current_context();
  if (!a.ptr || ctx != a.ctx) {
    // In host code g_static_stage is only a stand-in symbol; the device
    // address comes from the runtime, with the device current.
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_stage);
    if (e != cudaSuccess) return e;
    a.ptr = p;
    a.ctx = ctx;
  }
  *out = a.ptr;
  return cudaSuccess;
}

}  // namespace

extern "C" ponni_b200_status ponni_b200_forward_host_static(ponni_b200_model* m, const void* input, int64_t in_ld,
                                                            void* output, int64_t out_ld, int64_t batch) {
  if (!m) return PONNI_B200_ERR_INVALID_ARGUMENT;
  if (batch <= 0) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "Inference requires a nonzero batch size");
  if (!input || !output) return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "input/output pointer is NULL");
  if (in_ld < batch || out_ld < batch)
    return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT, "row stride smaller than the batch size");
  // Planning uploads the parameters (an allocation): it must have happened
  // already, through ponni_b200_model_kernel() or an earlier forward.
  if (!m->planned || m->params_dirty)
    return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT,
                   "model not prepared: call ponni_b200_model_kernel() once before the first "
                   "ponni_b200_forward_host_static() (and again after changing parameters)");
  const size_t esz = dtype_bytes(m->dtype);
  const int nin = ponni_b200_num_inputs(m), nout = ponni_b200_num_outputs(m);
  const size_t need = (size_t)batch * (size_t)(nin + nout) * esz;
  if (need > kStaticStageBytes) {
    return pb_fail(m, PONNI_B200_ERR_INVALID_ARGUMENT,
                   "batch of " + std::to_string(batch) + " columns needs " + std::to_string(need) +
                       " bytes of device staging; the static staging buffer holds " +
                       std::to_string(kStaticStageBytes) + " bytes (at most " +
                       std::to_string(kStaticStageBytes / ((size_t)(nin + nout) * esz)) +
                       " columns for this model)");
  }
  DeviceGuard guard(m->device);
  void* stage = nullptr;
  cudaError_t e = static_stage_address(m->device, &stage);
  if (e != cudaSuccess) return cuda_status(m, e, "cudaGetSymbolAddress(static staging)");
  // Staging row stride: the batch rounded up to 16 bytes when that fits (the
  // kernels' 16-byte vector paths need aligned rows), else the batch itself.
  const int64_t per16 = (int64_t)(16 / esz);
  int64_t ld = (batch + per16 - 1) / per16 * per16;
  auto layout_fits = [&](int64_t l, size_t* out_off) {
    const size_t in_bytes = (size_t)nin * (size_t)l * esz;
    size_t off = (in_bytes + 255) & ~(size_t)255;
    if (off + (size_t)nout * (size_t)l * esz > kStaticStageBytes) off = in_bytes;
    *out_off = off;
    return off + (size_t)nout * (size_t)l * esz <= kStaticStageBytes;
  };
  size_t out_off = 0;
  if (!layout_fits(ld, &out_off)) {
    ld = batch;
    layout_fits(ld, &out_off);
  }
  unsigned char* din = static_cast<unsigned char*>(stage);
  unsigned char* dout = din + out_off;
  cudaStream_t s = m->stream;
  e = cudaMemcpy2DAsync(din, (size_t)ld * esz, input, (size_t)in_ld * esz, (size_t)batch * esz, nin,
                        cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_status(m, e, "input copy");
  ponni_b200_status st = ponni_b200_forward(m, din, ld, dout, ld, batch, s);
  if (st) return st;
  e = cudaMemcpy2DAsync(output, (size_t)out_ld * esz, dout, (size_t)ld * esz, (size_t)batch * esz, nout,
                        cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return cuda_status(m, e, "output copy");
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(m, e, "forward_host_static");
  return pb_check_device_error(m);
}
