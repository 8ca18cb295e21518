// Test kernel of the in-kernel device API (include/ponni_b200_device.cuh):
// one thread per batch column calls forward_batch_parallel_in_kernel, as an
// application kernel embedding the model would.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ponni_b200_device.cuh"

namespace {

constexpr int kNbuf = 8;

template <class T, int MAXW>
__global__ void embedded_forward(ponni::device::Model m, const T* in, int64_t in_ld, T* out, int64_t out_ld,
                                 int64_t batch) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < batch) ponni::device::forward_batch_parallel_in_kernel<T, MAXW, kNbuf>(m, in, in_ld, out, out_ld, i);
}

template <class T>
cudaError_t launch(const ponni::device::Model& m, const void* in, int64_t in_ld, void* out, int64_t out_ld,
                   int64_t batch) {
  const int threads = 128;
  const int64_t blocks = (batch + threads - 1) / threads;
  const T* x = static_cast<const T*>(in);
  T* y = static_cast<T*>(out);
  if (m.max_width <= 16) embedded_forward<T, 16><<<blocks, threads>>>(m, x, in_ld, y, out_ld, batch);
  else if (m.max_width <= 64) embedded_forward<T, 64><<<blocks, threads>>>(m, x, in_ld, y, out_ld, batch);
  else embedded_forward<T, 256><<<blocks, threads>>>(m, x, in_ld, y, out_ld, batch);
  return cudaGetLastError();
}

}  // namespace

// Returns 0 on success, a ponni_b200_status (> 0), -1 for a model beyond
// this test kernel's bounds, or -2 for a CUDA error.
extern "C" int pb_test_embedded_forward(void* model, const void* in, int64_t in_ld, void* out, int64_t out_ld,
                                        int64_t batch) {
  auto* mdl = static_cast<ponni_b200_model*>(model);
  ponni::device::Model m;
  const ponni_b200_status s = ponni::device::get_model(mdl, &m);
  if (s != PONNI_B200_OK) return (int)s;
  if (m.max_width > 256 || m.num_buffers > kNbuf) return -1;
  cudaError_t e = cudaErrorInvalidValue;
  switch (ponni_b200_model_dtype(mdl)) {
    case PONNI_B200_F32: e = launch<float>(m, in, in_ld, out, out_ld, batch); break;
    case PONNI_B200_F64: e = launch<double>(m, in, in_ld, out, out_ld, batch); break;
    case PONNI_B200_F16: e = launch<__half>(m, in, in_ld, out, out_ld, batch); break;
    case PONNI_B200_BF16: e = launch<__nv_bfloat16>(m, in, in_ld, out, out_ld, batch); break;
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return e == cudaSuccess ? 0 : -2;
}
