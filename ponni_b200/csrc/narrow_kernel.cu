// Streaming kernel for narrow dense chains (every width <= 32).
//
// Narrow networks (the README's 2->3->1 MLP, the 8-wide benchmark network of
// the reference) do a few FLOPs per byte, so the roofline is HBM bandwidth:
// the kernel must move input in and output out at full speed and nothing
// else.  Each thread owns V consecutive batch columns; it loads each input
// feature row segment with one 16-byte load (a warp reads 512 contiguous
// bytes per row), keeps every intermediate state in registers, reads the
// (tiny) weights from shared memory as warp-wide broadcasts, and stores each
// output row segment with one 16-byte store.  Same program (steps, packed
// parameters, epilogue lists) and the same arithmetic as the tile kernel:
// FMA accumulation for fp32/fp64, per-operation rounding for fp16/bf16
// (reference Matvec::compute_output / apply_fused_epilogue,
// src/ponni_Inference.h:416-444).
#include <cuda_runtime.h>

#include <algorithm>

#include "device_math.cuh"
#include "narrow_kernel.h"
#include "program.h"

namespace ponni_b200 {
namespace {

constexpr int kNarrowThreads = 256;

template <class T> struct Vec16;  // 16 bytes of T
template <> struct Vec16<float> { static constexpr int N = 4; };
template <> struct Vec16<double> { static constexpr int N = 2; };
template <> struct Vec16<__half> { static constexpr int N = 8; };
template <> struct Vec16<__nv_bfloat16> { static constexpr int N = 8; };

// V elements of T as one load/store of V * sizeof(T) bytes (2..16).
template <int BYTES> struct VecType;
template <> struct VecType<16> { using type = uint4; };
template <> struct VecType<8> { using type = uint2; };
template <> struct VecType<4> { using type = unsigned int; };
template <> struct VecType<2> { using type = unsigned short; };

template <class T>
__device__ __forceinline__ typename Num<T>::C epi(const Program& p, int first, int n, int f, typename Num<T>::C v,
                                                 const T* params) {
  using C = typename Num<T>::C;
  for (int e = first; e < first + n; ++e) {
    const EpiDesc& d = p.epi[e];
    if (d.kind == EPI_BIAS) v = v + Num<T>::to_c(params[d.p_off + f]);
    else v = activation<C>(d.kind, d.flags, v, (C)d.s0, (C)d.s1);
    v = rnd<T>(v);
  }
  return v;
}

// MAXW: register width bound (>= every layer width); V: columns per thread.
template <class T, int MAXW, int V>
__global__ void __launch_bounds__(kNarrowThreads)
    narrow_forward_kernel(const __grid_constant__ Program p, const T* __restrict__ gparams, const T* __restrict__ in,
                          int64_t in_ld, T* __restrict__ out, int64_t out_ld, int64_t batch, int vec_io) {
  using C = typename Num<T>::C;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* params = reinterpret_cast<T*>(smem_raw);
  for (int i = threadIdx.x; i < p.n_params; i += kNarrowThreads) params[i] = gparams[i];
  __syncthreads();

  const int64_t ngroups = (batch + V - 1) / V;
  for (int64_t g = blockIdx.x * (int64_t)kNarrowThreads + threadIdx.x; g < ngroups;
       g += (int64_t)gridDim.x * kNarrowThreads) {
    const int64_t col = g * V;
    const bool full = vec_io && col + V <= batch;
    C x[MAXW][V];
    // ---- input ----
#pragma unroll
    for (int f = 0; f < MAXW; ++f) {
      if (f < p.nin) {
        const T* src = in + (int64_t)f * in_ld + col;
        if (full) {
          using VT = typename VecType<V * sizeof(T)>::type;
          const VT u = __ldg(reinterpret_cast<const VT*>(src));
          const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
          for (int j = 0; j < V; ++j) x[f][j] = Num<T>::to_c(e[j]);
        } else {
#pragma unroll
          for (int j = 0; j < V; ++j) x[f][j] = col + j < batch ? Num<T>::to_c(src[j]) : C(0);
        }
      }
    }
    // ---- steps ----
    int width = p.nin;
    for (int si = 0; si < p.n_steps; ++si) {
      const StepDesc& s = p.steps[si];
      if (s.kind == STEP_DENSE) {
        const T* W = params + s.w_off;
        C y[MAXW][V];
#pragma unroll
        for (int o = 0; o < MAXW; ++o) {
          if (o < s.nout) {
#pragma unroll
            for (int j = 0; j < V; ++j) y[o][j] = C(0);
#pragma unroll
            for (int k = 0; k < MAXW; ++k) {
              if (k < s.nin) {
                const C w = Num<T>::to_c(W[k * s.nout_pad + o]);
#pragma unroll
                for (int j = 0; j < V; ++j) {
                  if constexpr (sizeof(T) >= 4) y[o][j] = fma(w, x[k][j], y[o][j]);
                  else y[o][j] = rnd<T>(y[o][j] + rnd<T>(w * x[k][j]));
                }
              }
            }
#pragma unroll
            for (int j = 0; j < V; ++j) y[o][j] = epi<T>(p, s.epi_first, s.n_epi, o, y[o][j], params);
          }
        }
#pragma unroll
        for (int o = 0; o < MAXW; ++o)
#pragma unroll
          for (int j = 0; j < V; ++j) x[o][j] = y[o][j];
        width = s.nout;
      } else {  // STEP_POINTWISE
#pragma unroll
        for (int f = 0; f < MAXW; ++f)
          if (f < width)
#pragma unroll
            for (int j = 0; j < V; ++j) x[f][j] = epi<T>(p, s.epi_first, s.n_epi, f, x[f][j], params);
      }
    }
    // ---- output ----
#pragma unroll
    for (int f = 0; f < MAXW; ++f) {
      if (f < p.nout) {
        T* dst = out + (int64_t)f * out_ld + col;
        if (full) {
          using VT = typename VecType<V * sizeof(T)>::type;
          VT u;
          T* e = reinterpret_cast<T*>(&u);
#pragma unroll
          for (int j = 0; j < V; ++j) e[j] = Num<T>::from_c(x[f][j]);
          *reinterpret_cast<VT*>(dst) = u;
        } else {
#pragma unroll
          for (int j = 0; j < V; ++j)
            if (col + j < batch) dst[j] = Num<T>::from_c(x[f][j]);
        }
      }
    }
  }
}

template <class T, int MAXW, int V>
cudaError_t launch(const Program& p, const void* params, const void* in, int64_t in_ld, void* out, int64_t out_ld,
                   int64_t batch, int num_sms, cudaStream_t stream) {
  auto kern = narrow_forward_kernel<T, MAXW, V>;
  const size_t smem = ((size_t)p.n_params * sizeof(T) + 15) & ~(size_t)15;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const bool vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
                   ((in_ld * (int64_t)sizeof(T)) % 16 == 0) && ((out_ld * (int64_t)sizeof(T)) % 16 == 0);
  const int64_t groups = (batch + V - 1) / V;
  const int64_t want = (groups + kNarrowThreads - 1) / kNarrowThreads;
  const int grid = (int)std::min<int64_t>(want, (int64_t)num_sms * 8);
  kern<<<grid, kNarrowThreads, smem, stream>>>(p, static_cast<const T*>(params), static_cast<const T*>(in), in_ld,
                                                static_cast<T*>(out), out_ld, batch, vec ? 1 : 0);
  return cudaGetLastError();
}

// Columns per thread: a 16-byte vector, capped so that the two register
// state arrays hold at most 128 (fp64: 64) values.
template <class T, int MAXW>
constexpr int cols_per_thread() {
  constexpr int cap = (sizeof(T) == 8 ? 32 : 64) / MAXW;
  constexpr int v = Vec16<T>::N < cap ? Vec16<T>::N : cap;
  return v < 1 ? 1 : v;
}

template <class T>
cudaError_t dispatch_width(const Program& p, int maxw, const void* params, const void* in, int64_t in_ld, void* out,
                           int64_t out_ld, int64_t batch, int num_sms, cudaStream_t stream) {
  if (maxw <= 4) return launch<T, 4, cols_per_thread<T, 4>()>(p, params, in, in_ld, out, out_ld, batch, num_sms, stream);
  if (maxw <= 8) return launch<T, 8, cols_per_thread<T, 8>()>(p, params, in, in_ld, out, out_ld, batch, num_sms, stream);
  if (maxw <= 16)
    return launch<T, 16, cols_per_thread<T, 16>()>(p, params, in, in_ld, out, out_ld, batch, num_sms, stream);
  return launch<T, 32, cols_per_thread<T, 32>()>(p, params, in, in_ld, out, out_ld, batch, num_sms, stream);
}

}  // namespace

bool narrow_eligible(const Program& p, int* maxw_out) {
  int maxw = p.nin;
  for (int i = 0; i < p.n_steps; ++i) {
    const StepDesc& s = p.steps[i];
    if (s.kind != STEP_DENSE && s.kind != STEP_POINTWISE) return false;
    if (s.kind == STEP_DENSE && (s.flags & (DENSE_INIT_BIAS | DENSE_ADD_RESIDUAL))) return false;
    maxw = std::max(maxw, std::max(s.nin, s.nout));
  }
  if (maxw > 32) return false;
  if (maxw_out) *maxw_out = maxw;
  return true;
}

cudaError_t launch_narrow_forward(int dtype, const Program& p, int maxw, const void* params, const void* in,
                                  int64_t in_ld, void* out, int64_t out_ld, int64_t batch, int num_sms,
                                  cudaStream_t stream) {
  switch (dtype) {
    case 0: return dispatch_width<float>(p, maxw, params, in, in_ld, out, out_ld, batch, num_sms, stream);
    case 1: return dispatch_width<double>(p, maxw, params, in, in_ld, out, out_ld, batch, num_sms, stream);
    case 2: return dispatch_width<__half>(p, maxw, params, in, in_ld, out, out_ld, batch, num_sms, stream);
    case 3: return dispatch_width<__nv_bfloat16>(p, maxw, params, in, in_ld, out, out_ld, batch, num_sms, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ponni_b200
