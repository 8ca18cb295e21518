// Streaming kernel for narrow dense chains (every width <= 32).
//
// Narrow networks (the README's 2->3->1 MLP, the 8-wide benchmark network of
// the reference) do a few FLOPs per byte, so the roofline is HBM bandwidth:
// the kernel must move input in and output out at full speed and nothing
// else.  Each thread owns V consecutive batch columns; it loads each input
// feature row segment with 16-byte loads (a warp reads 512 contiguous bytes
// per row and vector), keeps every intermediate state in registers, reads the
// (tiny) weights from shared memory as warp-wide broadcasts, and stores each
// output row segment with 16-byte stores.  Same program (steps, packed
// parameters, epilogue lists) and the same arithmetic as the tile kernel:
// FMA accumulation for fp32/fp64, per-operation rounding for fp16/bf16
// (reference Matvec::compute_output / apply_fused_epilogue,
// src/ponni_Inference.h:416-444).
//
// The program lives in device memory and is decoded once per CTA into
// compact step and epilogue tables in shared memory.  Dynamically indexed
// reads of a kernel-parameter Program would go through the constant cache's
// address-divergence path, whose throughput (not HBM) then bounds the kernel;
// a ~10 KB kernel parameter would also cost host time on every launch.
#include <cuda_runtime.h>

#include <algorithm>

#include "device_math.cuh"
#include "narrow_kernel.h"
#include "program.h"

#ifndef PONNI_B200_NARROW_VEC
#define PONNI_B200_NARROW_VEC 1  // 16-byte vectors per row and thread
#endif

namespace ponni_b200 {
namespace {

constexpr int kNarrowThreads = 256;
constexpr size_t kNarrowMaxSmem = 200 * 1024;  // tables + staging rows + weights per CTA

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

// Compact step descriptor (two 16-byte shared-memory loads).
struct alignas(16) NStep {
  int32_t kind, nin, nout, ldw;
  int32_t w_off, epi_first, n_epi, in_regs;  // in_regs: epilogue is Bias/ReLU/LeakyReLU only
};

// Compact epilogue entry; s0/s1 in the compute type.
template <class C> struct alignas(16) NEpi {
  int32_t kind, flags, p_off, pad;
  C s0, s1;
};

template <class T> struct Tables {
  using C = typename Num<T>::C;
  const NStep* steps;
  const NEpi<C>* epi;
  const T* params;
  C* stage;  // [MAXW * V][threads] staging rows, or null
};

__host__ __device__ constexpr size_t align16(size_t b) { return (b + 15) & ~(size_t)15; }

// Apply Bias / ReLU / LeakyReLU entries to one feature row of V columns held
// in registers; each operation is rounded to T (reference
// apply_fused_epilogue, src/ponni_Inference.h:428-444).
template <class T, int V>
__device__ __forceinline__ void epi_row(const Tables<T>& t, int first, int n, int f, typename Num<T>::C (&v)[V]) {
  using C = typename Num<T>::C;
  for (int e = first; e < first + n; ++e) {
    const int kind = t.epi[e].kind;
    if (kind == EPI_BIAS) {
      const C b = Num<T>::to_c(t.params[t.epi[e].p_off + f]);
#pragma unroll
      for (int j = 0; j < V; ++j) v[j] = rnd<T>(v[j] + b);
    } else if (kind == EPI_RELU) {
#pragma unroll
      for (int j = 0; j < V; ++j) v[j] = v[j] > C(0) ? v[j] : C(0);
    } else {
      const C a = t.epi[e].s0;
#pragma unroll
      for (int j = 0; j < V; ++j) v[j] = rnd<T>(v[j] > C(0) ? v[j] : a * v[j]);
    }
  }
}

// General epilogue over rows [0, rows) staged in this thread's slots of
// shared memory (stage[(f * V + j) * threads + tid], conflict-free).  Not
// unrolled, so the activation code exists once per kernel instead of once
// per unrolled register element.
template <class T, int V>
__device__ __forceinline__ void epi_staged(const Tables<T>& t, int first, int n, int rows) {
  using C = typename Num<T>::C;
  for (int e = first; e < first + n; ++e) {
    const NEpi<C> d = t.epi[e];
#pragma unroll 1
    for (int f = 0; f < rows; ++f) {
      const C b = d.kind == EPI_BIAS ? Num<T>::to_c(t.params[d.p_off + f]) : C(0);
#pragma unroll 1
      for (int j = 0; j < V; ++j) {
        C& v = t.stage[(f * V + j) * kNarrowThreads + threadIdx.x];
        if (d.kind == EPI_BIAS) v = rnd<T>(v + b);
        else if (sizeof(T) == 2 && (d.flags & EPI_FLAG_REF16))
          v = rnd<T>(activation16(d.kind, d.flags, (float)v, (float)d.s0, (float)d.s1,
                                  [](float x) { return (float)rnd<T>(x); }));
        else v = rnd<T>(activation<C>(d.kind, d.flags, v, d.s0, d.s1));
      }
    }
  }
}

// Epilogue of one step on the register rows x[0..rows).
template <class T, int MAXW, int V>
__device__ __forceinline__ void epilogue(const Tables<T>& t, const NStep& s, int rows,
                                         typename Num<T>::C (&x)[MAXW][V]) {
  if (s.n_epi == 0) return;
  if (s.in_regs) {
#pragma unroll
    for (int f = 0; f < MAXW; ++f)
      if (f < rows) epi_row<T, V>(t, s.epi_first, s.n_epi, f, x[f]);
    return;
  }
#pragma unroll
  for (int f = 0; f < MAXW; ++f)
    if (f < rows)
#pragma unroll
      for (int j = 0; j < V; ++j) t.stage[(f * V + j) * kNarrowThreads + threadIdx.x] = x[f][j];
  epi_staged<T, V>(t, s.epi_first, s.n_epi, rows);
#pragma unroll
  for (int f = 0; f < MAXW; ++f)
    if (f < rows)
#pragma unroll
      for (int j = 0; j < V; ++j) x[f][j] = t.stage[(f * V + j) * kNarrowThreads + threadIdx.x];
}

// Four consecutive packed weights W[k][o..o+3]: one shared-memory vector load
// (weight rows are padded to multiples of 8 and start 16-element aligned).
template <class T> struct alignas(4 * sizeof(T) > 16 ? 16 : 4 * sizeof(T)) W4 { T w[4]; };

// One dense step dst = W^T src (before its epilogue), in registers.
// Reference order per output: acc from 0, k ascending (Matvec::compute_output,
// src/ponni_Inference.h:416-426); fma(w, x, 0) is exactly 0 + w*x.  Outputs
// past nout (row padding) are skipped by uniform branches.
template <class T, int MAXW, int V>
__device__ __forceinline__ void dense_step(const Tables<T>& t, const NStep& s, typename Num<T>::C (&src)[MAXW][V],
                                           typename Num<T>::C (&dst)[MAXW][V]) {
  using C = typename Num<T>::C;
  constexpr int MAXW4 = (MAXW + 3) / 4;
  const T* W = t.params + s.w_off;
#pragma unroll
  for (int k = 0; k < MAXW; ++k) {
    if (k < s.nin) {
#pragma unroll
      for (int o4 = 0; o4 < MAXW4; ++o4) {
        if (o4 * 4 < s.nout) {
          const W4<T> w4 = *reinterpret_cast<const W4<T>*>(W + k * s.ldw + o4 * 4);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int o = o4 * 4 + i;
            if (o < MAXW && o < s.nout) {
              const C w = Num<T>::to_c(w4.w[i]);
#pragma unroll
              for (int j = 0; j < V; ++j) {
                C& acc = dst[o < MAXW ? o : 0][j];
                if constexpr (sizeof(T) >= 4) acc = fma(w, src[k][j], k == 0 ? C(0) : acc);
                else acc = rnd<T>((k == 0 ? C(0) : acc) + rnd<T>(w * src[k][j]));
              }
            }
          }
        }
      }
    }
  }
}

// One step on the state in cur; returns true when the result is in nxt
// (dense steps), false when it stayed in cur (pointwise runs).
template <class T, int MAXW, int V>
__device__ __forceinline__ bool run_step(const Tables<T>& t, const NStep& s, int& width,
                                         typename Num<T>::C (&cur)[MAXW][V], typename Num<T>::C (&nxt)[MAXW][V]) {
  if (s.kind == STEP_DENSE) {
    dense_step<T, MAXW, V>(t, s, cur, nxt);
    width = s.nout;
    epilogue<T, MAXW, V>(t, s, width, nxt);
    return true;
  }
  epilogue<T, MAXW, V>(t, s, width, cur);  // a pointwise run that follows no dense layer
  return false;
}

template <class T, int MAXW, int V>
__device__ __forceinline__ void store_rows(int nout, typename Num<T>::C (&x)[MAXW][V], T* __restrict__ out,
                                           int64_t out_ld, int64_t col, int64_t batch, bool full) {
  constexpr int VN = Vec16<T>::N < V ? Vec16<T>::N : V;
  constexpr int NV = V / VN;
  using VT = typename VecType<VN * sizeof(T)>::type;
#pragma unroll
  for (int f = 0; f < MAXW; ++f) {
    if (f < nout) {
      T* dst = out + (int64_t)f * out_ld + col;
      if (full) {
#pragma unroll
        for (int q = 0; q < NV; ++q) {
          VT u;
          T* e = reinterpret_cast<T*>(&u);
#pragma unroll
          for (int j = 0; j < VN; ++j) e[j] = Num<T>::from_c(x[f][q * VN + j]);
          __stcs(reinterpret_cast<VT*>(dst) + q, u);
        }
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j)
          if (col + j < batch) dst[j] = Num<T>::from_c(x[f][j]);
      }
    }
  }
}

template <class T>
size_t table_bytes(const Program& p) {
  return align16((size_t)p.n_steps * sizeof(NStep)) + align16((size_t)p.n_epi * sizeof(NEpi<typename Num<T>::C>));
}

template <class T, int MAXW, int V>
constexpr size_t stage_bytes() {
  return (size_t)MAXW * V * sizeof(typename Num<T>::C) * kNarrowThreads;
}

// Staging rows are allocated only for programs with an activation other than
// ReLU / LeakyReLU (the register path needs none).
bool needs_stage(const Program& p) {
  for (int e = 0; e < p.n_epi; ++e)
    if (p.epi[e].kind > EPI_LEAKY_RELU) return true;
  return false;
}

// Dynamic shared memory: [step table][epilogue table][staging rows][weights].
template <class T, int MAXW, int V>
size_t smem_layout(const Program& p, size_t* stage_off, size_t* stage_size) {
  const size_t tables = table_bytes<T>(p);
  const size_t stage = needs_stage(p) ? stage_bytes<T, MAXW, V>() : 0;
  if (stage_off) *stage_off = tables;
  if (stage_size) *stage_size = stage;
  return tables + stage + align16((size_t)p.n_params * sizeof(T));
}

// MAXW: register width bound (>= every layer width); V: columns per thread.
template <class T, int MAXW, int V>
__global__ void __launch_bounds__(kNarrowThreads)
    narrow_forward_kernel(const Program* __restrict__ pg, const T* __restrict__ gparams, const T* __restrict__ in,
                          int64_t in_ld, T* __restrict__ out, int64_t out_ld, int64_t batch, int vec_io,
                          int stage_off, int stage_size) {
  using C = typename Num<T>::C;
  constexpr int VN = Vec16<T>::N < V ? Vec16<T>::N : V;  // elements per vector access
  constexpr int NV = V / VN;                              // vector accesses per row
  using VT = typename VecType<VN * sizeof(T)>::type;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const Program& p = *pg;
  const int n_steps = p.n_steps, n_epi = p.n_epi, n_params = p.n_params, nin = p.nin, nout = p.nout;
  NStep* steps = reinterpret_cast<NStep*>(smem_raw);
  NEpi<C>* epi = reinterpret_cast<NEpi<C>*>(smem_raw + align16((size_t)n_steps * sizeof(NStep)));
  Tables<T> t;
  t.steps = steps;
  t.epi = epi;
  t.stage = stage_size ? reinterpret_cast<C*>(smem_raw + stage_off) : nullptr;
  T* params = reinterpret_cast<T*>(smem_raw + stage_off + stage_size);
  t.params = params;
  // ---- decode the program once per CTA ----
  for (int i = threadIdx.x; i < n_params; i += kNarrowThreads) params[i] = gparams[i];
  for (int i = threadIdx.x; i < n_steps; i += kNarrowThreads) {
    const StepDesc& s = p.steps[i];
    NStep n;
    n.kind = s.kind;
    n.nin = s.nin;
    n.nout = s.nout;
    n.ldw = s.nout_pad;
    n.w_off = (int32_t)s.w_off;
    n.epi_first = s.epi_first;
    n.n_epi = s.n_epi;
    int regs = 1;
    for (int e = s.epi_first; e < s.epi_first + s.n_epi; ++e) regs &= p.epi[e].kind <= EPI_LEAKY_RELU;
    n.in_regs = regs;
    steps[i] = n;
  }
  for (int i = threadIdx.x; i < n_epi; i += kNarrowThreads) {
    const EpiDesc& d = p.epi[i];
    NEpi<C> n;
    n.kind = d.kind;
    n.flags = d.flags;
    n.p_off = (int32_t)d.p_off;
    n.pad = 0;
    n.s0 = (C)d.s0;
    n.s1 = (C)d.s1;
    epi[i] = n;
  }
  __syncthreads();

  const int64_t ngroups = (batch + V - 1) / V;
  for (int64_t g = blockIdx.x * (int64_t)kNarrowThreads + threadIdx.x; g < ngroups;
       g += (int64_t)gridDim.x * kNarrowThreads) {
    const int64_t col = g * V;
    const bool full = vec_io && col + V <= batch;
    // Two register state arrays used in turn (a dense step writes the other).
    C xa[MAXW][V], xb[MAXW][V];
#pragma unroll
    for (int f = 0; f < MAXW; ++f) {
      if (f < nin) {
        const T* src = in + (int64_t)f * in_ld + col;
        if (full) {
#pragma unroll
          for (int q = 0; q < NV; ++q) {
            const VT u = __ldcs(reinterpret_cast<const VT*>(src) + q);
            const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int j = 0; j < VN; ++j) xa[f][q * VN + j] = Num<T>::to_c(e[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < V; ++j) xa[f][j] = col + j < batch ? Num<T>::to_c(src[j]) : C(0);
        }
      }
    }
    int width = nin;
    bool in_a = true;
    for (int si = 0; si < n_steps; ++si) {
      const NStep s = steps[si];
      if (in_a) in_a = !run_step<T, MAXW, V>(t, s, width, xa, xb);
      else in_a = run_step<T, MAXW, V>(t, s, width, xb, xa);
    }
    if (in_a) store_rows<T, MAXW, V>(nout, xa, out, out_ld, col, batch, full);
    else store_rows<T, MAXW, V>(nout, xb, out, out_ld, col, batch, full);
  }
}

template <class T, int MAXW, int V>
cudaError_t prepare(const Program& p, int num_sms, NarrowLaunch* L) {
  static_assert(V >= 1, "columns per thread");
  auto kern = narrow_forward_kernel<T, MAXW, V>;
  size_t stage_off = 0, stage_size = 0;
  const size_t smem = smem_layout<T, MAXW, V>(p, &stage_off, &stage_size);
  // The attribute is the per-function maximum: set it to the kernel's limit,
  // so that models with different needs never lower it for each other.
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kNarrowMaxSmem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kNarrowThreads, smem);
  if (e != cudaSuccess) return e;
  L->maxw = MAXW;
  L->cols = V;
  L->smem = (int)smem;
  L->stage_off = (int)stage_off;
  L->stage_size = (int)stage_size;
  L->grid = num_sms * std::max(per_sm, 1);  // persistent: every resident CTA slot once
  return cudaSuccess;
}

template <class T, int MAXW, int V>
cudaError_t launch(const NarrowLaunch& L, const Program* prog_dev, const void* params, const void* in, int64_t in_ld,
                   void* out, int64_t out_ld, int64_t batch, cudaStream_t stream) {
  const bool vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
                   ((in_ld * (int64_t)sizeof(T)) % 16 == 0) && ((out_ld * (int64_t)sizeof(T)) % 16 == 0);
  const int64_t groups = (batch + V - 1) / V;
  const int64_t want = (groups + kNarrowThreads - 1) / kNarrowThreads;
  const int grid = (int)std::min<int64_t>(want, (int64_t)L.grid);
  narrow_forward_kernel<T, MAXW, V><<<grid, kNarrowThreads, L.smem, stream>>>(
      prog_dev, static_cast<const T*>(params), static_cast<const T*>(in), in_ld, static_cast<T*>(out), out_ld, batch,
      vec ? 1 : 0, L.stage_off, L.stage_size);
  return cudaGetLastError();
}

// Columns per thread: PONNI_B200_NARROW_VEC 16-byte vectors of input row,
// capped so that the two register state arrays hold at most 128 (fp64: 64)
// values, and at least two columns for 32-bit and 16-bit types (one
// shared-memory weight load then feeds eight FMAs).
template <class T, int MAXW>
constexpr int cols_per_thread() {
  constexpr int base = (sizeof(T) == 8 ? 32 : 64) / MAXW;
  constexpr int lo = sizeof(T) == 8 ? 1 : 2;
  constexpr int cap = base > lo ? base : lo;
  constexpr int want = PONNI_B200_NARROW_VEC * Vec16<T>::N;
  int v = want < cap ? want : cap;
  int p2 = 1;
  while (p2 * 2 <= v) p2 *= 2;
  return p2;
}

template <class T>
cudaError_t prepare_width(const Program& p, int maxw, int num_sms, NarrowLaunch* L) {
  if (maxw <= 4) return prepare<T, 4, cols_per_thread<T, 4>()>(p, num_sms, L);
  if (maxw <= 8) return prepare<T, 8, cols_per_thread<T, 8>()>(p, num_sms, L);
  if (maxw <= 16) return prepare<T, 16, cols_per_thread<T, 16>()>(p, num_sms, L);
  return prepare<T, 32, cols_per_thread<T, 32>()>(p, num_sms, L);
}

template <class T>
cudaError_t launch_width(const NarrowLaunch& L, const Program* prog_dev, const void* params, const void* in,
                         int64_t in_ld, void* out, int64_t out_ld, int64_t batch, cudaStream_t stream) {
  switch (L.maxw) {
    case 4: return launch<T, 4, cols_per_thread<T, 4>()>(L, prog_dev, params, in, in_ld, out, out_ld, batch, stream);
    case 8: return launch<T, 8, cols_per_thread<T, 8>()>(L, prog_dev, params, in, in_ld, out, out_ld, batch, stream);
    case 16:
      return launch<T, 16, cols_per_thread<T, 16>()>(L, prog_dev, params, in, in_ld, out, out_ld, batch, stream);
    case 32:
      return launch<T, 32, cols_per_thread<T, 32>()>(L, prog_dev, params, in, in_ld, out, out_ld, batch, stream);
  }
  return cudaErrorInvalidValue;
}

template <class T>
size_t smem_bytes(const Program& p, int maxw) {
  if (maxw <= 4) return smem_layout<T, 4, cols_per_thread<T, 4>()>(p, nullptr, nullptr);
  if (maxw <= 8) return smem_layout<T, 8, cols_per_thread<T, 8>()>(p, nullptr, nullptr);
  if (maxw <= 16) return smem_layout<T, 16, cols_per_thread<T, 16>()>(p, nullptr, nullptr);
  return smem_layout<T, 32, cols_per_thread<T, 32>()>(p, nullptr, nullptr);
}

}  // namespace

bool narrow_eligible(int dtype, const Program& p, int* maxw_out) {
  int maxw = p.nin;
  for (int i = 0; i < p.n_steps; ++i) {
    const StepDesc& s = p.steps[i];
    if (s.kind != STEP_DENSE && s.kind != STEP_POINTWISE) return false;
    if (s.kind == STEP_DENSE && (s.flags & (DENSE_INIT_BIAS | DENSE_ADD_RESIDUAL))) return false;
    maxw = std::max(maxw, std::max(s.nin, s.nout));
  }
  if (maxw > 32) return false;
  // Tables, staging rows and weights must fit one CTA's shared memory.
  size_t smem = 0;
  switch (dtype) {
    case 0: smem = smem_bytes<float>(p, maxw); break;
    case 1: smem = smem_bytes<double>(p, maxw); break;
    case 2: smem = smem_bytes<__half>(p, maxw); break;
    case 3: smem = smem_bytes<__nv_bfloat16>(p, maxw); break;
    default: return false;
  }
  if (smem > kNarrowMaxSmem) return false;
  if (maxw_out) *maxw_out = maxw;
  return true;
}

cudaError_t narrow_prepare(int dtype, const Program& p, int maxw, int num_sms, NarrowLaunch* L) {
  L->dtype = dtype;
  switch (dtype) {
    case 0: return prepare_width<float>(p, maxw, num_sms, L);
    case 1: return prepare_width<double>(p, maxw, num_sms, L);
    case 2: return prepare_width<__half>(p, maxw, num_sms, L);
    case 3: return prepare_width<__nv_bfloat16>(p, maxw, num_sms, L);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_narrow_forward(const NarrowLaunch& L, const Program* prog_dev, const void* params, const void* in,
                                  int64_t in_ld, void* out, int64_t out_ld, int64_t batch, cudaStream_t stream) {
  switch (L.dtype) {
    case 0: return launch_width<float>(L, prog_dev, params, in, in_ld, out, out_ld, batch, stream);
    case 1: return launch_width<double>(L, prog_dev, params, in, in_ld, out, out_ld, batch, stream);
    case 2: return launch_width<__half>(L, prog_dev, params, in, in_ld, out, out_ld, batch, stream);
    case 3: return launch_width<__nv_bfloat16>(L, prog_dev, params, in, in_ld, out, out_ld, batch, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ponni_b200
