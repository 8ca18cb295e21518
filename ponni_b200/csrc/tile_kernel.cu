// Fused tile kernel: the whole layer program per batch tile, on chip.
//
// Replaces the reference's single Kokkos kernel of
// Inference::forward_batch_parallel (src/ponni_Inference.h:384-388), which runs
// one thread per sample through traverse_mixed_batch_parallel (:454-555) and
// materialises every barrier state into HBM scratch (tmp1/tmp2/saved states).
//
// B200 design:
//  * persistent CTAs (grid = SMs x resident CTAs) walk batch tiles of BT
//    columns; the next tile's input is prefetched with cp.async while the
//    current tile is computed;
//  * every intermediate state lives in shared memory as [width][BT] (batch
//    contiguous, like the reference's LayoutRight Views), so HBM traffic is
//    input in + output out only; when they fit, the packed parameters are
//    staged in shared memory once per CTA as well;
//  * a dense layer is a register-tiled SIMT contraction: each thread owns
//    kTO=8 output features x kTB=4 batch columns and a warp covers a 32x32
//    tile (4 row groups x 8 column groups), so each 16-byte weight or
//    activation load is one shared-memory wavefront serving 4 or 8 lanes;
//  * the Bias/activation layers that follow a dense layer run on the
//    accumulators in registers (the reference's fused epilogue), with a
//    compile-time specialised path for [Bias][activation]; the final dense
//    block writes the caller's output directly;
//  * cross-feature barriers (LayerNorm, MinMaxNorm, Softmax, LogSoftmax) and
//    residual layers (Save_State, Binop_Add, Binop_Concatenate) run per column
//    on the shared tile in the reference's exact operation order;
//    Binop_Projection_Add is a dense step over the saved state that adds into
//    the main state.
#include <cuda_runtime.h>

#include "device_math.cuh"
#include "program.h"
#include "tile_kernel.h"

namespace ponni_b200 {

// ---------------------------------------------------------------------------
// cp.async helpers (16-byte, L2-only, zero fill beyond src_bytes).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Stage input columns [col0, col0+BT) of the feature-major input into the
// shared tile dst[nin][BT]; columns at or beyond `batch` are zero.
template <class T>
__device__ __forceinline__ void load_input_tile(T* dst, const T* __restrict__ in, int64_t in_ld, int nin,
                                                int bt, int64_t col0, int64_t batch, bool vec_ok) {
  constexpr int E = 16 / sizeof(T);  // elements per 16-byte chunk
  if (vec_ok) {
    const int chunks_per_row = bt / E;
    const int total = nin * chunks_per_row;
    for (int i = threadIdx.x; i < total; i += kThreads) {
      const int row = i / chunks_per_row;
      const int ch = i - row * chunks_per_row;
      const int64_t col = col0 + (int64_t)ch * E;
      const int64_t valid = batch - col;
      const int bytes = valid >= E ? 16 : (valid > 0 ? (int)valid * (int)sizeof(T) : 0);
      const T* src = in + (int64_t)row * in_ld + (bytes > 0 ? col : 0);
      cp_async16(dst + row * bt + ch * E, src, bytes);
    }
  } else {
    const int total = nin * bt;
    for (int i = threadIdx.x; i < total; i += kThreads) {
      const int row = i / bt;
      const int c = i - row * bt;
      const int64_t col = col0 + c;
      dst[i] = col < batch ? in[(int64_t)row * in_ld + col] : Num<T>::from_c(0);
    }
  }
}

// One activation: 16-bit models with the reference's rounding points when
// the entry asks for them, else in the compute type.
template <class T>
__device__ __forceinline__ typename Num<T>::C act_value(int kind, int flags, typename Num<T>::C v,
                                                         typename Num<T>::C s0, typename Num<T>::C s1) {
  if constexpr (sizeof(T) == 2) {
    if (flags & EPI_FLAG_REF16) return activation16(kind, flags, v, s0, s1, [](float x) { return rnd<T>(x); });
  }
  return activation<typename Num<T>::C>(kind, flags, v, s0, s1);
}

// Apply the pointwise epilogue list of a step to one value of feature f.
template <class T>
__device__ __forceinline__ typename Num<T>::C apply_epilogue(const Program& p, int first, int n, int f,
                                                              typename Num<T>::C v, const T* params) {
  using C = typename Num<T>::C;
  for (int e = first; e < first + n; ++e) {
    const EpiDesc& d = p.epi[e];
    if (d.kind == EPI_BIAS) {
      v = v + Num<T>::to_c(params[d.p_off + f]);
    } else {
      v = act_value<T>(d.kind, d.flags, v, (C)d.s0, (C)d.s1);
    }
    v = rnd<T>(v);
  }
  return v;
}

// ---------------------------------------------------------------------------
// Vector loads/stores used by the dense micro-tile.  Weights may sit in
// shared or global memory (generic loads); activations are in shared memory.
__device__ __forceinline__ void ld_w8(const float* p, float w[8]) {
  float4 a = reinterpret_cast<const float4*>(p)[0];
  float4 b = reinterpret_cast<const float4*>(p)[1];
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}
__device__ __forceinline__ void ld_w8(const double* p, double w[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    double2 a = reinterpret_cast<const double2*>(p)[i];
    w[2 * i] = a.x; w[2 * i + 1] = a.y;
  }
}
__device__ __forceinline__ void ld_x4(const float* p, float x[4]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
}
__device__ __forceinline__ void ld_x4(const double* p, double x[4]) {
  double2 a = reinterpret_cast<const double2*>(p)[0];
  double2 b = reinterpret_cast<const double2*>(p)[1];
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
__device__ __forceinline__ void st_x4(float* p, const float x[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
}
__device__ __forceinline__ void st_x4(double* p, const double x[4]) {
  reinterpret_cast<double2*>(p)[0] = make_double2(x[0], x[1]);
  reinterpret_cast<double2*>(p)[1] = make_double2(x[2], x[3]);
}
__device__ __forceinline__ void st_x4(__half* p, const float x[4]) {
  __half2 a = __floats2half2_rn(x[0], x[1]), b = __floats2half2_rn(x[2], x[3]);
  uint2 u;
  u.x = *reinterpret_cast<unsigned*>(&a);
  u.y = *reinterpret_cast<unsigned*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ void st_x4(__nv_bfloat16* p, const float x[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
  uint2 u;
  u.x = *reinterpret_cast<unsigned*>(&a);
  u.y = *reinterpret_cast<unsigned*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// Store one row segment of kTB results to the caller's output.
template <class T>
__device__ __forceinline__ void store_out4(T* __restrict__ out, int64_t out_ld, int o, int64_t col,
                                           int64_t batch, const typename Num<T>::C v[kTB], bool vec_ok) {
  T* dst = out + (int64_t)o * out_ld + col;
  if (vec_ok && col + kTB <= batch) {
    st_x4(dst, v);
  } else {
#pragma unroll
    for (int j = 0; j < kTB; ++j)
      if (col + j < batch) dst[j] = Num<T>::from_c(v[j]);
  }
}

// Epilogue of a dense micro-tile: optional residual, the pointwise layers,
// then the store to shared memory or to the caller's output.  ACT >= 0 is
// the compile-time [Bias][activation] fast path; ACT < 0 walks the generic
// epilogue list.
template <class T, int ACT>
__device__ __forceinline__ void dense_epilogue(const Program& p, const StepDesc& s,
                                               typename Num<T>::C (&acc)[kTO][kTB], int o0, int c0,
                                               const T* params, const T* res, T* dst, T* __restrict__ out,
                                               int64_t out_ld, int64_t col0, int64_t batch, bool out_vec_ok) {
  using C = typename Num<T>::C;
  const int bt = p.bt;
#pragma unroll
  for (int i = 0; i < kTO; ++i) {
    const int o = o0 + i;
    if (o >= s.nout) break;
    C v[kTB];
    C b = C(0);
    if (ACT >= 0 && s.fast_bias_off >= 0) b = Num<T>::to_c(params[s.fast_bias_off + o]);
#pragma unroll
    for (int j = 0; j < kTB; ++j) {
      C a = acc[i][j];
      if (s.flags & DENSE_ADD_RESIDUAL) a = rnd<T>(Num<T>::to_c(res[o * bt + c0 + j]) + a);
      if (ACT >= 0) {
        if (s.fast_bias_off >= 0) a = rnd<T>(a + b);
        if (ACT != EPI_NONE) a = rnd<T>(act_value<T>(ACT, s.fast_act_flags, a, (C)s.s0, (C)s.s1));
        v[j] = a;
      } else {
        v[j] = apply_epilogue<T>(p, s.epi_first, s.n_epi, o, a, params);
      }
    }
    if (s.flags & DENSE_TO_GLOBAL) store_out4<T>(out, out_ld, o, col0 + c0, batch, v, out_vec_ok);
    else st_x4(dst + o * bt + c0, v);
  }
}

// Work decomposition of a dense step: warp tiles of 4 row groups x 8 column
// groups; returns false for the idle lanes of a partial row tile.
__device__ __forceinline__ bool dense_item(int i, int ncg, int nrg, int& o0, int& c0) {
  const int wc_n = ncg >> 3;
  const int w = i >> 5, l = i & 31;
  const int wr = w / wc_n, wc = w - wr * wc_n;
  const int rg = wr * 4 + (l >> 3), cg = wc * 8 + (l & 7);
  o0 = rg * kTO;
  c0 = cg * kTB;
  return rg < nrg;
}

__device__ __forceinline__ int dense_items(int ncg, int nrg) { return ((nrg + 3) >> 2) * (ncg >> 3) * 32; }

// Dense step for float / double: out[o][c] = sum_k W[k][o] * in[k][c],
// accumulated in k-ascending order from 0 (reference Matvec::compute_output,
// src/layers/ponni_Matvec.h:71-79) or from the bias (Projection_Add,
// src/layers/ponni_Binop_Projection_Add.h:82-96).  Products are fused into
// the accumulation (FMA).
template <class T, int ACT>
__device__ __forceinline__ void dense_step_wide(const Program& p, const StepDesc& s, const T* params,
                                                const T* src, const T* res, T* dst, T* __restrict__ out,
                                                int64_t out_ld, int64_t col0, int64_t batch, bool out_vec_ok) {
  const int bt = p.bt;
  const int ncg = bt / kTB;
  const int nrg = s.nout_pad / kTO;
  const T* W = params + s.w_off;
  const int n_items = dense_items(ncg, nrg);
  for (int item = threadIdx.x; item < n_items; item += kThreads) {
    int o0, c0;
    if (!dense_item(item, ncg, nrg, o0, c0)) continue;
    T acc[kTO][kTB];
#pragma unroll
    for (int i = 0; i < kTO; ++i) {
      T b = T(0);
      if ((s.flags & DENSE_INIT_BIAS) && o0 + i < s.nout) b = params[s.b_off + o0 + i];
#pragma unroll
      for (int j = 0; j < kTB; ++j) acc[i][j] = b;
    }
    const T* wp = W + o0;
    const T* xp = src + c0;
    const int nout_pad = s.nout_pad;
#pragma unroll 4
    for (int k = 0; k < s.nin; ++k) {
      T w[kTO], x[kTB];
      ld_w8(wp + k * nout_pad, w);
      ld_x4(xp + k * bt, x);
#pragma unroll
      for (int i = 0; i < kTO; ++i)
#pragma unroll
        for (int j = 0; j < kTB; ++j) acc[i][j] = fma(w[i], x[j], acc[i][j]);
    }
    dense_epilogue<T, ACT>(p, s, acc, o0, c0, params, res, dst, out, out_ld, col0, batch, out_vec_ok);
  }
}

// Dense step for half / bfloat16.  The reference accumulates in `real`
// (Matvec::compute_output with real = half_t/bhalf_t): every product and every
// partial sum is rounded to the 16-bit type.  Two adjacent batch columns are
// processed as one packed pair (HMUL2 + HADD2; the _rn forms forbid
// contraction into an HFMA2, so both roundings happen as in the reference).
template <class T> struct Pair;
template <> struct Pair<__half> {
  using T2 = __half2;
  static __device__ __forceinline__ T2 lo(T2 v) { return __low2half2(v); }
  static __device__ __forceinline__ T2 hi(T2 v) { return __high2half2(v); }
  static __device__ __forceinline__ T2 splat(__half v) { return __half2half2(v); }
  static __device__ __forceinline__ float2 to_f2(T2 v) { return __half22float2(v); }
};
template <> struct Pair<__nv_bfloat16> {
  using T2 = __nv_bfloat162;
  static __device__ __forceinline__ T2 lo(T2 v) { return __low2bfloat162(v); }
  static __device__ __forceinline__ T2 hi(T2 v) { return __high2bfloat162(v); }
  static __device__ __forceinline__ T2 splat(__nv_bfloat16 v) { return __bfloat162bfloat162(v); }
  static __device__ __forceinline__ float2 to_f2(T2 v) { return __bfloat1622float2(v); }
};

template <class T, int ACT>
__device__ __forceinline__ void dense_step_pair(const Program& p, const StepDesc& s, const T* params,
                                                const T* src, const T* res, T* dst, T* __restrict__ out,
                                                int64_t out_ld, int64_t col0, int64_t batch, bool out_vec_ok) {
  using P = Pair<T>;
  using T2 = typename P::T2;
  const int bt = p.bt;
  const int ncg = bt / kTB;
  const int nrg = s.nout_pad / kTO;
  const T* W = params + s.w_off;
  const int n_items = dense_items(ncg, nrg);
  for (int item = threadIdx.x; item < n_items; item += kThreads) {
    int o0, c0;
    if (!dense_item(item, ncg, nrg, o0, c0)) continue;
    T2 acc[kTO][kTB / 2];
#pragma unroll
    for (int i = 0; i < kTO; ++i) {
      T b = Num<T>::from_c(0.0f);
      if ((s.flags & DENSE_INIT_BIAS) && o0 + i < s.nout) b = params[s.b_off + o0 + i];
#pragma unroll
      for (int j = 0; j < kTB / 2; ++j) acc[i][j] = P::splat(b);
    }
    const T* wp = W + o0;
    const T* xp = src + c0;
    const int nout_pad = s.nout_pad;
    const bool half_fma = (s.flags & DENSE_HALF_FMA) != 0;  // generated arithmetic: fused per product
#pragma unroll 4
    for (int k = 0; k < s.nin; ++k) {
      uint4 wr = *reinterpret_cast<const uint4*>(wp + k * nout_pad);
      uint2 xr = *reinterpret_cast<const uint2*>(xp + k * bt);
      T2 w2[4] = {*reinterpret_cast<T2*>(&wr.x), *reinterpret_cast<T2*>(&wr.y),
                  *reinterpret_cast<T2*>(&wr.z), *reinterpret_cast<T2*>(&wr.w)};
      T2 x2[2] = {*reinterpret_cast<T2*>(&xr.x), *reinterpret_cast<T2*>(&xr.y)};
#pragma unroll
      for (int i = 0; i < kTO; ++i) {
        const T2 wb = (i & 1) ? P::hi(w2[i >> 1]) : P::lo(w2[i >> 1]);
#pragma unroll
        for (int j = 0; j < kTB / 2; ++j)
          acc[i][j] = half_fma ? __hfma2(wb, x2[j], acc[i][j]) : __hadd2_rn(acc[i][j], __hmul2_rn(wb, x2[j]));
      }
    }
    float accf[kTO][kTB];
#pragma unroll
    for (int i = 0; i < kTO; ++i)
#pragma unroll
      for (int j = 0; j < kTB / 2; ++j) {
        float2 f = P::to_f2(acc[i][j]);
        accf[i][2 * j] = f.x;
        accf[i][2 * j + 1] = f.y;
      }
    dense_epilogue<T, ACT>(p, s, accf, o0, c0, params, res, dst, out, out_ld, col0, batch, out_vec_ok);
  }
}

template <class T, int ACT>
__device__ __forceinline__ void dense_step_act(const Program& p, const StepDesc& s, const T* params,
                                               const T* src, const T* res, T* dst, T* __restrict__ out,
                                               int64_t out_ld, int64_t col0, int64_t batch, bool out_vec_ok) {
  if constexpr (sizeof(T) == 2)
    dense_step_pair<T, ACT>(p, s, params, src, res, dst, out, out_ld, col0, batch, out_vec_ok);
  else
    dense_step_wide<T, ACT>(p, s, params, src, res, dst, out, out_ld, col0, batch, out_vec_ok);
}

// Dispatch to the compile-time epilogue specialisation (uniform branch).
template <class T>
__device__ __forceinline__ void dense_step(const Program& p, const StepDesc& s, const T* params, const T* src,
                                           const T* res, T* dst, T* __restrict__ out, int64_t out_ld,
                                           int64_t col0, int64_t batch, bool out_vec_ok) {
#define PONNI_DENSE(A) dense_step_act<T, A>(p, s, params, src, res, dst, out, out_ld, col0, batch, out_vec_ok)
  if (!(s.flags & DENSE_FAST_EPI)) {
    PONNI_DENSE(-1);
    return;
  }
  switch (s.fast_act) {
    case EPI_NONE: PONNI_DENSE(EPI_NONE); break;
    case EPI_RELU: PONNI_DENSE(EPI_RELU); break;
    case EPI_LEAKY_RELU: PONNI_DENSE(EPI_LEAKY_RELU); break;
    case EPI_SILU: PONNI_DENSE(EPI_SILU); break;
    case EPI_GELU: PONNI_DENSE(EPI_GELU); break;
    case EPI_TANH: PONNI_DENSE(EPI_TANH); break;
    case EPI_SIGMOID: PONNI_DENSE(EPI_SIGMOID); break;
    default: PONNI_DENSE(-1); break;
  }
#undef PONNI_DENSE
}

// ---------------------------------------------------------------------------
// Correctly rounded single operations that the compiler may not contract, so
// the barrier layers reproduce the reference's per-operation rounding.
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double div_rn(double a, double b) { return __ddiv_rn(a, b); }

template <class T> using CT = typename Num<T>::C;
template <class T> __device__ __forceinline__ CT<T> radd(CT<T> a, CT<T> b) { return rnd<T>(add_rn(a, b)); }
template <class T> __device__ __forceinline__ CT<T> rsub(CT<T> a, CT<T> b) { return rnd<T>(sub_rn(a, b)); }
template <class T> __device__ __forceinline__ CT<T> rmul(CT<T> a, CT<T> b) { return rnd<T>(mul_rn(a, b)); }
template <class T> __device__ __forceinline__ CT<T> rdiv(CT<T> a, CT<T> b) { return rnd<T>(div_rn(a, b)); }

// exp / log of the softmax barriers: 16-bit models take the correctly rounded
// float value (e16_exp / e16_log, the host C library's result).
template <class T> __device__ __forceinline__ CT<T> x_exp(CT<T> v) {
  if constexpr (sizeof(T) == 2) return e16_exp(v);
  else return m_exp(v);
}
template <class T> __device__ __forceinline__ CT<T> x_log(CT<T> v) {
  if constexpr (sizeof(T) == 2) return e16_log(v);
  else return m_log(v);
}

// LayerNorm per column: two-pass mean and biased variance,
// 1/sqrt(var + eps), gamma * xhat + beta (src/layers/ponni_LayerNorm.h:77-99).
template <class T>
__device__ void layernorm_step(const StepDesc& s, int bt, const T* params, T* x) {
  using C = CT<T>;
  const int n = s.nin;
  const C eps = (C)s.s0;
  const T* gamma = params + s.w_off;
  const T* beta = params + s.b_off;
  if (s.flags & LN_WELFORD) {
    // Generated LayerNormalization (src/generator/kokkos_nn/emitter.py:867-889):
    // one Welford pass in Scalar (16-bit models: in float, emitter.py:1161-1191,
    // the mean and 1/stddev rounded once to the model type), then
    // ((x - mean) * inv) * scale + bias with every operation rounded.
    for (int c = threadIdx.x; c < bt; c += kThreads) {
      C mean = C(0), m2 = C(0);
      for (int i = 0; i < n; ++i) {
        const C value = Num<T>::to_c(x[i * bt + c]);
        const C delta = sub_rn(value, mean);
        mean = add_rn(mean, div_rn(delta, (C)(i + 1)));
        m2 = add_rn(m2, mul_rn(delta, sub_rn(value, mean)));
      }
      const C var = div_rn(m2, (C)n);
      const C inv = rnd<T>(div_rn(C(1), m_sqrt(add_rn(var, eps))));
      mean = rnd<T>(mean);
      for (int i = 0; i < n; ++i) {
        C v = rmul<T>(rsub<T>(Num<T>::to_c(x[i * bt + c]), mean), inv);
        v = radd<T>(rmul<T>(v, Num<T>::to_c(gamma[i])), Num<T>::to_c(beta[i]));
        x[i * bt + c] = Num<T>::from_c(v);
      }
    }
    return;
  }
  for (int c = threadIdx.x; c < bt; c += kThreads) {
    C mean = C(0);
    for (int i = 0; i < n; ++i) mean = radd<T>(mean, Num<T>::to_c(x[i * bt + c]));
    mean = rdiv<T>(mean, (C)n);
    C var = C(0);
    for (int i = 0; i < n; ++i) {
      C d = rsub<T>(Num<T>::to_c(x[i * bt + c]), mean);
      var = radd<T>(var, rmul<T>(d, d));
    }
    var = rdiv<T>(var, (C)n);
    // 1 / std::sqrt(real): for 16-bit models the square root is a float and
    // only the quotient is rounded
    const C inv_std = rdiv<T>(C(1), m_sqrt(radd<T>(var, eps)));
    for (int i = 0; i < n; ++i) {
      C xhat = rmul<T>(rsub<T>(Num<T>::to_c(x[i * bt + c]), mean), inv_std);
      C v = radd<T>(rmul<T>(Num<T>::to_c(gamma[i]), xhat), Num<T>::to_c(beta[i]));
      x[i * bt + c] = Num<T>::from_c(v);
    }
  }
}

// MinMaxNorm per column (src/layers/ponni_MinMaxNorm.h:68-84).
template <class T>
__device__ void minmax_step(const StepDesc& s, int bt, T* x) {
  using C = CT<T>;
  const int n = s.nin;
  const C out_min = (C)s.s0, out_max = (C)s.s1, eps = (C)s.s2;
  for (int c = threadIdx.x; c < bt; c += kThreads) {
    C mn = Num<T>::to_c(x[c]), mx = mn;
    for (int i = 1; i < n; ++i) {
      C v = Num<T>::to_c(x[i * bt + c]);
      if (v < mn) mn = v;
      if (v > mx) mx = v;
    }
    const C scale = rdiv<T>(rsub<T>(out_max, out_min), radd<T>(rsub<T>(mx, mn), eps));
    for (int i = 0; i < n; ++i) {
      C v = Num<T>::to_c(x[i * bt + c]);
      x[i * bt + c] = Num<T>::from_c(radd<T>(out_min, rmul<T>(rsub<T>(v, mn), scale)));
    }
  }
}

// Softmax / LogSoftmax per column (src/layers/ponni_Softmax.h:46-57,
// src/layers/ponni_LogSoftmax.h:46-57).
template <class T, bool LOG>
__device__ void softmax_step(const StepDesc& s, int bt, T* x) {
  using C = CT<T>;
  const int n = s.nin;
  for (int c = threadIdx.x; c < bt; c += kThreads) {
    C mx = Num<T>::to_c(x[c]);
    for (int i = 1; i < n; ++i) {
      C v = Num<T>::to_c(x[i * bt + c]);
      mx = v > mx ? v : mx;
    }
    // std::exp / std::log of a 16-bit `real` are floats, rounded only where
    // the reference stores them (src/layers/ponni_Softmax.h:46-57)
    C sum = C(0);
    for (int i = 0; i < n; ++i)
      sum = radd<T>(sum, x_exp<T>(rsub<T>(Num<T>::to_c(x[i * bt + c]), mx)));
    if (LOG) {
      const C lse = radd<T>(x_log<T>(sum), mx);
      for (int i = 0; i < n; ++i)
        x[i * bt + c] = Num<T>::from_c(rsub<T>(Num<T>::to_c(x[i * bt + c]), lse));
    } else {
      for (int i = 0; i < n; ++i) {
        const C e = x_exp<T>(rsub<T>(Num<T>::to_c(x[i * bt + c]), mx));
        x[i * bt + c] = Num<T>::from_c(rdiv<T>(e, sum));
      }
    }
  }
}

// Pointwise layers that do not follow a dense layer, in place.
template <class T>
__device__ void pointwise_step(const Program& p, const StepDesc& s, const T* params, T* x) {
  const int bt = p.bt;
  const int total = s.nin * bt;
  for (int i = threadIdx.x; i < total; i += kThreads) {
    const int f = i / bt;
    x[i] = Num<T>::from_c(apply_epilogue<T>(p, s.epi_first, s.n_epi, f, Num<T>::to_c(x[i]), params));
  }
}

// Copy the final on-chip state to the caller's output.
template <class T>
__device__ void store_tile(const T* x, int nout, int bt, T* __restrict__ out, int64_t out_ld, int64_t col0,
                           int64_t batch) {
  const int total = nout * bt;
  for (int i = threadIdx.x; i < total; i += kThreads) {
    const int f = i / bt;
    const int c = i - f * bt;
    if (col0 + c < batch) out[(int64_t)f * out_ld + col0 + c] = x[i];
  }
}

// ---------------------------------------------------------------------------
template <class T>
__global__ void __launch_bounds__(kThreads)
    tile_forward_kernel(const __grid_constant__ Program p, const T* __restrict__ gparams,
                        const T* __restrict__ in, int64_t in_ld, T* __restrict__ out, int64_t out_ld,
                        int64_t batch, int in_vec, int out_vec) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sm = reinterpret_cast<T*>(smem_raw);
  const int bt = p.bt;
  const int64_t ntiles = (batch + bt - 1) / bt;
  int64_t tile = blockIdx.x;
  if (tile >= ntiles) return;
  const int in_off[2] = {p.buf_off[p.in_buf], p.buf_off[p.in_buf2]};
  int cur = 0;
  // Parameters: stage once per CTA when they fit (16-byte chunks; the packed
  // buffer is padded to a multiple of 16 bytes).
  const T* params = gparams;
  if (p.params_in_smem) {
    T* ps = sm + p.param_smem_off;
    const int chunks = (int)((p.n_params * sizeof(T)) / 16);
    for (int i = threadIdx.x; i < chunks; i += kThreads) cp_async16(ps + i * (16 / sizeof(T)), gparams + i * (16 / sizeof(T)), 16);
    params = ps;
  }
  load_input_tile<T>(sm + in_off[0], in, in_ld, p.nin, bt, tile * bt, batch, in_vec != 0);
  cp_async_commit();
  for (; tile < ntiles; tile += gridDim.x) {
    const int64_t col0 = tile * bt;
    const int64_t next = tile + gridDim.x;
    if (next < ntiles)
      load_input_tile<T>(sm + in_off[cur ^ 1], in, in_ld, p.nin, bt, next * bt, batch, in_vec != 0);
    cp_async_commit();
    cp_async_wait_1();
    __syncthreads();
    auto buf = [&](int id) -> T* {
      if (id < 0) return nullptr;
      return sm + (id == p.in_buf ? in_off[cur] : p.buf_off[id]);
    };
    for (int si = 0; si < p.n_steps; ++si) {
      const StepDesc& s = p.steps[si];
      T* src = buf(s.src);
      T* dst = buf(s.dst);
      T* aux = buf(s.aux);
      switch (s.kind) {
        case STEP_DENSE:
          dense_step<T>(p, s, params, src, aux, dst, out, out_ld, col0, batch, out_vec != 0);
          break;
        case STEP_POINTWISE: pointwise_step<T>(p, s, params, src); break;
        case STEP_LAYERNORM: layernorm_step<T>(s, bt, params, src); break;
        case STEP_MINMAXNORM: minmax_step<T>(s, bt, src); break;
        case STEP_SOFTMAX: softmax_step<T, false>(s, bt, src); break;
        case STEP_LOGSOFTMAX: softmax_step<T, true>(s, bt, src); break;
        case STEP_COPY:
          for (int i = threadIdx.x; i < s.nin * bt; i += kThreads) dst[i] = src[i];
          break;
        case STEP_ADD:
          for (int i = threadIdx.x; i < s.nin * bt; i += kThreads)
            src[i] = Num<T>::from_c(radd<T>(Num<T>::to_c(src[i]), Num<T>::to_c(aux[i])));
          break;
        case STEP_CONCAT: {
          // Distinct source and destination tiles (the reference's SArray form).
          const int n_main = s.nin, n_aux = s.nout - s.nin;
          const bool after = (s.flags & CONCAT_AFTER) != 0;
          for (int i = threadIdx.x; i < s.nout * bt; i += kThreads) {
            const int f = i / bt, c = i - f * bt;
            T v;
            if (after) v = f < n_main ? src[f * bt + c] : aux[(f - n_main) * bt + c];
            else v = f < n_aux ? aux[f * bt + c] : src[(f - n_aux) * bt + c];
            dst[i] = v;
          }
          break;
        }
        default: break;
      }
      __syncthreads();
    }
    if (p.final_buf >= 0) store_tile<T>(buf(p.final_buf), p.nout, bt, out, out_ld, col0, batch);
    __syncthreads();
    cur ^= 1;
  }
  cp_async_wait_0();
}

template <class T>
static cudaError_t launch_impl(const Program& p, const void* params, const void* in, int64_t in_ld, void* out,
                               int64_t out_ld, int64_t batch, int grid, size_t smem, cudaStream_t stream) {
  auto kern = tile_forward_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const bool in_vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && ((in_ld * sizeof(T)) % 16 == 0);
  const bool out_vec = (reinterpret_cast<uintptr_t>(out) % 16 == 0) && ((out_ld * sizeof(T)) % 16 == 0);
  kern<<<grid, kThreads, smem, stream>>>(p, static_cast<const T*>(params), static_cast<const T*>(in), in_ld,
                                         static_cast<T*>(out), out_ld, batch, in_vec, out_vec);
  return cudaGetLastError();
}

template <class T>
static int occupancy_impl(size_t smem) {
  auto kern = tile_forward_kernel<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kern, kThreads, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return blocks;
}

cudaError_t launch_tile_forward(int dtype, const Program& p, const void* params, const void* in, int64_t in_ld,
                                void* out, int64_t out_ld, int64_t batch, int grid, size_t smem,
                                cudaStream_t stream) {
  switch (dtype) {
    case 0: return launch_impl<float>(p, params, in, in_ld, out, out_ld, batch, grid, smem, stream);
    case 1: return launch_impl<double>(p, params, in, in_ld, out, out_ld, batch, grid, smem, stream);
    case 2: return launch_impl<__half>(p, params, in, in_ld, out, out_ld, batch, grid, smem, stream);
    case 3: return launch_impl<__nv_bfloat16>(p, params, in, in_ld, out, out_ld, batch, grid, smem, stream);
  }
  return cudaErrorInvalidValue;
}

int tile_forward_occupancy(int dtype, size_t smem) {
  switch (dtype) {
    case 0: return occupancy_impl<float>(smem);
    case 1: return occupancy_impl<double>(smem);
    case 2: return occupancy_impl<__half>(smem);
    case 3: return occupancy_impl<__nv_bfloat16>(smem);
  }
  return 0;
}

}  // namespace ponni_b200
