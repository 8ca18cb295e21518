// Per-dtype arithmetic of the tile kernel.
//
// Storage type T is the model's `real` (float, double, half_t, bhalf_t in the
// reference, src/ponni_create_model.h:70-98).  Compute type C is float for the
// 16-bit types and T otherwise.  Every reference operation on `real` rounds to
// `real`, so the 16-bit paths round after each operation (rnd()), which is the
// behaviour of Kokkos half_t/bhalf_t arithmetic; the transcendental functions
// are evaluated in float and rounded once, as PONNI's TwoHalf does for every
// non-linear function (reference src/utils/ponni_TwoHalf.h:138-370).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "program.h"

namespace ponni_b200 {

template <class T> struct Num;
template <> struct Num<float> {
  using C = float;
  static __device__ __forceinline__ float to_c(float x) { return x; }
  static __device__ __forceinline__ float from_c(float x) { return x; }
};
template <> struct Num<double> {
  using C = double;
  static __device__ __forceinline__ double to_c(double x) { return x; }
  static __device__ __forceinline__ double from_c(double x) { return x; }
};
template <> struct Num<__half> {
  using C = float;
  static __device__ __forceinline__ float to_c(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_c(float x) { return __float2half_rn(x); }
};
template <> struct Num<__nv_bfloat16> {
  using C = float;
  static __device__ __forceinline__ float to_c(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_c(float x) { return __float2bfloat16_rn(x); }
};

// Round a compute-type value to the storage type and back.
template <class T>
__device__ __forceinline__ typename Num<T>::C rnd(typename Num<T>::C x) {
  return Num<T>::to_c(Num<T>::from_c(x));
}

__device__ __forceinline__ float m_exp(float x) { return expf(x); }
__device__ __forceinline__ double m_exp(double x) { return exp(x); }
__device__ __forceinline__ float m_log(float x) { return logf(x); }
__device__ __forceinline__ double m_log(double x) { return log(x); }
__device__ __forceinline__ float m_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ double m_tanh(double x) { return tanh(x); }
__device__ __forceinline__ float m_erf(float x) { return erff(x); }
__device__ __forceinline__ double m_erf(double x) { return erf(x); }
__device__ __forceinline__ float m_sqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double m_sqrt(double x) { return sqrt(x); }

// Scalar activation formulas, each following the reference layer's apply():
//   ReLU        src/layers/ponni_Relu.h:49-51
//   LeakyReLU   src/layers/ponni_LeakyRelu.h:53-55
//   ELU         src/layers/ponni_Elu.h:48-50
//   SELU        src/layers/ponni_Selu.h:45-49
//   GELU        src/layers/ponni_Gelu.h:47-57 (exact erf form; tanh form when approximate)
//   SiLU        src/layers/ponni_Silu.h:45-49 (sign-split stable form)
//   Sigmoid     src/layers/ponni_Sigmoid.h:45-49
//   Tanh        src/layers/ponni_Tanh.h:44
//   Softplus    src/layers/ponni_Softplus.h:44-50
//   HardSigmoid src/layers/ponni_HardSigmoid.h:52-56
//   HardSwish   src/layers/ponni_HardSwish.h:42-47
//   Mish        src/layers/ponni_Mish.h:44-52
template <class C>
__device__ __forceinline__ C activation(int kind, int flags, C x, C s0, C s1) {
  const C zero = C(0), one = C(1);
  switch (kind) {
    case EPI_RELU: return x > zero ? x : zero;
    case EPI_LEAKY_RELU: return x > zero ? x : s0 * x;
    case EPI_ELU: return x > zero ? x : s0 * (m_exp(x) - one);
    case EPI_SELU: {
      const C alpha = C(1.6732632423543772848), scale = C(1.0507009873554804934);
      return x > zero ? scale * x : scale * alpha * (m_exp(x) - one);
    }
    case EPI_GELU: {
      if (flags & 0x2) {
        const C k = C(0.79788456080286535588);
        const C x3 = x * x * x;
        return C(0.5) * x * (one + m_tanh(k * (x + C(0.044715) * x3)));
      }
      const C sqrt2 = C(1.4142135623730950488);
      return C(0.5) * x * (one + m_erf(x / sqrt2));
    }
    case EPI_SILU: {
      if (x >= zero) return x / (one + m_exp(-x));
      const C e = m_exp(x);
      return x * e / (one + e);
    }
    case EPI_SIGMOID: {
      if (x >= zero) return one / (one + m_exp(-x));
      const C e = m_exp(x);
      return e / (one + e);
    }
    case EPI_TANH: return m_tanh(x);
    case EPI_SOFTPLUS: {
      const C sx = s0 * x;
      if (sx > zero) return (sx + m_log(one + m_exp(-sx))) / s0;
      return m_log(one + m_exp(sx)) / s0;
    }
    case EPI_HARD_SIGMOID: {
      C v = s0 * x + s1;
      v = v < zero ? zero : v;
      return v > one ? one : v;
    }
    case EPI_HARD_SWISH: {
      C r6 = x + C(3);
      r6 = r6 < zero ? zero : r6;
      r6 = r6 > C(6) ? C(6) : r6;
      return x * r6 / C(6);
    }
    case EPI_MISH: {
      C sp;
      if (x > zero) sp = x + m_log(one + m_exp(-x));
      else sp = m_log(one + m_exp(x));
      return x * m_tanh(sp);
    }
    default: return x;
  }
}

}  // namespace ponni_b200
