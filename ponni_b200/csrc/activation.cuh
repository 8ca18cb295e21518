// Scalar activation formulas shared by every kernel.  Only epi_kinds.h is
// included, so that the same text is compiled at run time (NVRTC) into the
// model-specialised narrow kernel and both agree bit for bit in their math.
#pragma once
#include "epi_kinds.h"

namespace ponni_b200 {

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
