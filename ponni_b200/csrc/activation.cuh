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

// The same activations for a 16-bit model (`real` = half_t / bhalf_t) with
// the reference's own rounding points: an operation between two `real`
// values rounds to the type (r), std:: functions and operations with a float
// operand run in float, and a float result is rounded where the reference
// stores it in a `real` (a local variable or the return value).  Each case
// follows the apply() of the file listed in activation() above.  `r` rounds
// a float to the model type and back.
// The float transcendental functions of the 16-bit path, evaluated in double
// and rounded once to float: the correctly rounded float value, which is what
// a host C library returns in all but rare cases, so that the 16-bit result
// (a rounding of that float) agrees with the reference's host arithmetic
// instead of flipping wherever two float implementations differ by a unit.
__device__ __forceinline__ float e16_exp(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float e16_log(float x) { return (float)log((double)x); }
__device__ __forceinline__ float e16_tanh(float x) { return (float)tanh((double)x); }
__device__ __forceinline__ float e16_erf(float x) { return (float)erf((double)x); }

template <class R>
__device__ __forceinline__ float activation16(int kind, int flags, float x, float s0, float s1, R r) {
  switch (kind) {
    case EPI_RELU: return x > 0.0f ? x : 0.0f;
    case EPI_LEAKY_RELU: return x > 0.0f ? x : r(s0 * x);
    case EPI_ELU: return x > 0.0f ? x : r(s0 * (e16_exp(x) - 1.0f));
    case EPI_SELU: {
      const float alpha = r(1.6732632423543772848f), scale = r(1.0507009873554804934f);
      return x > 0.0f ? r(scale * x) : r(r(scale * alpha) * (e16_exp(x) - 1.0f));
    }
    case EPI_GELU: {
      if (flags & 0x2) {
        const float k = r(0.79788456080286535588f), c = r(0.044715f);
        const float x3 = r(r(x * x) * x);
        const float t = e16_tanh(r(k * r(x + r(c * x3))));
        return r(r(0.5f * x) * (1.0f + t));
      }
      return r(r(0.5f * x) * (1.0f + e16_erf(r(x / r(1.4142135623730950488f)))));
    }
    case EPI_SILU: {
      if (x >= 0.0f) return r(x / (1.0f + e16_exp(-x)));
      const float e = r(e16_exp(x));
      return r(r(x * e) / r(1.0f + e));
    }
    case EPI_SIGMOID: {
      if (x >= 0.0f) return r(1.0f / (1.0f + e16_exp(-x)));
      const float e = r(e16_exp(x));
      return r(e / r(1.0f + e));
    }
    case EPI_TANH: return r(e16_tanh(x));
    case EPI_SOFTPLUS: {
      const float sx = r(s0 * x);
      if (sx > 0.0f) return r((sx + e16_log(1.0f + e16_exp(-sx))) / s0);
      return r(e16_log(1.0f + e16_exp(sx)) / s0);
    }
    case EPI_HARD_SIGMOID: {
      float v = r(r(s0 * x) + s1);
      v = v < 0.0f ? 0.0f : v;
      return v > 1.0f ? 1.0f : v;
    }
    case EPI_HARD_SWISH: {
      float r6 = r(x + 3.0f);
      r6 = r6 < 0.0f ? 0.0f : r6;
      r6 = r6 > 6.0f ? 6.0f : r6;
      return r(r(x * r6) / 6.0f);
    }
    case EPI_MISH: {
      const float sp = x > 0.0f ? r(x + e16_log(1.0f + e16_exp(-x))) : r(e16_log(1.0f + e16_exp(x)));
      return r(x * e16_tanh(sp));
    }
    default: return x;
  }
}

}  // namespace ponni_b200
