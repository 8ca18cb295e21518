/*
 * CPU oracle of PONNI's batched-inference hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference's per-sample traversal, used by the
 * tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the
 * checker and the timed CPU baseline.  It is never linked into or called by
 * libponni_b200.
 *
 * Semantics restated (paths inside mrnorman/ponni):
 *   traversal order            src/ponni_Inference.h:454-555 (layers applied in
 *                              tuple order; fusing a dense layer with its
 *                              pointwise epilogue does not change arithmetic,
 *                              every intermediate is a `real`)
 *   Matvec                     src/layers/ponni_Matvec.h:71-79
 *                              (value = 0; value += W(k,i) * x(k), k ascending)
 *   Bias                       src/layers/ponni_Bias.h:66-68
 *   activations                src/layers/ponni_{Relu,LeakyRelu,Elu,Selu,Gelu,Silu,Sigmoid,
 *                              Tanh,Softplus,HardSigmoid,HardSwish,Mish}.h apply()
 *   LayerNorm                  src/layers/ponni_LayerNorm.h:77-99
 *   MinMaxNorm                 src/layers/ponni_MinMaxNorm.h:68-84
 *   Softmax / LogSoftmax       src/layers/ponni_Softmax.h:46-57, src/layers/ponni_LogSoftmax.h:46-57
 *   Save_State / Binop_Add     src/layers/ponni_Save_State.h:58-67, src/layers/ponni_Binop_Add.h:58-68
 *   Binop_Concatenate          src/layers/ponni_Binop_Concatenate.h:64-86 (the SArray form:
 *                              input and output are distinct arrays)
 *   Binop_Projection_Add       src/layers/ponni_Binop_Projection_Add.h:82-96
 *
 * `real` arithmetic: every operation is rounded to the model type.  float and
 * double are native (compiled with -ffp-contract=off so a*b+c stays two
 * roundings, as g++ emits for x86-64 without -mfma); half and bfloat16 are
 * emulated by computing each operation in float and rounding the result
 * (round-to-nearest-even), which is how a host half_t/bhalf_t behaves.
 * Transcendentals use the C library in float (double for double models) and
 * are rounded once.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/ponni_b200.h"

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- binary16 / bfloat16 rounding (round to nearest even) ---- */
static uint16_t f32_to_f16_bits(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
  if (ax < 0x38800000u) {                                    /* subnormal half or zero */
    if (ax < 0x33000000u) return (uint16_t)sign;             /* <= 2^-25: rounds to 0 */
    /* value = m * 2^(e-150); in half subnormal units of 2^-24: m >> (126 - e) */
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    uint32_t sh = 126u - e;
    uint32_t r = m >> sh;
    uint32_t rem = m & ((1u << sh) - 1u);
    uint32_t halfway = 1u << (sh - 1u);
    if (rem > halfway || (rem == halfway && (r & 1u))) r++;
    return (uint16_t)(sign | r);
  }
  uint32_t e = (ax >> 23) - 112u; /* rebias 127 -> 15 */
  uint32_t m = ax & 0x7fffffu;
  uint32_t r = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
  return (uint16_t)(sign | r);
}

static float f16_bits_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else {
      float v = (float)m * 5.9604644775390625e-08f; /* m * 2^-24 */
      memcpy(&x, &v, 4);
      x |= sign;
    }
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static uint16_t f32_to_bf16_bits(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  uint32_t lsb = (x >> 16) & 1u;
  x += 0x7fffu + lsb;
  return (uint16_t)(x >> 16);
}

static float bf16_bits_to_f32(uint16_t h) {
  uint32_t x = (uint32_t)h << 16;
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static float round_f16(float v) { return f16_bits_to_f32(f32_to_f16_bits(v)); }
static float round_bf16(float v) { return bf16_bits_to_f32(f32_to_bf16_bits(v)); }

/* Exported for the tests of the rounding helpers. */
float ponni_oracle_round_f16(float v) { return round_f16(v); }
float ponni_oracle_round_bf16(float v) { return round_bf16(v); }

/* ---- per-sample traversal, instantiated for float and double compute ---- */
typedef struct {
  int kind, nin, nout, save_index, aux, flags;
  double s[3];
  double s_raw[3]; /* the scalars as given (generated 16-bit LayerNorm: epsilon in float) */
  double* pd; /* parameters as double (exact copies of the model-dtype values) */
} OLayer;

#define MAXSAVE 64

#define DEFINE_ORACLE(T, SUF, EXP, LOG, TANH, ERF, SQRT)                                                   \
  static inline T rnd_##SUF(int mode, T v) {                                                               \
    if (mode < 0) return v;                                                                                \
    if (mode == PONNI_B200_F16) return (T)round_f16((float)v);                                             \
    if (mode == PONNI_B200_BF16) return (T)round_bf16((float)v);                                           \
    return v;                                                                                              \
  }                                                                                                        \
  static T act_##SUF(int kind, int flags, T x, T s0, T s1) {                                               \
    const T zero = 0, one = 1;                                                                             \
    switch (kind) {                                                                                        \
      case PONNI_B200_RELU: return x > zero ? x : zero;                                                    \
      case PONNI_B200_LEAKY_RELU: return x > zero ? x : s0 * x;                                            \
      case PONNI_B200_ELU: return x > zero ? x : s0 * (EXP(x) - one);                                      \
      case PONNI_B200_SELU: {                                                                              \
        const T alpha = (T)1.6732632423543772848, scale = (T)1.0507009873554804934;                        \
        return x > zero ? scale * x : scale * alpha * (EXP(x) - one);                                      \
      }                                                                                                    \
      case PONNI_B200_GELU:                                                                                \
        if (flags & PONNI_B200_FLAG_APPROXIMATE) {                                                         \
          const T k = (T)0.79788456080286535588;                                                           \
          const T x3 = x * x * x;                                                                          \
          return (T)0.5 * x * (one + TANH(k * (x + (T)0.044715 * x3)));                                    \
        }                                                                                                  \
        return (T)0.5 * x * (one + ERF(x / (T)1.4142135623730950488));                                     \
      case PONNI_B200_SILU:                                                                                \
        if (x >= zero) return x / (one + EXP(-x));                                                         \
        { const T e = EXP(x); return x * e / (one + e); }                                                  \
      case PONNI_B200_SIGMOID:                                                                             \
        if (x >= zero) return one / (one + EXP(-x));                                                       \
        { const T e = EXP(x); return e / (one + e); }                                                      \
      case PONNI_B200_TANH: return TANH(x);                                                                \
      case PONNI_B200_SOFTPLUS: {                                                                          \
        const T sx = s0 * x;                                                                               \
        if (sx > zero) return (sx + LOG(one + EXP(-sx))) / s0;                                             \
        return LOG(one + EXP(sx)) / s0;                                                                    \
      }                                                                                                    \
      case PONNI_B200_HARD_SIGMOID: {                                                                      \
        T v = s0 * x + s1;                                                                                 \
        v = v < zero ? zero : v;                                                                           \
        return v > one ? one : v;                                                                          \
      }                                                                                                    \
      case PONNI_B200_HARD_SWISH: {                                                                        \
        T r6 = x + (T)3;                                                                                   \
        r6 = r6 < zero ? zero : r6;                                                                        \
        r6 = r6 > (T)6 ? (T)6 : r6;                                                                        \
        return x * r6 / (T)6;                                                                              \
      }                                                                                                    \
      case PONNI_B200_MISH: {                                                                              \
        T sp;                                                                                              \
        if (x > zero) sp = x + LOG(one + EXP(-x));                                                         \
        else sp = LOG(one + EXP(x));                                                                       \
        return x * TANH(sp);                                                                               \
      }                                                                                                    \
    }                                                                                                      \
    return x;                                                                                              \
  }                                                                                                        \
  /* 16-bit models: the activation with the reference's own rounding points */                           \
  /* (an operation between two `real` values rounds to the type; std::      */                           \
  /* functions and mixed operations with float run in float; a float result */                           \
  /* rounds where the reference stores it in a `real`): the apply() of     */                            \
  /* each src/layers/ponni_<Layer>.h instantiated with half_t / bhalf_t.    */                           \
  static T act16_##SUF(int md, int kind, int flags, T x, T s0, T s1) {                                     \
    _Pragma("GCC diagnostic push") _Pragma("GCC diagnostic ignored \"-Wunused-parameter\"")                \
    switch (kind) {                                                                                        \
      case PONNI_B200_RELU: return x > 0 ? x : 0;                                                          \
      case PONNI_B200_LEAKY_RELU: return x > 0 ? x : rnd_##SUF(md, s0 * x);                                \
      case PONNI_B200_ELU: return x > 0 ? x : rnd_##SUF(md, s0 * (EXP(x) - 1));                            \
      case PONNI_B200_SELU: {                                                                              \
        const T a = rnd_##SUF(md, (T)1.6732632423543772848), sc = rnd_##SUF(md, (T)1.0507009873554804934); \
        return x > 0 ? rnd_##SUF(md, sc * x) : rnd_##SUF(md, rnd_##SUF(md, sc * a) * (EXP(x) - 1));         \
      }                                                                                                    \
      case PONNI_B200_GELU:                                                                                \
        if (flags & PONNI_B200_FLAG_APPROXIMATE) {                                                         \
          const T k = rnd_##SUF(md, (T)0.79788456080286535588), c = rnd_##SUF(md, (T)0.044715);           \
          const T x3 = rnd_##SUF(md, rnd_##SUF(md, x * x) * x);                                            \
          const T t = TANH(rnd_##SUF(md, k * rnd_##SUF(md, x + rnd_##SUF(md, c * x3))));                   \
          return rnd_##SUF(md, rnd_##SUF(md, (T)0.5 * x) * (1 + t));                                       \
        }                                                                                                  \
        return rnd_##SUF(md, rnd_##SUF(md, (T)0.5 * x) *                                                   \
                                 (1 + ERF(rnd_##SUF(md, x / rnd_##SUF(md, (T)1.4142135623730950488)))));   \
      case PONNI_B200_SILU:                                                                                \
        if (x >= 0) return rnd_##SUF(md, x / (1 + EXP(-x)));                                               \
        {                                                                                                  \
          const T e = rnd_##SUF(md, EXP(x));                                                               \
          return rnd_##SUF(md, rnd_##SUF(md, x * e) / rnd_##SUF(md, 1 + e));                               \
        }                                                                                                  \
      case PONNI_B200_SIGMOID:                                                                             \
        if (x >= 0) return rnd_##SUF(md, 1 / (1 + EXP(-x)));                                               \
        {                                                                                                  \
          const T e = rnd_##SUF(md, EXP(x));                                                               \
          return rnd_##SUF(md, e / rnd_##SUF(md, 1 + e));                                                  \
        }                                                                                                  \
      case PONNI_B200_TANH: return rnd_##SUF(md, TANH(x));                                                 \
      case PONNI_B200_SOFTPLUS: {                                                                          \
        const T sx = rnd_##SUF(md, s0 * x);                                                                \
        if (sx > 0) return rnd_##SUF(md, (sx + LOG(1 + EXP(-sx))) / s0);                                   \
        return rnd_##SUF(md, LOG(1 + EXP(sx)) / s0);                                                       \
      }                                                                                                    \
      case PONNI_B200_HARD_SIGMOID: {                                                                      \
        T v = rnd_##SUF(md, rnd_##SUF(md, s0 * x) + s1);                                                   \
        v = v < 0 ? 0 : v;                                                                                 \
        return v > 1 ? 1 : v;                                                                              \
      }                                                                                                    \
      case PONNI_B200_HARD_SWISH: {                                                                        \
        T r6 = rnd_##SUF(md, x + 3);                                                                       \
        r6 = r6 < 0 ? 0 : r6;                                                                              \
        r6 = r6 > 6 ? 6 : r6;                                                                              \
        return rnd_##SUF(md, rnd_##SUF(md, x * r6) / 6);                                                   \
      }                                                                                                    \
      case PONNI_B200_MISH: {                                                                              \
        const T sp = x > 0 ? rnd_##SUF(md, x + LOG(1 + EXP(-x))) : rnd_##SUF(md, LOG(1 + EXP(x)));         \
        return rnd_##SUF(md, x * TANH(sp));                                                                \
      }                                                                                                    \
      default: return rnd_##SUF(md, x);                                                                    \
    }                                                                                                      \
    _Pragma("GCC diagnostic pop")                                                                          \
  }                                                                                                        \
  /* Run one sample: bufa holds the input; *res points at the result. */                                   \
  static void sample_##SUF(const OLayer* L, int nl, int smode, int mflags, T* bufa, T* bufb, T** saved,     \
                            T** res) {                                                                     \
    T* cur = bufa;                                                                                         \
    T* nxt = bufb;                                                                                         \
    const int acc32 = mflags & 1, gen = (mflags >> 1) & 1;                                                 \
    const int mode = acc32 ? -1 : smode; /* acc32: no per-operation rounding */                            \
    for (int li = 0; li < nl; ++li) {                                                                      \
      const OLayer* y = &L[li];                                                                            \
      const int n = y->nin;                                                                                \
      switch (y->kind) {                                                                                   \
        case PONNI_B200_MATVEC:                                                                            \
        {                                                                                                  \
          /* generated arithmetic: the sum starts at a following Bias, and    */                          \
          /* 16-bit products are fused multiply-adds (emitter.py:704-708,     */                          \
          /* :975-983)                                                        */                          \
          const OLayer* bl = (gen && li + 1 < nl && L[li + 1].kind == PONNI_B200_BIAS) ? &L[li + 1] : 0;   \
          const int fused = gen && (smode == PONNI_B200_F16 || smode == PONNI_B200_BF16);                 \
          for (int o = 0; o < y->nout; ++o) {                                                              \
            T v = bl ? (T)bl->pd[o] : 0;                                                                   \
            for (int k = 0; k < n; ++k) {                                                                  \
              const T w = (T)y->pd[(size_t)k * y->nout + o];                                               \
              if (fused) v = rnd_##SUF(mode, (T)((double)w * (double)cur[k] + (double)v));                 \
              else v = rnd_##SUF(mode, v + rnd_##SUF(mode, w * cur[k]));                                   \
            }                                                                                              \
            nxt[o] = v;                                                                                    \
          }                                                                                                \
          { T* t = cur; cur = nxt; nxt = t; }                                                              \
          if (bl) ++li; /* the Bias is consumed */                                                         \
          break;                                                                                           \
        }                                                                                                  \
        case PONNI_B200_BIAS:                                                                              \
          for (int f = 0; f < n; ++f) cur[f] = rnd_##SUF(mode, cur[f] + (T)y->pd[f]);                      \
          break;                                                                                           \
        case PONNI_B200_LAYER_NORM: {                                                                      \
          if (gen) {                                                                                       \
            /* generated LayerNormalization (emitter.py:867-889; 16-bit: :1161-1191): Welford */          \
            /* mean / second moment in Scalar (float for 16-bit models, which round the mean */           \
            /* and 1/stddev to the model type once), then ((x - mean) * inv) * scale + bias */            \
            const int half = smode == PONNI_B200_F16 || smode == PONNI_B200_BF16;                         \
            const int wm = half ? -1 : mode;                                                               \
            T mean = 0, m2 = 0;                                                                            \
            for (int i = 0; i < n; ++i) {                                                                  \
              const T value = cur[i];                                                                      \
              const T delta = rnd_##SUF(wm, value - mean);                                                 \
              mean = rnd_##SUF(wm, mean + rnd_##SUF(wm, delta / (T)(i + 1)));                             \
              m2 = rnd_##SUF(wm, m2 + rnd_##SUF(wm, delta * rnd_##SUF(wm, value - mean)));                 \
            }                                                                                              \
            const T eps = half ? (T)(float)y->s_raw[0] : (T)y->s[0];                                       \
            const T var = rnd_##SUF(wm, m2 / (T)n);                                                        \
            T inv = rnd_##SUF(wm, (T)1 / rnd_##SUF(wm, SQRT(rnd_##SUF(wm, var + eps))));                  \
            mean = rnd_##SUF(mode, mean);                                                                  \
            inv = rnd_##SUF(mode, inv);                                                                    \
            for (int i = 0; i < n; ++i) {                                                                  \
              T v = rnd_##SUF(mode, rnd_##SUF(mode, cur[i] - mean) * inv);                                 \
              v = rnd_##SUF(mode, v * (T)y->pd[i]);                                                        \
              cur[i] = rnd_##SUF(mode, v + (T)y->pd[n + i]);                                               \
            }                                                                                              \
            break;                                                                                         \
          }                                                                                                \
          T mean = 0, var = 0;                                                                             \
          for (int i = 0; i < n; ++i) mean = rnd_##SUF(mode, mean + cur[i]);                               \
          mean = rnd_##SUF(mode, mean / (T)n);                                                             \
          for (int i = 0; i < n; ++i) {                                                                    \
            T d = rnd_##SUF(mode, cur[i] - mean);                                                          \
            var = rnd_##SUF(mode, var + rnd_##SUF(mode, d * d));                                           \
          }                                                                                                \
          var = rnd_##SUF(mode, var / (T)n);                                                               \
          /* 1 / std::sqrt(real): the square root is a float, rounded once with the quotient */           \
          T inv = rnd_##SUF(mode, (T)1 / SQRT(rnd_##SUF(mode, var + (T)y->s[0])));                        \
          for (int i = 0; i < n; ++i) {                                                                    \
            T xh = rnd_##SUF(mode, rnd_##SUF(mode, cur[i] - mean) * inv);                                  \
            cur[i] = rnd_##SUF(mode, rnd_##SUF(mode, (T)y->pd[i] * xh) + (T)y->pd[n + i]);                 \
          }                                                                                                \
          break;                                                                                           \
        }                                                                                                  \
        case PONNI_B200_MIN_MAX_NORM: {                                                                    \
          T mn = cur[0], mx = cur[0];                                                                      \
          for (int i = 1; i < n; ++i) {                                                                    \
            if (cur[i] < mn) mn = cur[i];                                                                  \
            if (cur[i] > mx) mx = cur[i];                                                                  \
          }                                                                                                \
          T sc = rnd_##SUF(mode, rnd_##SUF(mode, (T)y->s[1] - (T)y->s[0]) /                                \
                                     rnd_##SUF(mode, rnd_##SUF(mode, mx - mn) + (T)y->s[2]));              \
          for (int i = 0; i < n; ++i)                                                                      \
            cur[i] = rnd_##SUF(mode, (T)y->s[0] + rnd_##SUF(mode, rnd_##SUF(mode, cur[i] - mn) * sc));     \
          break;                                                                                           \
        }                                                                                                  \
        case PONNI_B200_SOFTMAX:                                                                           \
        case PONNI_B200_LOG_SOFTMAX: {                                                                     \
          T mx = cur[0], sum = 0;                                                                          \
          for (int i = 1; i < n; ++i) mx = cur[i] > mx ? cur[i] : mx;                                      \
          for (int i = 0; i < n; ++i)                                                                      \
            sum = rnd_##SUF(mode, sum + EXP(rnd_##SUF(mode, cur[i] - mx)));                                \
          if (y->kind == PONNI_B200_LOG_SOFTMAX) {                                                         \
            T lse = rnd_##SUF(mode, LOG(sum) + mx);                                                        \
            for (int i = 0; i < n; ++i) cur[i] = rnd_##SUF(mode, cur[i] - lse);                            \
          } else {                                                                                         \
            for (int i = 0; i < n; ++i)                                                                    \
              cur[i] = rnd_##SUF(mode, EXP(rnd_##SUF(mode, cur[i] - mx)) / sum);                           \
          }                                                                                                \
          break;                                                                                           \
        }                                                                                                  \
        case PONNI_B200_SAVE_STATE:                                                                        \
          memcpy(saved[y->save_index], cur, sizeof(T) * (size_t)n);                                        \
          break;                                                                                           \
        case PONNI_B200_BINOP_ADD:                                                                         \
          for (int i = 0; i < n; ++i) cur[i] = rnd_##SUF(mode, cur[i] + saved[y->save_index][i]);          \
          break;                                                                                           \
        case PONNI_B200_BINOP_CONCATENATE: {                                                               \
          const T* s2 = saved[y->save_index];                                                              \
          const int n2 = y->nout - n;                                                                      \
          for (int i = 0; i < y->nout; ++i) {                                                              \
            if (y->flags & PONNI_B200_FLAG_AFTER) nxt[i] = i < n ? cur[i] : s2[i - n];                     \
            else nxt[i] = i < n2 ? s2[i] : cur[i - n2];                                                    \
          }                                                                                                \
          { T* t = cur; cur = nxt; nxt = t; }                                                              \
          break;                                                                                           \
        }                                                                                                  \
        case PONNI_B200_BINOP_PROJECTION_ADD: {                                                            \
          const T* sv = saved[y->save_index];                                                              \
          const int ns = y->aux;                                                                           \
          for (int i = 0; i < n; ++i) {                                                                    \
            T proj = (T)y->pd[(size_t)ns * n + i];                                                         \
            for (int k = 0; k < ns; ++k)                                                                   \
              proj = rnd_##SUF(mode, proj + rnd_##SUF(mode, (T)y->pd[(size_t)k * n + i] * sv[k]));         \
            cur[i] = rnd_##SUF(mode, cur[i] + proj);                                                       \
          }                                                                                                \
          break;                                                                                           \
        }                                                                                                  \
        default:                                                                                           \
          for (int f = 0; f < n; ++f)                                                                      \
            cur[f] = (!gen && (mode == PONNI_B200_F16 || mode == PONNI_B200_BF16))                        \
                         ? act16_##SUF(mode, y->kind, y->flags, cur[f], (T)y->s[0], (T)y->s[1])            \
                         : rnd_##SUF(mode, act_##SUF(y->kind, y->flags, cur[f], (T)y->s[0], (T)y->s[1]));  \
          break;                                                                                           \
      }                                                                                                    \
      /* acc32: the state is stored (rounded to the model type) where a fused  */                          \
      /* block ends, i.e. unless the next layer is pointwise.                  */                          \
      if (acc32 && !(li + 1 < nl && L[li + 1].kind >= PONNI_B200_BIAS && L[li + 1].kind <= PONNI_B200_MISH)) \
        for (int f = 0; f < y->nout; ++f) cur[f] = rnd_##SUF(smode, cur[f]);                              \
    }                                                                                                      \
    *res = cur;                                                                                            \
  }

DEFINE_ORACLE(float, f, expf, logf, tanhf, erff, sqrtf)
DEFINE_ORACLE(double, d, exp, log, tanh, erf, sqrt)

static double load_elem(int dtype, const void* p, size_t i) {
  switch (dtype) {
    case PONNI_B200_F32: return ((const float*)p)[i];
    case PONNI_B200_F64: return ((const double*)p)[i];
    case PONNI_B200_F16: return f16_bits_to_f32(((const uint16_t*)p)[i]);
    case PONNI_B200_BF16: return bf16_bits_to_f32(((const uint16_t*)p)[i]);
  }
  return 0.0;
}

static void store_elem(int dtype, void* p, size_t i, double v) {
  switch (dtype) {
    case PONNI_B200_F32: ((float*)p)[i] = (float)v; break;
    case PONNI_B200_F64: ((double*)p)[i] = v; break;
    case PONNI_B200_F16: ((uint16_t*)p)[i] = f32_to_f16_bits((float)v); break;
    case PONNI_B200_BF16: ((uint16_t*)p)[i] = f32_to_bf16_bits((float)v); break;
  }
}

static size_t n_params(const ponni_b200_layer_desc* d) {
  switch (d->kind) {
    case PONNI_B200_MATVEC: return (size_t)d->num_inputs * d->num_outputs;
    case PONNI_B200_BIAS: return (size_t)d->num_inputs;
    case PONNI_B200_LAYER_NORM: return 2 * (size_t)d->num_inputs;
    case PONNI_B200_BINOP_PROJECTION_ADD: return (size_t)d->aux * d->num_inputs + d->num_inputs;
  }
  return 0;
}

static double round_scalar(int dtype, double v) {
  unsigned char b[8];
  store_elem(dtype, b, 0, v);
  return load_elem(dtype, b, 0);
}

/*
 * out[f][c] = model(in[:, c]) for c in [0, batch).  Bit 1 of acc32 selects
 * the arithmetic of the reference's generated model (a Matvec followed by a
 * Bias starts its sum at the bias; 16-bit products are fused multiply-adds,
 * emitter.py:704-708, :975-983).  Bit 0 of acc32 selects the
 * fp32-accumulation semantics of the tensor-core path for 16-bit models:
 * every operation in float, the state rounded to the model type where each
 * fused block (dense layer + following pointwise layers, or a barrier) ends.  Same descriptor list and
 * dtype codes as ponni_b200_model_create; in/out are host arrays of the model
 * dtype with row strides in_ld/out_ld.  nthreads <= 0 uses all OpenMP threads.
 * Returns 0 on success.
 */
int ponni_oracle_forward_ex(const ponni_b200_layer_desc* layers, int n_layers, int dtype, const void* in,
                            int64_t in_ld, void* out, int64_t out_ld, int64_t batch, int nthreads, int acc32) {
  /* acc32: bit 0 fp32-accumulation semantics; bit 1 generated-model arithmetic */
  if (!layers || n_layers <= 0 || batch < 0) return 1;
  for (int i = 0; i < n_layers; ++i)
    if (layers[i].save_index >= MAXSAVE) return 2;
  OLayer* L = (OLayer*)calloc((size_t)n_layers, sizeof(OLayer));
  int maxw = 1;
  for (int i = 0; i < n_layers; ++i) {
    const ponni_b200_layer_desc* d = &layers[i];
    L[i].kind = d->kind;
    L[i].nin = d->num_inputs;
    L[i].nout = d->num_outputs;
    L[i].save_index = d->save_index;
    L[i].aux = d->aux;
    L[i].flags = d->flags;
    for (int k = 0; k < 3; ++k) {
      L[i].s[k] = round_scalar(dtype, d->scalar[k]);
      L[i].s_raw[k] = d->scalar[k];
    }
    size_t np = n_params(d);
    L[i].pd = (double*)malloc(sizeof(double) * (np ? np : 1));
    for (size_t k = 0; k < np; ++k) L[i].pd[k] = load_elem(dtype, d->params, k);
    if (d->num_inputs > maxw) maxw = d->num_inputs;
    if (d->num_outputs > maxw) maxw = d->num_outputs;
    if (d->aux > maxw) maxw = d->aux;
  }
  const int nin = layers[0].num_inputs, nout = layers[n_layers - 1].num_outputs;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
#pragma omp parallel
  {
    if (dtype == PONNI_B200_F64) {
      double* a = (double*)malloc(sizeof(double) * (size_t)maxw);
      double* b = (double*)malloc(sizeof(double) * (size_t)maxw);
      double* sv[MAXSAVE];
      for (int s = 0; s < MAXSAVE; ++s) sv[s] = NULL;
      for (int i = 0; i < n_layers; ++i)
        if (L[i].save_index >= 0 && !sv[L[i].save_index])
          sv[L[i].save_index] = (double*)calloc((size_t)maxw, sizeof(double));
#pragma omp for schedule(static)
      for (int64_t c = 0; c < batch; ++c) {
        for (int k = 0; k < nin; ++k) a[k] = ((const double*)in)[k * in_ld + c];
        double* r;
        sample_d(L, n_layers, dtype, acc32, a, b, sv, &r);
        for (int f = 0; f < nout; ++f) ((double*)out)[f * out_ld + c] = r[f];
      }
      free(a);
      free(b);
      for (int s = 0; s < MAXSAVE; ++s) free(sv[s]);
    } else {
      float* a = (float*)malloc(sizeof(float) * (size_t)maxw);
      float* b = (float*)malloc(sizeof(float) * (size_t)maxw);
      float* sv[MAXSAVE];
      for (int s = 0; s < MAXSAVE; ++s) sv[s] = NULL;
      for (int i = 0; i < n_layers; ++i)
        if (L[i].save_index >= 0 && !sv[L[i].save_index])
          sv[L[i].save_index] = (float*)calloc((size_t)maxw, sizeof(float));
#pragma omp for schedule(static)
      for (int64_t c = 0; c < batch; ++c) {
        for (int k = 0; k < nin; ++k) a[k] = (float)load_elem(dtype, in, (size_t)(k * in_ld + c));
        float* r;
        sample_f(L, n_layers, dtype, acc32, a, b, sv, &r);
        for (int f = 0; f < nout; ++f) store_elem(dtype, out, (size_t)(f * out_ld + c), r[f]);
      }
      free(a);
      free(b);
      for (int s = 0; s < MAXSAVE; ++s) free(sv[s]);
    }
  }
  for (int i = 0; i < n_layers; ++i) free(L[i].pd);
  free(L);
  return 0;
}

int ponni_oracle_forward(const ponni_b200_layer_desc* layers, int n_layers, int dtype, const void* in, int64_t in_ld,
                         void* out, int64_t out_ld, int64_t batch, int nthreads) {
  return ponni_oracle_forward_ex(layers, n_layers, dtype, in, in_ld, out, out_ld, batch, nthreads, 0);
}
