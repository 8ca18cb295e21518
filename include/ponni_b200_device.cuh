// In-kernel (device) API of libponni_b200: run a model on one sample inside
// an application's own CUDA kernel.
//
// Counterpart of the reference's Inference::forward_batch_parallel_in_kernel
// (src/ponni_Inference.h:392-408 for Views with a batch index, :592-604 for
// SArray samples) and of the generated model's infer_one: the application
// controls the launch and combines the model with its own per-sample work.
//
// Host side: plan the model once and obtain its device view with
// ponni::device::get_model() (C ABI ponni_b200_model_device_program); pass
// the view by value to the kernel.  Device side: each thread calls
// infer_one() (a sample in strided memory) or forward_batch_parallel_in_kernel()
// (column ibatch of feature-major [features, batch] arrays).
//
// The evaluation follows the model's lowered program one sample at a time
// with every state in thread-local arrays, in the reference's operation
// order and with the same arithmetic as libponni_b200's tile kernel
// (products fused into the accumulation for fp32/fp64; every operation
// rounded to the model type for fp16/bf16).  Template parameters bound the
// local arrays: MAXW >= the widest layer, NBUF >= the program's buffer count
// (both reported by get_model).  Compile with nvcc for sm_100a and link
// libponni_b200.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../ponni_b200/csrc/device_math.cuh"
#include "../ponni_b200/csrc/program.h"
#include "ponni_b200.h"

namespace ponni {
namespace device {

// Device view of a planned model (trivially copyable; pass by value).
struct Model {
  const ponni_b200::Program* program;  // lowered program, device memory
  const void* params;                  // packed parameters (model dtype), device memory
  int nin, nout;
  int max_width;                       // widest state (MAXW must be at least this)
  int num_buffers;                     // state buffers (NBUF must be at least this)
};

// Plan `m` and fill `out` (host).  The pointers stay valid until the model's
// parameters change or the model is destroyed.
inline ponni_b200_status get_model(ponni_b200_model* m, Model* out) {
  const void* prog = nullptr;
  const void* params = nullptr;
  int maxw = 0, nbuf = 0;
  const ponni_b200_status s = ponni_b200_model_device_program(m, &prog, &params, &maxw, &nbuf);
  if (s != PONNI_B200_OK) return s;
  out->program = static_cast<const ponni_b200::Program*>(prog);
  out->params = params;
  out->nin = ponni_b200_num_inputs(m);
  out->nout = ponni_b200_num_outputs(m);
  out->max_width = maxw;
  out->num_buffers = nbuf;
  return PONNI_B200_OK;
}

namespace detail {
using ponni_b200::Num;
using ponni_b200::rnd;

template <class T> using C = typename Num<T>::C;

__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double div_rn(double a, double b) { return __ddiv_rn(a, b); }
template <class T> __device__ __forceinline__ C<T> radd(C<T> a, C<T> b) { return rnd<T>(add_rn(a, b)); }
template <class T> __device__ __forceinline__ C<T> rsub(C<T> a, C<T> b) { return rnd<T>(sub_rn(a, b)); }
template <class T> __device__ __forceinline__ C<T> rmul(C<T> a, C<T> b) { return rnd<T>(mul_rn(a, b)); }
template <class T> __device__ __forceinline__ C<T> rdiv(C<T> a, C<T> b) { return rnd<T>(div_rn(a, b)); }

// Pointwise epilogue entries [first, first + n) on one value of feature f
// (reference apply_fused_epilogue, src/ponni_Inference.h:428-444).
template <class T>
__device__ __forceinline__ C<T> epilogue(const ponni_b200::Program& p, int first, int n, int f, C<T> v,
                                         const T* params) {
  for (int e = first; e < first + n; ++e) {
    const ponni_b200::EpiDesc& d = p.epi[e];
    if (d.kind == ponni_b200::EPI_BIAS) v = v + Num<T>::to_c(params[d.p_off + f]);
    else if (sizeof(T) == 2 && (d.flags & ponni_b200::EPI_FLAG_REF16))
      v = ponni_b200::activation16(d.kind, d.flags, (float)v, (float)d.s0, (float)d.s1,
                                   [](float x) { return (float)rnd<T>(x); });
    else v = ponni_b200::activation<C<T>>(d.kind, d.flags, v, (C<T>)d.s0, (C<T>)d.s1);
    v = rnd<T>(v);
  }
  return v;
}
}  // namespace detail

// One sample: x[i * x_stride] for i < nin -> y[i * y_stride] for i < nout.
template <class T, int MAXW, int NBUF = ponni_b200::kMaxBuffers>
__device__ void infer_one(const Model& m, const T* x, int64_t x_stride, T* y, int64_t y_stride) {
  using namespace ponni_b200;
  using detail::C;
  using detail::add_rn;
  using detail::div_rn;
  using detail::mul_rn;
  using detail::radd;
  using detail::rdiv;
  using detail::rmul;
  using detail::rsub;
  using detail::sub_rn;
  const Program& p = *m.program;
  const T* params = static_cast<const T*>(m.params);
  C<T> buf[NBUF][MAXW];
  auto slot = [&](int id) { return id == p.in_buf2 ? p.in_buf : id; };  // one input buffer per sample
  for (int i = 0; i < p.nin; ++i) buf[p.in_buf][i] = Num<T>::to_c(x[i * x_stride]);
  for (int si = 0; si < p.n_steps; ++si) {
    const StepDesc& s = p.steps[si];
    const int src = s.src >= 0 ? slot(s.src) : -1, dst = s.dst >= 0 ? slot(s.dst) : -1;
    const int aux = s.aux >= 0 ? slot(s.aux) : -1;
    switch (s.kind) {
      case STEP_DENSE: {
        // Reference Matvec::compute_output (src/layers/ponni_Matvec.h:71-79):
        // acc from 0 (or from the bias, Projection_Add), k ascending.
        const T* W = params + s.w_off;
        for (int o = 0; o < s.nout; ++o) {
          C<T> acc = (s.flags & DENSE_INIT_BIAS) ? Num<T>::to_c(params[s.b_off + o]) : C<T>(0);
          for (int k = 0; k < s.nin; ++k) {
            const C<T> w = Num<T>::to_c(W[k * s.nout_pad + o]);
            if constexpr (sizeof(T) >= 4) acc = fma(w, buf[src][k], acc);
            else if (s.flags & DENSE_HALF_FMA) acc = rnd<T>(fmaf(w, buf[src][k], acc));
            else acc = rnd<T>(acc + rnd<T>(w * buf[src][k]));
          }
          if (s.flags & DENSE_ADD_RESIDUAL) acc = rnd<T>(buf[aux][o] + acc);
          acc = detail::epilogue<T>(p, s.epi_first, s.n_epi, o, acc, params);
          if (s.flags & DENSE_TO_GLOBAL) y[o * y_stride] = Num<T>::from_c(acc);
          else buf[dst][o] = acc;
        }
        break;
      }
      case STEP_POINTWISE:
        for (int f = 0; f < s.nin; ++f) buf[src][f] = detail::epilogue<T>(p, s.epi_first, s.n_epi, f, buf[src][f], params);
        break;
      case STEP_LAYERNORM: {  // src/layers/ponni_LayerNorm.h:77-99
        const int n = s.nin;
        if (s.flags & LN_WELFORD) {  // generated LayerNormalization, emitter.py:867-889, :1161-1191
          C<T> mean = C<T>(0), m2 = C<T>(0);
          for (int i = 0; i < n; ++i) {
            const C<T> value = buf[src][i];
            const C<T> delta = sub_rn(value, mean);
            mean = add_rn(mean, div_rn(delta, (C<T>)(i + 1)));
            m2 = add_rn(m2, mul_rn(delta, sub_rn(value, mean)));
          }
          const C<T> inv = rnd<T>(div_rn(C<T>(1), m_sqrt(add_rn(div_rn(m2, (C<T>)n), (C<T>)s.s0))));
          mean = rnd<T>(mean);
          for (int i = 0; i < n; ++i) {
            const C<T> v = rmul<T>(rsub<T>(buf[src][i], mean), inv);
            buf[src][i] = radd<T>(rmul<T>(v, Num<T>::to_c(params[s.w_off + i])), Num<T>::to_c(params[s.b_off + i]));
          }
          break;
        }
        C<T> mean = C<T>(0);
        for (int i = 0; i < n; ++i) mean = radd<T>(mean, buf[src][i]);
        mean = rdiv<T>(mean, (C<T>)n);
        C<T> var = C<T>(0);
        for (int i = 0; i < n; ++i) {
          const C<T> d = rsub<T>(buf[src][i], mean);
          var = radd<T>(var, rmul<T>(d, d));
        }
        var = rdiv<T>(var, (C<T>)n);
        const C<T> inv_std = rdiv<T>(C<T>(1), m_sqrt(radd<T>(var, (C<T>)s.s0)));  // sqrt in float (16-bit)
        for (int i = 0; i < n; ++i) {
          const C<T> xhat = rmul<T>(rsub<T>(buf[src][i], mean), inv_std);
          buf[src][i] = radd<T>(rmul<T>(Num<T>::to_c(params[s.w_off + i]), xhat), Num<T>::to_c(params[s.b_off + i]));
        }
        break;
      }
      case STEP_MINMAXNORM: {  // src/layers/ponni_MinMaxNorm.h:68-84
        const int n = s.nin;
        C<T> mn = buf[src][0], mx = mn;
        for (int i = 1; i < n; ++i) {
          const C<T> v = buf[src][i];
          if (v < mn) mn = v;
          if (v > mx) mx = v;
        }
        const C<T> scale = rdiv<T>(rsub<T>((C<T>)s.s1, (C<T>)s.s0), radd<T>(rsub<T>(mx, mn), (C<T>)s.s2));
        for (int i = 0; i < n; ++i) buf[src][i] = radd<T>((C<T>)s.s0, rmul<T>(rsub<T>(buf[src][i], mn), scale));
        break;
      }
      case STEP_SOFTMAX:
      case STEP_LOGSOFTMAX: {  // src/layers/ponni_Softmax.h:46-57, ponni_LogSoftmax.h:46-57
        const int n = s.nin;
        C<T> mx = buf[src][0];
        for (int i = 1; i < n; ++i) mx = buf[src][i] > mx ? buf[src][i] : mx;
        C<T> sum = C<T>(0);
        for (int i = 0; i < n; ++i) sum = radd<T>(sum, sizeof(T) == 2 ? ponni_b200::e16_exp(rsub<T>(buf[src][i], mx)) : m_exp(rsub<T>(buf[src][i], mx)));
        if (s.kind == STEP_LOGSOFTMAX) {
          const C<T> lse = radd<T>(sizeof(T) == 2 ? ponni_b200::e16_log(sum) : m_log(sum), mx);
          for (int i = 0; i < n; ++i) buf[src][i] = rsub<T>(buf[src][i], lse);
        } else {
          for (int i = 0; i < n; ++i) buf[src][i] = rdiv<T>(sizeof(T) == 2 ? ponni_b200::e16_exp(rsub<T>(buf[src][i], mx)) : m_exp(rsub<T>(buf[src][i], mx)), sum);
        }
        break;
      }
      case STEP_COPY:  // Save_State (src/layers/ponni_Save_State.h:58-67)
        for (int i = 0; i < s.nin; ++i) buf[dst][i] = buf[src][i];
        break;
      case STEP_ADD:  // Binop_Add (src/layers/ponni_Binop_Add.h:58-68)
        for (int i = 0; i < s.nin; ++i) buf[src][i] = radd<T>(buf[src][i], buf[aux][i]);
        break;
      case STEP_CONCAT: {  // Binop_Concatenate, SArray form (ponni_Binop_Concatenate.h:80-86)
        const int n_main = s.nin, n_aux = s.nout - s.nin;
        const bool after = (s.flags & CONCAT_AFTER) != 0;
        for (int f = 0; f < s.nout; ++f) {
          if (after) buf[dst][f] = f < n_main ? buf[src][f] : buf[aux][f - n_main];
          else buf[dst][f] = f < n_aux ? buf[aux][f] : buf[src][f - n_aux];
        }
        break;
      }
      default: break;
    }
  }
  if (p.final_buf >= 0) {
    const int fb = slot(p.final_buf);
    for (int i = 0; i < p.nout; ++i) y[i * y_stride] = Num<T>::from_c(buf[fb][i]);
  }
}

// Column ibatch of feature-major arrays: in[f * in_ld + ibatch] ->
// out[f * out_ld + ibatch] (reference forward_batch_parallel_in_kernel with
// a batch index).
template <class T, int MAXW, int NBUF = ponni_b200::kMaxBuffers>
__device__ __forceinline__ void forward_batch_parallel_in_kernel(const Model& m, const T* in, int64_t in_ld, T* out,
                                                                 int64_t out_ld, int64_t ibatch) {
  infer_one<T, MAXW, NBUF>(m, in + ibatch, in_ld, out + ibatch, out_ld);
}

}  // namespace device
}  // namespace ponni
