// Tensor-core kernel for fp32 dense chains with LayerNorm and residual
// barriers (sm_100a, tcgen05 + TMEM), weights streamed from L2.
//
// One persistent CTA per SM, warp-specialised (576 threads):
//   producer (warp 16, one thread): streams the weight chunks of every job in
//     job order into a two-stage shared-memory ring with 1-D bulk copies
//     (cp.async.bulk, byte-counted mbarriers, no multicast).  A chunk is one
//     bf16 part of one K block of 64 of a layer's weights, N rows x 128 B,
//     pre-swizzled (SW128 K-major) on the host;
//   MMA issuer (warp 17, the whole warp, one elected lane issues): per job
//     (one Matvec of one tile of 128 batch columns) issues the six split
//     products chunk by chunk (tcgen05.mma kind::f16, bf16 operands, fp32
//     accumulators in the slot's first 128 TMEM columns): the five smaller
//     products first, then the dominant x0*w0 (the tensor core's fp32
//     accumulation truncates; summing the small products while the
//     accumulator is small keeps the result fp32-accurate), x0*w0 in groups
//     of one K block where the columns allow;
//   epilogue (warps 0-15, 4 TMEM lane quarters x 4 column quarters; a
//     thread holds one 32-column chunk of one row = one batch column): all
//     16 warps take the jobs one at a time in the issuer's order; per job
//     they sum the accumulators and run the job's epilogue operations in
//     tuple order (reference src/ponni_Inference.h:416-555):
//       Bias                    v += b                (ponni_Bias.h:66-68)
//       activations             v = f(v)              (activation.cuh)
//       Binop_Add<I>            v += saved[I]         (ponni_Binop_Add.h:58-68)
//       Save_State<I>           saved[I] = v          (ponni_Save_State.h:58-67)
//       LayerNorm               mean / biased variance (each column quarter
//                               two-pass over its values, quarters combined
//                               pairwise), gamma * (v - mean) / sqrt(var + eps)
//                               + beta (ponni_LayerNorm.h:77-99)
//     then split the result into the three bf16 parts of the next job's A
//     operand (shared memory, K-major SW128) or write the caller's output.
//     LayerNorm keeps the row's values in registers; the four column
//     quarters exchange (mean, squared deviations) pairs through two
//     already-read accumulator columns of TMEM, one barrier per lane
//     quarter.  A single saved state lives in the slot's other 128 TMEM
//     columns (tcgen05.st / tcgen05.ld by the thread that owns the row and
//     columns); models with two saved states keep them in a per-CTA, per-slot
//     global scratch area (64 KB per slot and state; L2-resident), written
//     and read back by the same thread.
// Two tiles are in flight and their jobs alternate Matvec by Matvec, so the
// epilogue of one tile's job overlaps the MMAs of the other tile's job.
//
// Arithmetic: fp32 model values; each operand x = x0 + x1 + x2 exactly
// (bf16 truncation parts); products of order <= 2 are kept (the dropped ones
// are below 2^-24 relative).  Epilogue arithmetic is IEEE fp32 without
// contraction where the reference rounds each operation (LayerNorm).
//
// Every wait is bounded: a role that gives up raises the CTA's abort flag,
// records an error code and the CTA drains its copies and MMAs before it
// frees TMEM; the epilogue warps of a lane quarter decide to leave together
// (a barrier reduction), so none is left waiting at a named barrier.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "device_math.cuh"
#include "f32x2.cuh"
#include "tc_common.cuh"
#include "tc_resid.h"

PONNI_B200_SKIP_ARRIVE_FLAG(tr)

#ifndef PONNI_B200_TR_DIAG
#define PONNI_B200_TR_DIAG 0
#endif

namespace ponni_b200 {
namespace {
using namespace tc;

constexpr long long kWaitCycles = PONNI_B200_WAIT_LIMIT;

// Optional phase timing (compiled only with -DPONNI_B200_TC_PROFILE): each
// role sums the cycles of its phases and adds them once per CTA to the
// diagnostic counters after the error word (1: MMA waits for the epilogue,
// 2: MMA waits for weights, 3: producer waits for a free stage, 4: epilogue
// waits for accumulators, 5: epilogue work, 6: LayerNorm passes 2-3,
// 7: MMA thread total).
#ifdef PONNI_B200_TC_PROFILE
#define TR_T(var) const long long var = clock64()
#define TR_ACC(acc, t0) acc += clock64() - (t0)
#define TR_FLUSH(idx, acc) atomicAdd(reinterpret_cast<unsigned long long*>(err) + (idx), (unsigned long long)(acc))
#else
#define TR_T(var)
#define TR_ACC(acc, t0)
#define TR_FLUSH(idx, acc)
#endif

__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(r) : "f"(x));
  return r;
}

// Exact GELU, x * Phi(x) = 0.5 x (1 + erf(x / sqrt 2)) (src/layers/ponni_Gelu.h:47-57),
// branch-free: with t = min(|x|, 12), Phi(-t) = 0.5 exp(-t^2 / 2) erfcx(t / sqrt 2)
// and erfcx(t / sqrt 2) = P4(t) / Q5(t), a rational fit with 4.8e-9 relative
// error on [0, 12] (fit_gelu.py).  In float its maximum absolute error is
// 3.8e-7 (the erf form in float: 4.5e-7) and its relative error in the left
// tail stays below 1.5e-6, where the erf form cancels.
// Two values at a time with packed fp32 arithmetic.
__device__ __forceinline__ void gelu_phi2(float& x0, float& x1) {
  const float t0 = fminf(fabsf(x0), 12.0f), t1 = fminf(fabsf(x1), 12.0f);
  float s0, s1;
  f2::mul(s0, s1, t0, t1, t0, t1);
  f2::mul(s0, s1, s0, s1, -0.72134752044448170f, -0.72134752044448170f);
  const float e0 = ex2_approx(s0), e1 = ex2_approx(s1);
  float p0, p1, q0, q1;
  f2::fma(p0, p1, 0.00794154778122902f, 0.00794154778122902f, t0, t1, 0.07927434146404266f, 0.07927434146404266f);
  f2::fma(p0, p1, p0, p1, t0, t1, 0.3605049252510071f, 0.3605049252510071f);
  f2::fma(p0, p1, p0, p1, t0, t1, 0.8684397339820862f, 0.8684397339820862f);
  f2::fma(p0, p1, p0, p1, t0, t1, 1.0f, 1.0f);
  f2::fma(q0, q1, 0.009953089989721775f, 0.009953089989721775f, t0, t1, 0.09936375170946121f, 0.09936375170946121f);
  f2::fma(q0, q1, q0, q1, t0, t1, 0.4616026282310486f, 0.4616026282310486f);
  f2::fma(q0, q1, q0, q1, t0, t1, 1.1900357007980347f, 1.1900357007980347f);
  f2::fma(q0, q1, q0, q1, t0, t1, 1.6663246154785156f, 1.6663246154785156f);
  f2::fma(q0, q1, q0, q1, t0, t1, 1.0f, 1.0f);
  float a0, a1;
  f2::mul(a0, a1, e0, e1, 0.5f, 0.5f);
  f2::mul(a0, a1, a0, a1, __fdividef(p0, q0), __fdividef(p1, q1));  // Phi(-|x|)
  const float f0 = x0 >= 0.0f ? 1.0f - a0 : a0, f1 = x1 >= 0.0f ? 1.0f - a1 : a1;
  f2::mul(x0, x1, x0, x1, f0, f1);
}

template <int K>
__device__ __forceinline__ void act32(float (&v)[32], int flags, float s0, float s1) {
  if constexpr (K == EPI_GELU) {
    if (!(flags & 0x2)) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) gelu_phi2(v[j], v[j + 1]);
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = activation<float>(K, flags, v[j], s0, s1);
}

__device__ __forceinline__ void act_dispatch(int kind, float (&v)[32], int flags, float s0, float s1) {
  switch (kind) {
    case EPI_RELU: act32<EPI_RELU>(v, flags, s0, s1); break;
    case EPI_LEAKY_RELU: act32<EPI_LEAKY_RELU>(v, flags, s0, s1); break;
    case EPI_ELU: act32<EPI_ELU>(v, flags, s0, s1); break;
    case EPI_SELU: act32<EPI_SELU>(v, flags, s0, s1); break;
    case EPI_GELU: act32<EPI_GELU>(v, flags, s0, s1); break;
    case EPI_SILU: act32<EPI_SILU>(v, flags, s0, s1); break;
    case EPI_SIGMOID: act32<EPI_SIGMOID>(v, flags, s0, s1); break;
    case EPI_TANH: act32<EPI_TANH>(v, flags, s0, s1); break;
    case EPI_SOFTPLUS: act32<EPI_SOFTPLUS>(v, flags, s0, s1); break;
    case EPI_HARD_SIGMOID: act32<EPI_HARD_SIGMOID>(v, flags, s0, s1); break;
    case EPI_HARD_SWISH: act32<EPI_HARD_SWISH>(v, flags, s0, s1); break;
    case EPI_MISH: act32<EPI_MISH>(v, flags, s0, s1); break;
    default: break;
  }
}

// Two TMEM columns of this warp's 32 lanes (one value per lane each).
__device__ __forceinline__ void tmem_st2(uint32_t taddr, float a, float b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};\n" ::"r"(taddr), "r"(__float_as_uint(a)),
               "r"(__float_as_uint(b))
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}
// Pairs of columns at four TMEM addresses of this warp's lanes, one wait.
__device__ __forceinline__ void tmem_ld2x4(const uint32_t (&t)[4], float (&a)[4], float (&b)[4]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%8];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x2.b32 {%2, %3}, [%9];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x2.b32 {%4, %5}, [%10];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x2.b32 {%6, %7}, [%11];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(t[0]), "r"(t[1]), "r"(t[2]), "r"(t[3])
      : "memory");
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    a[q] = __uint_as_float(r[2 * q]);
    b[q] = __uint_as_float(r[2 * q + 1]);
  }
}

// Per-thread context of the epilogue.  All 16 epilogue warps work on one
// job at a time: warp w reads TMEM lane quarter w % 4 (rows 32 (w % 4) ..)
// and handles accumulator columns 32 (w / 4) .. + 31, so each thread holds
// one 32-column chunk of one row in registers.
struct TrEpi {
  const unsigned char* image;
  float4* saved_cta;  // this CTA's saved states: [slot][state][f / 4][128 rows] float4
  int n_saved;
  int saved_tmem;     // the saved state lives in TMEM (columns kTrAccCols.. of the slot)
  int cq, m;          // column quarter, row
  int lq;             // TMEM lane quarter (warp % 4)
  // the job's slot
  float4* saved;      // the slot's saved states
  uint32_t a[3];      // the slot's A operand parts
  uint32_t tmem_row;  // the slot's accumulators + this warp's lane quarter
};

// Named barrier over the four epilogue warps of one TMEM lane quarter (the
// warps w, w + 4, w + 8, w + 12 that hold the four column quarters of the
// same rows; ids 1-4, 0 is __syncthreads).  Only these warps exchange data,
// so the quarters run independently of one another.
__device__ __forceinline__ void epi_sync(int lq) {
  asm volatile("bar.sync %0, 128;\n" ::"r"(1 + lq) : "memory");
}
__device__ __forceinline__ int epi_sync_or(int lq, int pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 128, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(pred), "r"(1 + lq)
      : "memory");
  return r;
}

// 32 columns of this warp's 32 TMEM lanes, completed before returning.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
      "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]),
      "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]),
      "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// Element-wise operations [o0, o1) on the 32 columns c0.. of this row.
__device__ __forceinline__ void tr_ops(const TrOp* ops, int o0, int o1, float (&v)[32], int c0, const TrEpi& E) {
  for (int i = o0; i < o1; ++i) {
    const TrOp o = ops[i];
#if PONNI_B200_TR_DIAG & 8  // diagnostic builds: bit 8 skips the saved-state traffic
    if (o.kind == TR_ADD || o.kind == TR_SAVE) continue;
#endif
    if (o.kind == TR_BIAS) {
      const float4* b4 = reinterpret_cast<const float4*>(E.image + o.off) + c0 / 4;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b = __ldg(b4 + q);
        f2::add(v[4 * q], v[4 * q + 1], v[4 * q], v[4 * q + 1], b.x, b.y);
        f2::add(v[4 * q + 2], v[4 * q + 3], v[4 * q + 2], v[4 * q + 3], b.z, b.w);
      }
    } else if (o.kind == TR_ACT) {
#if !(PONNI_B200_TR_DIAG & 1)  // diagnostic builds: bit 1 skips activations
      act_dispatch(o.arg, v, o.flags, o.s0, o.s1);
#endif
    } else if (o.kind == TR_ADD && E.saved_tmem) {
      float t[32];
      tmem_ld32(E.tmem_row + kTrAccCols + (uint32_t)c0, t);
      f2::add_n(v, t);
    } else if (o.kind == TR_SAVE && E.saved_tmem) {
      tmem_st32(E.tmem_row + kTrAccCols + (uint32_t)c0, v);
    } else if (o.kind == TR_ADD) {
      const float4* sv = E.saved + (size_t)o.arg * (kTrMaxN / 4) * 128 + (c0 / 4) * 128 + E.m;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 t = sv[q * 128];
        f2::add(v[4 * q], v[4 * q + 1], v[4 * q], v[4 * q + 1], t.x, t.y);
        f2::add(v[4 * q + 2], v[4 * q + 3], v[4 * q + 2], v[4 * q + 3], t.z, t.w);
      }
    } else if (o.kind == TR_SAVE) {
      float4* sv = E.saved + (size_t)o.arg * (kTrMaxN / 4) * 128 + (c0 / 4) * 128 + E.m;
#pragma unroll
      for (int q = 0; q < 8; ++q) sv[q * 128] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  }
}

// The row's 32 values c0.. go to the next job's A operand (split into three
// bf16 parts) or, after the last Matvec, to the caller's output.
__device__ __forceinline__ void tr_finish(const float (&v)[32], int c0, bool last, int nout, const TrEpi& E,
                                          float* __restrict__ out, int64_t out_ld, int64_t col, int64_t batch) {
  if (last) {
    if (col < batch) {
      const int nv = min(32, nout - c0);
      float* o = out + (int64_t)c0 * out_ld + col;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j >= nv) break;
        o[(int64_t)j * out_ld] = v[j];
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#if PONNI_B200_TR_DIAG & 4  // diagnostic builds: bit 4 stores part 0 only, unsplit
      st_shared_v4(E.a[0] + kmajor_chunk(E.m, (uint32_t)(c0 + 8 * q) * 2), __float_as_uint(v[8 * q]),
                   __float_as_uint(v[8 * q + 2]), __float_as_uint(v[8 * q + 4]), __float_as_uint(v[8 * q + 6]));
#else
      store_row8<float>(E.a, E.m, c0 + 8 * q, v + 8 * q);
#endif
    }
  }
}

// Epilogue of job (layer l) for this thread's row and 32-column chunk.
__device__ __forceinline__ void tr_epilogue(const TrProgram& p, int l, const TrEpi& E, float* __restrict__ out,
                                            int64_t out_ld, int64_t col, int64_t batch) {
  const TrLayer& L = p.layers[l];
  const int n_pad = L.n_pad, nout = L.nout, groups = L.groups;
  const bool last = l == p.n_layers - 1;
  const int o0 = L.op_first, o_end = o0 + L.n_ops;
  const bool has_ln = L.ln >= 0 && !(PONNI_B200_TR_DIAG & 2);  // diagnostic builds: bit 2 skips LayerNorm
  const int o_ln = has_ln ? o0 + L.ln : o_end;
  const int c0 = E.cq * 32;
  const bool active = c0 < n_pad;  // warp-uniform
  const int nv = min(32, nout - c0);  // valid columns of the chunk
  float v[32];
  if (active) {
    if (groups == 1) {
      tmem_ld32(E.tmem_row + (uint32_t)c0, v);
    } else {
      float w[32];
      tmem_ld32x2(E.tmem_row + (uint32_t)c0, E.tmem_row + (uint32_t)(n_pad + c0), v, w);
      f2::add_n(v, w);
    }
    tr_ops(p.ops, o0, o_ln, v, c0, E);
  }
  if (has_ln) {
    // LayerNorm over the row (src/layers/ponni_LayerNorm.h:77-99): the four
    // column quarters of a row combine their partial statistics.
    // Each column quarter's mean and sum of squared deviations (two passes
    // over its registers), combined across the row's quarters with the
    // pairwise update of Chan, Golub and LeVeque (mean = sum n_q m_q / n,
    // M2 = sum M2_q + sum n_q (m_q - mean)^2, var = M2 / n).  The pairs go
    // through TMEM: each warp writes its pair into the first two of its own,
    // already read, accumulator columns; one barrier; each warp reads the
    // pairs of the row's quarters.
    const uint32_t xrow = E.tmem_row;  // exchange columns: the first two of each warp's own, already read, columns
    if (active) {
      float qmean, qm2;
      if (nv >= 32) {
        float s0 = v[0], s1 = v[1];
#pragma unroll
        for (int j = 2; j < 32; j += 2) f2::add(s0, s1, s0, s1, v[j], v[j + 1]);
        qmean = __fdiv_rn(__fadd_rn(s0, s1), 32.0f);
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float d0, d1;
          f2::sub(d0, d1, v[j], v[j + 1], qmean, qmean);
          f2::mul(d0, d1, d0, d1, d0, d1);
          f2::add(t0, t1, t0, t1, d0, d1);
        }
        qm2 = __fadd_rn(t0, t1);
      } else {
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nv) sum = __fadd_rn(sum, v[j]);
        qmean = __fdiv_rn(sum, (float)nv);
        qm2 = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nv) {
            const float d = __fsub_rn(v[j], qmean);
            qm2 = __fadd_rn(qm2, __fmul_rn(d, d));
          }
      }
      tmem_st2(xrow + (uint32_t)c0, qmean, qm2);
    }
    tc_fence_before();
    epi_sync(E.lq);
    tc_fence_after();
    float mean = 0.f, var = 0.f;
    if (active) {
      float qm[4], q2[4];
      uint32_t ta[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)  // quarters past n_pad read quarter 0 (ignored below)
        ta[q] = xrow + (uint32_t)(32 * q < n_pad ? 32 * q : 0);
      tmem_ld2x4(ta, qm, q2);
      const float n = (float)nout;
      float tot = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int nq = min(32, nout - 32 * q);
        if (nq > 0) tot = __fadd_rn(tot, __fmul_rn((float)nq, qm[q]));
      }
      mean = __fdiv_rn(tot, n);
      float m2 = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int nq = min(32, nout - 32 * q);
        if (nq > 0) {
          const float d = __fsub_rn(qm[q], mean);
          m2 = __fadd_rn(m2, __fadd_rn(q2[q], __fmul_rn((float)nq, __fmul_rn(d, d))));
        }
      }
      var = __fdiv_rn(m2, n);
    }
    if (active) {
      const TrOp ln = p.ops[o_ln];
      const float inv_std = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, ln.s0)));
      const float4* g4 = reinterpret_cast<const float4*>(E.image + ln.off) + c0 / 4;
      const float4* b4 = g4 + 32;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 g = __ldg(g4 + q), b = __ldg(b4 + q);
        const float gg[4] = {g.x, g.y, g.z, g.w}, bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          float& x0 = v[4 * q + e];
          float& x1 = v[4 * q + e + 1];
          f2::sub(x0, x1, x0, x1, mean, mean);
          f2::mul(x0, x1, x0, x1, inv_std, inv_std);  // xhat
          f2::mul(x0, x1, x0, x1, gg[e], gg[e + 1]);
          f2::add(x0, x1, x0, x1, bb[e], bb[e + 1]);
        }
      }
      tr_ops(p.ops, o_ln + 1, o_end, v, c0, E);
    }
    // (the exchange columns belong to this job's accumulators, which the MMA
    // issuer reuses only after every epilogue warp has released the slot)
  }
  if (active) tr_finish(v, c0, last, nout, E, out, out_ld, col, batch);
}

// Stage this row's input column as layer 0's A operand (three bf16 parts);
// column quarter cq takes the 8-feature groups cq, cq + 4, ...
__device__ __forceinline__ void tr_stage_input(const float* __restrict__ in, int64_t in_ld, int nin, int k_pad,
                                               int64_t col, int64_t batch, const TrEpi& E) {
  const bool live = col < batch;
  const float* src = in + col;
#pragma unroll 1
  for (int g = E.cq; g < k_pad / 8; g += 4) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int f = 8 * g + e;
      v[e] = (live && f < nin) ? __ldg(src + (int64_t)f * in_ld) : 0.0f;
    }
    store_row8<float>(E.a, E.m, 8 * g, v);
  }
}

// MMA issue state of one job.
struct TrIssue {
  uint32_t a0, a1, a2;  // low descriptor halves of the slot's A operand parts
  uint32_t hi;          // shared upper descriptor half
  uint32_t d;           // the job's accumulator group 0 (group 1 at d + n_pad)
  uint32_t n_pad, idesc;
};

// Wait (bounded, whole warp) for the weight chunk of ring use `use`.
__device__ __forceinline__ bool tr_wait_chunk(uint32_t use, uint32_t b_full, volatile int* abort_flag,
                                              long long& w_full) {
  (void)w_full;
  TR_T(tf);
  const bool ok =
      __all_sync(0xffffffffu, wait_phase_abort(b_full + 8u * (use & 1u), (use >> 1) & 1u, abort_flag, kWaitCycles));
  TR_ACC(w_full, tf);
  tc_fence_after();
  return ok;
}

// One job's MMAs (NS K steps of 16, accumulator groups of GS steps), all
// offsets and accumulate flags compile-time constants.  Ring chunks in
// image order: parts 2 and 1 of each K block (x0 w2 | x1 w1, x0 w1), then
// part 0 of each K block (x2 w0, x1 w0; the stage is held), then the
// dominant x0 w0 products from the held stages, each stage released after
// its last MMA.  The five small products all go into group 0 before any
// x0 w0 product, so the truncating accumulation loses nothing of them that
// matters; group g takes x0 w0 of K steps [g GS, (g + 1) GS).
template <int NS, int GS>
__device__ __forceinline__ bool tr_job(const TrIssue& I, uint32_t& use, uint32_t ring_lo, uint32_t b_full,
                                       uint32_t b_empty, volatile int* abort_flag, long long& w_full) {
  constexpr int KB = (NS + 3) / 4;
  static_assert(KB <= kTrStages, "part-0 chunks of every K block are held in the ring at once");
#pragma unroll
  for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {  // part 2, then part 1
      if (!tr_wait_chunk(use, b_full, abort_flag, w_full)) return false;
      const uint32_t b = ring_lo + (use & 1u) * (kTrChunkBytes >> 4);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (kb * 4 + kk < NS) {
          const uint32_t ao = (uint32_t)kb * 1024u + (uint32_t)kk * 2u;  // K block: 16 KB; K step: 32 B
          const uint32_t bk = b + (uint32_t)kk * 2u;
          if (j == 0) {
            umma_f16_lh_warp(I.d, I.a0 + ao, bk, I.hi, I.idesc, (kb | kk) ? 1u : 0u);
          } else {
            umma_f16_lh_warp(I.d, I.a1 + ao, bk, I.hi, I.idesc, 1u);
            umma_f16_lh_warp(I.d, I.a0 + ao, bk, I.hi, I.idesc, 1u);
          }
        }
      }
      umma_commit_warp(b_empty + 8u * (use & 1u));
      ++use;
    }
  }
  uint32_t held[KB];
#pragma unroll
  for (int kb = 0; kb < KB; ++kb) {  // part 0: the small products x2 w0, x1 w0
    if (!tr_wait_chunk(use, b_full, abort_flag, w_full)) return false;
    held[kb] = use & 1u;
    const uint32_t b = ring_lo + held[kb] * (kTrChunkBytes >> 4);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      if (kb * 4 + kk < NS) {
        const uint32_t ao = (uint32_t)kb * 1024u + (uint32_t)kk * 2u;
        umma_f16_lh_warp(I.d, I.a2 + ao, b + (uint32_t)kk * 2u, I.hi, I.idesc, 1u);
        umma_f16_lh_warp(I.d, I.a1 + ao, b + (uint32_t)kk * 2u, I.hi, I.idesc, 1u);
      }
    }
    ++use;
  }
#pragma unroll
  for (int kb = 0; kb < KB; ++kb) {  // the dominant products x0 w0
    const uint32_t b = ring_lo + held[kb] * (kTrChunkBytes >> 4);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      constexpr int kGS = GS;
      const int step = kb * 4 + kk;
      if (step < NS) {
        const int g = step / kGS;
        const uint32_t acc = (g == 0 || step % kGS != 0) ? 1u : 0u;
        umma_f16_lh_warp(I.d + (uint32_t)g * I.n_pad, I.a0 + (uint32_t)kb * 1024u + (uint32_t)kk * 2u,
                         b + (uint32_t)kk * 2u, I.hi, I.idesc, acc);
      }
    }
    umma_commit_warp(b_empty + 8u * held[kb]);
  }
  return true;
}

// Tile order shared by the three roles: rounds of two tiles (one per slot);
// within a round, Matvec by Matvec, slot 0's job then slot 1's.
struct TrJobs {
  int64_t first, stride;
  int64_t c0, c1;  // tiles of slot 0 and slot 1
  __device__ TrJobs(int64_t ntiles, int64_t first_, int64_t stride_) : first(first_), stride(stride_) {
    const int64_t mine = first_ < ntiles ? (ntiles - first_ + stride_ - 1) / stride_ : 0;
    c0 = (mine + 1) / 2;
    c1 = mine / 2;
  }
  __device__ int64_t tile(int s, int64_t r) const { return first + (2 * r + s) * stride; }
};

__global__ void __launch_bounds__(kTrThreads, 1)
    tr_forward_kernel(const __grid_constant__ TrProgram p, const unsigned char* __restrict__ image,
                      float* __restrict__ scratch, const float* __restrict__ in, int64_t in_ld,
                      float* __restrict__ out, int64_t out_ld, int64_t batch, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t base = smem_u32(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (base & 1023u) {  // the operand layouts need 1024-byte alignment
    if (tid == 0) atomicExch(err, 5);
    return;
  }
  const uint32_t s_ring = base + kTrSlots * 3 * kTrPartBytes;
  const uint32_t s_bars = s_ring + kTrStages * kTrChunkBytes;
  const uint32_t b_full = s_bars;        // [stage]
  const uint32_t b_empty = s_bars + 16;  // [stage]
  const uint32_t b_accf = s_bars + 32;   // [slot] accumulator ready (MMA -> epilogue)
  const uint32_t b_epid = s_bars + 48;   // [slot] operand written and TMEM free (epilogue -> MMA)
  const uint32_t b_drain = s_bars + 64;
  const uint32_t s_tmem = s_bars + 72;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem_raw + (s_tmem - base));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem_raw + (s_tmem + 4 - base));

  const int64_t ntiles = (batch + kTcM - 1) / kTcM;
  if ((int64_t)blockIdx.x >= ntiles) return;
  const TrJobs jobs(ntiles, blockIdx.x, gridDim.x);
  const int nl = p.n_layers;

  if (warp == kTrMmaWarp) tmem_alloc(s_tmem, 2 * kTrSlotTmem);
  if (tid == 0) {
    for (int r = 0; r < kTrStages; ++r) {
      mbar_init(b_full + 8u * r, 1);
      mbar_init(b_empty + 8u * r, 1);
    }
    for (int s = 0; s < kTrSlots; ++s) {
      mbar_init(b_accf + 8u * s, 1);
      mbar_init(b_epid + 8u * s, kTrEpiWarps);
    }
    mbar_init(b_drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kTrProducerWarp) {
    // ------------------------------------------------ producer ----
    if (lane == 0) {
      uint32_t use = 0;
      bool ok = true;
      [[maybe_unused]] long long w_empty = 0;
      (void)w_empty;
      for (int64_t r = 0; r < jobs.c0 && ok; ++r)
        for (int l = 0; l < nl && ok; ++l)
          for (int s = 0; s < kTrSlots && ok; ++s) {
            if (r >= (s ? jobs.c1 : jobs.c0)) continue;
            const TrLayer& L = p.layers[l];
            const uint32_t bytes = (uint32_t)L.n_pad * 128u;
            for (int c = 0; c < L.kblk * 3; ++c) {
              const uint32_t st = use % kTrStages;
              TR_T(tw);
              if (use >= (uint32_t)kTrStages &&
                  !wait_phase_abort(b_empty + 8u * st, ((use / kTrStages) - 1) & 1u, abort_flag, kWaitCycles)) {
                ok = false;
                break;
              }
              TR_ACC(w_empty, tw);
              mbar_expect_tx(b_full + 8u * st, bytes);
              bulk_load(s_ring + st * kTrChunkBytes, image + L.w_off + (uint64_t)c * bytes, bytes, b_full + 8u * st);
              ++use;
            }
          }
      // Drain: the copies issued last must have landed before the CTA exits.
      const uint32_t n = use < (uint32_t)kTrStages ? use : (uint32_t)kTrStages;
      for (uint32_t u = use - n; u < use; ++u) {
        const long long t0 = clock64();
        while (!mbar_try_wait(b_full + 8u * (u % kTrStages), (u / kTrStages) & 1u))
          if (clock64() - t0 > kWaitCycles) break;
      }
      if (!ok) atomicExch(err, 2);
      TR_FLUSH(3, w_empty);
    }
    __syncwarp();
  } else if (warp == kTrMmaWarp) {
    // --------------------------------------------- MMA issuer ----
    // The whole warp runs the issue loop (its values stay warp-uniform); one
    // elected lane issues each MMA and commit.
    {
      uint32_t use = 0, ep0 = 0, ep1 = 0;
      bool ok = true;
      bool skip = PONNI_B200_SKIP_ARRIVE();  // wait-bound test build: drop the first job's signal
      [[maybe_unused]] long long w_epi = 0, w_full = 0;
      TR_T(t_all);
      // Descriptors as 32-bit halves: start addresses advance in the low half.
      const uint32_t hi = (uint32_t)(smem_desc(0, 16, 1024) >> 32);
      const uint32_t lo_flags = (uint32_t)smem_desc(0, 16, 1024);
      const uint32_t ring_lo = lo_flags | ((s_ring >> 4) & 0x3FFFu);
      for (int64_t r = 0; r < jobs.c0 && ok; ++r)
        for (int l = 0; l < nl && ok; ++l) {
          const TrLayer& L = p.layers[l];
          const uint32_t n_pad = (uint32_t)L.n_pad, gs = (uint32_t)L.group_steps, idesc = L.idesc;
          const int nsteps = L.nsteps;
          for (int s = 0; s < kTrSlots && ok; ++s) {
            if (r >= (s ? jobs.c1 : jobs.c0)) continue;
            // The slot's operand is written and its accumulators are free.
            TR_T(te);
            if (!(ok = __all_sync(0xffffffffu, wait_phase_abort(b_epid + 8u * s, s ? ep1 : ep0, abort_flag, kWaitCycles))))
              break;
            if (s) ep1 ^= 1u;
            else ep0 ^= 1u;
            TR_ACC(w_epi, te);
            tc_fence_after();
            TrIssue I;
            I.d = tmem_base + (uint32_t)s * kTrSlotTmem;
            I.n_pad = n_pad;
            I.idesc = idesc;
            I.hi = hi;
            const uint32_t a_base = base + (uint32_t)(s * 3) * kTrPartBytes;
            I.a0 = lo_flags | ((a_base >> 4) & 0x3FFFu);
            I.a1 = I.a0 + (kTrPartBytes >> 4);
            I.a2 = I.a0 + 2 * (kTrPartBytes >> 4);
            switch (nsteps * 16 + (int)gs) {
#define TR_JOB(n, g) \
  case n * 16 + g: ok = tr_job<n, g>(I, use, ring_lo, b_full, b_empty, abort_flag, w_full); break;
              TR_JOB(1, 1) TR_JOB(2, 2) TR_JOB(3, 3) TR_JOB(4, 4) TR_JOB(5, 5) TR_JOB(6, 6) TR_JOB(7, 7)
              TR_JOB(8, 8) TR_JOB(5, 4) TR_JOB(6, 4) TR_JOB(7, 4) TR_JOB(8, 4)
#undef TR_JOB
              default: ok = false; break;
            }
            if (ok && !skip) umma_commit_warp(b_accf + 8u * s);
            skip = false;
          }
        }
      // Drain: every MMA issued has completed before TMEM is freed.
      umma_commit_warp(b_drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(b_drain, 0))
        if (clock64() - t0 > kWaitCycles) break;
      if (lane == 0) {
        if (!ok) atomicExch(err, 3);
        TR_FLUSH(1, w_epi);
        TR_FLUSH(2, w_full);
#ifdef PONNI_B200_TC_PROFILE
        TR_FLUSH(7, clock64() - t_all);
#endif
      }
    }
    __syncwarp();
  } else {
    // ----------------------------------------------- epilogue ----
    // All 16 warps take the jobs in the MMA issuer's order, one job at a
    // time, so that one job's epilogue runs while the tensor core works on
    // the other slot's job.
    TrEpi E;
    E.cq = warp >> 2;
    E.lq = warp & 3;
    E.m = (warp & 3) * 32 + lane;
    E.image = image;
    E.n_saved = p.n_saved;
    E.saved_tmem = p.saved_tmem;
    E.saved_cta = reinterpret_cast<float4*>(scratch + (size_t)blockIdx.x * (p.scratch_per_cta / 4));
    auto select_slot = [&](int s) {
      E.saved = E.saved_cta + (size_t)s * p.n_saved * (kTrMaxN / 4) * 128;
      for (int q = 0; q < 3; ++q) E.a[q] = base + (uint32_t)(s * 3 + q) * kTrPartBytes;
      E.tmem_row = tmem_base + (uint32_t)s * kTrSlotTmem + ((uint32_t)((warp & 3) * 32) << 16);
    };
    const int k0 = p.layers[0].k_pad;
    // Operand written and accumulators read: hand the slot to the MMA issuer.
    auto release = [&](int s) {
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_epid + 8u * s);
    };
    for (int s = 0; s < kTrSlots; ++s)
      if ((s ? jobs.c1 : jobs.c0) > 0) {
        select_slot(s);
        tr_stage_input(in, in_ld, p.nin, k0, jobs.tile(s, 0) * kTcM + E.m, batch, E);
        release(s);
      }
    bool ok = true;
    uint32_t ph0 = 0, ph1 = 0;
    [[maybe_unused]] long long w_acc = 0, c_work = 0;
    for (int64_t r = 0; r < jobs.c0 && ok; ++r)
      for (int l = 0; l < nl && ok; ++l)
        for (int s = 0; s < kTrSlots; ++s) {
          const int64_t tiles = s ? jobs.c1 : jobs.c0;
          if (r >= tiles) continue;
          TR_T(ta);
          int got = 0;
          if (lane == 0) got = wait_phase_abort(b_accf + 8u * s, s ? ph1 : ph0, abort_flag, kWaitCycles) ? 1 : 0;
          got = __shfl_sync(0xffffffffu, got, 0);
          // The warps of a lane quarter leave together (none is left at a named barrier).
          if (epi_sync_or(E.lq, !got)) {
            ok = false;
            break;
          }
          if (s) ph1 ^= 1u;
          else ph0 ^= 1u;
          TR_ACC(w_acc, ta);
          TR_T(tw);
          tc_fence_after();
          select_slot(s);
          tr_epilogue(p, l, E, out, out_ld, jobs.tile(s, r) * kTcM + E.m, batch);
          TR_ACC(c_work, tw);
          if (l + 1 < nl) {
            release(s);
          } else if (r + 1 < tiles) {
            // The slot's MMAs are done with its operand and its accumulators
            // are read: stage its next tile.
            tr_stage_input(in, in_ld, p.nin, k0, jobs.tile(s, r + 1) * kTcM + E.m, batch, E);
            release(s);
          }
        }
    if (!ok && tid == 0) atomicExch(err, 4);
    if (tid == 0) {
      TR_FLUSH(4, w_acc);
      TR_FLUSH(5, c_work);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kTrMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kTrSlotTmem);
  }
}

}  // namespace

cudaError_t launch_tr_forward(const TrProgram& p, const void* image, void* scratch, const void* in, int64_t in_ld,
                              void* out, int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  if (p.dtype != 0) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(tr_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)p.smem_bytes);
  if (e != cudaSuccess) return e;
  tr_forward_kernel<<<grid, kTrThreads, p.smem_bytes, stream>>>(
      p, static_cast<const unsigned char*>(image), static_cast<float*>(scratch), static_cast<const float*>(in), in_ld,
      static_cast<float*>(out), out_ld, batch, err);
  return cudaGetLastError();
}

}  // namespace ponni_b200
