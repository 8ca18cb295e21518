// Body of the resident-weights tensor-core kernel (sm_100a, tcgen05 + TMEM),
// shared by the library's generic kernel (tc_kernel.cu) and by the
// model-specialised kernel generated and compiled with NVRTC at plan time
// (tc_jit.cpp), so both run the same code.  The algorithm is described at
// the top of tc_kernel.cu.
#pragma once
#include "device_math.cuh"
#include "tc_common.cuh"
#include "tc_program.h"

namespace ponni_b200 {
namespace tck {
using namespace tc;

#ifdef PONNI_B200_TC_PROFILE
__device__ int* prof_ptr;
#endif

// The fields of a layer the epilogue needs, held in registers (a reference
// into shared memory would be re-read after every shared-memory store).
struct EpiArgs {
  int n_pad, nout, groups, has_bias, act_flags;
  float s0, s1;
};

template <int ACT>
__device__ __forceinline__ float epi_act(float v, const EpiArgs& E) {
  if constexpr (ACT == EPI_NONE) return v;
  else return activation<float>(ACT, E.act_flags, v, E.s0, E.s1);
}

// ReLU on two packed 16-bit values: max(x, 0) after rounding equals the
// rounding of max(x, 0) (rounding is monotonic and keeps the sign).
__device__ __forceinline__ uint32_t relu2(uint32_t w, __half*) {
  uint32_t r;
  asm("max.f16x2 %0, %1, %2;\n" : "=r"(r) : "r"(w), "r"(0u));
  return r;
}
__device__ __forceinline__ uint32_t relu2(uint32_t w, __nv_bfloat16*) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(w), "r"(0u));
  return r;
}

// Epilogue of one layer for this thread's TMEM lane (= batch column m):
// sum the layer's accumulators, add the bias, apply the activation (fp32),
// then write the next layer's operand, or the caller's output.  Padding
// columns (nout..n_pad) need no masking: their weights and biases are zero
// and the next layer's padded K rows of B are zero.
template <class T, int TPS, int ACT>
__device__ __forceinline__ void epilogue(const EpiArgs E, bool last, uint32_t tmem_lane, const float* bias,
                                         const uint32_t* a, T* __restrict__ out, int64_t out_ld, int64_t col,
                                         int64_t batch, int m, int half) {
  using Op = typename OperandOf<T>::type;
  constexpr int kStep = 32 * (TPS / 128);  // 256-thread slots split the columns in two halves
  for (int c0 = 32 * half; c0 < E.n_pad; c0 += kStep) {
    float v[32];
#ifdef PONNI_B200_TC_PROFILE
    const long long t_ld = clock64();
#endif
    int g = 1;
    if (sizeof(T) != 4 || E.groups == 1) {  // 16-bit models keep one accumulator per layer
      tmem_ld32(tmem_lane + (uint32_t)c0, v);
    } else {
      float w[32];
      tmem_ld32x2(tmem_lane + (uint32_t)c0, tmem_lane + (uint32_t)(E.n_pad + c0), v, w);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += w[j];
      g = 2;
    }
    for (; sizeof(T) == 4 && g + 1 < E.groups; g += 2) {
      float w0[32], w1[32];
      tmem_ld32x2(tmem_lane + (uint32_t)(g * E.n_pad + c0), tmem_lane + (uint32_t)((g + 1) * E.n_pad + c0), w0, w1);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += w0[j] + w1[j];
    }
    for (; sizeof(T) == 4 && g < E.groups; ++g) {
      float w[32];
      tmem_ld32(tmem_lane + (uint32_t)(g * E.n_pad + c0), w);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += w[j];
    }
#ifdef PONNI_B200_TC_PROFILE
    if ((threadIdx.x & (TPS - 1)) == 0)
      atomicAdd(reinterpret_cast<unsigned long long*>(prof_ptr) + 7, (unsigned long long)(clock64() - t_ld));
#endif
    if (E.has_bias) {
      const float4* b4 = reinterpret_cast<const float4*>(bias + c0);  // zero-padded to 32 columns
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b = b4[q];
        if constexpr (sizeof(T) == 2) {  // packed fp32 (fp32 models: register pressure, slower)
          f2::add(v[4 * q], v[4 * q + 1], v[4 * q], v[4 * q + 1], b.x, b.y);
          f2::add(v[4 * q + 2], v[4 * q + 3], v[4 * q + 2], v[4 * q + 3], b.z, b.w);
        } else {
          v[4 * q] += b.x;
          v[4 * q + 1] += b.y;
          v[4 * q + 2] += b.z;
          v[4 * q + 3] += b.w;
        }
      }
    }
    if (last) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = epi_act<ACT>(v[j], E);
      if (col < batch) {
        // Rows c0 .. c0 + nv of the output (a warp stores 32 consecutive
        // columns of each row).
        const int nv = min(32, E.nout - c0);
        T* o = out + (int64_t)c0 * out_ld + col;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (j >= nv) break;
          o[(int64_t)j * out_ld] = Store<T>::from(v[j]);
        }
      }
    } else if constexpr (sizeof(T) == 2 && ACT == EPI_RELU) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = relu2(pack2(v[8 * q + 2 * e], v[8 * q + 2 * e + 1], (Op*)0), (Op*)0);
        st_shared_v4(a[0] + kmajor_chunk(m, (uint32_t)(c0 + 8 * q) * 2), w[0], w[1], w[2], w[3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = epi_act<ACT>(v[j], E);
#pragma unroll
      for (int q = 0; q < 4; ++q) store_row8<T>(a, m, c0 + 8 * q, v + 8 * q);
    }
  }
}

template <class T, int TPS>
__device__ __forceinline__ void epilogue_dispatch(int act, const EpiArgs E, bool last, uint32_t tmem_lane,
                                                  const float* bias, const uint32_t* a, T* __restrict__ out,
                                                  int64_t out_ld, int64_t col, int64_t batch, int m, int half) {
#define PONNI_TC_EPI(A) epilogue<T, TPS, A>(E, last, tmem_lane, bias, a, out, out_ld, col, batch, m, half)
  switch (act) {
    case EPI_RELU: PONNI_TC_EPI(EPI_RELU); break;
    case EPI_LEAKY_RELU: PONNI_TC_EPI(EPI_LEAKY_RELU); break;
    case EPI_SILU: PONNI_TC_EPI(EPI_SILU); break;
    case EPI_GELU: PONNI_TC_EPI(EPI_GELU); break;
    case EPI_TANH: PONNI_TC_EPI(EPI_TANH); break;
    case EPI_SIGMOID: PONNI_TC_EPI(EPI_SIGMOID); break;
    default: PONNI_TC_EPI(EPI_NONE); break;
  }
#undef PONNI_TC_EPI
}

// Named barrier over one slot's threads (ids 1..slots; 0 is __syncthreads).
template <int TPS>
__device__ __forceinline__ void wg_sync(int wg) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(wg + 1), "r"(TPS) : "memory");
}
template <int TPS>
__device__ __forceinline__ int wg_sync_or(int wg, int pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %2, 0;\n\t"
      "bar.red.or.pred q, %1, %3, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(wg + 1), "r"(pred), "r"(TPS)
      : "memory");
  return r;
}

// Issue the UMMA chain of layer L for one slot (one warp, elected lane).  The
// descriptors of each operand are built once per layer; the K steps then only
// add the step offset to the 14-bit start-address field (>> 4), which never
// carries out of the field for shared-memory addresses.
// No-swizzle K-major descriptor (8-row core matrices of 16 bytes: `lbo`
// between the two K halves of a 16-element K step, `sbo` between row groups).
__device__ __forceinline__ uint64_t smem_desc_plain(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

template <bool SPLIT>
__device__ __forceinline__ void issue_layer(const TcLayer& L, bool layer0, uint32_t d_tmem, const uint32_t* s_a,
                                            uint32_t s_image, uint32_t stage, uint32_t s_ones, uint32_t s_zero) {
  const int nsteps = L.k_pad / 16;  // UMMA K = 16 for 16-bit operands (32 bytes)
  const uint64_t b_step_kb = (uint64_t)L.n_pad * 8;  // (n_pad * 128) >> 4 per K block
  const uint32_t gstep = (uint32_t)L.group_steps, n_pad = (uint32_t)L.n_pad;
  const uint32_t idesc = L.idesc;
  uint32_t d = d_tmem, in_group = 0;
  if constexpr (SPLIT) {
    uint64_t a0[3], b0[3];
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      a0[q] = smem_desc(s_a[q], 16, 1024);
      b0[q] = smem_desc(s_image + L.w_off[q], 16, 1024);
    }
    // Accumulators: groups - 1 "main" ones, each summing the dominant
    // products a0*b0 of gstep consecutive K steps, and one "correction"
    // accumulator for the five smaller products of every step (their
    // truncation errors are 2^-8 smaller).  The tensor core's fp32
    // accumulation truncates, so bounding the additions into each main
    // accumulator keeps the result fp32-accurate; the epilogue sums all.
    const uint32_t dc = d_tmem + (uint32_t)(L.groups - 1) * n_pad;
    for (int s = 0; s < nsteps; ++s) {
      const uint64_t ao = (uint64_t)(s >> 2) * 1024 + (uint64_t)(s & 3) * 2;
      const uint64_t bo = (uint64_t)(s >> 2) * b_step_kb + (uint64_t)(s & 3) * 2;
      umma_f16_warp(dc, a0[1] + ao, b0[1] + bo, idesc, s > 0 ? 1u : 0u);  // smallest products first
      umma_f16_warp(dc, a0[0] + ao, b0[2] + bo, idesc, 1u);
      umma_f16_warp(dc, a0[2] + ao, b0[0] + bo, idesc, 1u);
      umma_f16_warp(dc, a0[0] + ao, b0[1] + bo, idesc, 1u);
      umma_f16_warp(dc, a0[1] + ao, b0[0] + bo, idesc, 1u);
      umma_f16_warp(d, a0[0] + ao, b0[0] + bo, idesc, in_group ? 1u : 0u);
      if (++in_group == gstep) {
        in_group = 0;
        d += n_pad;
      }
    }
  } else {
    const uint64_t b0 = smem_desc(s_image + L.w_off[0], 16, 1024);
    // The bias first: D = ones x bias block (every row of A is e_0).
    uint32_t acc0 = 0;
    if (L.bias_mma) {
      const uint32_t s_bias = s_image + L.bias_off;
      umma_f16_warp(d, smem_desc_plain(s_ones, s_zero - s_ones, 0), smem_desc_plain(s_bias, s_zero - s_bias, 128),
                    idesc, 0u);
      acc0 = 1;
    }
    if (layer0) {
      // The staged input tile is the MN-major layer-0 operand: one K step =
      // 32 bytes of K for 128 rows = 4096 bytes.
      const uint64_t a0 = smem_desc(stage, 1024, 2048);
      for (int s = 0; s < nsteps; ++s) {
        const uint64_t bo = (uint64_t)(s >> 2) * b_step_kb + (uint64_t)(s & 3) * 2;
        umma_f16_warp(d, a0 + (uint64_t)s * 256, b0 + bo, L.idesc_mn, (s > 0 || acc0) ? 1u : 0u);
      }
    } else {
      const uint64_t a0 = smem_desc(s_a[0], 16, 1024);
      for (int s = 0; s < nsteps; ++s) {
        const uint64_t ao = (uint64_t)(s >> 2) * 1024 + (uint64_t)(s & 3) * 2;
        const uint64_t bo = (uint64_t)(s >> 2) * b_step_kb + (uint64_t)(s & 3) * 2;
        umma_f16_warp(d, a0 + ao, b0 + bo, idesc, (s > 0 || acc0) ? 1u : 0u);
      }
    }
  }
}

// Optional phase timing (compiled only with -DPONNI_B200_TC_PROFILE): thread
// 0 of each warpgroup adds the cycles of each phase to `prof` (6 counters).
#ifdef PONNI_B200_TC_PROFILE
#define TC_PROF_T(var) const long long var = clock64()
#define TC_PROF_ADD(idx, t0) \
  if (lt == 0) atomicAdd(reinterpret_cast<unsigned long long*>(err) + 1 + (idx), (unsigned long long)(clock64() - (t0)))
#else
#define TC_PROF_T(var)
#define TC_PROF_ADD(idx, t0)
#endif

// --------------------------------------------------------------- kernel --
// Up to four slots per CTA, each run by 4 or 8 warps (4 TMEM lane quarters,
// x 2 column halves with 8) that own the slot's operand buffers, input stage, mbarrier and TMEM
// accumulators and walk their own tiles; while one slot runs its epilogue the
// tensor core works on the other's chain.
//
// `Shape` fixes the layer loop: RuntimeShape walks the program's layer table;
// a generated shape (the model-specialised kernel compiled at plan time)
// gives the layer count and every layer's widths, accumulator groups,
// activation and bias flag as compile-time constants, so that the loop
// unrolls and the epilogue's bookkeeping folds away.
struct RuntimeShape {
  static constexpr bool kStatic = false;
  static constexpr int kNL = 0;
  static __device__ __forceinline__ void fix(int, TcLayer&) {}
};

template <class T, int TPS, class Shape>
__device__ __forceinline__ void tc_forward_body(const TcProgram& p, const unsigned char* __restrict__ image,
                                                const T* __restrict__ in, int64_t in_ld, T* __restrict__ out,
                                                int64_t out_ld, int64_t batch, int in_vec, int* __restrict__ err) {
  constexpr bool SPLIT = sizeof(T) == 4;
  constexpr int NP = SPLIT ? 3 : 1;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzle atoms need 1024-byte alignment
  unsigned char* base_ptr = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int kWarps = TPS / 32;
  const int wg = warp / kWarps, lt = tid & (TPS - 1);
  const int half = TPS == 256 ? (warp >> 2) & 1 : 0;  // column half of the epilogue this warp handles
  const uint32_t s_image = base;
  const uint32_t s_slot = s_image + p.image_bytes + (uint32_t)wg * p.slot_bytes;
  uint32_t s_a[3];
#pragma unroll
  for (int q = 0; q < 3; ++q) s_a[q] = s_slot + (uint32_t)(q < NP ? q : 0) * p.a_bytes;
  const uint32_t stage = s_slot + (uint32_t)NP * p.a_bytes;
  const int nslots = p.slots, nthreads = nslots * TPS;
  const uint32_t s_bars = s_image + p.image_bytes + (uint32_t)nslots * p.slot_bytes;
  const uint32_t s_bar = s_bars + 8u * (uint32_t)wg;
  const uint32_t s_tmem = s_bars + 8u * kTcMaxSlots;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(base_ptr + (s_tmem - base));
  // Layer table copied to shared memory: the layer loop indexes it with a
  // run-time index, which on the kernel-parameter copy would go through the
  // constant cache's slow address-divergence path.
  TcLayer* layers = reinterpret_cast<TcLayer*>(base_ptr + (s_bars + 128u - base));

  const int64_t ntiles = (batch + kTcM - 1) / kTcM;
  if ((int64_t)blockIdx.x * nslots >= ntiles) return;
#ifdef PONNI_B200_TC_PROFILE
  if (tid == 0) prof_ptr = err;
#endif

  // ---- set-up (whole CTA): TMEM, mbarriers, zeroed stages, parameter image ----
  if (warp == 0) tmem_alloc(s_tmem, p.tmem_cols);
  if (tid == 0) {
    for (int q = 0; q < nslots; ++q) mbar_init(s_bars + 8u * q, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  for (int q = 0; q < nslots; ++q) {
    uint4* z = reinterpret_cast<uint4*>(base_ptr + (s_image + p.image_bytes + q * p.slot_bytes + NP * p.a_bytes - base));
    for (int i = tid; i < (int)(p.stage_bytes / 16); i += nthreads) z[i] = make_uint4(0, 0, 0, 0);
  }
  for (uint32_t i = tid; i < p.image_bytes / 16; i += nthreads) cp_async16(s_image + i * 16, image + i * 16, 16);
  for (int i = tid; i < p.n_layers; i += nthreads) layers[i] = p.layers[i];
  cp_async_commit();
  cp_async_wait_0();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot + (uint32_t)wg * p.slot_cols;
  const uint32_t tmem_lane = tmem_base + ((uint32_t)((warp & 3) * 32) << 16);
  const int m = (warp & 3) * 32 + lane;  // this thread's batch row in its slot's tile

  // ---- per-warpgroup tile loop ----
  const int64_t stride = (int64_t)gridDim.x * nslots;
  int64_t tile = (int64_t)blockIdx.x * nslots + wg;
  uint32_t phase = 0;
  if (!SPLIT && tile < ntiles) {
    load_input<T, TPS>(stage, in, in_ld, p.nin, tile * kTcM, batch, in_vec != 0, lt);
    cp_async_commit();
  }
  for (; tile < ntiles; tile += stride) {
    const int64_t col0 = tile * kTcM;
    const int64_t next = tile + stride;
    TC_PROF_T(t_in);
    cp_async_wait_0();
    wg_sync<TPS>(wg);
    TC_PROF_ADD(0, t_in);
    TC_PROF_T(t_split);
    if constexpr (SPLIT) {
      // Thread m reads column m of the input straight from global memory (a
      // warp reads 32 consecutive columns of a feature row: coalesced) and
      // splits it into the K-major bf16 operand parts of layer 0.  No input
      // stage: the shared memory goes to more tile slots, whose work hides
      // this load's latency.
      TcLayer L0 = layers[0];
      Shape::fix(0, L0);
      const int k0 = L0.k_pad, nin = p.nin;
      const int64_t col = col0 + m;
      const bool live = col < batch;
      const float* src = reinterpret_cast<const float*>(in) + col;
      for (int f = 16 * half; f < k0; f += 16 * (TPS / 128)) {
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = (live && f + e < nin) ? __ldg(src + (int64_t)(f + e) * in_ld) : 0.0f;
        store_row8<T>(s_a, m, f, v);
        if (f + 8 < k0) store_row8<T>(s_a, m, f + 8, v + 8);
      }
    }
    TC_PROF_ADD(1, t_split);
    // One layer of this tile; false when the slot gives up (bounded wait).
    auto layer_step = [&](int l, const TcLayer& L, int nl) -> bool {
      const EpiArgs E{L.n_pad, L.nout, L.groups, L.has_bias, L.act_flags, L.s0, L.s1};
      const int act = L.act;
      const uint32_t bias_off = L.bias_off;
      TC_PROF_T(t_bar);
      fence_proxy_async();
      tc_fence_before();
      wg_sync<TPS>(wg);
      // The slot's first warp issues the chain (one elected lane per MMA,
      // descriptors in uniform registers) and waits for its completion; the
      // rest of the slot parks on the named barrier (no issue slots spent
      // spinning while the other slots' epilogues run).
      TC_PROF_ADD(2, t_bar);
      bool ok = true;
      if (lt < 32) {  // the slot's first warp issues (one elected lane per MMA) and waits
        TC_PROF_T(t_issue);
        tc_fence_after();
        issue_layer<SPLIT>(L, l == 0, tmem_base, s_a, s_image, stage, s_image + p.ones_off, s_image + p.zero_off);
        // (the wait-bound test build drops the first layer's signal of the first tile)
        if (!(PONNI_B200_SKIP_ARRIVE() && l == 0 && tile == (int64_t)blockIdx.x * nslots + wg)) umma_commit_warp(s_bar);
        TC_PROF_ADD(3, t_issue);
        TC_PROF_T(t_mma);
        int w = 0;
        if (lane == 0) w = mbar_wait_bounded(s_bar, phase) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, w, 0) != 0;
        TC_PROF_ADD(4, t_mma);
      }
      phase ^= 1u;
      TC_PROF_T(t_post);
      const int bad = wg_sync_or<TPS>(wg, !ok);
      tc_fence_after();
      if (bad) {
        if (lt == 0) atomicExch(err, 1);
        return false;
      }
      if constexpr (!SPLIT) {
        if (l == 0) {  // layer 0 has consumed the stage: prefetch the next tile
          if (next < ntiles) load_input<T, TPS>(stage, in, in_ld, p.nin, next * kTcM, batch, in_vec != 0, lt);
          cp_async_commit();
        }
        TC_PROF_ADD(1, t_post);  // 16-bit models have no split phase: slot 1 times the hand-off
      }
      const float* bias = reinterpret_cast<const float*>(base_ptr + bias_off);
      TC_PROF_T(t_epi);
      epilogue_dispatch<T, TPS>(act, E, l == nl - 1, tmem_lane, bias, s_a, out, out_ld, col0 + m, batch, m, half);
      TC_PROF_ADD(5, t_epi);
      return true;
    };
    bool failed = false;
    if constexpr (Shape::kStatic) {
#pragma unroll
      for (int l = 0; l < Shape::kNL; ++l) {
        if (!failed) {
          TcLayer L = layers[l];
          Shape::fix(l, L);
          failed = !layer_step(l, L, Shape::kNL);
        }
      }
    } else {
      for (int l = 0; l < p.n_layers && !failed; ++l) failed = !layer_step(l, layers[l], p.n_layers);
    }
    if (failed) break;
  }
  cp_async_wait_0();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(*tmem_slot, p.tmem_cols);
  }
}


}  // namespace tck
}  // namespace ponni_b200
