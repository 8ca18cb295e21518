// Body of the streamed-weights tensor-core kernel (sm_100a, tcgen05 + TMEM),
// shared by the library's generic kernel (tc_stream.cu, which describes the
// algorithm) and by the model-specialised kernel compiled with NVRTC at plan
// time (narrow_jit.cpp), so both run the same code.
#pragma once
#include <cuda.h>

#include "device_math.cuh"
#include "tc_common.cuh"
#include "tc_stream_program.h"

#ifndef PONNI_B200_TS_DIAG
#define PONNI_B200_TS_DIAG 0
#endif
#if PONNI_B200_TS_DIAG & 4  // diagnostic builds: bit 4 removes the epilogue work
#define PONNI_B200_TS_NO_EPI
#endif

namespace ponni_b200 {
namespace tsk {
using namespace tc;

constexpr long long kWaitCycles = PONNI_B200_WAIT_LIMIT;

// Epilogue organisation: all 16 epilogue warps on every job (4 TMEM lane
// quarters x 4 column quarters of 64), or (diagnostic builds, bit 8) one
// group of 8 warps per slot (4 lane quarters x 2 column halves of 128).
#if PONNI_B200_TS_DIAG & 8
constexpr bool kTsEpiAll = false;
#else
constexpr bool kTsEpiAll = true;
#endif
constexpr int kTsEpiCols = kTsEpiAll ? kTsMaxN / 4 : kTsMaxN / 2;     // accumulator columns per warp and job
constexpr int kTsEpiLoaders = kTsEpiAll ? kTsEpiWarps * 32 : kTsGroupThreads;  // threads staging a tile
constexpr int kTsEpiHalfWarps = kTsEpiAll ? 8 : 4;                   // warps signalling one column half

// Optional phase timing (compiled only with -DPONNI_B200_TC_PROFILE): each
// role sums the cycles of its waits locally and adds them once per CTA to
// the diagnostic counters after the error word.
#ifdef PONNI_B200_TC_PROFILE
#define TS_T(var) const long long var = clock64()
#define TS_ACC(acc, t0) acc += clock64() - (t0)
#define TS_FLUSH(idx, acc) atomicAdd(reinterpret_cast<unsigned long long*>(err) + (idx), (unsigned long long)(acc))
#else
#define TS_T(var)
#define TS_ACC(acc, t0)
#define TS_FLUSH(idx, acc)
#endif

// Bounded wait that also leaves when another role has aborted.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  return wait_phase_abort(bar, parity, abort_flag, kWaitCycles);
}

__device__ __forceinline__ uint32_t idesc_of(int dtype, int n, bool a_mn) {
  const uint32_t fmt = dtype == 2 ? 0u : 1u;  // f16 : bf16
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((a_mn ? 1u : 0u) << 15) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kTcM >> 4) << 24);
}

__device__ __forceinline__ float tanh_fast(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;\n" : "=f"(t) : "f"(x));
  return t;
}

template <int ACT>
__device__ __forceinline__ float ts_act(float x, int fast, int flags, float s0, float s1) {
  if constexpr (ACT == EPI_NONE) {
    return x;
  } else if constexpr (ACT == EPI_RELU) {
    return x > 0.f ? x : 0.f;
  } else if constexpr (ACT == EPI_SILU || ACT == EPI_SIGMOID || ACT == EPI_TANH) {
    if (fast) {
      if constexpr (ACT == EPI_TANH) return tanh_fast(x);
      else return x * 0.f;  // SiLU / sigmoid take ts_act32's fast path
    }
    return activation<float>(ACT, flags, x, s0, s1);
  } else {
    return activation<float>(ACT, flags, x, s0, s1);
  }
}

// sigmoid(x) = (1 + tanh(x / 2)) / 2 with the hardware tanh approximation:
// one MUFU operation per value (absolute error near 2^-11, below one
// fp16/bf16 unit of the activations the next layer consumes).
// Activation of 32 values; in the fast mode SiLU and sigmoid use
// the sigmoid above (two values at a time), tanh the fp32 tanh approximation.
template <int ACT>
__device__ __forceinline__ void ts_act32(float (&v)[32], int fast, int flags, float s0, float s1) {
  if constexpr (ACT == EPI_SILU || ACT == EPI_SIGMOID) {
    if (fast) {
      // packed fp32 for the multiplies and the fma
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float h0, h1, g0, g1;
        f2::mul(h0, h1, v[j], v[j + 1], 0.5f, 0.5f);
        f2::fma(g0, g1, 0.5f, 0.5f, tanh_fast(h0), tanh_fast(h1), 0.5f, 0.5f);
        if (ACT == EPI_SILU) f2::mul(v[j], v[j + 1], v[j], v[j + 1], g0, g1);
        else v[j] = g0, v[j + 1] = g1;
      }
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = ts_act<ACT>(v[j], fast, flags, s0, s1);
}

// Epilogue of the columns [c_begin, c_begin + kTsEpiCols) of one job
// for this thread's row m: accumulator -> bias -> activation -> the tile's
// K-major operand (in place: the job's MMAs have completed) or the output.
template <class T, int ACT>
__device__ __forceinline__ void ts_epilogue(const TsLayer& L, int fast, bool last, uint32_t tmem_row, int c_begin,
                                            const float* __restrict__ bias, uint32_t a_out, T* __restrict__ out,
                                            int64_t out_ld, int64_t col, int64_t batch, int m, long long (&t_ph)[3]) {
  (void)t_ph;
  const int n_pad = L.n_pad, nout = L.nout, has_bias = L.has_bias, flags = L.act_flags;
  const float s0 = L.s0, s1 = L.s1;
#pragma unroll 1
  for (int c0 = c_begin; c0 < c_begin + kTsEpiCols && c0 < n_pad; c0 += 32) {
    float v[32];
    TS_T(tl);
    tmem_ld32(tmem_row + (uint32_t)c0, v);
    TS_ACC(t_ph[0], tl);
    TS_T(ta);
    if (has_bias) {
      const float4* b4 = reinterpret_cast<const float4*>(bias + c0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b = __ldg(b4 + q);
        f2::add(v[4 * q], v[4 * q + 1], v[4 * q], v[4 * q + 1], b.x, b.y);
        f2::add(v[4 * q + 2], v[4 * q + 3], v[4 * q + 2], v[4 * q + 3], b.z, b.w);
      }
    }
#if !(PONNI_B200_TS_DIAG & 2)  // diagnostic builds: bit 2 skips activations
    ts_act32<ACT>(v, fast, flags, s0, s1);
#endif
    TS_ACC(t_ph[1], ta);
    if (last) {
      if (col < batch) {
        const int nv = min(32, nout - c0);
        T* o = out + (int64_t)c0 * out_ld + col;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (j >= nv) break;
          o[(int64_t)j * out_ld] = Store<T>::from(v[j]);
        }
      }
    } else {
      const uint32_t a[1] = {a_out};
#pragma unroll
      for (int q = 0; q < 4; ++q) store_row8<T>(a, m, c0 + 8 * q, v + 8 * q);
    }
  }
}

template <class T>
__device__ __forceinline__ void ts_epilogue_dispatch(const TsLayer& L, int fast, bool last, uint32_t tmem_row,
                                                     int c_begin, const float* bias, uint32_t a_out,
                                                     T* __restrict__ out, int64_t out_ld, int64_t col, int64_t batch,
                                                     int m, long long (&t_ph)[3]) {
#define PONNI_TS_EPI(A) \
  ts_epilogue<T, A>(L, fast, last, tmem_row, c_begin, bias, a_out, out, out_ld, col, batch, m, t_ph)
  switch (L.act) {
    case EPI_RELU: PONNI_TS_EPI(EPI_RELU); break;
    case EPI_LEAKY_RELU: PONNI_TS_EPI(EPI_LEAKY_RELU); break;
    case EPI_SILU: PONNI_TS_EPI(EPI_SILU); break;
    case EPI_GELU: PONNI_TS_EPI(EPI_GELU); break;
    case EPI_TANH: PONNI_TS_EPI(EPI_TANH); break;
    case EPI_SIGMOID: PONNI_TS_EPI(EPI_SIGMOID); break;
    default: PONNI_TS_EPI(EPI_NONE); break;
  }
#undef PONNI_TS_EPI
}

// Layer-0 operand (MN-major, 128-byte swizzle) of one tile: two 64-column
// halves, each k0 feature rows of 128 B (row f at f * 128, its 16-byte
// chunks XOR-ed with f % 8), half h at h * k0 * 128.  This is the layout a
// 2-D tensor copy with 128-byte swizzle writes for a box of 64 columns x k0
// features, so the loader warp fills it with two copies; the fallback below
// writes the same bytes with cp.async.
__device__ __forceinline__ uint32_t ts_stage_off(int f, int j, int k0) {
  return (uint32_t)(j >> 3) * (uint32_t)(k0 * 128) + (uint32_t)f * 128u + ((((uint32_t)j & 7u) ^ ((uint32_t)f & 7u)) << 4);
}

// Stage tile `t`'s input into a slot's operand buffer with cp.async (the
// epilogue threads; used when the input cannot go through a tensor map),
// and zero its padding K rows nin..k0 (the buffer holds the previous
// tile's activations).
template <class T>
__device__ __forceinline__ void ts_load_tile(uint32_t buf, unsigned char* buf_ptr, const T* in, int64_t in_ld,
                                             int nin, int k0, int64_t t, int64_t batch, bool vec, int tid) {
  const int64_t col0 = t * kTcM;
  if (vec) {
    for (int i = tid; i < nin * 16; i += kTsEpiLoaders) {
      const int f = i >> 4, j = i & 15;
      const int64_t col = col0 + (int64_t)j * 8;
      const int64_t valid = batch - col;
      const int bytes = valid >= 8 ? 16 : (valid > 0 ? (int)valid * 2 : 0);
      cp_async16(buf + ts_stage_off(f, j, k0), in + (int64_t)f * in_ld + (bytes > 0 ? col : 0), bytes);
    }
  } else {
    for (int i = tid; i < nin * kTcM; i += kTsEpiLoaders) {
      const int f = i / kTcM, mm = i - f * kTcM;
      const int64_t col = col0 + mm;
      const T v = col < batch ? in[(int64_t)f * in_ld + col] : Store<T>::from(0.0f);
      const uint32_t dst = buf + ts_stage_off(f, mm >> 3, k0) + (uint32_t)(mm & 7) * 2;
      asm volatile("st.shared.b16 [%0], %1;\n" ::"r"(dst), "h"(*reinterpret_cast<const unsigned short*>(&v)) : "memory");
    }
  }
  cp_async_commit();
  for (int i = tid; i < (k0 - nin) * 16; i += kTsEpiLoaders) {
    const int f = nin + (i >> 4), j = i & 15;
    *reinterpret_cast<uint4*>(buf_ptr + ts_stage_off(f, j, k0)) = make_uint4(0, 0, 0, 0);
  }
}

// One box of the input tensor map (64 columns x k0 features, 128-byte
// swizzle) into shared memory, completion counted in bytes on `bar`.  No
// multicast; the column coordinate is a multiple of 64 (the 16-byte rule).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Job order shared by the three roles: rounds of two tiles (one per slot);
// within a round, layer by layer, slot 0's job then slot 1's.  Slot s's
// j-th tile is this CTA's tile 2j + s of the grid-strided sequence.  In pair
// mode the sequence runs over pairs of adjacent tiles, one per cluster of
// two CTAs, and CTA r of the pair takes tile 2 * pair + r (a tile past the
// batch is computed on zero columns and not stored).
struct TsJobs {
  int64_t first, stride, units;
  int64_t count[kTsSlots];
  int per, rank;
  __device__ TsJobs(int64_t units_, int64_t first_, int64_t stride_, int per_, int rank_)
      : first(first_), stride(stride_), units(units_), per(per_), rank(rank_) {
    const int64_t mine = first_ < units_ ? (units_ - first_ + stride_ - 1) / stride_ : 0;
    count[0] = (mine + 1) / 2;
    count[1] = mine / 2;
  }
  __device__ int64_t rounds() const { return count[0]; }
  __device__ int64_t tile(int s, int64_t r) const { return (first + (2 * r + s) * stride) * per + rank; }
};

// Single CTA (PAIR false): the CTA issues M = 128 MMAs over its own tile.
// CTA pair (PAIR true, clusters of two): the even CTA issues M = 256 MMAs
// (cta_group::2) over both CTAs' tiles; each CTA streams half of every
// weight chunk (N / 2 rows) into its own ring with its own bulk copies, the
// odd CTA's MMA warp relays "my half has landed" to the even CTA, the
// commits signal both CTAs, and the odd CTA's epilogue warps arrive on the
// even CTA's operand barriers.  Per SM this halves the weight bytes staged
// and the MMA instructions issued.
// `Shape` fixes the epilogue's layer loop: TsRuntimeShape walks the layer
// table; a generated shape (the model-specialised build compiled at plan
// time) unrolls it with every layer's widths, bias flag and activation as
// compile-time constants.
struct TsRuntimeShape {
  static constexpr bool kStatic = false;
  static constexpr int kNL = 0;
  static __device__ __forceinline__ void fix(int, TsLayer&) {}
  template <class T>
  static __device__ __forceinline__ void epilogue(int, const TsLayer& L, int fast, bool last, uint32_t tmem_row,
                                                  int c_begin, const float* bias, uint32_t a_out,
                                                  T* __restrict__ out, int64_t out_ld, int64_t col, int64_t batch,
                                                  int m, long long (&t_ph)[3]) {
    ts_epilogue_dispatch<T>(L, fast, last, tmem_row, c_begin, bias, a_out, out, out_ld, col, batch, m, t_ph);
  }
};

template <class T, bool PAIR, class Shape>
__device__ __forceinline__ void ts_forward_body(const TsProgram& p, const unsigned char* __restrict__ image,
                                                const T* __restrict__ in, int64_t in_ld, T* __restrict__ out,
                                                int64_t out_ld, int64_t batch, int in_vec, const CUtensorMap& in_map,
                                                int in_tma, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* base_ptr = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int R = (int)p.ring_stages;
  const uint32_t crank = PAIR ? cluster_rank() : 0u;
  const bool leader = crank == 0;
  constexpr uint32_t kStage = PAIR ? kTsChunkBytes / 2 : kTsChunkBytes;

  const uint32_t s_a[kTsSlots] = {base, base + p.a_bytes};  // per-slot operand buffer (input stage inside)
  const uint32_t s_ring = base + kTsSlots * p.a_bytes;
  const uint32_t s_bars = s_ring + (uint32_t)R * kStage;
  const uint32_t b_full = s_bars;          // [R]
  const uint32_t b_empty = s_bars + 64;    // [R]
  const uint32_t b_accf = s_bars + 128;    // [slot]
  const uint32_t b_kbar = s_bars + 144;    // [slot][2 column halves]
  const uint32_t b_stage = s_bars + 208;   // [slot]
  const uint32_t b_free = s_bars + 176;    // [slot] the slot's last layer has read its operand buffer
  const uint32_t b_drain = s_bars + 224;
  const uint32_t s_tmem = s_bars + 232;
  const uint32_t b_pfull = s_bars + 256;   // [R] pair mode: the odd CTA's half of the stage has landed
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(base_ptr + (s_tmem - base));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base_ptr + (s_tmem + 4 - base));
  TsLayer* layers = reinterpret_cast<TsLayer*>(base_ptr + (s_bars + kTsBarBytes - base));

  const int64_t ntiles = (batch + kTcM - 1) / kTcM;
  const int64_t units = PAIR ? (ntiles + 1) / 2 : ntiles;
  const int64_t unit = PAIR ? (int64_t)(blockIdx.x >> 1) : (int64_t)blockIdx.x;
  const int64_t nunits_grid = PAIR ? (int64_t)(gridDim.x >> 1) : (int64_t)gridDim.x;
  if (unit >= units) return;  // both CTAs of a pair leave together
  const TsJobs jobs(units, unit, nunits_grid, PAIR ? 2 : 1, (int)crank);

  // Where this CTA's epilogue signals the MMA issuer: its own barriers, or
  // in pair mode the even CTA's.
  const uint32_t kbar_sig = PAIR ? mapa_shared(b_kbar, 0) : b_kbar;
  const uint32_t stage_sig = PAIR ? mapa_shared(b_stage, 0) : b_stage;

  // ---- set-up ----
  if (warp == kTsMmaWarp) {
    if constexpr (PAIR) tmem_alloc_pair(s_tmem, 512);
    else tmem_alloc(s_tmem, 512);
  }
  if (tid == 0) {
    const uint32_t peers = PAIR ? 2u : 1u;
    for (int r = 0; r < R; ++r) {
      mbar_init(b_full + 8u * r, 1);
      mbar_init(b_empty + 8u * r, 1);
      mbar_init(b_pfull + 8u * r, 1);
    }
    for (int s = 0; s < kTsSlots; ++s) {
      mbar_init(b_accf + 8u * s, 1);
      for (int h = 0; h < 2; ++h) mbar_init(b_kbar + 8u * (2 * s + h), kTsEpiHalfWarps * peers);
      mbar_init(b_stage + 8u * s, in_tma ? 1u : (kTsEpiLoaders / 32) * peers);
      mbar_init(b_free + 8u * s, 1);
    }
    mbar_init(b_drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  for (int i = tid; i < p.n_layers; i += kTsThreads) layers[i] = p.layers[i];
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before any remote arrive
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nl = p.n_layers;

  if (warp == kTsProducerWarp) {
    // ------------------------------------------------ producer ----
    if (lane == 0) {
      uint32_t use = 0;
      bool ok = true;
      for (int64_t r = 0; r < jobs.rounds() && ok; ++r)
        for (int l = 0; l < nl && ok; ++l)
          for (int s = 0; s < kTsSlots && ok; ++s) {
            if (r >= jobs.count[s]) continue;
            const TsLayer& L = layers[l];
            // pair mode: this CTA's half of the chunk's n_pad rows
            const uint32_t bytes = (uint32_t)L.n_pad * (PAIR ? 64u : 128u);
            const uint64_t half = PAIR ? (uint64_t)crank * bytes : 0u;
            for (int kb = 0; kb < L.kblk; ++kb) {
              const uint32_t st = use % (uint32_t)R;
              if (use >= (uint32_t)R && !wait_phase(b_empty + 8u * st, ((use / R) - 1) & 1u, abort_flag)) {
                ok = false;
                break;
              }
              mbar_expect_tx(b_full + 8u * st, bytes);
              bulk_load(s_ring + st * kStage, image + L.w_off + (uint64_t)kb * kTsChunkBytes + half, bytes,
                        b_full + 8u * st);
              ++use;
            }
          }
      // Drain: the last copies issued must have landed before the CTA exits.
      const uint32_t n = use < (uint32_t)R ? use : (uint32_t)R;
      for (uint32_t u = use - n; u < use; ++u) {
        const long long t0 = clock64();
        while (!mbar_try_wait(b_full + 8u * (u % R), (u / R) & 1u))
          if (clock64() - t0 > kWaitCycles) break;
      }
      if (!ok) atomicExch(err, 2);
    }
    __syncwarp();
  } else if (warp == kTsLoaderWarp) {
    // -------------------------------------------------- loader ----
    // Input tiles through the input tensor map (single CTA, aligned input):
    // a slot's next tile as soon as its previous tile's last layer has read
    // the operand buffer, two boxes of 64 columns x k0 features per tile.
    if (in_tma && lane == 0) {
      const int k0 = layers[0].k_pad;
      const uint32_t bytes = 2u * 64u * (uint32_t)k0 * 2u;
      uint32_t fr_ph[kTsSlots] = {0, 0}, n_issued[kTsSlots] = {0, 0};
      bool ok = true;
      for (int64_t r = 0; r < jobs.rounds() && ok; ++r)
        for (int s = 0; s < kTsSlots && ok; ++s) {
          if (r >= jobs.count[s]) continue;
          if (r > 0) {
            if (!(ok = wait_phase(b_free + 8u * s, fr_ph[s], abort_flag))) break;
            fr_ph[s] ^= 1u;
          }
          const int32_t x = (int32_t)(jobs.tile(s, r) * kTcM);
          mbar_expect_tx(b_stage + 8u * s, bytes);
          for (int h = 0; h < 2; ++h)
            tma_load_2d(s_a[s] + (uint32_t)h * (uint32_t)k0 * 128u, &in_map, x + 64 * h, 0, b_stage + 8u * s);
          ++n_issued[s];
        }
      // Drain: a copy still in flight (after an abort) lands before the CTA
      // exits.  Load k of a slot completes phase k of its stage barrier, and
      // load k - 1 had landed before load k was issued (the MMAs of its tile
      // had run), so the parity of the last load identifies its phase.
      for (int s = 0; s < kTsSlots; ++s) {
        if (n_issued[s] == 0) continue;
        const long long t0 = clock64();
        while (!mbar_try_wait(b_stage + 8u * s, (n_issued[s] - 1) & 1u))
          if (clock64() - t0 > kWaitCycles) break;
      }
      if (!ok) atomicExch(err, 2);
    }
    __syncwarp();
  } else if (warp == kTsMmaWarp && PAIR && !leader) {
    // ----------------------------- relay (odd CTA of a pair) ----
    // Tell the even CTA, stage by stage and in job order, that this CTA's
    // half of the chunk has landed.
    if (lane == 0) {
      const uint32_t pfull_sig = mapa_shared(b_pfull, 0);
      uint32_t use = 0;
      bool ok = true;
      for (int64_t r = 0; r < jobs.rounds() && ok; ++r)
        for (int l = 0; l < nl && ok; ++l)
          for (int s = 0; s < kTsSlots && ok; ++s) {
            if (r >= jobs.count[s]) continue;
            for (int kb = 0; kb < layers[l].kblk; ++kb) {
              const uint32_t st = use % (uint32_t)R;
              if (!(ok = wait_phase(b_full + 8u * st, (use / R) & 1u, abort_flag))) break;
              mbar_arrive_cluster(pfull_sig + 8u * st);
              ++use;
            }
          }
      if (!ok) atomicExch(err, 3);
    }
    __syncwarp();
  } else if (warp == kTsMmaWarp) {
    // --------------------------------------------- MMA issuer ----
    // The whole warp runs the issue loop (warp-uniform values), one elected
    // lane issues each MMA and commit.
    {
      uint32_t use = 0, st_ph[kTsSlots] = {0, 0}, k_ph[kTsSlots] = {0, 0};
      bool has_prev[kTsSlots] = {false, false};
      bool ok = true;
      bool skip = PONNI_B200_SKIP_ARRIVE();  // wait-bound test build: drop the first job's signal
      long long w_epi = 0, w_full = 0;
      (void)w_epi; (void)w_full;
      TS_T(t_all);
      // Cluster-scope acquire where the odd CTA arrives (pair mode).
      auto wait_x = [&](uint32_t bar, uint32_t par) -> bool {
        const bool got = PAIR ? wait_phase_abort_cluster(bar, par, abort_flag, kWaitCycles)
                              : wait_phase(bar, par, abort_flag);
        return __all_sync(0xffffffffu, got);
      };
      const uint32_t hi_k = (uint32_t)(smem_desc(0, 16, 1024) >> 32);
      const uint32_t lo_k = (uint32_t)smem_desc(0, 16, 1024);
      // layer 0 (MN-major input stage): 64-column halves k0 * 128 B apart,
      // 8-feature groups 1024 B apart
      const uint32_t k0b = (uint32_t)layers[0].k_pad * 128u;
      const uint32_t hi_mn = (uint32_t)(smem_desc(0, k0b, 1024) >> 32);
      const uint32_t lo_mn = (uint32_t)smem_desc(0, k0b, 1024);
      const uint32_t ring_lo = lo_k | ((s_ring >> 4) & 0x3FFFu);
      // One job (layer l of slot s's tile); false when a wait gave up.
      auto mma_job = [&](int l, int s, const TsLayer& L) -> bool {
          {
            TS_T(tw);
            if (l == 0) {
              if (!(ok = wait_x(b_stage + 8u * s, st_ph[s]))) return false;
              st_ph[s] ^= 1u;
            }
            // The slot's previous epilogue has read its accumulator and
            // written the operand (both column halves, both CTAs).
            if (has_prev[s]) {
              for (int h = 0; h < 2 && ok; ++h) ok = wait_x(b_kbar + 8u * (2 * s + h), k_ph[s]);
              k_ph[s] ^= 1u;
            }
            if (!ok) return false;
            TS_ACC(w_epi, tw);
            has_prev[s] = true;
            tc_fence_after();
            const int nsteps = L.k_pad / 16;
            uint32_t idesc = idesc_of(p.dtype, L.n_pad, l == 0);
            if constexpr (PAIR) idesc = (idesc & ~(0x1Fu << 24)) | ((uint32_t)(2 * kTcM >> 4) << 24);  // M = 256
            const uint32_t d = tmem_base + (uint32_t)(s * kTsMaxN);
            const uint32_t a_lo = (l == 0 ? lo_mn : lo_k) | ((s_a[s] >> 4) & 0x3FFFu);
            const uint32_t a_hi = l == 0 ? hi_mn : hi_k;  // the weights (B) are always K-major
            for (int kb = 0; kb < L.kblk; ++kb) {
              const uint32_t st = use % (uint32_t)R;
              TS_T(t2);
              ok = __all_sync(0xffffffffu, wait_phase(b_full + 8u * st, (use / R) & 1u, abort_flag));
              if (PAIR && ok) ok = wait_x(b_pfull + 8u * st, (use / R) & 1u);
              if (!ok) break;
              TS_ACC(w_full, t2);
              tc_fence_after();
              const uint32_t b_lo = ring_lo + st * (kStage >> 4);
              const int s_end = min(nsteps, kb * 4 + 4);
              for (int k = kb * 4; k < s_end; ++k) {
                // start-address advance in 16-byte units: MN-major, 2 KB per K step of 16;
                // K-major, 16 KB per K block of 64 and 32 B per K step
                const uint32_t ao = l == 0 ? (uint32_t)k * 128u : (uint32_t)(k >> 2) * 1024u + (uint32_t)(k & 3) * 2u;
                const uint32_t bk = b_lo + (uint32_t)(k & 3) * 2u;
                if constexpr (PAIR) umma_f16_pair_warp(d, a_lo + ao, a_hi, bk, hi_k, idesc, k > 0 ? 1u : 0u);
                else umma_f16_desc_warp(d, a_lo + ao, a_hi, bk, hi_k, idesc, k > 0 ? 1u : 0u);
              }
              if constexpr (PAIR) umma_commit_pair_warp(b_empty + 8u * st);
              else umma_commit_warp(b_empty + 8u * st);
              ++use;
            }
            if (ok && !skip) {
              if constexpr (PAIR) umma_commit_pair_warp(b_accf + 8u * s);
              else umma_commit_warp(b_accf + 8u * s);
            }
            if (!PAIR && in_tma && ok && l == nl - 1) umma_commit_warp(b_free + 8u * s);  // stage the next tile
            skip = false;
          }
          return ok;
      };
      for (int64_t r = 0; r < jobs.rounds() && ok; ++r) {
        if constexpr (Shape::kStatic) {
#pragma unroll
          for (int l = 0; l < Shape::kNL; ++l) {
            TsLayer L = layers[l];
            Shape::fix(l, L);
            for (int s = 0; s < kTsSlots; ++s)
              if (ok && r < jobs.count[s]) ok = mma_job(l, s, L);
          }
        } else {
          for (int l = 0; l < nl && ok; ++l)
            for (int s = 0; s < kTsSlots && ok; ++s)
              if (r < jobs.count[s]) ok = mma_job(l, s, layers[l]);
        }
      }
      // Drain: every MMA issued has completed before TMEM is freed (both CTAs).
      if constexpr (PAIR) umma_commit_pair_warp(b_drain);
      else umma_commit_warp(b_drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(b_drain, 0))
        if (clock64() - t0 > kWaitCycles) break;
      if (lane == 0) {
        if (!ok) atomicExch(err, 3);
        TS_FLUSH(1, w_epi);
        TS_FLUSH(6, w_full);
#ifdef PONNI_B200_TC_PROFILE
        TS_FLUSH(7, clock64() - t_all);
#endif
      }
    }
    __syncwarp();
  } else {
    // ----------------------------------------------- epilogue ----
    // Every epilogue warp runs the jobs in the MMA issuer's order (both slots)
    // or, with per-slot groups, only its slot's jobs.
    const int q = warp & 3;
    const int cq = kTsEpiAll ? (warp >> 2) : ((warp >> 2) & 1);  // column quarter / half
    const int ch = kTsEpiAll ? (cq >> 1) : cq;                     // column half (signals)
    const int gs = kTsEpiAll ? -1 : warp / kTsGroupWarps;          // group's slot (per-slot groups)
    const int ltid = kTsEpiAll ? tid : (tid & (kTsGroupThreads - 1));
    const int m = q * 32 + lane;
    const bool vec = in_vec != 0;
    const int k0 = layers[0].k_pad;
    uint32_t acc_ph[kTsSlots] = {0, 0};
    bool ok = true;
    long long w_acc = 0, c_epi = 0, t_ph[3] = {0, 0, 0};
    (void)w_acc; (void)c_epi;
    // Operand written / accumulator read: local arrive, or in pair mode a
    // cluster-scope arrive on the even CTA's barrier.
    auto signal = [&](uint32_t bar) {
      if constexpr (PAIR) mbar_arrive_cluster(bar);
      else mbar_arrive(bar);
    };
    for (int s = 0; s < kTsSlots; ++s)
      if (!in_tma && (gs < 0 || gs == s) && jobs.count[s] > 0) {
        ts_load_tile<T>(s_a[s], base_ptr + (s_a[s] - base), in, in_ld, p.nin, k0, jobs.tile(s, 0), batch, vec, ltid);
        cp_async_wait_0();
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) signal(stage_sig + 8u * s);
      }
    // One job (tile round r, layer l, slot s) of this warp; false when a wait gave up.
    auto job = [&](int64_t r, int l, int s, bool last) -> bool {
      {
          const TsLayer& L = layers[l];
          const int64_t t = jobs.tile(s, r);
          // One lane waits, the warp follows (the TMEM loads are warp-collective).
          TS_T(t0);
          int got = 0;
          if (lane == 0) got = wait_phase(b_accf + 8u * s, acc_ph[s], abort_flag) ? 1 : 0;
          got = __shfl_sync(0xffffffffu, got, 0);
          if (got == 0) return false;
          acc_ph[s] ^= 1u;
          TS_ACC(w_acc, t0);
          TS_T(t1);
          tc_fence_after();
          const bool refill = !in_tma && last && r + 1 < jobs.count[s];
          if (refill && !(PONNI_B200_TS_DIAG & 1))  // (diagnostic builds: bit 1 skips the input loads)
            // the slot's MMAs are done with its operand buffer: stage the next tile
            ts_load_tile<T>(s_a[s], base_ptr + (s_a[s] - base), in, in_ld, p.nin, k0, jobs.tile(s, r + 1), batch,
                            vec, ltid);
          const uint32_t tmem_row = tmem_base + (uint32_t)(s * kTsMaxN) + ((uint32_t)(q * 32) << 16);
#ifndef PONNI_B200_TS_NO_EPI  // diagnostic build: handoffs only, no epilogue work
          Shape::template epilogue<T>(l, L, p.fast_act, last, tmem_row, cq * kTsEpiCols,
                                      reinterpret_cast<const float*>(image + L.bias_off), s_a[s], out, out_ld,
                                      t * kTcM + m, batch, m, t_ph);
#else
          (void)tmem_row;
#endif
          fence_proxy_async();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) signal(kbar_sig + 8u * (2 * s + ch));
          if (refill) {
            cp_async_wait_0();
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) signal(stage_sig + 8u * s);
          }
          TS_ACC(c_epi, t1);
      }
      return true;
    };
    for (int64_t r = 0; r < jobs.rounds() && ok; ++r) {
      if constexpr (Shape::kStatic) {
#pragma unroll
        for (int l = 0; l < Shape::kNL; ++l)
          for (int s = 0; s < kTsSlots; ++s)
            if (ok && r < jobs.count[s] && (gs < 0 || gs == s)) ok = job(r, l, s, l == Shape::kNL - 1);
      } else {
        for (int l = 0; l < nl && ok; ++l)
          for (int s = 0; s < kTsSlots && ok; ++s)
            if (r < jobs.count[s] && (gs < 0 || gs == s)) ok = job(r, l, s, l == nl - 1);
      }
    }
    cp_async_wait_0();
    if (!ok && lane == 0) atomicExch(err, 4);
    if (tid == 0) {
      TS_FLUSH(3, t_ph[0]);
      TS_FLUSH(2, t_ph[1]);
      TS_FLUSH(4, w_acc);
      TS_FLUSH(5, c_epi);
    }
  }

  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // the even CTA's MMAs (which read this CTA's memory) are complete
  else __syncthreads();
  if (warp == kTsMmaWarp) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, 512);
    else tmem_dealloc(tmem_base, 512);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).

}  // namespace tsk
}  // namespace ponni_b200
