// Tensor-core dense-chain kernel with streamed weights (sm_100a, tcgen05).
//
// For 16-bit Matvec[Bias][activation] chains whose weights do not fit in
// shared memory next to the operand tiles (e.g. 64->256x5->32 bf16: 573 KB).
// One persistent CTA per SM, warp-specialised:
//   producer (warp 16, one thread): streams the pre-swizzled weight chunks of
//     every job, in job order, from global memory (L2-resident: every CTA
//     reads the same image) into a ring of shared-memory stages with 1-D bulk
//     copies (cp.async.bulk, completion counted in bytes on the stage's
//     "full" mbarrier; no multicast);
//   MMA issuer (warp 17, one thread): per job (layer l, column block nb of
//     128) issues D[128 x N] += A[128 x K] * B[N x K]^T chunk by chunk
//     (tcgen05.mma kind::f16, fp32 accumulator in TMEM columns nb*128...),
//     frees each ring stage with tcgen05.commit and signals the finished job
//     on the block's "acc full" mbarrier;
//   epilogue (warps 0-15: 4 TMEM lane quarters x 4 column quarters): per job,
//     tcgen05.ld of the accumulator, bias, activation (reference fused
//     epilogue, src/ponni_Inference.h:416-444), and the next layer's K-major
//     operand (ping-pong buffers A0/A1) or the caller's output; then signals
//     "epi done" for the block.  They also stage each tile's input (cp.async
//     into the MN-major layer-0 operand) as soon as layer 0 has consumed the
//     previous one.
// A job's epilogue overlaps the MMAs of the next column block; a layer's
// MMAs start when every block of the previous layer has been written.
//
// In this fp32-accumulation mode SiLU and sigmoid use the hardware base-2
// exponential and reciprocal approximations (two full-rate MUFU operations
// per value) and tanh the hardware tanh approximation; their errors are far
// below one unit of the 16-bit model type.
//
// Every wait is bounded; a role that gives up raises a shared abort flag
// (the others see it and leave), records an error code, and the CTA drains
// its bulk copies and MMAs before it frees TMEM and returns.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "device_math.cuh"
#include "tc_common.cuh"
#include "tc_stream.h"

namespace ponni_b200 {
namespace {
using namespace tc;

constexpr long long kWaitCycles = 1ll << 31;

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

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory, completion on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Bounded wait that also leaves when another role has aborted.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
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

// sigmoid(x) = 1 / (1 + 2^(-x log2 e)) with the hardware base-2 exponential
// and reciprocal approximations (relative error near 2^-22 each): two
// full-rate MUFU operations per value.
__device__ __forceinline__ float sigmoid_fast(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(e) : "f"(x * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;\n" : "=f"(r) : "f"(1.0f + e));
  return r;
}

// Activation of 32 values; in the fast mode SiLU and sigmoid use
// sigmoid_fast, tanh the fp32 tanh approximation.
template <int ACT>
__device__ __forceinline__ void ts_act32(float (&v)[32], int fast, int flags, float s0, float s1) {
  if constexpr (ACT == EPI_SILU || ACT == EPI_SIGMOID) {
    if (fast) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float g = sigmoid_fast(v[j]);
        v[j] = ACT == EPI_SILU ? v[j] * g : g;
      }
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = ts_act<ACT>(v[j], fast, flags, s0, s1);
}

struct TsShared {
  uint32_t a[2], stage, ring, full, empty, accf, epi_done, stage_full, drain;
};

// Epilogue of the columns [c_begin, c_begin + kTsColsPerWarp) of job
// (l, nb) for this thread's row m.
template <class T, int ACT>
__device__ __forceinline__ void ts_epilogue(const TsLayer& L, int fast, bool last, uint32_t tmem_row, int c_begin,
                                            const float* __restrict__ bias, uint32_t a_out, T* __restrict__ out,
                                            int64_t out_ld, int64_t col, int64_t batch, int m, long long (&t_ph)[3]) {
  (void)t_ph;
  using Op = typename OperandOf<T>::type;
  const int n_pad = L.n_pad, nout = L.nout, has_bias = L.has_bias, flags = L.act_flags;
  const float s0 = L.s0, s1 = L.s1;
#pragma unroll 1
  for (int c0 = c_begin; c0 < c_begin + kTsColsPerWarp && c0 < n_pad; c0 += 32) {
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
        v[4 * q] += b.x;
        v[4 * q + 1] += b.y;
        v[4 * q + 2] += b.z;
        v[4 * q + 3] += b.w;
      }
    }
    if (last) {
      ts_act32<ACT>(v, fast, flags, s0, s1);
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
      ts_act32<ACT>(v, fast, flags, s0, s1);
#ifdef PONNI_B200_TC_PROFILE
      // make the timing see the activation results before the stores
      float sink = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) sink += v[j];
      if (sink == 12345.678f) v[0] += 1e-30f;
#endif
      TS_ACC(t_ph[1], ta);
      TS_T(ts);
      const uint32_t a[1] = {a_out};
#pragma unroll
      for (int q = 0; q < 4; ++q) store_row8<T>(a, m, c0 + 8 * q, v + 8 * q);
      TS_ACC(t_ph[2], ts);
    }
  }
  (void)sizeof(Op);
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

template <class T>
__global__ void __launch_bounds__(kTsThreads, 1)
    ts_forward_kernel(const __grid_constant__ TsProgram p, const unsigned char* __restrict__ image,
                      const T* __restrict__ in, int64_t in_ld, T* __restrict__ out, int64_t out_ld, int64_t batch,
                      int in_vec, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* base_ptr = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int R = (int)p.ring_stages;

  TsShared S;
  S.a[0] = base;
  S.a[1] = base + p.a_bytes;
  S.stage = base + 2 * p.a_bytes;
  S.ring = S.stage + p.stage_bytes;
  const uint32_t s_bars = S.ring + (uint32_t)R * kTsChunkBytes;
  S.full = s_bars;                 // [R]
  S.empty = s_bars + 64;           // [R]
  S.accf = s_bars + 128;           // [2]
  S.epi_done = s_bars + 144;       // [2]
  S.stage_full = s_bars + 160;
  S.drain = s_bars + 168;
  const uint32_t s_tmem = s_bars + 176;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(base_ptr + (s_tmem - base));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base_ptr + (s_tmem + 4 - base));
  TsLayer* layers = reinterpret_cast<TsLayer*>(base_ptr + (s_bars + 256 - base));

  const int64_t ntiles = (batch + kTcM - 1) / kTcM;
  if ((int64_t)blockIdx.x >= ntiles) return;

  // ---- set-up ----
  if (warp == kTsMmaWarp) tmem_alloc(s_tmem, 256);
  if (tid == 0) {
    for (int r = 0; r < R; ++r) {
      mbar_init(S.full + 8u * r, 1);
      mbar_init(S.empty + 8u * r, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(S.accf + 8u * b, 1);
      mbar_init(S.epi_done + 8u * b, kTsEpiWarps);
    }
    mbar_init(S.stage_full, kTsEpiWarps);
    mbar_init(S.drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  for (int i = tid; i < p.n_layers; i += kTsThreads) layers[i] = p.layers[i];
  {
    uint4* z = reinterpret_cast<uint4*>(base_ptr + (S.stage - base));
    for (int i = tid; i < (int)(p.stage_bytes / 16); i += kTsThreads) z[i] = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nl = p.n_layers;
  const int64_t stride = gridDim.x;

  if (warp == kTsProducerWarp) {
    // ------------------------------------------------ producer ----
    if (lane == 0) {
      uint32_t use = 0;
      bool ok = true;
      long long w_empty = 0;
      (void)w_empty;
      for (int64_t t = blockIdx.x; t < ntiles && ok; t += stride) {
        for (int l = 0; l < nl && ok; ++l) {
          const TsLayer& L = layers[l];
          for (int nb = 0; nb < L.nblk && ok; ++nb) {
            const uint32_t bytes = (uint32_t)min(kTsBlockN, L.n_pad - nb * kTsBlockN) * 128u;
            for (int kb = 0; kb < L.kblk; ++kb) {
              const uint32_t r = use % (uint32_t)R;
              TS_T(t0);
              if (use >= (uint32_t)R && !wait_phase(S.empty + 8u * r, ((use / R) - 1) & 1u, abort_flag)) {
                ok = false;
                break;
              }
              TS_ACC(w_empty, t0);
              mbar_expect_tx(S.full + 8u * r, bytes);
              bulk_load(S.ring + r * kTsChunkBytes,
                        image + L.w_off + ((uint64_t)nb * L.kblk + kb) * kTsChunkBytes, bytes, S.full + 8u * r);
              ++use;
            }
          }
        }
      }
      // Drain: the last copies issued must have landed before the CTA exits.
      const uint32_t n = use < (uint32_t)R ? use : (uint32_t)R;
      for (uint32_t u = use - n; u < use; ++u) {
        const long long t0 = clock64();
        while (!mbar_try_wait(S.full + 8u * (u % R), (u / R) & 1u))
          if (clock64() - t0 > kWaitCycles) break;
      }
      if (!ok) atomicExch(err, 2);
    }
    __syncwarp();
  } else if (warp == kTsMmaWarp) {
    // --------------------------------------------- MMA issuer ----
    if (lane == 0) {
      uint32_t use = 0, st_ph = 0, epi_ph[2] = {0, 0};
      int prev_nblk = 0;
      bool ok = true;
      long long w_stage = 0, w_epi = 0, w_full = 0;
      (void)w_stage; (void)w_epi; (void)w_full;
      TS_T(t_all);
      const uint64_t a_stage = smem_desc(S.stage, 1024, 2048);
      for (int64_t t = blockIdx.x; t < ntiles && ok; t += stride) {
        for (int l = 0; l < nl && ok; ++l) {
          const TsLayer& L = layers[l];
          if (l == 0) {
            TS_T(t0);
            if (!(ok = wait_phase(S.stage_full, st_ph, abort_flag))) break;
            TS_ACC(w_stage, t0);
            st_ph ^= 1u;
          }
          // Dependencies on the previous job layer (l - 1, or the last layer
          // of the previous tile), per chunk: the accumulator block nb must
          // have been read out, and for l >= 1 the operand K block kb must
          // have been written (by the epilogue of block kb*64/128).  So a
          // layer's first chunks start while the previous layer's last block
          // is still in its epilogue.
          bool waited[2] = {false, false};
          auto need = [&](int b) {
            if (ok && b < prev_nblk && !waited[b]) {
              TS_T(tw);
              ok = wait_phase(S.epi_done + 8u * b, epi_ph[b], abort_flag);
              TS_ACC(w_epi, tw);
              epi_ph[b] ^= 1u;
              waited[b] = true;
              tc_fence_after();
            }
          };
          const int nsteps = L.k_pad / 16;
          const uint64_t a_in = smem_desc(S.a[(l + 1) & 1], 16, 1024);  // written by the epilogue of layer l-1
          for (int nb = 0; nb < L.nblk && ok; ++nb) {
            const int rows = min(kTsBlockN, L.n_pad - nb * kTsBlockN);
            const uint32_t idesc = idesc_of(p.dtype, rows, l == 0);
            const uint32_t d = tmem_base + (uint32_t)(nb * kTsBlockN);
            need(nb);
            for (int kb = 0; kb < L.kblk && ok; ++kb) {
              if (l > 0) need(kb * kTsBlockK / kTsBlockN);
              if (!ok) break;
              const uint32_t r = use % (uint32_t)R;
              TS_T(t2);
              if (!(ok = wait_phase(S.full + 8u * r, (use / R) & 1u, abort_flag))) break;
              TS_ACC(w_full, t2);
              tc_fence_after();
              const uint64_t b0 = smem_desc(S.ring + r * kTsChunkBytes, 16, 1024);
              const int s_end = min(nsteps, kb * 4 + 4);
              for (int s = kb * 4; s < s_end; ++s) {
                const uint64_t a = l == 0 ? a_stage + (uint64_t)s * 256
                                          : a_in + (uint64_t)(s >> 2) * 1024 + (uint64_t)(s & 3) * 2;
                umma_f16(d, a, b0 + (uint64_t)(s & 3) * 2, idesc, s > 0 ? 1u : 0u);
              }
              umma_commit(S.empty + 8u * r);
              ++use;
            }
            if (ok) umma_commit(S.accf + 8u * nb);
          }
          // Consume the remaining completions of the previous layer's blocks
          // (keeps every barrier's phase accounting one-to-one).
          for (int b = 0; b < prev_nblk; ++b) need(b);
          prev_nblk = L.nblk;
        }
      }
      // Drain: every MMA issued has completed before TMEM is freed.
      umma_commit(S.drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(S.drain, 0))
        if (clock64() - t0 > kWaitCycles) break;
      if (!ok) atomicExch(err, 3);
      TS_FLUSH(1, w_epi);
      TS_FLUSH(6, w_full);
#ifdef PONNI_B200_TC_PROFILE
      TS_FLUSH(7, clock64() - t_all);
#endif
    }
    __syncwarp();
  } else {
    // ----------------------------------------------- epilogue ----
    const int q = warp & 3, ch = warp >> 2;
    const int m = q * 32 + lane;
    const uint32_t tmem_row = tmem_base + ((uint32_t)(q * 32) << 16);
    const bool vec = in_vec != 0;
    uint32_t acc_ph[2] = {0, 0};
    bool ok = true;
    long long w_acc = 0, c_epi = 0, c_sig = 0, t_ph[3] = {0, 0, 0};
    (void)w_acc; (void)c_epi; (void)c_sig;
    int64_t t = blockIdx.x;
    load_input<T, kTsEpiWarps * 32>(S.stage, in, in_ld, p.nin, t * kTcM, batch, vec, tid);
    cp_async_commit();
    cp_async_wait_0();
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive(S.stage_full);
    for (; t < ntiles && ok; t += stride) {
      const int64_t next = t + stride;
      const int64_t col = t * kTcM + m;
      for (int l = 0; l < nl && ok; ++l) {
        const TsLayer& L = layers[l];
        const bool last = l == nl - 1;
        const float* bias = reinterpret_cast<const float*>(image + L.bias_off);
        const uint32_t a_out = S.a[l & 1];
        for (int nb = 0; nb < L.nblk; ++nb) {
          // One lane waits, the warp follows (the TMEM loads are warp-collective).
          int got = 0;
          TS_T(t0);
          if (lane == 0) got = wait_phase(S.accf + 8u * nb, acc_ph[nb], abort_flag) ? 1 : 0;
          got = __shfl_sync(0xffffffffu, got, 0);
          if (!(ok = got != 0)) break;
          TS_ACC(w_acc, t0);
          TS_T(t1);
          acc_ph[nb] ^= 1u;
          tc_fence_after();
          if (l == 0 && nb == L.nblk - 1 && next < ntiles) {
            // layer 0 has consumed the stage: fetch the next tile's input
            load_input<T, kTsEpiWarps * 32>(S.stage, in, in_ld, p.nin, next * kTcM, batch, vec, tid);
            cp_async_commit();
          }
          ts_epilogue_dispatch<T>(L, p.fast_act, last, tmem_row, nb * kTsBlockN + ch * kTsColsPerWarp, bias, a_out, out, out_ld,
                                  col, batch, m, t_ph);
          TS_T(t2);
          fence_proxy_async();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(S.epi_done + 8u * nb);
          TS_ACC(c_sig, t2);
          TS_ACC(c_epi, t1);
        }
      }
      if (ok && next < ntiles) {
        cp_async_wait_0();
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(S.stage_full);
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
  __syncthreads();
  if (warp == kTsMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

template <class T>
cudaError_t launch_impl(const TsProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                        int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  auto kern = ts_forward_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
  if (e != cudaSuccess) return e;
  const bool vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && ((in_ld * (int64_t)sizeof(T)) % 16 == 0);
  kern<<<grid, kTsThreads, p.smem_bytes, stream>>>(p, static_cast<const unsigned char*>(image),
                                                   static_cast<const T*>(in), in_ld, static_cast<T*>(out), out_ld,
                                                   batch, vec ? 1 : 0, err);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_ts_forward(const TsProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                              int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  switch (p.dtype) {
    case 2: return launch_impl<__half>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
    case 3: return launch_impl<__nv_bfloat16>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ponni_b200
