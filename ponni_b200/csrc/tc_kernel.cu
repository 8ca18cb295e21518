// Tensor-core dense-chain kernel for sm_100a (tcgen05 UMMA + TMEM).
//
// One persistent CTA per SM, 4 warps.  Per batch tile of 128 columns:
//   input  : cp.async (16 B, zero-filled tail) of the batch-contiguous input
//            rows straight into an MN-major SW128 tile (prefetched one tile
//            ahead into a second staging buffer); 16-bit models use it as the
//            layer-0 operand directly, fp32 models split it into tf32 hi/lo
//            K-major operands (the tf32 MMA reads K-major operands here);
//   layer l: thread 0 issues the UMMA chain D[128 x N] = A[128 x K] B[N x K]^T
//            (tcgen05.mma, fp32 accumulator in TMEM) and commits it to an
//            mbarrier; all threads wait (bounded), then each warp reads its 32
//            TMEM lanes (= 32 batch columns) with tcgen05.ld, applies bias and
//            activation in fp32 (the reference's fused epilogue,
//            src/ponni_Inference.h:416-444) and writes the next layer's
//            K-major operand to shared memory, or the caller's output for the
//            last layer (coalesced: a warp writes 32 consecutive columns).
// Weights and biases are staged once per CTA (the packed image built on the
// host is byte-for-byte the swizzled operand layout).
//
// Arithmetic:
//   fp32 models: 3xTF32 -- every operand x is split into hi = tf32(x) and
//     lo = tf32(x - hi) and D accumulates lo*HI + hi*LO + hi*HI (the
//     error-compensated TF32 scheme; the dropped lo*lo term is below 2^-22
//     relative), giving fp32-level accuracy on the TF32 tensor pipe;
//   fp16/bf16 models: operands in the model type, fp32 accumulation, states
//     rounded to the model type where the reference stores them.
//
// Every wait is bounded: on timeout the kernel records an error code in
// `err`, stops issuing work, frees its TMEM and returns.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "device_math.cuh"
#include "tc_kernel.h"

namespace ponni_b200 {
namespace {

// ---------------------------------------------------------------- PTX ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase; false when the limit is reached.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (it > 32) __nanosleep(64);
  }
  return false;
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

// UMMA, A and B from shared memory descriptors, D in TMEM.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return r;
}

// Shared-memory matrix descriptor, SW128, sm_100 version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// ------------------------------------------------------------ helpers ----
template <class T> struct Store;
template <> struct Store<float> {
  static __device__ __forceinline__ float from(float v) { return v; }
};
template <> struct Store<__half> {
  static __device__ __forceinline__ __half from(float v) { return __float2half_rn(v); }
};
template <> struct Store<__nv_bfloat16> {
  static __device__ __forceinline__ __nv_bfloat16 from(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of element (row m, column f) of a K-major SW128 operand with
// 128 rows, for a 16-byte-chunk aligned column group.
__device__ __forceinline__ uint32_t kmajor_chunk(int m, uint32_t byte_in_row_total) {
  const uint32_t kb = byte_in_row_total >> 7;  // 128-byte K block
  const uint32_t chunk = (byte_in_row_total >> 4) & 7;
  return kb * (kTcM * 128) + (uint32_t)m * 128 + ((chunk ^ ((uint32_t)m & 7)) << 4);
}

// Stage input columns [col0, col0+128) into the MN-major SW128 layout.
template <class T>
__device__ __forceinline__ void load_input(uint32_t stage, const T* __restrict__ in, int64_t in_ld, int nin,
                                           int64_t col0, int64_t batch, bool vec) {
  constexpr int esz = sizeof(T);
  constexpr int chunks_per_row = kTcM * esz / 16;  // 32 (fp32) or 16 (16-bit)
  constexpr uint32_t sbo = esz * 1024;
  if (vec) {
    for (int i = threadIdx.x; i < nin * chunks_per_row; i += kTcThreads) {
      const int f = i / chunks_per_row, j = i - f * chunks_per_row;
      const int64_t col = col0 + (int64_t)j * (16 / esz);
      const int64_t valid = batch - col;
      const int bytes = valid >= 16 / esz ? 16 : (valid > 0 ? (int)valid * esz : 0);
      const T* src = in + (int64_t)f * in_ld + (bytes > 0 ? col : 0);
      const uint32_t dst = stage + (uint32_t)(f >> 3) * sbo + (uint32_t)(j >> 3) * 1024 + (uint32_t)(f & 7) * 128 +
                           ((((uint32_t)j & 7) ^ ((uint32_t)f & 7)) << 4);
      cp_async16(dst, src, bytes);
    }
  } else {
    for (int i = threadIdx.x; i < nin * kTcM; i += kTcThreads) {
      const int f = i / kTcM, m = i - f * kTcM;
      const int64_t col = col0 + m;
      T v = col < batch ? in[(int64_t)f * in_ld + col] : Store<T>::from(0.0f);
      const uint32_t byte = (uint32_t)m * esz;
      const uint32_t j = byte >> 4;
      const uint32_t dst = stage + (uint32_t)(f >> 3) * sbo + (j >> 3) * 1024 + (uint32_t)(f & 7) * 128 +
                           (((j & 7) ^ ((uint32_t)f & 7)) << 4) + (byte & 15);
      if constexpr (esz == 4) {
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(dst), "r"(__float_as_uint(*reinterpret_cast<float*>(&v)))
                     : "memory");
      } else {
        asm volatile("st.shared.b16 [%0], %1;\n" ::"r"(dst), "h"(*reinterpret_cast<unsigned short*>(&v))
                     : "memory");
      }
    }
  }
}

template <int ACT>
__device__ __forceinline__ float epi_act(float v, const TcLayer& L) {
  if constexpr (ACT == EPI_NONE) return v;
  else return activation<float>(ACT, L.act_flags, v, L.s0, L.s1);
}

// Epilogue of one layer for this thread's TMEM lane (= batch column m).
template <class T, int ACT>
__device__ __forceinline__ void epilogue(const TcLayer& L, bool last, uint32_t tmem_lane, const float* bias,
                                         uint32_t a_hi, uint32_t a_lo, T* __restrict__ out, int64_t out_ld,
                                         int64_t col, int64_t batch, int m) {
  constexpr bool TF32 = sizeof(T) == 4;
  for (int c0 = 0; c0 < L.n_pad; c0 += 32) {
    float v[32];
    tmem_ld32(tmem_lane + (uint32_t)c0, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int f = c0 + j;
      float x = v[j];
      if (L.has_bias) x += bias[f];  // bias is zero-padded to the 32-column boundary
      x = epi_act<ACT>(x, L);
      v[j] = f < L.nout ? x : 0.0f;
    }
    if (last) {
      if (col < batch) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < L.nout) out[(int64_t)(c0 + j) * out_ld + col] = Store<T>::from(v[j]);
      }
    } else if constexpr (TF32) {
      // 32 fp32 columns = one 128-byte K block row: 8 chunks of 4.
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[e] = to_tf32(v[4 * q + e]);
          l[e] = to_tf32(v[4 * q + e] - __uint_as_float(h[e]));
        }
        const uint32_t off = kmajor_chunk(m, (uint32_t)(c0 + 4 * q) * 4);
        st_shared_v4(a_hi + off, h[0], h[1], h[2], h[3]);
        st_shared_v4(a_lo + off, l[0], l[1], l[2], l[3]);
      }
    } else {
      // 32 16-bit columns = 64 bytes: 4 chunks of 8.
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t off = kmajor_chunk(m, (uint32_t)(c0 + 8 * q) * 2);
        st_shared_v4(a_hi + off, pack2(v[8 * q], v[8 * q + 1], (T*)nullptr),
                     pack2(v[8 * q + 2], v[8 * q + 3], (T*)nullptr), pack2(v[8 * q + 4], v[8 * q + 5], (T*)nullptr),
                     pack2(v[8 * q + 6], v[8 * q + 7], (T*)nullptr));
      }
    }
  }
}

template <class T>
__device__ __forceinline__ void epilogue_dispatch(const TcLayer& L, bool last, uint32_t tmem_lane, const float* bias,
                                                  uint32_t a_hi, uint32_t a_lo, T* __restrict__ out, int64_t out_ld,
                                                  int64_t col, int64_t batch, int m) {
#define PONNI_TC_EPI(A) epilogue<T, A>(L, last, tmem_lane, bias, a_hi, a_lo, out, out_ld, col, batch, m)
  switch (L.act) {
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

// --------------------------------------------------------------- kernel --
template <class T>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_forward_kernel(const __grid_constant__ TcProgram p, const unsigned char* __restrict__ image,
                      const T* __restrict__ in, int64_t in_ld, T* __restrict__ out, int64_t out_ld, int64_t batch,
                      int in_vec, int* __restrict__ err) {
  constexpr bool TF32 = sizeof(T) == 4;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // Swizzled operands need 1024-byte aligned atoms.
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* base_ptr = smem_raw + (base - raw);
  const uint32_t s_image = base;
  const uint32_t s_ahi = s_image + p.image_bytes;
  const uint32_t s_alo = s_ahi + p.a_bytes;
  const uint32_t s_stage0 = s_alo + (TF32 ? p.a_bytes : 0u);
  const uint32_t s_stage1 = s_stage0 + p.stage_bytes;
  const uint32_t s_bar = s_stage1 + p.stage_bytes;
  const uint32_t s_tmem = s_bar + 8;
  const float* bias_base = reinterpret_cast<const float*>(base_ptr);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(base_ptr + (s_tmem - base));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t ntiles = (batch + kTcM - 1) / kTcM;
  int64_t tile = blockIdx.x;
  if (tile >= ntiles) return;

  // ---- set-up: TMEM, mbarrier, zeroed staging, parameter image ----
  if (warp == 0) tmem_alloc(s_tmem, p.tmem_cols);
  if (tid == 0) {
    mbar_init(s_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  {
    uint4* z = reinterpret_cast<uint4*>(base_ptr + (s_stage0 - base));
    const int n16 = (int)(2 * p.stage_bytes / 16);
    for (int i = tid; i < n16; i += kTcThreads) z[i] = make_uint4(0, 0, 0, 0);
  }
  for (uint32_t i = tid; i < p.image_bytes / 16; i += kTcThreads) cp_async16(s_image + i * 16, image + i * 16, 16);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_lane = tmem_base + ((uint32_t)(warp * 32) << 16);
  const int m = warp * 32 + lane;  // this thread's batch row in the tile

  load_input<T>(s_stage0, in, in_ld, p.nin, tile * kTcM, batch, in_vec != 0);
  cp_async_commit();
  uint32_t phase = 0;
  int cur = 0;
  bool failed = false;
  const int kstep = 32 / p.esz;  // UMMA K elements per instruction (32 bytes)

  for (; tile < ntiles && !failed; tile += gridDim.x) {
    const int64_t col0 = tile * kTcM;
    const int64_t next = tile + gridDim.x;
    const uint32_t stage = cur ? s_stage1 : s_stage0;
    if (next < ntiles) load_input<T>(cur ? s_stage0 : s_stage1, in, in_ld, p.nin, next * kTcM, batch, in_vec != 0);
    cp_async_commit();
    cp_async_wait_1();
    __syncthreads();
    if constexpr (TF32) {
      // Split the fp32 input tile into tf32 hi/lo operands and transpose it
      // to K-major (the MN-major operand form is used for 16-bit inputs
      // only): thread m builds row m from column m of the staged tile.
      const int k0 = p.layers[0].k_pad;
      const unsigned char* st = base_ptr + (stage - base);
      const uint32_t mo = (uint32_t)(tid >> 5) * 1024 + (uint32_t)(tid & 3) * 4;
      const uint32_t mc = (uint32_t)(tid & 31) >> 2;
      for (int f = 0; f < k0; f += 4) {
        uint32_t h[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t fe = (uint32_t)(f + e);
          const float x = *reinterpret_cast<const float*>(st + (fe >> 3) * 4096 + mo + (fe & 7) * 128 +
                                                          ((mc ^ (fe & 7)) << 4));
          h[e] = to_tf32(x);
          lo[e] = to_tf32(x - __uint_as_float(h[e]));
        }
        const uint32_t off = kmajor_chunk(tid, (uint32_t)f * 4);
        st_shared_v4(s_ahi + off, h[0], h[1], h[2], h[3]);
        st_shared_v4(s_alo + off, lo[0], lo[1], lo[2], lo[3]);
      }
    }
    for (int l = 0; l < p.n_layers; ++l) {
      const TcLayer& L = p.layers[l];
      fence_proxy_async();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        const int nsteps = L.k_pad / kstep;
        const uint32_t w_hi = s_image + L.w_hi_off, w_lo = s_image + L.w_lo_off;
        const uint32_t b_block = (uint32_t)L.n_pad * 128;
        for (int s = 0; s < nsteps; ++s) {
          const uint32_t kb = (uint32_t)s >> 2, ks = (uint32_t)s & 3;
          const uint32_t b_off = kb * b_block + ks * 32;
          uint64_t ad_hi, ad_lo;
          uint32_t idesc;
          if (!TF32 && l == 0) {
            // 16-bit layer 0 reads the staged input tile as an MN-major
            // operand: one K step = 32 bytes of K for 128 rows = 4096 bytes.
            ad_hi = smem_desc(stage + (uint32_t)s * 4096, 1024, (uint32_t)p.esz * 1024);
            ad_lo = ad_hi;
            idesc = L.idesc_mn;
          } else {
            const uint32_t a_off = kb * (kTcM * 128) + ks * 32;
            ad_hi = smem_desc(s_ahi + a_off, 16, 1024);
            ad_lo = smem_desc(s_alo + a_off, 16, 1024);
            idesc = L.idesc;
          }
          const uint64_t bd_hi = smem_desc(w_hi + b_off, 16, 1024);
          if constexpr (TF32) {
            const uint64_t bd_lo = smem_desc(w_lo + b_off, 16, 1024);
            umma_tf32(tmem_base, ad_lo, bd_hi, idesc, s > 0 ? 1u : 0u);
            umma_tf32(tmem_base, ad_hi, bd_lo, idesc, 1u);
            umma_tf32(tmem_base, ad_hi, bd_hi, idesc, 1u);
          } else {
            umma_f16(tmem_base, ad_hi, bd_hi, idesc, s > 0 ? 1u : 0u);
          }
        }
        umma_commit(s_bar);
      }
      const bool ok = mbar_wait_bounded(s_bar, phase);
      phase ^= 1u;
      tc_fence_after();
      if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicExch(err, 1);
        failed = true;
        break;
      }
      const bool last = l == p.n_layers - 1;
      const float* bias = reinterpret_cast<const float*>(reinterpret_cast<const unsigned char*>(bias_base) + L.bias_off);
      epilogue_dispatch<T>(L, last, tmem_lane, bias, s_ahi, s_alo, out, out_ld, col0 + m, batch, m);
    }
    cur ^= 1;
  }
  cp_async_wait_0();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

template <class T>
cudaError_t launch_impl(const TcProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                        int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  auto kern = tc_forward_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
  if (e != cudaSuccess) return e;
  const bool vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && ((in_ld * (int64_t)sizeof(T)) % 16 == 0);
  kern<<<grid, kTcThreads, p.smem_bytes, stream>>>(p, static_cast<const unsigned char*>(image),
                                                    static_cast<const T*>(in), in_ld, static_cast<T*>(out), out_ld,
                                                    batch, vec ? 1 : 0, err);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_tc_forward(const TcProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                              int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  switch (p.dtype) {
    case 0: return launch_impl<float>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
    case 2: return launch_impl<__half>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
    case 3: return launch_impl<__nv_bfloat16>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ponni_b200
