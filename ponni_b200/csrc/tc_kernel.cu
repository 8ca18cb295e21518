// Tensor-core dense-chain kernel for sm_100a (tcgen05 UMMA + TMEM).
//
// One persistent CTA per SM with up to four thread groups, each owning one
// tile slot, so that the slots' epilogues overlap the others' MMAs.  Per batch tile of 128
// columns:
//   input  : cp.async (16 B, zero-filled tail) of the batch-contiguous input
//            rows into a staging tile, prefetched one tile ahead into a
//            second buffer; 16-bit models stage it as an MN-major SW128
//            operand and use it for layer 0 directly, fp32 models stage it
//            row-major and split it into K-major bf16 operand parts;
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
//   fp32 models: every operand x is split exactly into three bfloat16 parts
//     x = b0 + b1 + b2 (b0 = bf16(x), b1 = bf16(x - b0), b2 = x - b0 - b1;
//     8 + 8 + 8 significand bits cover fp32's 24) and D accumulates the six
//     products whose parts sum to order <= 2 (a1B1, a0B2, a2B0, a0B1, a1B0,
//     a0B0, smallest first); the three dropped products are below 2^-24
//     relative.  Six bf16 MMAs cost the same tensor time as three TF32 ones
//     and, unlike a two-way TF32 split (22 bits), represent the operands
//     exactly, so the result is fp32-accurate;
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

// Bounded wait on an mbarrier phase (try_wait suspends the thread for a
// hardware-chosen window per attempt); false after about 2^31 cycles.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > (1ll << 31)) return false;
  }
  return true;
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

// Two 32-column accumulator loads (addresses a0, a1) completed by one wait.
__device__ __forceinline__ void tmem_ld32x2(uint32_t a0, uint32_t a1, float (&v)[32], float (&w)[32]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = __uint_as_float(r[i]);
    w[i] = __uint_as_float(r[32 + i]);
  }
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


// Shared-memory matrix descriptor, SW128, sm_100 version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  // No "memory" clobber: ordering against the MMAs that read these operands
  // comes from the proxy fence and barrier asm statements (all volatile).
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d));
}

#ifdef PONNI_B200_TC_PROFILE
__device__ int* prof_ptr;
#endif

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

// Operand type of a model type: bf16 parts for fp32, else the type itself.
template <class T> struct OperandOf { using type = T; };
template <> struct OperandOf<float> { using type = __nv_bfloat16; };

__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Exact three-way split of an fp32 value into bfloat16 parts by truncation:
// b0 keeps the top 8 significant bits, b1 the next 8, b2 the rest (at most 8
// bits, so exactly representable).  Integer masks and two FADDs, no
// conversion instructions.  Returns the three parts as fp32 bit patterns
// whose low 16 bits are zero.
__device__ __forceinline__ void split3(float x, uint32_t& h0, uint32_t& h1, uint32_t& h2) {
  h0 = __float_as_uint(x) & 0xFFFF0000u;
  const float r1 = x - __uint_as_float(h0);
  h1 = __float_as_uint(r1) & 0xFFFF0000u;
  h2 = __float_as_uint(r1 - __uint_as_float(h1));
}

// Two bf16 parts (as fp32 bit patterns) -> one packed bf16x2 word (lo first).
__device__ __forceinline__ uint32_t pack_hi16(uint32_t lo, uint32_t hi) { return __byte_perm(lo, hi, 0x7632); }

// Byte offset of the 16-byte chunk holding byte `byte` of row m of a K-major
// SW128 operand with 128 rows.
__device__ __forceinline__ uint32_t kmajor_chunk(int m, uint32_t byte) {
  const uint32_t kb = byte >> 7;
  const uint32_t chunk = (byte >> 4) & 7;
  return kb * (kTcM * 128) + (uint32_t)m * 128 + ((chunk ^ ((uint32_t)m & 7)) << 4);
}

// Write 8 consecutive K values (k0 multiple of 8) of row m into the operand
// part(s).
template <class T>
__device__ __forceinline__ void store_row8(const uint32_t* a, int m, int k0, const float* v) {
  using Op = typename OperandOf<T>::type;
  const uint32_t off = kmajor_chunk(m, (uint32_t)k0 * 2);
  if constexpr (sizeof(T) == 4) {
    uint32_t p0[8], p1[8], p2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) split3(v[e], p0[e], p1[e], p2[e]);
    st_shared_v4(a[0] + off, pack_hi16(p0[0], p0[1]), pack_hi16(p0[2], p0[3]), pack_hi16(p0[4], p0[5]),
                 pack_hi16(p0[6], p0[7]));
    st_shared_v4(a[1] + off, pack_hi16(p1[0], p1[1]), pack_hi16(p1[2], p1[3]), pack_hi16(p1[4], p1[5]),
                 pack_hi16(p1[6], p1[7]));
    st_shared_v4(a[2] + off, pack_hi16(p2[0], p2[1]), pack_hi16(p2[2], p2[3]), pack_hi16(p2[4], p2[5]),
                 pack_hi16(p2[6], p2[7]));
  } else {
    st_shared_v4(a[0] + off, pack2(v[0], v[1], (Op*)0), pack2(v[2], v[3], (Op*)0), pack2(v[4], v[5], (Op*)0),
                 pack2(v[6], v[7], (Op*)0));
  }
}

// Stage input columns [col0, col0+128).  fp32: row-major [k][128] fp32;
// 16-bit: MN-major SW128 operand layout.
template <class T, int TPS>
__device__ __forceinline__ void load_input(uint32_t stage, const T* __restrict__ in, int64_t in_ld, int nin,
                                           int64_t col0, int64_t batch, bool vec, int lt) {
  constexpr int esz = sizeof(T);
  constexpr int per16 = 16 / esz;
  constexpr int chunks_per_row = kTcM / per16;  // 32 (fp32) or 16 (16-bit)
  if (vec) {
    for (int i = lt; i < nin * chunks_per_row; i += TPS) {
      const int f = i / chunks_per_row, j = i - f * chunks_per_row;
      const int64_t col = col0 + (int64_t)j * per16;
      const int64_t valid = batch - col;
      const int bytes = valid >= per16 ? 16 : (valid > 0 ? (int)valid * esz : 0);
      const T* src = in + (int64_t)f * in_ld + (bytes > 0 ? col : 0);
      uint32_t dst;
      if constexpr (esz == 4) dst = stage + (uint32_t)f * 512 + (uint32_t)j * 16;
      else
        dst = stage + (uint32_t)(f >> 3) * 2048 + (uint32_t)(j >> 3) * 1024 + (uint32_t)(f & 7) * 128 +
              ((((uint32_t)j & 7) ^ ((uint32_t)f & 7)) << 4);
      cp_async16(dst, src, bytes);
    }
  } else {
    for (int i = lt; i < nin * kTcM; i += TPS) {
      const int f = i / kTcM, m = i - f * kTcM;
      const int64_t col = col0 + m;
      T v = col < batch ? in[(int64_t)f * in_ld + col] : Store<T>::from(0.0f);
      if constexpr (esz == 4) {
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(stage + (uint32_t)f * 512 + (uint32_t)m * 4),
                     "r"(__float_as_uint(*reinterpret_cast<float*>(&v)))
                     : "memory");
      } else {
        const uint32_t byte = (uint32_t)m * 2, j = byte >> 4;
        const uint32_t dst = stage + (uint32_t)(f >> 3) * 2048 + (j >> 3) * 1024 + (uint32_t)(f & 7) * 128 +
                             (((j & 7) ^ ((uint32_t)f & 7)) << 4) + (byte & 15);
        asm volatile("st.shared.b16 [%0], %1;\n" ::"r"(dst), "h"(*reinterpret_cast<unsigned short*>(&v)) : "memory");
      }
    }
  }
}

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
    if (E.groups == 1) {
      tmem_ld32(tmem_lane + (uint32_t)c0, v);
    } else {
      float w[32];
      tmem_ld32x2(tmem_lane + (uint32_t)c0, tmem_lane + (uint32_t)(E.n_pad + c0), v, w);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += w[j];
      g = 2;
    }
    for (; g + 1 < E.groups; g += 2) {
      float w0[32], w1[32];
      tmem_ld32x2(tmem_lane + (uint32_t)(g * E.n_pad + c0), tmem_lane + (uint32_t)((g + 1) * E.n_pad + c0), w0, w1);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += w0[j] + w1[j];
    }
    for (; g < E.groups; ++g) {
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
        v[4 * q] += b.x;
        v[4 * q + 1] += b.y;
        v[4 * q + 2] += b.z;
        v[4 * q + 3] += b.w;
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

// Issue the UMMA chain of layer L for one slot (one elected thread).  The
// descriptors of each operand are built once per layer; the K steps then only
// add the step offset to the 14-bit start-address field (>> 4), which never
// carries out of the field for shared-memory addresses.
template <bool SPLIT>
__device__ __forceinline__ void issue_layer(const TcLayer& L, bool layer0, uint32_t d_tmem, const uint32_t* s_a,
                                            uint32_t s_image, uint32_t stage) {
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
    for (int s = 0; s < nsteps; ++s) {
      const uint64_t ao = (uint64_t)(s >> 2) * 1024 + (uint64_t)(s & 3) * 2;
      const uint64_t bo = (uint64_t)(s >> 2) * b_step_kb + (uint64_t)(s & 3) * 2;
      const uint32_t acc = in_group ? 1u : 0u;
      // smallest products first
      umma_f16(d, a0[1] + ao, b0[1] + bo, idesc, acc);
      umma_f16(d, a0[0] + ao, b0[2] + bo, idesc, 1u);
      umma_f16(d, a0[2] + ao, b0[0] + bo, idesc, 1u);
      umma_f16(d, a0[0] + ao, b0[1] + bo, idesc, 1u);
      umma_f16(d, a0[1] + ao, b0[0] + bo, idesc, 1u);
      umma_f16(d, a0[0] + ao, b0[0] + bo, idesc, 1u);
      if (++in_group == gstep) {
        in_group = 0;
        d += n_pad;
      }
    }
  } else {
    const uint64_t b0 = smem_desc(s_image + L.w_off[0], 16, 1024);
    if (layer0) {
      // The staged input tile is the MN-major layer-0 operand: one K step =
      // 32 bytes of K for 128 rows = 4096 bytes.
      const uint64_t a0 = smem_desc(stage, 1024, 2048);
      for (int s = 0; s < nsteps; ++s) {
        const uint64_t bo = (uint64_t)(s >> 2) * b_step_kb + (uint64_t)(s & 3) * 2;
        umma_f16(d, a0 + (uint64_t)s * 256, b0 + bo, L.idesc_mn, s > 0 ? 1u : 0u);
      }
    } else {
      const uint64_t a0 = smem_desc(s_a[0], 16, 1024);
      for (int s = 0; s < nsteps; ++s) {
        const uint64_t ao = (uint64_t)(s >> 2) * 1024 + (uint64_t)(s & 3) * 2;
        const uint64_t bo = (uint64_t)(s >> 2) * b_step_kb + (uint64_t)(s & 3) * 2;
        umma_f16(d, a0 + ao, b0 + bo, idesc, s > 0 ? 1u : 0u);
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
template <class T, int TPS>
__global__ void __launch_bounds__(kTcMaxThreads, 1)
    tc_forward_kernel(const __grid_constant__ TcProgram p, const unsigned char* __restrict__ image,
                      const T* __restrict__ in, int64_t in_ld, T* __restrict__ out, int64_t out_ld, int64_t batch,
                      int in_vec, int* __restrict__ err) {
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
  TcLayer* layers = reinterpret_cast<TcLayer*>(base_ptr + (s_bars + 64u - base));

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
  if (tile < ntiles) {
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
      // Thread m splits column m of the staged fp32 tile into the K-major
      // bf16 operand parts of layer 0; then the stage is free for the next tile.
      const int k0 = p.layers[0].k_pad;
      const float* st = reinterpret_cast<const float*>(base_ptr + (stage - base));
      for (int f = 8 * half; f < k0; f += 8 * (TPS / 128)) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = st[(f + e) * kTcM + m];
        store_row8<T>(s_a, m, f, v);
      }
      wg_sync<TPS>(wg);
      if (next < ntiles) load_input<T, TPS>(stage, in, in_ld, p.nin, next * kTcM, batch, in_vec != 0, lt);
      cp_async_commit();
    }
    TC_PROF_ADD(1, t_split);
    bool failed = false;
    for (int l = 0; l < p.n_layers; ++l) {
      const TcLayer& L = layers[l];
      const EpiArgs E{L.n_pad, L.nout, L.groups, L.has_bias, L.act_flags, L.s0, L.s1};
      const int act = L.act;
      const uint32_t bias_off = L.bias_off;
      TC_PROF_T(t_bar);
      fence_proxy_async();
      tc_fence_before();
      wg_sync<TPS>(wg);
      // One elected thread issues the chain and waits for its completion;
      // the rest of the warpgroup parks on the named barrier (no issue slots
      // spent spinning while the other slot's epilogue runs).
      TC_PROF_ADD(2, t_bar);
      bool ok = true;
      if (lt == 0) {
        TC_PROF_T(t_issue);
        tc_fence_after();
        issue_layer<SPLIT>(L, l == 0, tmem_base, s_a, s_image, stage);
        umma_commit(s_bar);
        TC_PROF_ADD(3, t_issue);
        TC_PROF_T(t_mma);
        ok = mbar_wait_bounded(s_bar, phase);
        TC_PROF_ADD(4, t_mma);
      }
      phase ^= 1u;
      const int bad = wg_sync_or<TPS>(wg, !ok);
      tc_fence_after();
      if (bad) {
        if (lt == 0) atomicExch(err, 1);
        failed = true;
        break;
      }
      if constexpr (!SPLIT) {
        if (l == 0) {  // layer 0 has consumed the stage: prefetch the next tile
          if (next < ntiles) load_input<T, TPS>(stage, in, in_ld, p.nin, next * kTcM, batch, in_vec != 0, lt);
          cp_async_commit();
        }
      }
      const float* bias = reinterpret_cast<const float*>(base_ptr + bias_off);
      TC_PROF_T(t_epi);
      epilogue_dispatch<T, TPS>(act, E, l == p.n_layers - 1, tmem_lane, bias, s_a, out, out_ld, col0 + m, batch, m, half);
      TC_PROF_ADD(5, t_epi);
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

template <class T, int TPS>
cudaError_t launch_tps(const TcProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                       int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  auto kern = tc_forward_kernel<T, TPS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem_bytes);
  if (e != cudaSuccess) return e;
  const bool vec = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && ((in_ld * (int64_t)sizeof(T)) % 16 == 0);
  kern<<<grid, p.slots * TPS, p.smem_bytes, stream>>>(p, static_cast<const unsigned char*>(image),
                                                     static_cast<const T*>(in), in_ld, static_cast<T*>(out), out_ld,
                                                     batch, vec ? 1 : 0, err);
  return cudaGetLastError();
}

template <class T>
cudaError_t launch_impl(const TcProgram& p, const void* image, const void* in, int64_t in_ld, void* out,
                        int64_t out_ld, int64_t batch, int grid, int* err, cudaStream_t stream) {
  if (p.slot_threads == 128) return launch_tps<T, 128>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
  return launch_tps<T, 256>(p, image, in, in_ld, out, out_ld, batch, grid, err, stream);
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
