// PTX wrappers and operand helpers shared by the tensor-core kernels
// (tc_kernel.cu: weights resident in shared memory; tc_stream_kernel.cu:
// weights streamed per layer).  sm_100a only.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tc_program.h"
#include "f32x2.cuh"

// Bound of every spin-wait of the tensor-core kernels, in SM cycles (about
// one second).  The wait-bound test build (PONNI_B200_WAIT_TEST) shortens it.
#ifndef PONNI_B200_WAIT_LIMIT
#ifdef PONNI_B200_WAIT_TEST
#define PONNI_B200_WAIT_LIMIT (1ll << 20)
#else
#define PONNI_B200_WAIT_LIMIT (1ll << 31)
#endif
#endif

// Wait-bound test build only (PONNI_B200_WAIT_TEST, never the default
// library): each tensor-core translation unit holds a flag that the host
// sets through ponni_b200_debug_skip_arrive_<kernel>(); a launch that sees it
// leaves out the completion signal of its first job, so that the waiting role
// runs into its bound and the kernel reports PONNI_B200_ERR_DEVICE.
#ifdef PONNI_B200_WAIT_TEST
#define PONNI_B200_SKIP_ARRIVE_FLAG(kernel)                                                     \
  namespace {                                                                                   \
  __device__ int g_skip_arrive;                                                                 \
  }                                                                                             \
  extern "C" __attribute__((visibility("default"))) int ponni_b200_debug_skip_arrive_##kernel(int on) { \
    return (int)cudaMemcpyToSymbol(g_skip_arrive, &on, sizeof(int));                            \
  }
#define PONNI_B200_SKIP_ARRIVE() (g_skip_arrive != 0)
#else
#define PONNI_B200_SKIP_ARRIVE_FLAG(kernel)
#define PONNI_B200_SKIP_ARRIVE() false
#endif

namespace ponni_b200 {
namespace tc {

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
    if (clock64() - t0 > PONNI_B200_WAIT_LIMIT) return false;
  }
  return true;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory, completion on `bar`
// (no multicast).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Bounded wait on an mbarrier phase that also leaves when another role of
// the CTA has raised `abort_flag`; raises it itself after `limit` cycles.
__device__ __forceinline__ bool wait_phase_abort(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                 long long limit) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// ------------------------------------------- CTA pairs (cta_group::2) ----
// Two CTAs of a cluster of two share one MMA of M = 256: the even CTA issues
// it, each CTA holds its 128 rows of A, half of the N rows of B and its 128
// rows of the accumulator.  The helpers below are the cluster-scope pieces
// of that handshake (no multicast loads anywhere: each CTA fills its own
// shared memory with its own bulk copies).
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// Address of this CTA's shared-memory location `addr` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive (release, cluster scope) on an mbarrier given by its cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(cluster_addr) : "memory");
}
// try_wait with acquire at cluster scope (arrivals from the peer CTA).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait_phase_abort_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                         long long limit) {
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}
// Cluster-wide barrier of every thread of both CTAs.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
// M = 256 MMA over the pair (issued by the even CTA only), warp-level form:
// every lane of the converged warp calls it, one elected lane issues.
__device__ __forceinline__ void umma_f16_pair_warp(uint32_t d_tmem, uint32_t alo, uint32_t ahi, uint32_t blo,
                                                   uint32_t bhi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 da, db;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "mov.b64 da, {%1, %2};\n\t"
      "mov.b64 db, {%3, %4};\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %5, p;\n\t}\n" ::"r"(d_tmem),
      "r"(alo), "r"(ahi), "r"(blo), "r"(bhi), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same for one CTA (M <= 128).
__device__ __forceinline__ void umma_f16_desc_warp(uint32_t d_tmem, uint32_t alo, uint32_t ahi, uint32_t blo,
                                                   uint32_t bhi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 da, db;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "mov.b64 da, {%1, %2};\n\t"
      "mov.b64 db, {%3, %4};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}\n" ::"r"(d_tmem),
      "r"(alo), "r"(ahi), "r"(blo), "r"(bhi), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Completion of the pair's MMAs issued so far, signalled on the mbarrier at
// offset `bar` in both CTAs (commit multicast; not a load).
__device__ __forceinline__ void umma_commit_pair_warp(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}\n" ::"r"(bar)
      : "memory");
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
// UMMA issued by the calling thread (single-thread issue loops).
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

// Same, with both descriptors given as 32-bit halves: `alo` / `blo` carry
// the start address (advanced by the caller, no carry out of the 14-bit
// field), `hi` the shared upper half (stride, version, swizzle).
__device__ __forceinline__ void umma_f16_lh(uint32_t d_tmem, uint32_t alo, uint32_t blo, uint32_t hi, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 da, {%1, %3};\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %4, p;\n\t}\n" ::"r"(d_tmem),
      "r"(alo), "r"(blo), "r"(hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Warp-level forms: every lane of a converged warp calls them (elect.sync
// over the full warp), one elected lane issues; the whole warp runs the issue
// loop so the descriptors stay in uniform registers.  Never call these from
// a divergent branch: elect.sync waits for all 32 lanes.
__device__ __forceinline__ void umma_f16_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_f16_lh_warp(uint32_t d_tmem, uint32_t alo, uint32_t blo, uint32_t hi,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 da, db;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 da, {%1, %3};\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %4, p;\n\t}\n" ::"r"(d_tmem),
      "r"(alo), "r"(blo), "r"(hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit_warp(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(bar)
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

// split3 of two values with packed fp32 subtractions (the same results).
__device__ __forceinline__ void split3x2(float x, float y, uint32_t& h0, uint32_t& h1, uint32_t& h2, uint32_t& g0,
                                         uint32_t& g1, uint32_t& g2) {
  h0 = __float_as_uint(x) & 0xFFFF0000u;
  g0 = __float_as_uint(y) & 0xFFFF0000u;
  float r, t;
  f2::sub(r, t, x, y, __uint_as_float(h0), __uint_as_float(g0));
  h1 = __float_as_uint(r) & 0xFFFF0000u;
  g1 = __float_as_uint(t) & 0xFFFF0000u;
  f2::sub(r, t, r, t, __uint_as_float(h1), __uint_as_float(g1));
  h2 = __float_as_uint(r);
  g2 = __float_as_uint(t);
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
    for (int e = 0; e < 8; e += 2)
      split3x2(v[e], v[e + 1], p0[e], p1[e], p2[e], p0[e + 1], p1[e + 1], p2[e + 1]);
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


}  // namespace tc
}  // namespace ponni_b200
