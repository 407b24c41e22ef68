// Shared device helpers for the sm_100a kernels: bf16 conversion, warp reductions,
// mbarrier / TMA / tcgen05 inline PTX, bounded waits and the library error word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/qw200.h"

#define QW_DEV __device__ __forceinline__

namespace qw {

// ------------------------------------------------------------------ error reporting
// One library-wide error word in device memory (defined in gemm.cu). Kernels receive its
// address as a parameter; one that gives up on a bounded wait or sees an out-of-range
// index records a code there (first writer wins). The host reads and clears it with
// qw_take_device_error().
int* device_error_ptr();  // host: address of the error word on the current device

QW_DEV void set_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

QW_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Spin limit for every wait in this library: 2 seconds of wall time.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ------------------------------------------------------------------ bf16 helpers
QW_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
QW_DEV float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
QW_DEV __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

QW_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// barrier `id` (1..15) among `n` threads (a multiple of 32) of the CTA
QW_DEV void named_bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// 2^x with the approximate hardware exponential, subnormal results flushed to zero
// (ex2.approx.ftz.f32; 2^-inf = 0): softmax weights in the log2 domain
QW_DEV float ex2_ftz(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// approximate reciprocal (rcp.approx.ftz.f32: relative error below 2^-23; 1/inf = 0)
QW_DEV float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// fp32 pairs in one 64-bit register (low float first) and the sm_100 packed arithmetic on
// them: one instruction for both lanes, each rounded as the scalar operation
QW_DEV unsigned long long f2_pack(float lo, float hi) {
  return ((unsigned long long)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
QW_DEV float f2_lo(unsigned long long v) { return __uint_as_float((uint32_t)v); }
QW_DEV float f2_hi(unsigned long long v) { return __uint_as_float((uint32_t)(v >> 32)); }
QW_DEV unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
QW_DEV unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// a bf16 pair (packed) as an fp32 pair: exact bit shifts
QW_DEV unsigned long long bf16x2_to_f2(uint32_t u) {
  return ((unsigned long long)(u & 0xffff0000u) << 32) | (u << 16);
}

// the two bf16 of a packed pair as floats (low half first): exact bit shifts
QW_DEV float2 bf16x2_to_float2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
QW_DEV void unpack_bf16x2(uint32_t u, float& lo, float& hi) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  lo = __low2float(v);
  hi = __high2float(v);
}

// 8 bf16 <-> 8 floats through one 16-byte vector
QW_DEV void load_bf16x8(const __nv_bfloat16* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  unpack_bf16x2(u.x, f[0], f[1]);
  unpack_bf16x2(u.y, f[2], f[3]);
  unpack_bf16x2(u.z, f[4], f[5]);
  unpack_bf16x2(u.w, f[6], f[7]);
}
QW_DEV void store_bf16x8(__nv_bfloat16* p, const float* f) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

QW_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
QW_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// silu(x) = x / (1 + e^-x), fp32 (the activation of the reference's SwiGLU and conv)
QW_DEV float silu(float x) { return x / (1.0f + __expf(-x)); }
QW_DEV float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }

// ------------------------------------------------------------------ shared-memory addresses
QW_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ------------------------------------------------------------------ mbarrier
QW_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
QW_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
QW_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
QW_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
QW_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase completes or up to
// kWaitSuspendNs passes, instead of re-issuing the test (waiting warps cost fewer issue
// slots and less power). Builds with QW_MBAR_SPIN defined test without the hint.
#ifndef QW_MBAR_SPIN
constexpr uint32_t kWaitSuspendNs = 100000;  // 100 us
#endif
QW_DEV bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
#ifdef QW_MBAR_SPIN
  return mbar_try_wait(bar, parity);
#else
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kWaitSuspendNs)
      : "memory");
  return ok != 0;
#endif
}
// Bounded wait: returns false (and records `code`) if the phase did not complete within
// kWaitLimitNs, or if `abort` (shared flag) was raised by another role of the CTA.
QW_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((it & 15u) == 15u) {
      if (abort != nullptr && *abort) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        set_error(err, code);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------ cp.async (16-byte, L2 only)
// pred false copies nothing and zero-fills the 16 destination bytes
QW_DEV void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
QW_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
QW_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------------ TMA (no multicast anywhere)
QW_DEV void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
QW_DEV void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// TMA store of a box from this CTA's shared memory to global memory (bulk-group completion):
// rows and columns of the box outside the tensor map's extent are not written.
QW_DEV void tma_store_2d(const CUtensorMap* m, uint32_t smem_src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_src), "r"(x), "r"(y)
               : "memory");
}
QW_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N committed bulk groups of this thread still read their shared source
template <int N>
QW_DEV void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// wait until at most N committed bulk groups of this thread are incomplete
template <int N>
QW_DEV void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// generic-proxy writes to shared memory made visible to the async proxy (TMA, tcgen05)
QW_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 fp32 of one row as bf16 into a 64-column (128-byte) row of a SWIZZLE_128B staging box
// (16-byte chunk j of row r at chunk j ^ (r % 8)); half = which 32 columns of the 64
QW_DEV void stage_row_bf16_sw128(uint8_t* box, int r, int half, const float* f) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    u.x = pack_bf16x2(f[8 * j], f[8 * j + 1]);
    u.y = pack_bf16x2(f[8 * j + 2], f[8 * j + 3]);
    u.z = pack_bf16x2(f[8 * j + 4], f[8 * j + 5]);
    u.w = pack_bf16x2(f[8 * j + 6], f[8 * j + 7]);
    const int chunk = (half * 4 + j) ^ (r & 7);
    *reinterpret_cast<uint4*>(box + r * 128 + chunk * 16) = u;
  }
}

// ------------------------------------------------------------------ tcgen05 (cta_group::1)
QW_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
}
QW_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
QW_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
QW_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
QW_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 x bf16 -> fp32)
QW_DEV void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16; A in tensor memory with one row per lane
// and bf16 pairs (k = 2c, 2c + 1) in 32-bit column c (a K step of 16 spans 8 columns).
QW_DEV void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
QW_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Instruction descriptor, kind::f16: A=B=bf16, D=f32, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with SWIZZLE_128B:
// rows of 128 bytes, 8-row swizzle atoms of 1024 bytes (stride byte offset), version 1.
QW_DEV uint64_t umma_sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;  // stride byte offset
  d |= (uint64_t)1u << 46;            // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;            // SWIZZLE_128B
  return d;
}

// 32 lanes x 32 consecutive fp32 columns of TMEM into 32 registers per thread.
QW_DEV void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
QW_DEV void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
QW_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 registers per thread into 32 lanes x 32 consecutive fp32 columns of TMEM.
QW_DEV void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
QW_DEV void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
QW_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory descriptor for an MN-major operand (N contiguous) stored as 64-element
// SWIZZLE_128B column blocks of `block_bytes` each, rows of 128 bytes: the leading byte
// offset is the stride between column blocks, the stride byte offset the stride between
// 8-row groups along K (1024 bytes).
QW_DEV uint64_t umma_sdesc_mn_sw128(uint32_t saddr, uint32_t block_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((block_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// ------------------------------------------------------------------ CTA pairs (cluster of 2)
QW_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// address of the same shared-memory object in CTA `rank` of the cluster
QW_DEV uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
QW_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
QW_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on the mbarrier at
// `bar_cluster` (which may be the pair leader's); no multicast
QW_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
QW_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
}
QW_DEV void tmem_relinquish_pair() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
QW_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (both CTAs' TMEM) (+)= A (each CTA's 128 rows) * B (each CTA's half of N)^T, M = 256
QW_DEV void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` in every CTA of `mask` once the pair's MMAs issued so far complete.
// The .multicast::cluster qualifier here only signals the mbarriers of the pair's two CTAs
// (this GPU's shared memory, same offset in each CTA); it loads nothing. Every TMA load in
// this library is a per-CTA copy without multicast (tma_load_2d, tma_load_2d_pair), so the
// same code runs in multi-GPU jobs.
QW_DEV void umma_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "h"(mask)
               : "memory");
}

QW_DEV bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\telect.sync r|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ------------------------------------------------------------------ programmatic dependent launch
// A kernel launched with programmatic stream serialization (launch_k with pdl = true) may start
// while the kernel before it on the stream still runs. It must execute griddep_wait() before
// it reads anything an earlier kernel wrote and before it writes anything an earlier kernel
// reads: the wait returns once every earlier grid has completed and its memory is visible.
// Without the launch attribute the wait returns at once. griddep_launch_dependents() lets the
// next kernel's CTAs start; a CTA executes it only once it holds everything it allocates
// (shared memory comes with the launch, tensor memory is allocated before it), so a dependent
// CTA that became resident can never keep an earlier grid's CTA from running.
QW_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
QW_DEV void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace qw

// Launch a kernel; with pdl, with programmatic stream serialization (the kernel calls
// qw::griddep_wait before touching memory that earlier kernels use). PDL is on unless the
// environment variable QW_PDL=0 turns it off (a tuning knob).
bool qw_pdl_enabled();
// the same for the small kernels of the decode step (norms, attention, merge, GDN step): off
// unless QW_PDL_SMALL=1 (a tuning knob). Measured on the B32 decode graph (27B, 1024 context,
// replay after idle): 13.44 ms without PDL, 13.10 ms with the weight-streaming GEMMs alone
// under PDL, 13.53 ms with every kernel under it. The small kernels still execute
// griddep_launch_dependents at their start, so the GEMM after one of them starts early.
bool qw_pdl_small();
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_k(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                   cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl && qw_pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ host-side argument checks
#define QW_CHECK_ARG(cond, code) \
  do {                           \
    if (!(cond)) return (code);  \
  } while (0)

#define QW_LAUNCH_CHECK()                                   \
  do {                                                      \
    cudaError_t _e = cudaGetLastError();                    \
    if (_e != cudaSuccess) return QW_ERR_CUDA_BASE + (int)_e; \
  } while (0)
