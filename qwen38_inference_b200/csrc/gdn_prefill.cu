// Chunked gated delta rule for prefill (replaces flashinfer chunk_gated_delta_rule,
// REF:4852/5084, plus the gating kernel REF:1258-1323, the state gather/scatter
// REF:5082-5085 and the gated RMSNorm REF:5086: the state is read and written in place at
// the request's slot and the output goes straight through the norm).
//
// Recurrence per token t (state S is [dv, dk], fp32):
//   S_t = a_t S_{t-1} (I - b_t k_t k_t^T) + b_t v_t k_t^T,   o_t = S_t q_t * scale
// with a_t = exp(g_t), g_t = -exp(A_log) softplus(a + dt_bias), b_t = bf16(sigmoid(b)).
// Chunk form (C = 64 tokens, G = within-chunk cumsum of g, S0 = state before the chunk):
//   A_ts = b_t e^{G_t - G_s} k_t.k_s (s < t),   T = (I + A)^-1
//   W = T diag(b e^G) K,   U = T diag(b) V - W S0^T
//   O = scale diag(e^G) Q S0^T + ([s <= t] scale e^{G_t - G_s} Q K^T) U
//   S_C = e^{G_C} S0 + U^T diag(e^{G_C - G}) K
//
// One CTA of 16 warps per (sequence, value head), two warp groups in a software pipeline:
//  * prep warps 0-7 work one chunk ahead on everything that does not depend on the state:
//    gating, K K^T and Q K^T (mma.sync), T by a blocked inverse (16 x 16 diagonal blocks by
//    forward substitution in fp32, off-diagonal blocks on tf32 tensor cores), b e^G K,
//    W = T (b e^G K), b V and e^{G_C - G} K; the chunk is handed over on an mbarrier;
//  * state warps 8-15 keep S in tensor memory (one value row dv per TMEM lane, fp32) and run
//    the state products on tcgen05 with dv as the MMA M dimension (128):
//      warps 8-11 (one elected thread issues the MMAs): S0 = bf16(S) and S <- e^{G_C} S
//      (tcgen05.ld / st), U^T = (bV)^T T^T + S0 (-W)^T (A = bV MN-major from shared memory,
//      then S0 from TMEM), O1^T = S0 Q^T, U^T to bf16 in TMEM, O2^T = U^T P^T and
//      S += U^T (e^{G_C-G} K) (B MN-major);
//      warps 12-15: O = bf16(scale e^G O1 + O2) out of TMEM, the gated RMSNorm over the 128
//      value rows of each token (halving exchange in the warp, then shared memory) and
//      y = o rstd w silu(z) through a double-buffered z / y staging tile.
// Q, K, V chunks arrive by TMA (128-byte swizzle) into two chunk buffers; the state warps
// release a buffer and issue the loads of the chunk two ahead. Every mbarrier wait is bounded
// (QW_DEV_ERR_TIMEOUT_GDN); after a timeout all waits return at once and both groups run
// their remaining iterations on whatever is in shared memory, so every named barrier is still
// reached by all its warps and the kernel ends.
#include "common.cuh"
#include "tmap.cuh"

namespace qw {
namespace gdn {

constexpr int CH = 64;  // chunk length
constexpr int D = 128;  // key / value head dim
constexpr int TILE = CH * D * 2;      // [64][128] bf16 = two 64-column halves of 8 KB
constexpr int TILE64 = CH * CH * 2;   // [64][64] bf16
// one chunk buffer: Q | K (then e^{G_C-G} K) | V (then b V) | b e^G K (then -W) | T | P
constexpr int B_Q = 0, B_K = TILE, B_V = 2 * TILE, B_W = 3 * TILE, B_T = 4 * TILE, B_P = B_T + TILE64;
constexpr int BUF = B_P + TILE64;     // multiple of 1024 (TMA swizzle atoms)
constexpr int BLD = 20;               // row stride (floats) of a compact 16 x 16 fp32 block
constexpr int BLK = 16 * BLD;         // floats per block
constexpr int S_BLK = 2 * BUF;        // 20 blocks: [0,6) A_ij then T_ij (i > j), [6,10) A_ii, [10,14) T_ii, [14,20) M_ik
// gating of a chunk (written by the state warps two chunks ahead, four slots: the output
// warps read a chunk's e^G up to two chunks after the MMA warps move on):
// G * log2(e), beta, e^{G_C - G}, e^G (64 each), e^{G_C}
constexpr int GB_G2 = 0, GB_BETA = CH, GB_EGL = 2 * CH, GB_EG = 3 * CH, GB_EC = 4 * CH, GB_FLOATS = 4 * CH + 4;
constexpr int GB_SLOTS = 4;
constexpr int S_GB = S_BLK + 20 * BLK * 4;
constexpr int S_RED = S_GB + GB_SLOTS * GB_FLOATS * 4;      // output warps: [4][64] sums of squares, rstd [64]
constexpr int S_Z = (S_RED + 5 * CH * 4 + 127) / 128 * 128;  // output warps: two z / y tiles [64 tokens][128] bf16
constexpr int ZBUF = CH * D * 2;
constexpr int S_BAR = S_Z + 2 * ZBUF;
constexpr int SMEM = S_BAR + 128 + 1024;                     // + slack to align the base to 1024
static_assert(BUF % 1024 == 0 && S_Z % 128 == 0, "layout alignment");
// tensor memory columns: S fp32, S0 = bf16(S) pairs, U^T fp32, U^T bf16 pairs, O1^T, O2^T
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t T_S = 0, T_S0 = 128, T_U = 192, T_UB = 256, T_O1 = 320, T_O2 = 384;
constexpr uint32_t IDESC_N64 = umma_idesc_bf16(128, 64);
constexpr uint32_t IDESC_U_AMN = umma_idesc_bf16(128, 64) | (1u << 15);  // A (bV) MN-major
constexpr uint32_t IDESC_S_BMN = umma_idesc_bf16(128, 128) | (1u << 16);  // B (e^{G_C-G} K) MN-major

QW_DEV int blk_lo(int i, int j) { return i * (i - 1) / 2 + j; }  // i > j

// byte offset of 16-byte chunk c (0..15) of row r (0..63) of a 64-row bf16 tile stored as
// 64-column halves of 8 KB, each with the TMA 128-byte swizzle (chunk ^= row % 8)
QW_DEV uint32_t swz(int r, int c) { return (uint32_t)(((c >> 3) << 13) | (r << 7) | (((c & 7) ^ (r & 7)) << 4)); }
QW_DEV uint32_t swz_elem(int r, int col) { return swz(r, col >> 3) + ((col & 7) << 1); }

QW_DEV void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
QW_DEV void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
QW_DEV void stsm_x4(uint32_t addr, const uint32_t* r) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}
QW_DEV void stsm_x4_t(uint32_t addr, const uint32_t* r) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}
QW_DEV void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
QW_DEV uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
QW_DEV void mma1688_tf32(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
QW_DEV void cpa16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0) : "memory");
}
// Register split between the warp groups: the CTA is launched with 512 x 128 registers
// (ptxas is held to 128 by the launch bounds); the prep warpgroups give 32 back and the
// state warpgroups take 32 more (the output warps hold a token row of O, 64 values, and its
// squares while they reduce them): 256 x 96 + 256 x 160 = 512 x 128. At 96 the prep code
// does not spill (at 88 it did, and a B32 x L1024 launch took 2.7 % longer).
#ifndef QW_GDN_PREP_REGS
#define QW_GDN_PREP_REGS 96
#endif
constexpr int PREP_REGS = QW_GDN_PREP_REGS, STATE_REGS = 256 - QW_GDN_PREP_REGS;
static_assert(256 * PREP_REGS + 256 * STATE_REGS == 512 * 128, "register split must equal the launch allocation");
QW_DEV void named_bar(int id) { asm volatile("bar.sync %0, 256;" ::"r"(id) : "memory"); }
QW_DEV void named_bar_n(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// a[0, 2W) -> a[0, W): partner lanes (lane ^ bit) add their halves; lanes with `bit` set keep
// the upper half
template <int W>
QW_DEV void halve(float* a, int lane, int bit) {
  const bool up = (lane & bit) != 0;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const float send = up ? a[i] : a[i + W];
    const float keep = up ? a[i + W] : a[i];
    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
  }
}
QW_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// mma.sync fragments from swizzled 64-row tiles
QW_DEV void frag_a(uint32_t base, int m0, int k0, int lane, uint32_t* a) {  // tile [M][K]
  ldsm_x4(base + swz(m0 + (lane & 15), (k0 >> 3) + (lane >> 4)), a);
}
QW_DEV void frag_a_t(uint32_t base, int m0, int k0, int lane, uint32_t* a) {  // tile [K][M]
  ldsm_x4_t(base + swz(k0 + (lane & 7) + ((lane >> 4) << 3), (m0 >> 3) + ((lane >> 3) & 1)), a);
}
// b[0],b[1]: n-tile n0; b[2],b[3]: n-tile n0+8
QW_DEV void frag_b(uint32_t base, int n0, int k0, int lane, uint32_t* b) {  // tile [N][K]
  ldsm_x4(base + swz(n0 + (lane & 7) + ((lane >> 4) << 3), (k0 >> 3) + ((lane >> 3) & 1)), b);
}
QW_DEV void frag_b_t(uint32_t base, int n0, int k0, int lane, uint32_t* b) {  // tile [K][N]
  ldsm_x4_t(base + swz(k0 + (lane & 7) + (((lane >> 3) & 1) << 3), (n0 >> 3) + (lane >> 4)), b);
}
// acc[NT][4] += A(16 x 16*KS at rows m0) * B(16*KS x 8*NT at cols n0)
template <int NT, int KS, bool AT, bool BT>
QW_DEV void mma_tile(float (*acc)[4], uint32_t sa, uint32_t sb, int m0, int n0, int lane) {
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    uint32_t a[4];
    if constexpr (AT) frag_a_t(sa, m0, ks * 16, lane, a);
    else frag_a(sa, m0, ks * 16, lane, a);
#pragma unroll
    for (int nt = 0; nt < NT; nt += 2) {
      uint32_t b[4];
      if constexpr (BT) frag_b_t(sb, n0 + nt * 8, ks * 16, lane, b);
      else frag_b(sb, n0 + nt * 8, ks * 16, lane, b);
      mma16816(acc[nt], a, b[0], b[1]);
      mma16816(acc[nt + 1], a, b[2], b[3]);
    }
  }
}
template <int NT>
QW_DEV void store_tile_bf16(uint8_t* tile, float (*acc)[4], int m0, int n0, int lane, float mul) {
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int col = n0 + nt * 8 + c * 2;
    *reinterpret_cast<uint32_t*>(tile + swz_elem(m0 + g, col)) = pack_bf16x2(acc[nt][0] * mul, acc[nt][1] * mul);
    *reinterpret_cast<uint32_t*>(tile + swz_elem(m0 + g + 8, col)) = pack_bf16x2(acc[nt][2] * mul, acc[nt][3] * mul);
  }
}
// bf16 A-operand fragment of k-step ks from a 16-row accumulator strip held in registers
QW_DEV void acc_to_a(const float (*s)[4], int ks, uint32_t* a) {
  a[0] = pack_bf16x2(s[2 * ks][0], s[2 * ks][1]);
  a[1] = pack_bf16x2(s[2 * ks][2], s[2 * ks][3]);
  a[2] = pack_bf16x2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
  a[3] = pack_bf16x2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
}
// acc[2][4] += X * Y for compact 16 x 16 fp32 blocks, tf32 tensor cores
QW_DEV void blk_mma(float (*acc)[4], const float* X, const float* Y, int lane) {
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int kk = 0; kk < 16; kk += 8) {
    uint32_t a[4] = {to_tf32(X[g * BLD + kk + c]), to_tf32(X[(g + 8) * BLD + kk + c]),
                     to_tf32(X[g * BLD + kk + c + 4]), to_tf32(X[(g + 8) * BLD + kk + c + 4])};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
      mma1688_tf32(acc[nt], a, to_tf32(Y[(kk + c) * BLD + nt * 8 + g]), to_tf32(Y[(kk + c + 4) * BLD + nt * 8 + g]));
  }
}
// store mul * acc as a compact fp32 block and, when tile != nullptr, as bf16 at (r0, c0)
QW_DEV void blk_store(float* out, float (*acc)[4], float mul, uint8_t* tile, int r0, int c0, int lane) {
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int col = nt * 8 + 2 * c;
    const float v0 = acc[nt][0] * mul, v1 = acc[nt][1] * mul, v2 = acc[nt][2] * mul, v3 = acc[nt][3] * mul;
    out[g * BLD + col] = v0;
    out[g * BLD + col + 1] = v1;
    out[(g + 8) * BLD + col] = v2;
    out[(g + 8) * BLD + col + 1] = v3;
    if (tile) {
      *reinterpret_cast<uint32_t*>(tile + swz_elem(r0 + g, c0 + col)) = pack_bf16x2(v0, v1);
      *reinterpret_cast<uint32_t*>(tile + swz_elem(r0 + g + 8, c0 + col)) = pack_bf16x2(v2, v3);
    }
  }
}

// Gating of one chunk by one warp (lane owns tokens lane and lane + 32; nc valid tokens):
// g = -exp(A_log) softplus(a + dt_bias), beta = bf16(sigmoid(b)), G = inclusive cumsum of g.
// The exponentials and logarithm use the approximate hardware forms, as the reference's
// Triton gating kernel does.
QW_DEV void chunk_gating(float* gb, const float* rb, const float* ra, int nc, float a_log, float dtb, int lane) {
  float gg[2], bt[2];
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    gg[hf] = bt[hf] = 0.f;
    if (lane + 32 * hf < nc) {
      const float xa = ra[hf] + dtb;
      const float sp = xa <= 20.f ? __logf(1.f + __expf(xa)) : xa;
      gg[hf] = -a_log * sp;
      bt[hf] = bf16_round(__fdividef(1.f, 1.f + __expf(-rb[hf])));
    }
  }
  float x0 = gg[0], x1 = gg[1];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y0 = __shfl_up_sync(0xffffffffu, x0, o), y1 = __shfl_up_sync(0xffffffffu, x1, o);
    if (lane >= o) {
      x0 += y0;
      x1 += y1;
    }
  }
  x1 += __shfl_sync(0xffffffffu, x0, 31);
  const float G_last = __shfl_sync(0xffffffffu, x1, 31);
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int t = lane + 32 * hf;
    const float G = hf ? x1 : x0;
    gb[GB_G2 + t] = G * 1.4426950408889634f;
    gb[GB_BETA + t] = bt[hf];
    gb[GB_EGL + t] = __expf(G_last - G);
    gb[GB_EG + t] = __expf(G);
  }
  if (lane == 0) gb[GB_EC] = __expf(G_last);
}
// raw b, a of tokens lane and lane + 32 of chunk c (zero past the request)
QW_DEV void load_gating_inputs(float* rb, float* ra, const __nv_bfloat16* ba, int64_t ldba, int t_begin, int n, int c,
                               int hv, int HV, int lane) {
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int t = c * CH + lane + 32 * hf;
    rb[hf] = ra[hf] = 0.f;
    if (t < n) {
      rb[hf] = bf2f(ba[(int64_t)(t_begin + t) * ldba + hv]);
      ra[hf] = bf2f(ba[(int64_t)(t_begin + t) * ldba + HV + hv]);
    }
  }
}

QW_DEV void issue_chunk_loads(uint8_t* buf, uint64_t* bar, const CUtensorMap* tq, const CUtensorMap* tk,
                              const CUtensorMap* tv, int h, int hv, int row) {
  mbar_arrive_expect_tx(bar, 3 * TILE);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    tma_load_2d(buf + B_Q + half * (TILE / 2), tq, bar, h * D + half * 64, row);
    tma_load_2d(buf + B_K + half * (TILE / 2), tk, bar, h * D + half * 64, row);
    tma_load_2d(buf + B_V + half * (TILE / 2), tv, bar, hv * D + half * 64, row);
  }
}

}  // namespace gdn

using namespace gdn;

__global__ void __launch_bounds__(512, 1) gdn_prefill_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const __nv_bfloat16* __restrict__ ba, int64_t ldba,
    const float* __restrict__ A_log, const __nv_bfloat16* __restrict__ dt_bias, const int32_t* __restrict__ cu,
    const int32_t* __restrict__ slots, int n_slots, float* __restrict__ state, const __nv_bfloat16* __restrict__ z,
    int64_t ldz, const __nv_bfloat16* __restrict__ norm_w, __nv_bfloat16* __restrict__ y, int64_t ldy, int H, int HV,
    float scale, float eps, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  uint64_t* loaded = reinterpret_cast<uint64_t*>(smem + S_BAR);  // [2] chunk tiles landed
  uint64_t* ready = loaded + 2;                                  // [2] chunk prepared
  uint64_t* bar_u = ready + 2;                                   // U^T products complete
  uint64_t* bar_o = bar_u + 1;                                   // O1^T and O2^T complete
  uint64_t* bar_s = bar_o + 1;                                   // state update complete
  uint64_t* o_free = bar_s + 1;                                  // output warps have read O
  uint64_t* gate_pub = o_free + 1;                               // [4] gating slot written
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gate_pub + GB_SLOTS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gate_pub + GB_SLOTS) + 1;

  // value heads vary fastest: the CTAs resident together read whole token rows of q, k, v, z
  // (DRAM page locality) and the value heads of one key head share its q, k tiles in L2
  const int hv = blockIdx.x, seq = blockIdx.y;
  const int h = hv / (HV / H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g4 = lane >> 2, c4 = lane & 3;
  const int t_begin = cu[seq], n = cu[seq + 1] - t_begin;
  const int slot = slots[seq];
  if (slot < 0 || slot >= n_slots) {
    if (tid == 0) set_error(err, QW_DEV_ERR_INDEX);
    return;
  }
  const int n_chunks = (n + CH - 1) / CH;

  if (tid == 0) {
    mbar_init(&loaded[0], 1);
    mbar_init(&loaded[1], 1);
    mbar_init(&ready[0], 256);
    mbar_init(&ready[1], 256);
    mbar_init(bar_u, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_s, 1);
    mbar_init(o_free, 128);
    for (int i = 0; i < GB_SLOTS; ++i) mbar_init(&gate_pub[i], 32);
    *abort_flag = 0;
    fence_barrier_init();
  }
  float* gbuf = reinterpret_cast<float*>(smem + S_GB);
  const float a_log = expf(A_log[hv]);
  const float dtb = bf2f(dt_bias[hv]);
  // blocks of T above the diagonal stay zero in both buffers
  for (int e = tid; e < 2 * CH * CH; e += 512) {
    const int bb = e / (CH * CH), r = (e / CH) % CH, cc = e % CH;
    if ((cc >> 4) > (r >> 4))
      *reinterpret_cast<__nv_bfloat16*>(smem + bb * BUF + B_T + swz_elem(r, cc)) = f2bf(0.f);
  }
  fence_proxy_async_smem();  // T is an operand of the state warps' tensor-core products
  __syncthreads();

  if (warp < 8) {
    // =============================================================== prep warps
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(PREP_REGS));
    const int mt = warp & 3, nh = warp >> 2;
    float* blk = reinterpret_cast<float*>(smem + S_BLK);
    for (int c = 0; c < n_chunks; ++c) {
      const int b = c & 1;
      uint8_t* buf = smem + b * BUF;
      const uint32_t sb = s0 + b * BUF;
      const int nc = min(CH, n - c * CH);
      // gating of this chunk (written by the state warps before they issued its loads)
      const float* gb = gbuf + (c % GB_SLOTS) * GB_FLOATS;
      const float* sG = gb + GB_G2;
      const float* sBeta = gb + GB_BETA;
      const float* sEGl = gb + GB_EGL;
      const float* sEG = gb + GB_EG;
      mbar_wait(&loaded[b], (c >> 1) & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
      if (nc < CH) {
        // rows past the request hold the next request's tokens (or TMA zero fill): clear them
        for (int e = tid; e < (CH - nc) * 16 * 3; e += 256) {
          const int tile = e % 3, rc = e / 3;
          *reinterpret_cast<uint4*>(buf + tile * TILE + swz(nc + (rc >> 4), rc & 15)) = make_uint4(0, 0, 0, 0);
        }
      }
      named_bar(1);
      // ---- K K^T -> A (fp32 blocks), Q K^T -> P (bf16)
      {
        float kk[4][4], qk[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) kk[i][e] = qk[i][e] = 0.f;
        if (nh * 32 <= mt * 16 + 15) {  // tiles wholly above the diagonal stay zero
          mma_tile<4, 8, false, false>(kk, sb + B_K, sb + B_K, mt * 16, nh * 32, lane);
          mma_tile<4, 8, false, false>(qk, sb + B_Q, sb + B_K, mt * 16, nh * 32, lane);
        }
        // rows t = mt*16 + g4 (+8), columns s = s0, s0 + 1 of each n-tile
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int t = mt * 16 + g4 + 8 * rr;
          const float gt = sG[t], bt = sBeta[t];
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            const int s0 = nh * 32 + nt * 8 + 2 * c4;
            const int bj = (nh * 32 + nt * 8) >> 4;
            const float2 gs = *reinterpret_cast<const float2*>(sG + s0);
            const float d0 = (s0 <= t) ? exp2f(gt - gs.x) : 0.f;
            const float d1 = (s0 + 1 <= t) ? exp2f(gt - gs.y) : 0.f;
            const float a0 = (s0 < t) ? bt * d0 * kk[nt][2 * rr] : 0.f;
            const float a1 = (s0 + 1 < t) ? bt * d1 * kk[nt][2 * rr + 1] : 0.f;
            qk[nt][2 * rr] = scale * d0 * qk[nt][2 * rr];
            qk[nt][2 * rr + 1] = scale * d1 * qk[nt][2 * rr + 1];
            if (bj <= mt)
              *reinterpret_cast<float2*>(blk + (bj < mt ? blk_lo(mt, bj) : 6 + mt) * BLK + (g4 + 8 * rr) * BLD +
                                         (s0 & 15)) = make_float2(a0, a1);
          }
        }
        store_tile_bf16<4>(buf + B_P, qk, mt * 16, nh * 32, lane, 1.f);
      }
      named_bar(1);
      // ---- diagonal blocks of T (warps 0-3) || b e^G K, e^{G_C-G} K, b V (warps 4-7 take rows
      // 0-47 of the tiles, warps 0-3 rows 48-63 once their inverse is done: the two halves of
      // the phase then take about the same time)
      constexpr int SCALE_SPLIT = 48 * 16;  // 16-byte items (row, 8 columns) done by warps 4-7
      auto scale_items = [&](int e_begin, int e_end, int t) {
        for (int e = e_begin + t; e < e_end; e += 128) {
          const int r = e >> 4;
          const uint32_t off = swz(r, e & 15);
          float kf[8], vf[8], kb[8], kd[8];
          load_bf16x8(reinterpret_cast<const __nv_bfloat16*>(buf + B_K + off), kf);
          load_bf16x8(reinterpret_cast<const __nv_bfloat16*>(buf + B_V + off), vf);
          const float fb = sBeta[r], fk = fb * sEG[r], fd = sEGl[r];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            kb[jj] = kf[jj] * fk;
            kd[jj] = kf[jj] * fd;
            vf[jj] *= fb;
          }
          store_bf16x8(reinterpret_cast<__nv_bfloat16*>(buf + B_W + off), kb);
          store_bf16x8(reinterpret_cast<__nv_bfloat16*>(buf + B_K + off), kd);
          store_bf16x8(reinterpret_cast<__nv_bfloat16*>(buf + B_V + off), vf);
        }
      };
      if (warp < 4) {
        const int i = warp, j = lane;  // lane j < 16 owns column j of T_ii
        const float* a = blk + (6 + i) * BLK;
        float tcol[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          // row r of A_ii as float4s (rows are 16-byte aligned); acc[e] sums the columns
          // kx = 4 q + e < r in increasing kx, tcol[kx] = 0 for kx < j
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            if (4 * q4 < r) {
              const float4 a4 = *reinterpret_cast<const float4*>(a + r * BLD + 4 * q4);
              if (4 * q4 + 0 < r) acc[0] += a4.x * tcol[4 * q4 + 0];
              if (4 * q4 + 1 < r) acc[1] += a4.y * tcol[4 * q4 + 1];
              if (4 * q4 + 2 < r) acc[2] += a4.z * tcol[4 * q4 + 2];
              if (4 * q4 + 3 < r) acc[3] += a4.w * tcol[4 * q4 + 3];
            }
          }
          const float sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
          tcol[r] = (r == j) ? 1.f : (r > j ? -sum : 0.f);
        }
        if (j < 16) {
          float* td = blk + (10 + i) * BLK;
#pragma unroll
          for (int r = 0; r < 16; ++r) {
            td[r * BLD + j] = tcol[r];
            *reinterpret_cast<__nv_bfloat16*>(buf + B_T + swz_elem(16 * i + r, 16 * i + j)) = f2bf(tcol[r]);
          }
        }
        scale_items(SCALE_SPLIT, CH * 16, tid);
      } else {
        scale_items(0, SCALE_SPLIT, tid - 128);
      }
      named_bar(1);
      // ---- M_ik = T_ii A_ik for the six blocks below the diagonal (warps 0-5)
      if (warp < 6) {
        const int p = warp, i = p < 1 ? 1 : (p < 3 ? 2 : 3);
        float acc[2][4] = {};
        blk_mma(acc, blk + (10 + i) * BLK, blk + p * BLK, lane);
        blk_store(blk + (14 + p) * BLK, acc, 1.f, nullptr, 0, 0, lane);
      }
      named_bar(1);
      // ---- T_ij = -sum_{k=j}^{i-1} M_ik T_kj, one level of i - j at a time
#pragma unroll 1
      for (int d = 1; d < 4; ++d) {
        if (warp < 4 - d) {
          const int j = warp, i = warp + d;
          float acc[2][4] = {};
          for (int k = j; k < i; ++k)
            blk_mma(acc, blk + (14 + blk_lo(i, k)) * BLK, blk + (k == j ? 10 + j : blk_lo(k, j)) * BLK, lane);
          blk_store(blk + blk_lo(i, j) * BLK, acc, -1.f, buf + B_T, 16 * i, 16 * j, lane);
        }
        named_bar(1);
      }
      // ---- W = T (b e^G K), stored negated over b e^G K
      {
        float w[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i][0] = w[i][1] = w[i][2] = w[i][3] = 0.f;
#pragma unroll 1
        for (int ks = 0; ks <= mt; ++ks) {  // T is lower triangular by 16-row blocks
          uint32_t a[4];
          frag_a(sb + B_T, mt * 16, ks * 16, lane, a);
#pragma unroll
          for (int nt = 0; nt < 8; nt += 2) {
            uint32_t bq[4];
            frag_b_t(sb + B_W, nh * 64 + nt * 8, ks * 16, lane, bq);
            mma16816(w[nt], a, bq[0], bq[1]);
            mma16816(w[nt + 1], a, bq[2], bq[3]);
          }
        }
        named_bar(1);
        store_tile_bf16<8>(buf + B_W, w, mt * 16, nh * 64, lane, -1.f);
      }
      fence_proxy_async_smem();  // the tiles written here are read by tcgen05.mma (async proxy)
      mbar_arrive(&ready[b]);
    }
  } else {
    // =============================================================== state warps
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(STATE_REGS));
    const int sw = warp - 8, stid = tid - 256;
    const int quarter = warp & 3;                             // TMEM lanes 32 quarter .. + 31
    const int dv = 32 * quarter + lane;                       // the value row this thread owns
    const uint32_t lanes = (uint32_t)(32 * quarter) << 16;  // lane field of its TMEM addresses
    if (sw == 0) {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
    tc_fence_before();
    named_bar_n(3, 256);
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    float* Sg = state + ((int64_t)slot * HV + hv) * D * D;
    if (sw < 4) {
      // ------------------------------------------------------------- MMA warps 8-11
      {
        const float4* src = reinterpret_cast<const float4*>(Sg + (int64_t)dv * D);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 v = src[8 * j + i];
            r[4 * i] = __float_as_uint(v.x);
            r[4 * i + 1] = __float_as_uint(v.y);
            r[4 * i + 2] = __float_as_uint(v.z);
            r[4 * i + 3] = __float_as_uint(v.w);
          }
          tmem_st_32x32b_x32(tmem + lanes + T_S + 32 * j, r);
        }
        tmem_st_wait();
      }
      float rb[2] = {0.f, 0.f}, ra[2] = {0.f, 0.f};  // warp 8: raw gating inputs of chunk c + 2
      if (sw == 0) {
        // gating of chunks 0 and 1, then their loads (the load mbarrier publishes the gating
        // to the prep warps, gate_pub to the output warps)
        for (int c = 0; c < 2 && c < n_chunks; ++c) {
          load_gating_inputs(rb, ra, ba, ldba, t_begin, n, c, hv, HV, lane);
          chunk_gating(gbuf + c * GB_FLOATS, rb, ra, min(CH, n - c * CH), a_log, dtb, lane);
          __syncwarp();
          mbar_arrive(&gate_pub[c]);
        }
        __syncwarp();
        if (lane == 0) {
          tma_prefetch_desc(&tm_q);
          tma_prefetch_desc(&tm_k);
          tma_prefetch_desc(&tm_v);
          for (int c = 0; c < 2 && c < n_chunks; ++c)
            issue_chunk_loads(smem + c * BUF, &loaded[c], &tm_q, &tm_k, &tm_v, h, hv, t_begin + c * CH);
        }
        load_gating_inputs(rb, ra, ba, ldba, t_begin, n, 2, hv, HV, lane);
      }
      for (int c = 0; c < n_chunks; ++c) {
        const int b = c & 1;
        const uint32_t sb = s0 + b * BUF;
        const float* gb = gbuf + (c % GB_SLOTS) * GB_FLOATS;
        if (sw == 0 && c + 2 < n_chunks) {
          // gating of chunk c + 2 into the slot of chunk c - 2, which the output warps have
          // finished with (the MMA warps passed o_free of chunk c - 2 in the last iteration)
          const int g2 = (c + 2) % GB_SLOTS;
          chunk_gating(gbuf + g2 * GB_FLOATS, rb, ra, min(CH, n - (c + 2) * CH), a_log, dtb, lane);
          __syncwarp();
          mbar_arrive(&gate_pub[g2]);
          load_gating_inputs(rb, ra, ba, ldba, t_begin, n, c + 3, hv, HV, lane);
        }
        // ---- S after chunk c - 1: S0 = bf16(S) for this chunk's products, S <- e^{G_C} S
        // (e^{G_C} from this chunk's gating, which warp 8 may have written just now)
        mbar_wait(&gate_pub[c % GB_SLOTS], (c / GB_SLOTS) & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
        if (c > 0) mbar_wait(bar_s, (c - 1) & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
        tc_fence_after();
        {
          const float eC = gb[GB_EC];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t r[32], pk[16];
            tmem_ld_32x32b_x32(tmem + lanes + T_S + 32 * j, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * eC);
            tmem_st_32x32b_x16(tmem + lanes + T_S0 + 16 * j, pk);
            tmem_st_32x32b_x32(tmem + lanes + T_S + 32 * j, r);
          }
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_wait(&ready[b], (c >> 1) & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
        named_bar_n(4, 128);
        if (stid == 0) {
          tc_fence_after();
          // U^T = (bV)^T T^T + S0 (-W)^T
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16(tmem + T_U, umma_sdesc_mn_sw128(sb + B_V + ks * 2048, TILE / 2),
                      umma_sdesc_sw128(sb + B_T + ks * 32), IDESC_U_AMN, ks > 0 ? 1u : 0u);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_bf16_ts(tmem + T_U, tmem + T_S0 + ks * 8,
                         umma_sdesc_sw128(sb + B_W + (ks >> 2) * (TILE / 2) + (ks & 3) * 32), IDESC_N64, 1u);
          umma_commit(bar_u);
          // O1^T = S0 Q^T, once the output warps have read the previous chunk's O
          if (c > 0) mbar_wait(o_free, (c - 1) & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_bf16_ts(tmem + T_O1, tmem + T_S0 + ks * 8,
                         umma_sdesc_sw128(sb + B_Q + (ks >> 2) * (TILE / 2) + (ks & 3) * 32), IDESC_N64,
                         ks > 0 ? 1u : 0u);
        }
        // ---- U^T rounded to bf16 into TMEM: the A operand of O2^T and of the state update
        mbar_wait(bar_u, c & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t r[32], pk[16];
          tmem_ld_32x32b_x32(tmem + lanes + T_U + 32 * j, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
          tmem_st_32x32b_x16(tmem + lanes + T_UB + 16 * j, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        named_bar_n(4, 128);
        if (stid == 0) {
          tc_fence_after();
          // O2^T = U^T P^T, then S += U^T (e^{G_C-G} K)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16_ts(tmem + T_O2, tmem + T_UB + ks * 8, umma_sdesc_sw128(sb + B_P + ks * 32), IDESC_N64,
                         ks > 0 ? 1u : 0u);
          umma_commit(bar_o);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16_ts(tmem + T_S, tmem + T_UB + ks * 8, umma_sdesc_mn_sw128(sb + B_K + ks * 2048, TILE / 2),
                         IDESC_S_BMN, 1u);
          umma_commit(bar_s);
          if (c + 2 < n_chunks) {
            // every product reading buffer b is complete once the state update is: refill it
            mbar_wait(bar_s, c & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
            fence_proxy_async_smem();
            if (!*abort_flag)
              issue_chunk_loads(smem + b * BUF, &loaded[b], &tm_q, &tm_k, &tm_v, h, hv, t_begin + (c + 2) * CH);
          }
        }
      }
      // ---- final state, in place
      if (n_chunks > 0) mbar_wait(bar_s, (n_chunks - 1) & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
      tc_fence_after();
      {
        float4* dst = reinterpret_cast<float4*>(Sg + (int64_t)dv * D);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lanes + T_S + 32 * j, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[8 * j + i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                         __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
        }
      }
      tc_fence_before();
    } else {
      // ------------------------------------------------------------- output warps 12-15
      const int otid = tid - 384;
      float* sRed = reinterpret_cast<float*>(smem + S_RED);  // [4][64] sums of squares
      float* sRstd = sRed + 4 * CH;
      const float wdv = bf2f(norm_w[dv]);
      // z tile of chunk c: row t = token t (256 bytes), filled by 16-byte copies
      auto prefetch_z = [&](int c) {
        const int64_t tz = t_begin + (int64_t)c * CH;
        const int ncz = min(CH, n - c * CH);
        const uint32_t base = s0 + S_Z + (c & 1) * ZBUF;
        for (int i = otid; i < CH * 16; i += 128) {
          const int t = i >> 4, part = i & 15;
          const bool ok = t < ncz;
          cpa16(base + t * 256 + part * 16, z + (tz + (ok ? t : 0)) * ldz + (int64_t)hv * D + part * 8, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
      };
      if (n_chunks > 0) prefetch_z(0);
      for (int c = 0; c < n_chunks; ++c) {
        const int nc = min(CH, n - c * CH);
        const int64_t tc = t_begin + (int64_t)c * CH;
        if (c + 1 < n_chunks) prefetch_z(c + 1);  // into the tile chunk c - 1 used
        const float* gb = gbuf + (c % GB_SLOTS) * GB_FLOATS;
        mbar_wait(&gate_pub[c % GB_SLOTS], (c / GB_SLOTS) & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
        mbar_wait(bar_o, c & 1, abort_flag, err, QW_DEV_ERR_TIMEOUT_GDN);
        tc_fence_after();
        // ---- o = bf16(scale e^G O1 + O2): this thread's value row for the 64 tokens
        float o[CH];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t r1[32], r2[32];
          tmem_ld_32x32b_x32(tmem + lanes + T_O1 + 32 * j, r1);
          tmem_ld_32x32b_x32(tmem + lanes + T_O2 + 32 * j, r2);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            o[32 * j + i] =
                bf16_round(__uint_as_float(r1[i]) * (scale * gb[GB_EG + 32 * j + i]) + __uint_as_float(r2[i]));
        }
        tc_fence_before();
        mbar_arrive(o_free);
        // ---- sum of o^2 over the 128 value rows of each token: halving exchange in the warp
        // (lane l ends with tokens 2l and 2l + 1), then the four warps through shared memory
        {
          float a[CH];
#pragma unroll
          for (int i = 0; i < CH; ++i) a[i] = o[i] * o[i];
          halve<32>(a, lane, 16);
          halve<16>(a, lane, 8);
          halve<8>(a, lane, 4);
          halve<4>(a, lane, 2);
          halve<2>(a, lane, 1);
          *reinterpret_cast<float2*>(sRed + quarter * CH + 2 * lane) = make_float2(a[0], a[1]);
        }
        named_bar_n(5, 128);
        if (otid < CH)
          sRstd[otid] = rsqrtf(((sRed[otid] + sRed[CH + otid]) + (sRed[2 * CH + otid] + sRed[3 * CH + otid])) /
                                   (float)D + eps);
        if (c + 1 < n_chunks) asm volatile("cp.async.wait_group 1;" ::: "memory");  // this chunk's z
        else asm volatile("cp.async.wait_group 0;" ::: "memory");
        named_bar_n(5, 128);
        // ---- y = o rstd w silu(z), written over z in the staging tile
        uint8_t* zt = smem + S_Z + (c & 1) * ZBUF;
#pragma unroll
        for (int t = 0; t < CH; ++t) {
          __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(zt + t * 256) + dv;
          const float zv = bf2f(*p);
          *p = f2bf(o[t] * sRstd[t] * wdv * __fdividef(zv, 1.f + __expf(-zv)));
        }
        named_bar_n(5, 128);
        for (int i = otid; i < CH * 16; i += 128) {
          const int t = i >> 4, part = i & 15;
          if (t < nc)
            *reinterpret_cast<uint4*>(y + (tc + t) * ldy + (int64_t)hv * D + part * 8) =
                *reinterpret_cast<const uint4*>(zt + t * 256 + part * 16);
        }
        named_bar_n(5, 128);  // the tile is refilled by the prefetch of chunk c + 2
      }
    }
  }
  __syncthreads();
  if (tid == 0 && *abort_flag) {
    // a wait gave up: leave time for any bulk copy or tensor-core product still in flight
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 200000ull) {
    }
  }
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(*tmem_slot, TMEM_COLS);
  }
}

}  // namespace qw

using namespace qw;

extern "C" int qw_gdn_prefill(const void* q, const void* k, const void* v, const void* ba, int64_t ldba,
                              const float* A_log, const void* dt_bias, const int32_t* cu_seqlens,
                              const int32_t* slots, int64_t B, int64_t T, int64_t n_slots, float* state,
                              const void* z, int64_t ldz, const void* norm_w, void* y, int64_t ldy, int64_t H,
                              int64_t HV, int64_t dk, int64_t dv, float scale, float eps, qw_stream_t stream) {
  QW_CHECK_ARG(q && k && v && ba && A_log && dt_bias && cu_seqlens && slots && state && z && norm_w && y, QW_ERR_ARG);
  QW_CHECK_ARG(B > 0 && T > 0 && T < (1ll << 31) && H > 0 && HV % H == 0 && n_slots > 0 && B <= 65535, QW_ERR_ARG);
  if (dk != gdn::D || dv != gdn::D) return QW_ERR_UNSUPPORTED;
  QW_CHECK_ARG(((uintptr_t)q % 16) == 0 && ((uintptr_t)k % 16) == 0 && ((uintptr_t)v % 16) == 0 &&
                   ((uintptr_t)state % 16) == 0 && ((uintptr_t)y % 16) == 0 && (ldy % 8) == 0 &&
                   ((uintptr_t)z % 16) == 0 && (ldz % 8) == 0,
               QW_ERR_ALIGN);
  CUtensorMap tq, tk, tv;
  if (!tmap_bf16_2d_sw128(&tq, q, T, H * dk, H * dk, 64, gdn::CH) ||
      !tmap_bf16_2d_sw128(&tk, k, T, H * dk, H * dk, 64, gdn::CH) ||
      !tmap_bf16_2d_sw128(&tv, v, T, HV * dv, HV * dv, 64, gdn::CH))
    return QW_ERR_DRIVER;
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  static bool cfg = false;
  if (!cfg) {
    cudaFuncSetAttribute(gdn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gdn::SMEM);
    cfg = true;
  }
  dim3 grid((unsigned)HV, (unsigned)B);
  gdn_prefill_kernel<<<grid, 512, gdn::SMEM, s>>>(
      tq, tk, tv, static_cast<const __nv_bfloat16*>(ba), ldba, A_log, static_cast<const __nv_bfloat16*>(dt_bias),
      cu_seqlens, slots, (int)n_slots, state, static_cast<const __nv_bfloat16*>(z), ldz,
      static_cast<const __nv_bfloat16*>(norm_w), static_cast<__nv_bfloat16*>(y), ldy, (int)H, (int)HV, scale, eps,
      device_error_ptr());
  QW_LAUNCH_CHECK();
  return QW_OK;
}
