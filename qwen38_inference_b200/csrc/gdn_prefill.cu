// Chunked gated delta rule for prefill (replaces flashinfer chunk_gated_delta_rule,
// REF:4852/5084, plus the gating kernel REF:1258-1323 and the state gather/scatter
// REF:5082-5085: the state is read and written in place at the request's slot).
//
// Recurrence per token t (state S is [dv, dk], fp32):
//   S_t = a_t S_{t-1} (I - b_t k_t k_t^T) + b_t v_t k_t^T,   o_t = S_t q_t * scale
// with a_t = exp(g_t), g_t = -exp(A_log) softplus(a + dt_bias), b_t = bf16(sigmoid(b)).
// Chunk form (C = 64 tokens, G = within-chunk cumsum of g, S0 = state before the chunk):
//   A_ts = b_t e^{G_t - G_s} k_t.k_s (s < t),   T = (I + A)^-1
//   W = T diag(b e^G) K,   U = T diag(b) V - W S0^T
//   O = scale (diag(e^G) Q S0^T + [s <= t] e^{G_t - G_s} (Q K^T) U)
//   S_C = e^{G_C} S0 + U^T diag(e^{G_C - G}) K
// The 64 x 64 and 64 x 128 products run on tensor cores (mma.sync m16n8k16, bf16 operands,
// fp32 accumulation); T is a blocked fp32 forward substitution; S stays in registers as
// the accumulator of the state update across all chunks of the sequence.
// One CTA (8 warps) per (sequence, value head).
#include "common.cuh"

namespace qw {

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
QW_DEV void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
QW_DEV void cpa16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0) : "memory");
}

// swizzled byte offset of 16-byte chunk c of row r in a tile with RL bf16 per row
template <int RL>
QW_DEV uint32_t sw(int r, int c) {
  return (uint32_t)(r * RL * 2 + ((c ^ (r & 7)) << 4));
}
template <int RL>
QW_DEV uint32_t sw_elem(int r, int col) {  // byte offset of element (r, col)
  return sw<RL>(r, col >> 3) + ((col & 7) << 1);
}
// A fragment, tile stored [M][K]
template <int RL>
QW_DEV void frag_a(uint32_t base, int m0, int k0, int lane, uint32_t* a) {
  ldsm_x4(base + sw<RL>(m0 + (lane & 15), (k0 >> 3) + (lane >> 4)), a);
}
// A fragment, tile stored [K][M]
template <int RL>
QW_DEV void frag_a_t(uint32_t base, int m0, int k0, int lane, uint32_t* a) {
  ldsm_x4_t(base + sw<RL>(k0 + (lane & 7) + ((lane >> 4) << 3), (m0 >> 3) + ((lane >> 3) & 1)), a);
}
// B fragments of n-tiles n0 and n0+8: b[0],b[1] (tile n0), b[2],b[3] (tile n0+8); tile stored [N][K]
template <int RL>
QW_DEV void frag_b(uint32_t base, int n0, int k0, int lane, uint32_t* b) {
  ldsm_x4(base + sw<RL>(n0 + (lane & 7) + ((lane >> 4) << 3), (k0 >> 3) + ((lane >> 3) & 1)), b);
}
// same, tile stored [K][N]
template <int RL>
QW_DEV void frag_b_t(uint32_t base, int n0, int k0, int lane, uint32_t* b) {
  ldsm_x4_t(base + sw<RL>(k0 + (lane & 7) + (((lane >> 3) & 1) << 3), (n0 >> 3) + (lane >> 4)), b);
}
// acc[NT][4] += A(16 x 16*KS at rows m0) * B(16*KS x 8*NT at cols n0)
template <int NT, int KS, int RLA, int RLB, bool AT, bool BT>
QW_DEV void mma_tile(float (*acc)[4], uint32_t sa, uint32_t sb, int m0, int n0, int lane) {
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    uint32_t a[4];
    if constexpr (AT) frag_a_t<RLA>(sa, m0, ks * 16, lane, a);
    else frag_a<RLA>(sa, m0, ks * 16, lane, a);
#pragma unroll
    for (int nt = 0; nt < NT; nt += 2) {
      uint32_t b[4];
      if constexpr (BT) frag_b_t<RLB>(sb, n0 + nt * 8, ks * 16, lane, b);
      else frag_b<RLB>(sb, n0 + nt * 8, ks * 16, lane, b);
      mma16816(acc[nt], a, b[0], b[1]);
      mma16816(acc[nt + 1], a, b[2], b[3]);
    }
  }
}
// store a 16 x 8*NT accumulator tile as bf16 (times `mul`) into a swizzled [rows][RL] tile
template <int NT, int RL>
QW_DEV void store_tile_bf16(uint8_t* smem_base, float (*acc)[4], int m0, int n0, int lane, float mul) {
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int col = n0 + nt * 8 + c * 2;
    *reinterpret_cast<uint32_t*>(smem_base + sw_elem<RL>(m0 + g, col)) = pack_bf16x2(acc[nt][0] * mul, acc[nt][1] * mul);
    *reinterpret_cast<uint32_t*>(smem_base + sw_elem<RL>(m0 + g + 8, col)) =
        pack_bf16x2(acc[nt][2] * mul, acc[nt][3] * mul);
  }
}
constexpr int CH = 64;   // chunk length
constexpr int DKc = 128; // key / value head dim
constexpr int LDA = 65;  // fp32 row stride of the A / T matrices

struct GdnSmem {
  static constexpr int TILE = CH * DKc * 2;       // 16 KB
  static constexpr int QKV = 0;                   // [2 buffers][Q | K | V]
  static constexpr int KB = QKV + 6 * TILE;       // b e^G K, later e^{G_C-G} K
  static constexpr int R = KB + TILE;             // A32 | T32 during the inverse; then -W | U
  static constexpr int W = R;
  static constexpr int U = R + TILE;
  static constexpr int A32 = R;
  static constexpr int T32 = R + CH * LDA * 4;
  static constexpr int R_BYTES = 2 * CH * LDA * 4;  // >= 2 * TILE
  static constexpr int S = R + R_BYTES;           // S0 bf16 [dv][dk], 32 KB
  static constexpr int P = S + 2 * TILE;          // [t][s] bf16, 8 KB
  static constexpr int T = P + CH * CH * 2;
  static constexpr int X32 = T + CH * CH * 2;     // 6 x 16 x 16 fp32 scratch (T_ii A_ik)
  static constexpr int VEC = X32 + 6 * 256 * 4;   // G, eG, eGl, beta: 4 x 64 fp32; row sums 4 x 64
  static constexpr int ZLD = DKc + 8;             // padded row of the z tile (bf16)
  static constexpr int Z = VEC + 8 * CH * 4;      // z rows of the chunk [64][ZLD] bf16
  static constexpr int TOTAL = Z + CH * ZLD * 2;
};
static_assert(GdnSmem::R_BYTES >= 2 * GdnSmem::TILE, "W and U must fit in the inverse's scratch");

// Issue the loads of chunk `ch` (rows beyond the request are zero-filled) into buffer `b`.
template <int NTHR>
QW_DEV void gdn_load_chunk(uint32_t s0, int b, const __nv_bfloat16* q, const __nv_bfloat16* k,
                           const __nv_bfloat16* v, int64_t tc, int nc, int h, int hv, int H, int HV, int tid) {
  const uint32_t base = s0 + GdnSmem::QKV + b * 3 * GdnSmem::TILE;
  for (int i = tid; i < CH * 16; i += NTHR) {
    const int r = i >> 4, c = i & 15;
    const bool ok = r < nc;
    const int64_t t = tc + (ok ? r : 0);
    cpa16(base + sw<DKc>(r, c), q + (t * H + h) * DKc + c * 8, ok);
    cpa16(base + GdnSmem::TILE + sw<DKc>(r, c), k + (t * H + h) * DKc + c * 8, ok);
    cpa16(base + 2 * GdnSmem::TILE + sw<DKc>(r, c), v + (t * HV + hv) * DKc + c * 8, ok);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// NW warps per CTA (8 or 16): the 64-row products are split into 4 m-tiles x NW/4 column
// groups, the 128 x 128 state into 8 m-tiles x NW/8 column groups.
template <int NW>
__global__ void __launch_bounds__(NW * 32, 1) gdn_prefill_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const __nv_bfloat16* __restrict__ ba, int64_t ldba, const float* __restrict__ A_log,
    const __nv_bfloat16* __restrict__ dt_bias, const int32_t* __restrict__ cu, const int32_t* __restrict__ slots,
    int n_slots, float* __restrict__ state, const __nv_bfloat16* __restrict__ z, int64_t ldz,
    const __nv_bfloat16* __restrict__ norm_w, __nv_bfloat16* __restrict__ y, int64_t ldy, int H, int HV, float scale,
    float eps, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t s0 = smem_u32(smem);
  float* A32 = reinterpret_cast<float*>(smem + GdnSmem::A32);
  float* T32 = reinterpret_cast<float*>(smem + GdnSmem::T32);
  float* X32 = reinterpret_cast<float*>(smem + GdnSmem::X32);
  float* sG = reinterpret_cast<float*>(smem + GdnSmem::VEC);
  float* sEG = sG + CH;
  float* sEGl = sEG + CH;
  float* sBeta = sEGl + CH;
  float* sSS = sBeta + CH;  // [NW/4][64] partial sums of squares of the output rows
  constexpr int NT_ = NW * 32;          // threads
  constexpr int NQ = NW / 4;            // column groups of the 64-row products
  constexpr int KK_NT = 8 / NQ;         // n-tiles per warp, 64-column outputs
  constexpr int V_NT = 16 / NQ;         // n-tiles per warp, 128-column outputs
  constexpr int S_NT = 16 / (NW / 8);   // n-tiles per warp of the state

  const int seq = blockIdx.x, hv = blockIdx.y;
  const int h = hv / (HV / H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g4 = lane >> 2, c4 = lane & 3;
  const int t_begin = cu[seq], n = cu[seq + 1] - t_begin;
  const int slot = slots[seq];
  if (slot < 0 || slot >= n_slots) {
    if (tid == 0) set_error(err, QW_DEV_ERR_INDEX);
    return;
  }
  float* Sg = state + ((int64_t)slot * HV + hv) * DKc * DKc;
  const float a_log = expf(A_log[hv]);
  const float dtb = bf2f(dt_bias[hv]);
  const int n_chunks = (n + CH - 1) / CH;
  gdn_load_chunk<NT_>(s0, 0, q, k, v, t_begin, min(CH, n), h, hv, H, HV, tid);
  const __nv_bfloat16* zrow = z + (int64_t)hv * DKc;
  const int mt = warp & 3, nh = warp >> 2;  // 64-row products: m-tile and column group
  uint32_t wpair[V_NT];  // norm weight pairs of this thread's output columns
#pragma unroll
  for (int nt = 0; nt < V_NT; ++nt)
    wpair[nt] = *reinterpret_cast<const uint32_t*>(norm_w + nh * (V_NT * 8) + nt * 8 + c4 * 2);

  // state accumulator: warp w owns dv rows [16 (w % 8), +16) and dk columns of group w / 8
  const int smt = warp & 7, sng = warp >> 3;
  float sacc[S_NT][4];
#pragma unroll
  for (int nt = 0; nt < S_NT; ++nt) {
    const int col = sng * (S_NT * 8) + nt * 8 + c4 * 2;
    const float2 lo = *reinterpret_cast<const float2*>(Sg + (int64_t)(smt * 16 + g4) * DKc + col);
    const float2 hi = *reinterpret_cast<const float2*>(Sg + (int64_t)(smt * 16 + g4 + 8) * DKc + col);
    sacc[nt][0] = lo.x;
    sacc[nt][1] = lo.y;
    sacc[nt][2] = hi.x;
    sacc[nt][3] = hi.y;
  }
  store_tile_bf16<S_NT, DKc>(smem + GdnSmem::S, sacc, smt * 16, sng * (S_NT * 8), lane, 1.f);

  // blocks of T above the diagonal stay zero for every chunk
  for (int e = tid; e < CH * CH; e += NT_) {
    const int r = e / CH, c = e % CH;
    if ((c >> 4) > (r >> 4))
      *reinterpret_cast<__nv_bfloat16*>(smem + GdnSmem::T + sw_elem<CH>(r, c)) = f2bf(0.f);
  }
  // raw b, a of the gating for token tid of the chunk, loaded one chunk ahead
  float g_b = 0.f, g_a = 0.f;
  if (tid < CH && tid < n) {
    g_b = bf2f(ba[(int64_t)(t_begin + tid) * ldba + hv]);
    g_a = bf2f(ba[(int64_t)(t_begin + tid) * ldba + HV + hv]);
  }
  for (int ch = 0; ch < n_chunks; ++ch) {
    const int tc = t_begin + ch * CH;
    const int nc = min(CH, n - ch * CH);
    const int b = ch & 1;
    const float cur_b = g_b, cur_a = g_a;
    if (tid < CH) {
      g_b = g_a = 0.f;
      if ((ch + 1) * CH + tid < n) {
        g_b = bf2f(ba[(int64_t)(tc + CH + tid) * ldba + hv]);
        g_a = bf2f(ba[(int64_t)(tc + CH + tid) * ldba + HV + hv]);
      }
    }
    const uint32_t sQ = s0 + GdnSmem::QKV + b * 3 * GdnSmem::TILE;
    const uint32_t sK = sQ + GdnSmem::TILE, sV = sK + GdnSmem::TILE;
    uint8_t* pK = smem + GdnSmem::QKV + b * 3 * GdnSmem::TILE + GdnSmem::TILE;
    uint8_t* pV = pK + GdnSmem::TILE;
    // z rows of this chunk (consumed by the epilogue), then the next chunk's q/k/v into the
    // other buffer (its previous contents are dead)
    for (int i = tid; i < CH * 16; i += NT_) {
      const int r = i >> 4, c = i & 15;
      const bool ok = r < nc;
      cpa16(s0 + GdnSmem::Z + (uint32_t)(r * GdnSmem::ZLD + c * 8) * 2, zrow + (int64_t)(tc + (ok ? r : 0)) * ldz + c * 8, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (ch + 1 < n_chunks) {
      gdn_load_chunk<NT_>(s0, b ^ 1, q, k, v, tc + CH, min(CH, n - (ch + 1) * CH), h, hv, H, HV, tid);
    } else {
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // gating (threads 0..63) and the within-chunk cumulative log decay
    if (tid < CH) {
      float gg = 0.f, bb = 0.f;
      if (tid < nc) {
        const float xa = cur_a + dtb;
        const float sp = xa <= 20.f ? logf(1.f + expf(xa)) : xa;
        gg = -a_log * sp;
        bb = bf16_round(1.f / (1.f + expf(-cur_b)));
      }
      sBeta[tid] = bb;
      float x = gg;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float yv = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += yv;
      }
      sG[tid] = x;
    }
    asm volatile("cp.async.wait_group 2;" ::: "memory");  // this chunk's q/k/v tiles have landed
    __syncthreads();
    if (tid >= 32 && tid < CH) sG[tid] += sG[31];
    __syncthreads();
    const float G_last = sG[CH - 1];
    if (tid < CH) {
      sEG[tid] = expf(sG[tid]);
      sEGl[tid] = expf(G_last - sG[tid]);
    }
    // ---------------------------------------------------------------- K K^T -> A,  Q K^T -> P
    {
      float kk[KK_NT][4], qk[KK_NT][4];
#pragma unroll
      for (int i = 0; i < KK_NT; ++i) kk[i][0] = kk[i][1] = kk[i][2] = kk[i][3] = qk[i][0] = qk[i][1] = qk[i][2] = qk[i][3] = 0.f;
      mma_tile<KK_NT, 8, DKc, DKc, false, false>(kk, sK, sK, mt * 16, nh * (KK_NT * 8), lane);
      mma_tile<KK_NT, 8, DKc, DKc, false, false>(qk, sQ, sK, mt * 16, nh * (KK_NT * 8), lane);
#pragma unroll
      for (int nt = 0; nt < KK_NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = mt * 16 + g4 + ((e >> 1) << 3);
          const int s = nh * (KK_NT * 8) + nt * 8 + c4 * 2 + (e & 1);
          const float dec = (s <= t) ? expf(sG[t] - sG[s]) : 0.f;
          A32[t * LDA + s] = (s < t) ? sBeta[t] * dec * kk[nt][e] : 0.f;
          qk[nt][e] = (s <= t) ? scale * dec * qk[nt][e] : 0.f;
        }
      }
      store_tile_bf16<KK_NT, CH>(smem + GdnSmem::P, qk, mt * 16, nh * (KK_NT * 8), lane, 1.f);
    }
    __syncthreads();

    // ---------------------------------------------------------------- T = (I + A)^-1, blocked
    if (warp < 4) {
      // invert the unit lower-triangular diagonal block b = warp; lane j < 16 owns column j
      const int bb = warp, j = lane;
      float tcol[16];
      const float* arow = A32 + (bb * 16) * LDA + bb * 16;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        // row i of the block: i broadcast loads issued together, then a predicated dot
        // product with the column computed so far (T[k][j] = 0 for k < j)
        float a[16];
#pragma unroll
        for (int kx = 0; kx < i; ++kx) a[kx] = arow[i * LDA + kx];
        float acc = 0.f;
#pragma unroll
        for (int kx = 0; kx < i; ++kx) acc += (kx >= j) ? a[kx] * tcol[kx] : 0.f;
        tcol[i] = (i == j) ? 1.f : (i > j ? -acc : 0.f);
      }
      if (j < 16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          T32[(bb * 16 + i) * LDA + bb * 16 + j] = tcol[i];
          *reinterpret_cast<__nv_bfloat16*>(smem + GdnSmem::T + sw_elem<CH>(bb * 16 + i, bb * 16 + j)) = f2bf(tcol[i]);
        }
      }
    } else {
      // meanwhile: b e^G K into KB and b V in place (inputs of W and U)
      for (int i = tid - 128; i < CH * 16; i += NT_ - 128) {
        const int r = i >> 4, c = i & 15;
        float kf[8], vf[8];
        load_bf16x8(reinterpret_cast<const __nv_bfloat16*>(pK + sw<DKc>(r, c)), kf);
        load_bf16x8(reinterpret_cast<const __nv_bfloat16*>(pV + sw<DKc>(r, c)), vf);
        const float fk = sBeta[r] * sEG[r], fv = sBeta[r];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          kf[jj] *= fk;
          vf[jj] *= fv;
        }
        store_bf16x8(reinterpret_cast<__nv_bfloat16*>(smem + GdnSmem::KB + sw<DKc>(r, c)), kf);
        store_bf16x8(reinterpret_cast<__nv_bfloat16*>(pV + sw<DKc>(r, c)), vf);
      }
    }
    __syncthreads();
    // below-diagonal blocks: with M_ik = T_ii A_ik, T_ij = -sum_{k=j}^{i-1} M_ik T_kj.
    // M for the six blocks (1,0) (2,0) (2,1) (3,0) (3,1) (3,2) in one pass, then one pass
    // per distance i - j; each T_ij goes to T32 (read by later levels) and to bf16 T.
    for (int e = tid; e < 6 * 256; e += NT_) {
      const int pi = e >> 8, r = (e >> 4) & 15, c = e & 15;
      const int i = pi < 1 ? 1 : (pi < 3 ? 2 : 3);
      const int kk = pi < 1 ? 0 : (pi < 3 ? pi - 1 : pi - 3);
      float acc = 0.f;
#pragma unroll
      for (int x = 0; x < 16; ++x) acc += T32[(i * 16 + r) * LDA + i * 16 + x] * A32[(i * 16 + x) * LDA + kk * 16 + c];
      X32[pi * 256 + r * 16 + c] = acc;
    }
    __syncthreads();
#pragma unroll 1
    for (int d = 1; d < 4; ++d) {
      const int nb = 4 - d;  // number of blocks at this distance
      for (int e = tid; e < nb * 256; e += NT_) {
        const int bi = e >> 8, r = (e >> 4) & 15, c = e & 15;
        const int j = bi, i = bi + d;
        float acc = 0.f;
        for (int kb = j; kb < i; ++kb) {
          const int pi = (i == 1) ? 0 : (i == 2 ? 1 + kb : 3 + kb);  // M_{i,kb}
#pragma unroll
          for (int x = 0; x < 16; ++x) acc += X32[pi * 256 + r * 16 + x] * T32[(kb * 16 + x) * LDA + j * 16 + c];
        }
        T32[(i * 16 + r) * LDA + j * 16 + c] = -acc;
        *reinterpret_cast<__nv_bfloat16*>(smem + GdnSmem::T + sw_elem<CH>(i * 16 + r, j * 16 + c)) = f2bf(-acc);
      }
      __syncthreads();
    }

    // ---------------------------------------------------------------- W = T (b e^G K), stored negated
    {
      float w[V_NT][4];
#pragma unroll
      for (int i = 0; i < V_NT; ++i) w[i][0] = w[i][1] = w[i][2] = w[i][3] = 0.f;
      mma_tile<V_NT, 4, CH, DKc, false, true>(w, s0 + GdnSmem::T, s0 + GdnSmem::KB, mt * 16, nh * (V_NT * 8), lane);
      store_tile_bf16<V_NT, DKc>(smem + GdnSmem::W, w, mt * 16, nh * (V_NT * 8), lane, -1.f);
    }
    __syncthreads();
    // ---------------------------------------------------------------- U = T (b V) - W S0^T
    {
      float u[V_NT][4];
#pragma unroll
      for (int i = 0; i < V_NT; ++i) u[i][0] = u[i][1] = u[i][2] = u[i][3] = 0.f;
      mma_tile<V_NT, 4, CH, DKc, false, true>(u, s0 + GdnSmem::T, sV, mt * 16, nh * (V_NT * 8), lane);
      mma_tile<V_NT, 8, DKc, DKc, false, false>(u, s0 + GdnSmem::W, s0 + GdnSmem::S, mt * 16, nh * (V_NT * 8), lane);
      store_tile_bf16<V_NT, DKc>(smem + GdnSmem::U, u, mt * 16, nh * (V_NT * 8), lane, 1.f);
    }
    __syncthreads();
    // ---------------------------------------------------------------- O, gated RMSNorm; e^{G_C - G} K into KB
    {
      float o[V_NT][4];
#pragma unroll
      for (int i = 0; i < V_NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      mma_tile<V_NT, 8, DKc, DKc, false, false>(o, sQ, s0 + GdnSmem::S, mt * 16, nh * (V_NT * 8), lane);
      const float f0 = scale * sEG[mt * 16 + g4], f1 = scale * sEG[mt * 16 + g4 + 8];
#pragma unroll
      for (int i = 0; i < V_NT; ++i) {
        o[i][0] *= f0;
        o[i][1] *= f0;
        o[i][2] *= f1;
        o[i][3] *= f1;
      }
      mma_tile<V_NT, 4, CH, DKc, false, true>(o, s0 + GdnSmem::P, s0 + GdnSmem::U, mt * 16, nh * (V_NT * 8), lane);
      // o rounds to bf16 (the reference's GDN output dtype), then y = o rstd w z sigmoid(z)
      float ss[2] = {0.f, 0.f};
#pragma unroll
      for (int i = 0; i < V_NT; ++i) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o[i][e] = bf16_round(o[i][e]);
          ss[e >> 1] += o[i][e] * o[i][e];
        }
      }
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        ss[rr] += __shfl_xor_sync(0xffffffffu, ss[rr], 1);
        ss[rr] += __shfl_xor_sync(0xffffffffu, ss[rr], 2);
      }
      if (c4 == 0) {
        sSS[nh * CH + mt * 16 + g4] = ss[0];
        sSS[nh * CH + mt * 16 + g4 + 8] = ss[1];
      }
      for (int i = tid; i < CH * 16; i += NT_) {
        const int r = i >> 4, c = i & 15;
        float kf[8];
        load_bf16x8(reinterpret_cast<const __nv_bfloat16*>(pK + sw<DKc>(r, c)), kf);
        const float f = sEGl[r];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) kf[jj] *= f;
        store_bf16x8(reinterpret_cast<__nv_bfloat16*>(smem + GdnSmem::KB + sw<DKc>(r, c)), kf);
      }
      asm volatile("cp.async.wait_group 1;" ::: "memory");  // this chunk's z rows
      __syncthreads();
      const __nv_bfloat16* sZ = reinterpret_cast<const __nv_bfloat16*>(smem + GdnSmem::Z);
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int t = mt * 16 + g4 + rr * 8;
        if (t >= nc) continue;
        float ssum = 0.f;
#pragma unroll
        for (int gq = 0; gq < NQ; ++gq) ssum += sSS[gq * CH + t];
        const float rstd = rsqrtf(ssum / (float)DKc + eps);
        const int64_t tok = tc + t;
        const __nv_bfloat16* zr = sZ + t * GdnSmem::ZLD + nh * (V_NT * 8);
        __nv_bfloat16* dst = y + tok * ldy + (int64_t)hv * DKc + nh * (V_NT * 8);
#pragma unroll
        for (int nt = 0; nt < V_NT; ++nt) {
          const int col = nt * 8 + c4 * 2;
          float z0, z1, w0, w1;
          unpack_bf16x2(*reinterpret_cast<const uint32_t*>(zr + col), z0, z1);
          unpack_bf16x2(wpair[nt], w0, w1);
          const float y0 = o[nt][rr * 2] * rstd * w0 * (z0 / (1.f + __expf(-z0)));
          const float y1 = o[nt][rr * 2 + 1] * rstd * w1 * (z1 / (1.f + __expf(-z1)));
          *reinterpret_cast<uint32_t*>(dst + col) = pack_bf16x2(y0, y1);
        }
      }
    }
    // ---------------------------------------------------------------- S <- e^{G_C} S + U^T (e^{G_C-G} K)
    {
      const float eC = expf(G_last);
#pragma unroll
      for (int nt = 0; nt < S_NT; ++nt) {
        sacc[nt][0] *= eC;
        sacc[nt][1] *= eC;
        sacc[nt][2] *= eC;
        sacc[nt][3] *= eC;
      }
      mma_tile<S_NT, 4, DKc, DKc, true, true>(sacc, s0 + GdnSmem::U, s0 + GdnSmem::KB, smt * 16, sng * (S_NT * 8), lane);
      store_tile_bf16<S_NT, DKc>(smem + GdnSmem::S, sacc, smt * 16, sng * (S_NT * 8), lane, 1.f);
    }
    __syncthreads();
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  // ---------------------------------------------------------------- final state, in place
#pragma unroll
  for (int nt = 0; nt < S_NT; ++nt) {
    const int col = sng * (S_NT * 8) + nt * 8 + c4 * 2;
    *reinterpret_cast<float2*>(Sg + (int64_t)(smt * 16 + g4) * DKc + col) = make_float2(sacc[nt][0], sacc[nt][1]);
    *reinterpret_cast<float2*>(Sg + (int64_t)(smt * 16 + g4 + 8) * DKc + col) = make_float2(sacc[nt][2], sacc[nt][3]);
  }
}

}  // namespace qw

using namespace qw;

extern "C" int qw_gdn_prefill(const void* q, const void* k, const void* v, const void* ba, int64_t ldba,
                              const float* A_log, const void* dt_bias, const int32_t* cu_seqlens,
                              const int32_t* slots, int64_t B, int64_t n_slots, float* state, const void* z,
                              int64_t ldz, const void* norm_w, void* y, int64_t ldy, int64_t H, int64_t HV,
                              int64_t dk, int64_t dv, float scale, float eps, qw_stream_t stream) {
  QW_CHECK_ARG(q && k && v && ba && A_log && dt_bias && cu_seqlens && slots && state && z && norm_w && y, QW_ERR_ARG);
  QW_CHECK_ARG(B > 0 && H > 0 && HV % H == 0 && n_slots > 0, QW_ERR_ARG);
  if (dk != 128 || dv != 128) return QW_ERR_UNSUPPORTED;
  QW_CHECK_ARG(((uintptr_t)q % 16) == 0 && ((uintptr_t)k % 16) == 0 && ((uintptr_t)v % 16) == 0 &&
                   ((uintptr_t)state % 16) == 0 && ((uintptr_t)y % 4) == 0 &&
                   ((uintptr_t)z % 16) == 0 && (ldz % 8) == 0 && (ldy % 2) == 0,
               QW_ERR_ALIGN);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  constexpr int NW = 16;
  static bool cfg = false;
  if (!cfg) {
    cudaFuncSetAttribute(gdn_prefill_kernel<NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, GdnSmem::TOTAL);
    cfg = true;
  }
  dim3 grid((unsigned)B, (unsigned)HV);
  gdn_prefill_kernel<NW><<<grid, NW * 32, GdnSmem::TOTAL, s>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
      static_cast<const __nv_bfloat16*>(ba), ldba, A_log, static_cast<const __nv_bfloat16*>(dt_bias), cu_seqlens,
      slots, (int)n_slots, state, static_cast<const __nv_bfloat16*>(z), ldz,
      static_cast<const __nv_bfloat16*>(norm_w), static_cast<__nv_bfloat16*>(y), ldy, (int)H, (int)HV, scale, eps,
      device_error_ptr());
  QW_LAUNCH_CHECK();
  return QW_OK;
}
