// Gated GQA attention over the slot-contiguous paged KV cache.
//
//   qw_qk_norm_rope_store  per-head Gemma RMSNorm of q and k, NeoX RoPE on the first
//                          rotary dims, q written back in place, k and v stored at their
//                          cache rows (REF:83-190 fused with the KV store REF:2656-2687)
//   qw_attn_prefill        causal varlen attention, tensor cores (mma.sync m16n8k16 bf16),
//                          epilogue out = bf16(bf16(o) * sigmoid(gate)) (L5 + REF:2105-2121)
//   qw_attn_decode         one query per request, split over the KV length, CUDA cores;
//                          partials combined by qw_attn_decode's second kernel (L6 + K10)
//
// Cache layout (the reference's, REF:4966-4983): K and V are [rows, nkv, d] with rows
// 64 + slot*capacity + position; page 0 (rows 0..63) is reserved. A request's keys are
// therefore contiguous from row kv_base = 64 + slot*capacity, which is what the kernels
// address; the page table of REF:5038-5040 is implied by that layout.
#include "common.cuh"
#include "tmap.cuh"

namespace qw {

// ============================================================== q/k norm + rope + kv store
// E consecutive bf16 per lane moved as one vector (E = 8: 16 bytes, 4: 8 bytes, 2: 4 bytes)
template <int E>
QW_DEV void ld_vec(const __nv_bfloat16* p, float* f) {
  if constexpr (E == 8) {
    load_bf16x8(p, f);
  } else if constexpr (E == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    unpack_bf16x2(u.x, f[0], f[1]);
    unpack_bf16x2(u.y, f[2], f[3]);
  } else {
    unpack_bf16x2(*reinterpret_cast<const uint32_t*>(p), f[0], f[1]);
  }
}
template <int E>
QW_DEV void st_vec(__nv_bfloat16* p, const float* f) {
  if constexpr (E == 8) {
    store_bf16x8(p, f);
  } else if constexpr (E == 4) {
    uint2 u;
    u.x = pack_bf16x2(f[0], f[1]);
    u.y = pack_bf16x2(f[2], f[3]);
    *reinterpret_cast<uint2*>(p) = u;
  } else {
    *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(f[0], f[1]);
  }
}

// One warp per (token, head); lane owns E = D/32 consecutive dims.
template <int D>
__global__ void qk_norm_rope_store_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ldq, int nq, int nkv,
                                          const __nv_bfloat16* __restrict__ q_w, const __nv_bfloat16* __restrict__ k_w,
                                          const float* __restrict__ rope, int rd, int64_t rope_rows,
                                          const int32_t* __restrict__ positions, const int32_t* __restrict__ locs,
                                          __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                                          int64_t cache_rows, int T, float eps, int* err) {
  constexpr int E = D / 32;
  const int gw = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int heads = nq + nkv;
  if (gw >= T * heads) return;
  const int t = gw / heads, h = gw % heads;
  const bool is_k = h >= nq;
  const int kh = h - nq;
  __nv_bfloat16* row = qkv + (int64_t)t * ldq;
  __nv_bfloat16* src = is_k ? row + (int64_t)2 * nq * D + kh * D : row + (int64_t)h * 2 * D;
  const __nv_bfloat16* wt = is_k ? k_w : q_w;
  const int c0 = lane * E;
  float x[E], w[E];
  ld_vec<E>(src + c0, x);
  ld_vec<E>(wt + c0, w);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < E; ++j) ss += x[j] * x[j];
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
  float xn[E];
#pragma unroll
  for (int j = 0; j < E; ++j) xn[j] = bf16_round(x[j] * inv * (w[j] + 1.0f));
  // rotate-half on [0, rd): pair (i, i + rd/2); partner lane holds the matching elements
  const int half = rd / 2;
  const int off = half / E;  // lane distance between partners
  int pos = positions[t];
  if (pos < 0 || pos >= rope_rows) {
    set_error(err, QW_DEV_ERR_INDEX);
    pos = 0;
  }
  float o[E];
  float partner[E];
#pragma unroll
  for (int j = 0; j < E; ++j) partner[j] = __shfl_sync(0xffffffffu, xn[j], (c0 < half) ? lane + off : lane - off);
  if (c0 < rd) {
    // this lane's E dims are all rotary (rd is a multiple of 2E); cos/sin index = dim mod half
    const int ci = c0 < half ? c0 : c0 - half;
    const float* cs = rope + (int64_t)pos * rd + ci;
    const float* sn = cs + half;
    const float sign = c0 < half ? -1.f : 1.f;
#pragma unroll
    for (int j = 0; j < E; ++j) o[j] = xn[j] * cs[j] + sign * partner[j] * sn[j];
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) o[j] = xn[j];
  }
  if (!is_k) {
    st_vec<E>(src + c0, o);
    return;
  }
  const int64_t loc = locs[t];
  if (loc < 0 || loc >= cache_rows) {
    set_error(err, QW_DEV_ERR_INDEX);
    return;
  }
  if (loc == 0) return;  // reserved row, skipped like the reference store (REF:2683)
  const __nv_bfloat16* vs = row + (int64_t)2 * nq * D + (int64_t)nkv * D + kh * D;
  st_vec<E>(kc + (loc * nkv + kh) * D + c0, o);
  if constexpr (E == 8) {
    *reinterpret_cast<uint4*>(vc + (loc * nkv + kh) * D + c0) = *reinterpret_cast<const uint4*>(vs + c0);
  } else {
    float vv[E];
    ld_vec<E>(vs + c0, vv);
    st_vec<E>(vc + (loc * nkv + kh) * D + c0, vv);
  }
}

// ============================================================== prefill attention (tensor cores)
QW_DEV void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
QW_DEV void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
QW_DEV void mma_bf16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// byte offset of 16-byte chunk `c` of row `r` in a tile whose rows are D bf16 long,
// with the chunk index XOR-swizzled by (r % 8) so ldmatrix reads are conflict free
template <int D>
QW_DEV uint32_t swz(int r, int c) {
  return (uint32_t)(r * (D * 2) + ((c ^ (r & 7)) << 4));
}

struct PrefillTile {
  int32_t req;    // request index
  int32_t q0;     // first query (within the request) of this tile
};

// ============================================================== prefill attention (tcgen05)
// CTA = (query head, 128-query tile), 7 warps:
//  * warp 0 issues the TMA loads of the Q tile, then K in blocks of 64 keys (three stages,
//    SWIZZLE_128B boxes of 64 columns), and after the last S MMA the gate tile into the Q
//    buffer; warp 6 loads V (two stages, its own stream, so K never waits behind V);
//  * warp 1 issues tcgen05.mma from one lane: S_j = Q K_j^T (M 128, N 64) into one of two TMEM
//    S buffers, then O += P_{j-1} V_{j-1} (M 128, N = head dim) with P read from TMEM and V as
//    the MN-major shared-memory operand;
//  * warps 2-5 own one query row each (TMEM lane = row) and run the online softmax: S row from
//    TMEM, causal mask, scores in log2 units, P = exp2(s - m) rounded to bf16 pairs into one
//    of two TMEM P buffers (the A operand of P V). The running max m is raised only when a block's max
//    exceeds it by more than 8, so P < 2^8 and the O row in TMEM is rescaled rarely (after the
//    previous P V has completed). Epilogue: out = bf16(bf16(O / l) * sigmoid(gate)).
// Every wait is a bounded mbarrier wait (QW_DEV_ERR_TIMEOUT_ATTN).
template <int D>
struct AttnTc {
  static constexpr int BM = 128, BN = 64, NB = D / 64;  // 64-column boxes per row
  static constexpr int QB = BM * 128;                   // bytes of one Q box
  static constexpr int KVB = BN * 128;                  // bytes of one K or V box
  static constexpr int Q = 0;
  static constexpr int KST = 2;                         // K stages
  static constexpr int K0 = Q + NB * QB;                // KST stages x NB boxes
  static constexpr int V0 = K0 + KST * NB * KVB;        // 2 stages x NB boxes
  static constexpr int BAR = V0 + 2 * NB * KVB;
  // exchange of the two softmax halves: block maxima [2 parities][2 halves][BM], then the
  // row sums [2 halves][BM] at the end
  static constexpr int XMAX = BAR + 256;
  static constexpr int XSUM = XMAX + 2 * 2 * BM * 4;
  static constexpr int SMEM = XSUM + 2 * BM * 4 + 1024;  // + slack to align the base to 1024
  static constexpr int THREADS = 352;
  static constexpr int TMEM_O = 2 * BN;                 // S buffers at TMEM columns 0 and 64
  static constexpr int TMEM_P = TMEM_O + D;             // P buffers: 32 columns (64 bf16) each
  static constexpr uint32_t TMEM_COLS = (TMEM_P + BN <= 256) ? 256 : 512;
};

template <int D>
__global__ void __launch_bounds__(352, 1) attn_prefill_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, const PrefillTile* __restrict__ tiles, const int32_t* __restrict__ cu,
    const int32_t* __restrict__ prefix, const int32_t* __restrict__ kv_base, const __nv_bfloat16* __restrict__ qkv,
    int64_t ldq, __nv_bfloat16* __restrict__ out, int64_t ldo, int nq, int nkv, float scale_log2,
    float* __restrict__ part_o, float* __restrict__ part_ml, int* err) {
  using L = AttnTc<D>;
  constexpr int CODE = QW_DEV_ERR_TIMEOUT_ATTN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // [3]
  uint64_t* k_empty = bars + 4;  // [3]
  uint64_t* v_full = bars + 7;
  uint64_t* v_empty = bars + 9;
  uint64_t* s_full = bars + 11;
  uint64_t* s_empty = bars + 13;
  uint64_t* p_full = bars + 15;
  uint64_t* p_empty = bars + 17;
  uint64_t* mma_done = bars + 19;
  uint64_t* q_free = bars + 20;  // the last S MMA has read Q
  uint64_t* g_full = bars + 21;  // gate tile landed in the Q buffer
  uint64_t* x_full = bars + 22;  // [2] both softmax halves have published a block's maxima
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int h = blockIdx.x, kvh = h / (nq / nkv);
  const PrefillTile tile = tiles[blockIdx.y];
  const int t0 = cu[tile.req], n = cu[tile.req + 1] - t0;
  const int q0 = tile.q0;
  const int pre = prefix[tile.req];
  const int kend = min(pre + q0 + L::BM, pre + n);  // keys any valid row of the tile can see
  const int nblk_all = (kend + L::BN - 1) / L::BN;
  // split-KV (gridDim.z > 1): this CTA takes key blocks [jb, jb + nblk) of the tile and writes
  // an unnormalized partial (O, running max, sum) per row; the gate is applied at the merge
  const int nsplit = gridDim.z, split = blockIdx.z;
  int jb = 0, nblk = nblk_all;
  if (nsplit > 1) {
    const int per = (nblk_all + nsplit - 1) / nsplit;
    jb = min(nblk_all, split * per);
    nblk = min(nblk_all, jb + per) - jb;
  }
  const int kvrow = kv_base[tile.req];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < L::KST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 256);
      mbar_init(&p_full[i], 256);
      mbar_init(&p_empty[i], 1);
      mbar_init(&x_full[i], 256);
    }
    mbar_init(mma_done, 1);
    mbar_init(q_free, 1);
    mbar_init(g_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA: Q, K, then the gate
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, L::NB * L::QB);
      for (int i = 0; i < L::NB; ++i)
        tma_load_2d(smem + L::Q + i * L::QB, &tmQ, q_full, h * 2 * D + i * 64, t0 + q0);
      bool okp = true;
      for (int j = 0; j < nblk; ++j) {
        const int s = j % L::KST;
        const uint32_t ph = (j / L::KST) & 1;
        if (!mbar_wait(&k_empty[s], ph ^ 1, abort_flag, err, CODE)) {
          okp = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[s], L::NB * L::KVB);
        for (int i = 0; i < L::NB; ++i)
          tma_load_2d(smem + L::K0 + (s * L::NB + i) * L::KVB, &tmK, &k_full[s], kvh * D + i * 64,
                      kvrow + (jb + j) * L::BN);
      }
      // the output gate of the tile goes where Q was, once the last S MMA has read Q
      if (okp && nsplit == 1 && mbar_wait(q_free, 0, abort_flag, err, CODE)) {
        mbar_arrive_expect_tx(g_full, L::NB * L::QB);
        for (int i = 0; i < L::NB; ++i)
          tma_load_2d(smem + L::Q + i * L::QB, &tmQ, g_full, h * 2 * D + D + i * 64, t0 + q0);
      }
    }
  } else if (warp == 6) {
    // ---------------------------------------------------------------- TMA: V
    if (elect_one()) {
      for (int j = 0; j < nblk; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&v_empty[s], ph ^ 1, abort_flag, err, CODE)) break;
        mbar_arrive_expect_tx(&v_full[s], L::NB * L::KVB);
        for (int i = 0; i < L::NB; ++i)
          tma_load_2d(smem + L::V0 + (s * L::NB + i) * L::KVB, &tmV, &v_full[s], kvh * D + i * 64,
                      kvrow + (jb + j) * L::BN);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC_S = umma_idesc_bf16(128, L::BN);
      constexpr uint32_t IDESC_O = umma_idesc_bf16(128, D) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(q_full, 0, abort_flag, err, CODE);
      for (int j = 0; ok && j <= nblk; ++j) {
        if (j < nblk) {
          // S_j = Q K_j^T
          const int s = j & 1, ks3 = j % L::KST;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(&k_full[ks3], (j / L::KST) & 1, abort_flag, err, CODE) ||
              !mbar_wait(&s_empty[s], ph ^ 1, abort_flag, err, CODE)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ad = umma_sdesc_sw128(smem_u32(smem + L::Q + (kk >> 2) * L::QB) + (kk & 3) * 32);
            const uint64_t bd =
                umma_sdesc_sw128(smem_u32(smem + L::K0 + (ks3 * L::NB + (kk >> 2)) * L::KVB) + (kk & 3) * 32);
            umma_bf16(tmem + s * L::BN, ad, bd, IDESC_S, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[s]);
          umma_commit(&k_empty[ks3]);
          if (j == nblk - 1) umma_commit(q_free);
        }
        if (j >= 1) {
          // O += P_{j-1} V_{j-1}
          const int jp = j - 1, s = jp & 1;
          const uint32_t ph = (jp >> 1) & 1;
          if (!mbar_wait(&v_full[s], ph, abort_flag, err, CODE) || !mbar_wait(&p_full[s], ph, abort_flag, err, CODE)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < L::BN / 16; ++ks) {
            const uint64_t bd = umma_sdesc_mn_sw128(smem_u32(smem + L::V0 + s * L::NB * L::KVB) + ks * 2048, L::KVB);
            umma_bf16_ts(tmem + L::TMEM_O, tmem + L::TMEM_P + s * (L::BN / 2) + ks * 8, bd, IDESC_O,
                         (jp > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(&p_empty[s]);
          umma_commit(&v_empty[s]);
        }
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, err, CODE);  // every MMA of this CTA has completed
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- softmax + epilogue (warps 2-5, 7-10)
    // Two warps per TMEM lane quarter: warps 2-5 own the first 32 keys of every S block and
    // the first half of O's columns, warps 7-10 the rest. A row's block maximum is the max of
    // both halves (published in shared memory behind the x_full mbarrier), so both keep the
    // same running max and rescale decisions; each keeps the sum of its half of P, and the
    // two sums are added in the epilogue. tcgen05.ld/st are warp-collective: every decision
    // that guards them is made per warp (__any_sync / __all_sync).
    const int hf = warp >= 7 ? 1 : 0;
    const int row = 32 * (warp & 3) + lane;  // TMEM lane = query row of the tile
    const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    const int qpos = pre + q0 + row;  // keys at positions <= qpos are visible
    float* xmax = reinterpret_cast<float*>(smem + L::XMAX);
    float* xsum = reinterpret_cast<float*>(smem + L::XSUM);
    constexpr int OC = D / 2;  // O columns of a half
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[s], ph, abort_flag, err, CODE))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[32];
      tmem_ld_32x32b_x32(trow + s * L::BN + hf * 32, sr);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_empty[s]);
      const int key0 = (jb + j) * L::BN + hf * 32;
      float mx8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx8[e] = -INFINITY;
      // scores stay unscaled (the scale is positive, so the max commutes with it); a block
      // below the diagonal for every row of the tile needs no mask (CTA-uniform test)
      if ((jb + j) * L::BN + L::BN - 1 <= pre + q0) {
#pragma unroll
        for (int i = 0; i < 32; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(sr[i]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float v = (key0 + i <= qpos) ? __uint_as_float(sr[i]) : -INFINITY;
          sr[i] = __float_as_uint(v);
          mx8[i & 7] = fmaxf(mx8[i & 7], v);
        }
      }
      const float mine = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      xmax[(s * 2 + hf) * L::BM + row] = mine;
      mbar_arrive(&x_full[s]);
      if (!__all_sync(0xffffffffu, mbar_wait(&x_full[s], ph, abort_flag, err, CODE))) {
        ok = false;
        break;
      }
      const float mx = scale_log2 * fmaxf(mine, xmax[(s * 2 + (hf ^ 1)) * L::BM + row]);
      // the running max of a row is raised only when the block's max exceeds it by more
      // than 8; rows of O are rescaled in TMEM by the whole warp (factor 1 on rows whose
      // max stayed), once P V_{j-1} has completed
      const bool grow = mx > m_used + 8.f;
      const float m_new = grow ? mx : m_used;
      if (__any_sync(0xffffffffu, grow && j > 0)) {
        const int jp = j - 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&p_empty[jp & 1], (jp >> 1) & 1, abort_flag, err, CODE))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = (grow && j > 0) ? exp2f(m_used - m_new) : 1.f;
#pragma unroll 1
        for (int c0 = hf * OC; c0 < (hf + 1) * OC; c0 += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(trow + L::TMEM_O + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st_32x32b_x32(trow + L::TMEM_O + c0, r);
        }
        tmem_st_wait();
        l *= alpha;
      }
      m_used = m_new;
      const float mu = (m_used == -INFINITY) ? 0.f : m_used;
      // the P buffer is free once P V_{j-2} has completed
      if (!__all_sync(0xffffffffu, mbar_wait(&p_empty[s], ph ^ 1, abort_flag, err, CODE))) {
        ok = false;
        break;
      }
      float ps8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t pk[16];  // bf16 pairs (keys 2c, 2c + 1) of this half of the row
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float p0 = ex2_ftz(fmaf(__uint_as_float(sr[2 * c]), scale_log2, -mu));
        const float p1 = ex2_ftz(fmaf(__uint_as_float(sr[2 * c + 1]), scale_log2, -mu));
        ps8[(2 * c) & 7] += p0;
        ps8[(2 * c + 1) & 7] += p1;
        pk[c] = pack_bf16x2(p0, p1);
      }
      tmem_st_32x32b_x16(trow + L::TMEM_P + s * (L::BN / 2) + hf * 16, pk);
      tmem_st_wait();
      l += ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      tc_fence_before();  // P (and any O rescale) in TMEM before the P V issue
      mbar_arrive(&p_full[s]);
    }
    // ---- epilogue once the last P V has completed
    if (ok && nblk > 0) {
      const int jp = nblk - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[jp & 1], (jp >> 1) & 1, abort_flag, err, CODE));
    }
    if (ok && nsplit == 1) ok = __all_sync(0xffffffffu, mbar_wait(g_full, 0, abort_flag, err, CODE));
    // the row's sum over both halves (every softmax warp reaches this barrier once)
    xsum[hf * L::BM + row] = l;
    named_bar_sync(2, 256);
    l = xsum[row] + xsum[L::BM + row];
    __syncwarp();
    tc_fence_after();
    const bool valid = ok && q0 + row < n;
    const float inv_l = l > 0.f ? 1.f / l : 0.f;
    const int64_t t = t0 + q0 + row;
    if (nsplit > 1) {
      // partial of this split in the layout of the decode merge: slot (t * nq + h) * nsplit + split;
      // O is in TMEM only if a P V ran (nblk > 0, uniform over the CTA); rows that saw no key
      // have m = -inf and l = 0 and are ignored by the merge
      const int64_t slot = ((int64_t)t * nq + h) * nsplit + split;
#pragma unroll 1
      for (int c0 = hf * OC; c0 < (hf + 1) * OC; c0 += 32) {
        uint32_t r[32];
        if (nblk > 0) {
          tmem_ld_32x32b_x32(trow + L::TMEM_O + c0, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
        if (valid) {
          float4* dst = reinterpret_cast<float4*>(part_o + slot * D + c0);
#pragma unroll
          for (int v = 0; v < 8; ++v)
            dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                 __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
        }
      }
      if (valid && hf == 0) {
        part_ml[slot * 2 + 0] = nblk > 0 ? m_used : -INFINITY;
        part_ml[slot * 2 + 1] = nblk > 0 ? l : 0.f;
      }
    }
#pragma unroll 1
    for (int c0 = hf * OC; c0 < (hf + 1) * OC && nsplit == 1; c0 += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(trow + L::TMEM_O + c0, r);
      tmem_ld_wait();
      if (valid) {
        // gate row from the swizzled [128][64] boxes in the Q buffer
        const uint8_t* grow = smem + L::Q + (c0 >> 6) * L::QB + row * 128;
        __nv_bfloat16* dst = out + t * ldo + (int64_t)h * D + c0;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float g[8], y[8];
          const int chunk = ((c0 & 63) >> 3) + v;
          load_bf16x8(reinterpret_cast<const __nv_bfloat16*>(grow + ((chunk ^ (row & 7)) << 4)), g);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float a = bf16_round(__uint_as_float(r[v * 8 + e]) * inv_l);
            y[e] = __fdividef(a, 1.f + __expf(-g[e]));
          }
          store_bf16x8(dst + v * 8, y);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// Decode attention (one query token per request) on tensor cores. CTA = (request, kv head,
// split of the keys), 2 warps (64 KB of shared memory at d = 256, three CTAs per SM); each
// warp takes a contiguous half of the split's keys,
// 16 at a time: S^T = K Q^T ([16 keys] x [8 query heads of the group], Q held as register B
// fragments), an online softmax per head in the log2 domain, P^T rounded to bf16 through
// shared memory, and O^T += V^T P^T ([d] x [heads]). K and V rows stream through a per-warp
// double buffer of cp.async copies. The warps' (max, sum, O) merge in shared memory into
// the split's partial; attn_decode_combine_kernel merges the splits and applies the gate.
template <int D>
struct DecodeSmem {
  static constexpr int NW = 2;                    // warps per CTA
  static constexpr int KB = 16;                   // keys per warp step
  static constexpr int TK = KB * D * 2;           // one K (or V) step tile
  static constexpr int WARP = 4 * TK;             // two stages of K and V
  static constexpr int P = NW * WARP;             // per-warp P^T tiles [8 heads][16 keys] bf16
  static constexpr int ML = P + NW * 8 * KB * 2;  // per-warp max and sum of the 8 head columns
  static constexpr int TOTAL = ML + 2 * NW * 8 * 4;
  static_assert(NW * 8 * D * 4 <= P, "the warps' O^T merge reuses the K/V stages");
};

QW_DEV void ldmatrix_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

template <int D, int G>
__global__ void __launch_bounds__(64) attn_decode_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t ldq, int nq, int nkv, const __nv_bfloat16* __restrict__ kc,
    const __nv_bfloat16* __restrict__ vc, const int32_t* __restrict__ seq_len, const int32_t* __restrict__ kv_base,
    int keys_per_split, float scale_log2, float* __restrict__ part_o, float* __restrict__ part_ml, int splits) {
  griddep_launch_dependents();  // programmatic dependent launch (launch_k): see common.cuh
  griddep_wait();
  static_assert(G <= 8 && D % 16 == 0, "the query heads of a group fill one 8-wide n-tile");
  using L_ = DecodeSmem<D>;
  constexpr int KB = L_::KB, TK = L_::TK, NCH = D / 8, MT = D / 16, NW = L_::NW;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int b = blockIdx.x / nkv, kvh = blockIdx.x % nkv, split = blockIdx.y;
  const int L = seq_len[b];
  const int64_t base = kv_base[b];
  const int k_begin = split * keys_per_split;
  const int k_end = min(L, k_begin + keys_per_split);
  const int span = (keys_per_split + NW * KB - 1) / (NW * KB) * KB;  // keys per warp, multiple of 16
  const int w_begin = k_begin + warp * span;
  const int w_end = min(k_end, w_begin + span);
  const int steps = w_end > w_begin ? (w_end - w_begin + KB - 1) / KB : 0;
  const uint32_t ws0 = smem_u32(smem + warp * L_::WARP);
  __nv_bfloat16* sP = reinterpret_cast<__nv_bfloat16*>(smem + L_::P + warp * 8 * KB * 2);

  // Q of the group as B fragments: b0 = (d = 16 ks + 2c, +1; head g), b1 = (d + 8; head g)
  uint32_t qf[MT][2];
  {
    const bool ok = g < G;
    const __nv_bfloat16* qr = qkv + (int64_t)b * ldq + (int64_t)(kvh * G + (ok ? g : 0)) * 2 * D;
#pragma unroll
    for (int ks = 0; ks < MT; ++ks) {
      qf[ks][0] = ok ? *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 2 * c) : 0u;
      qf[ks][1] = ok ? *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 8 + 2 * c) : 0u;
    }
  }
  auto load_step = [&](int st) {
    const int key0 = w_begin + st * KB;
    const uint32_t kd = ws0 + (st & 1) * 2 * TK, vd = kd + TK;
    for (int i = lane; i < KB * NCH; i += 32) {
      const int r = i / NCH, ch = i % NCH;
      const bool ok = key0 + r < w_end;
      const int64_t row = (base + (ok ? key0 + r : 0)) * nkv + kvh;
      cp_async16(kd + swz<D>(r, ch), kc + row * D + ch * 8, ok);
      cp_async16(vd + swz<D>(r, ch), vc + row * D + ch * 8, ok);
    }
    cp_async_commit();
  };

  float o[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_j[2] = {-INFINITY, -INFINITY}, l_j[2] = {0.f, 0.f};  // heads 2c, 2c+1
  if (steps > 0) load_step(0);
  for (int st = 0; st < steps; ++st) {
    if (st + 1 < steps) {
      load_step(st + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();
    const uint32_t kd = ws0 + (st & 1) * 2 * TK, vd = kd + TK;
    // ---- S^T = K Q^T
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < MT; ++ks) {
      uint32_t a[4];
      ldmatrix_x4(kd + swz<D>(lane & 15, 2 * ks + (lane >> 4)), a[0], a[1], a[2], a[3]);
      mma_bf16_16816(sc, a, qf[ks][0], qf[ks][1]);
    }
    // ---- online softmax per head column (keys g and g + 8 of the step)
    const int key0 = w_begin + st * KB;
    const bool v0 = key0 + g < w_end, v1 = key0 + g + 8 < w_end;
    const float x[4] = {v0 ? sc[0] * scale_log2 : -INFINITY, v0 ? sc[1] * scale_log2 : -INFINITY,
                        v1 ? sc[2] * scale_log2 : -INFINITY, v1 ? sc[3] * scale_log2 : -INFINITY};
    float pr[4], alpha[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float mx = fmaxf(x[j], x[2 + j]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mn = fmaxf(m_j[j], mx);  // finite: key0 is always a valid key
      alpha[j] = ex2_ftz(m_j[j] - mn);
      pr[j] = ex2_ftz(x[j] - mn);
      pr[2 + j] = ex2_ftz(x[2 + j] - mn);
      float ps = pr[j] + pr[2 + j];
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      ps += __shfl_xor_sync(0xffffffffu, ps, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      l_j[j] = l_j[j] * alpha[j] + ps;
      m_j[j] = mn;
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      o[mt][0] *= alpha[0];
      o[mt][1] *= alpha[1];
      o[mt][2] *= alpha[0];
      o[mt][3] *= alpha[1];
    }
    // ---- P^T as [head][key] bf16, read back as the B fragments of V^T P^T
    sP[(2 * c) * KB + g] = f2bf(pr[0]);
    sP[(2 * c + 1) * KB + g] = f2bf(pr[1]);
    sP[(2 * c) * KB + g + 8] = f2bf(pr[2]);
    sP[(2 * c + 1) * KB + g + 8] = f2bf(pr[3]);
    __syncwarp();
    uint32_t pb0, pb1;
    ldmatrix_x2(smem_u32(sP) + (lane & 7) * (KB * 2) + ((lane >> 3) & 1) * 16, pb0, pb1);
    // ---- O^T += V^T P^T
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      uint32_t a[4];
      ldmatrix_x4_trans(vd + swz<D>((lane & 7) + ((lane >> 4) << 3), 2 * mt + ((lane >> 3) & 1)), a[0], a[1], a[2],
                        a[3]);
      mma_bf16_16816(o[mt], a, pb0, pb1);
    }
    __syncwarp();  // this stage and P are refilled next
  }
  // ---- merge the warps into the split's partial
  __syncthreads();  // every warp is done with its K/V stages
  float* sO = reinterpret_cast<float*>(smem);  // [NW warps][8 heads][D]
  float* sM = reinterpret_cast<float*>(smem + L_::ML);
  float* sL = sM + NW * 8;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) sO[(warp * 8 + 2 * c + (e & 1)) * D + 16 * mt + g + 8 * (e >> 1)] = o[mt][e];
  }
  if (g == 0) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      sM[warp * 8 + 2 * c + j] = m_j[j];
      sL[warp * 8 + 2 * c + j] = l_j[j];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int gi = i / D, d = i % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mm = fmaxf(mm, sM[w * 8 + gi]);
    float ll = 0.f, oo = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float f = (sM[w * 8 + gi] == -INFINITY) ? 0.f : exp2f(sM[w * 8 + gi] - mm);
      ll += sL[w * 8 + gi] * f;
      oo += sO[(w * 8 + gi) * D + d] * f;
    }
    const int h = kvh * G + gi;
    const int64_t slot = ((int64_t)b * nq + h) * splits + split;
    part_o[slot * D + d] = oo;
    if (d == 0) {
      part_ml[slot * 2 + 0] = mm;
      part_ml[slot * 2 + 1] = ll;
    }
  }
}

template <int D>
__global__ void attn_decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                           int splits, const __nv_bfloat16* __restrict__ qkv, int64_t ldq, int nq,
                                           __nv_bfloat16* __restrict__ out, int64_t ldo) {
  griddep_launch_dependents();  // programmatic dependent launch (launch_k): see common.cuh
  griddep_wait();
  const int bh = blockIdx.x;  // b * nq + h
  const int b = bh / nq, h = bh % nq;
  // the loops over splits are unrolled so that their independent loads are in flight together
  float mm = -INFINITY;
#pragma unroll 8
  for (int s = 0; s < splits; ++s) mm = fmaxf(mm, part_ml[((int64_t)bh * splits + s) * 2]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float ll = 0.f, oo = 0.f;
#pragma unroll 8
    for (int s = 0; s < splits; ++s) {
      const int64_t slot = (int64_t)bh * splits + s;
      const float ms = part_ml[slot * 2];
      const float f = (ms == -INFINITY) ? 0.f : exp2f(ms - mm);
      ll += part_ml[slot * 2 + 1] * f;
      oo += part_o[slot * D + d] * f;
    }
    const float a = bf16_round(ll > 0.f ? oo / ll : 0.f);
    const float gt = bf2f(qkv[(int64_t)b * ldq + (int64_t)h * 2 * D + D + d]);
    out[(int64_t)b * ldo + (int64_t)h * D + d] = f2bf(a / (1.f + expf(-gt)));
  }
}

}  // namespace qw

using namespace qw;

extern "C" int qw_qk_norm_rope_store(void* qkv, int64_t ldq, int64_t T, int64_t nq, int64_t nkv, int64_t d,
                                     const void* q_w, const void* k_w, const float* rope, int64_t rotary_dim,
                                     int64_t rope_rows, const int32_t* positions, const int32_t* locations,
                                     void* k_cache, void* v_cache, int64_t cache_rows, float eps,
                                     qw_stream_t stream) {
  QW_CHECK_ARG(qkv && q_w && k_w && rope && positions && locations && k_cache && v_cache && T > 0, QW_ERR_ARG);
  QW_CHECK_ARG(nq > 0 && nkv > 0 && nq % nkv == 0 && rotary_dim > 0 && rotary_dim <= d && rotary_dim % 2 == 0,
               QW_ERR_ARG);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t warps = T * (nq + nkv);
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  auto* q = static_cast<__nv_bfloat16*>(qkv);
  const auto* qw_ = static_cast<const __nv_bfloat16*>(q_w);
  const auto* kw_ = static_cast<const __nv_bfloat16*>(k_w);
  auto* kc = static_cast<__nv_bfloat16*>(k_cache);
  auto* vc = static_cast<__nv_bfloat16*>(v_cache);
  int* err = device_error_ptr();
#define QW_ROPE_LAUNCH(DD)                                                                                          \
  do {                                                                                                              \
    QW_CHECK_ARG(((rotary_dim / 2) % (DD / 32)) == 0, QW_ERR_UNSUPPORTED);                                          \
    qk_norm_rope_store_kernel<DD><<<blocks, 256, 0, s>>>(q, ldq, (int)nq, (int)nkv, qw_, kw_, rope, (int)rotary_dim, \
                                                         rope_rows, positions, locations, kc, vc, cache_rows,       \
                                                         (int)T, eps, err);                                         \
  } while (0)
  if (d == 256) QW_ROPE_LAUNCH(256);
  else if (d == 128) QW_ROPE_LAUNCH(128);
  else if (d == 64) QW_ROPE_LAUNCH(64);
  else return QW_ERR_UNSUPPORTED;
#undef QW_ROPE_LAUNCH
  QW_LAUNCH_CHECK();
  return QW_OK;
}

static int attn_prefill_launch(const void* qkv, int64_t ldq, int64_t nq, int64_t nkv, int64_t d, const void* k_cache,
                               const void* v_cache, const void* tiles, int64_t n_tiles, const int32_t* cu_seqlens,
                               const int32_t* prefix, const int32_t* kv_base, void* out, int64_t ldo, float scale,
                               int64_t T, int64_t cache_rows, int64_t splits, float* part_o, float* part_ml,
                               qw_stream_t stream) {
  QW_CHECK_ARG(qkv && k_cache && v_cache && tiles && cu_seqlens && prefix && kv_base && out, QW_ERR_ARG);
  QW_CHECK_ARG(n_tiles > 0 && n_tiles <= 65535 && nq > 0 && nkv > 0 && nq % nkv == 0, QW_ERR_ARG);
  QW_CHECK_ARG(T > 0 && T < (1ll << 31) && cache_rows > 0 && cache_rows < (1ll << 31) && ldq >= 2 * nq * d, QW_ERR_ARG);
  QW_CHECK_ARG(splits >= 1 && splits <= 65535, QW_ERR_ARG);
  QW_CHECK_ARG(((uintptr_t)qkv % 16) == 0 && (ldq % 8) == 0 && ((uintptr_t)out % 16) == 0 && (ldo % 8) == 0 &&
                   ((uintptr_t)k_cache % 16) == 0 && ((uintptr_t)v_cache % 16) == 0,
               QW_ERR_ALIGN);
  if (d != 64 && d != 128 && d != 256) return QW_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv;
  if (!tmap_bf16_2d_sw128(&tq, qkv, T, ldq, ldq, 64, 128) ||
      !tmap_bf16_2d_sw128(&tk, k_cache, cache_rows, nkv * d, nkv * d, 64, 64) ||
      !tmap_bf16_2d_sw128(&tv, v_cache, cache_rows, nkv * d, nkv * d, 64, 64))
    return QW_ERR_DRIVER;
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const float sl2 = scale * 1.4426950408889634f;
  // heads fastest: a kv group's heads share K/V in L2; key splits slowest
  dim3 grid((unsigned)nq, (unsigned)n_tiles, (unsigned)splits);
#define QW_ATTN_LAUNCH(DD)                                                                                        \
  do {                                                                                                            \
    static bool cfg = false;                                                                                      \
    if (!cfg) {                                                                                                   \
      cudaFuncSetAttribute(attn_prefill_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize,                 \
                           AttnTc<DD>::SMEM);                                                                     \
      cfg = true;                                                                                                 \
    }                                                                                                             \
    attn_prefill_kernel<DD><<<grid, AttnTc<DD>::THREADS, AttnTc<DD>::SMEM, s>>>(                                  \
        tq, tk, tv, static_cast<const PrefillTile*>(tiles), cu_seqlens, prefix, kv_base,                         \
        static_cast<const __nv_bfloat16*>(qkv), ldq, static_cast<__nv_bfloat16*>(out), ldo, (int)nq, (int)nkv,   \
        sl2, part_o, part_ml, device_error_ptr());                                                                \
  } while (0)
  if (d == 256) QW_ATTN_LAUNCH(256);
  else if (d == 128) QW_ATTN_LAUNCH(128);
  else QW_ATTN_LAUNCH(64);
#undef QW_ATTN_LAUNCH
  QW_LAUNCH_CHECK();
  if (splits == 1) return QW_OK;
  const auto* q = static_cast<const __nv_bfloat16*>(qkv);
  auto* o = static_cast<__nv_bfloat16*>(out);
  if (d == 256)
    launch_k(qw_pdl_small(), attn_decode_combine_kernel<256>, dim3((unsigned)(T * nq)), dim3(128), 0, s, part_o, part_ml, (int)splits, q, ldq, (int)nq, o, ldo);
  else if (d == 128)
    launch_k(qw_pdl_small(), attn_decode_combine_kernel<128>, dim3((unsigned)(T * nq)), dim3(128), 0, s, part_o, part_ml, (int)splits, q, ldq, (int)nq, o, ldo);
  else
    launch_k(qw_pdl_small(), attn_decode_combine_kernel<64>, dim3((unsigned)(T * nq)), dim3(64), 0, s, part_o, part_ml, (int)splits, q, ldq, (int)nq, o, ldo);
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_attn_prefill(const void* qkv, int64_t ldq, int64_t nq, int64_t nkv, int64_t d, const void* k_cache,
                               const void* v_cache, const void* tiles, int64_t n_tiles, const int32_t* cu_seqlens,
                               const int32_t* prefix, const int32_t* kv_base, void* out, int64_t ldo, float scale,
                               int64_t T, int64_t cache_rows, qw_stream_t stream) {
  return attn_prefill_launch(qkv, ldq, nq, nkv, d, k_cache, v_cache, tiles, n_tiles, cu_seqlens, prefix, kv_base, out,
                             ldo, scale, T, cache_rows, 1, nullptr, nullptr, stream);
}

extern "C" size_t qw_attn_prefill_split_workspace_bytes(int64_t T, int64_t nq, int64_t d, int64_t splits) {
  return (size_t)(T * nq * splits) * (size_t)(d + 2) * sizeof(float) + 256;
}

extern "C" int qw_attn_prefill_split(const void* qkv, int64_t ldq, int64_t nq, int64_t nkv, int64_t d,
                                     const void* k_cache, const void* v_cache, const void* tiles, int64_t n_tiles,
                                     const int32_t* cu_seqlens, const int32_t* prefix, const int32_t* kv_base,
                                     void* out, int64_t ldo, float scale, int64_t T, int64_t cache_rows,
                                     int64_t splits, void* workspace, size_t ws_bytes, qw_stream_t stream) {
  QW_CHECK_ARG(splits >= 1 && T > 0 && nq > 0, QW_ERR_ARG);
  if (splits == 1)
    return attn_prefill_launch(qkv, ldq, nq, nkv, d, k_cache, v_cache, tiles, n_tiles, cu_seqlens, prefix, kv_base,
                               out, ldo, scale, T, cache_rows, 1, nullptr, nullptr, stream);
  QW_CHECK_ARG(workspace && ws_bytes >= qw_attn_prefill_split_workspace_bytes(T, nq, d, splits), QW_ERR_WORKSPACE);
  QW_CHECK_ARG(((uintptr_t)workspace % 16) == 0, QW_ERR_ALIGN);
  float* part_o = static_cast<float*>(workspace);
  float* part_ml = part_o + T * nq * splits * d;
  return attn_prefill_launch(qkv, ldq, nq, nkv, d, k_cache, v_cache, tiles, n_tiles, cu_seqlens, prefix, kv_base, out,
                             ldo, scale, T, cache_rows, splits, part_o, part_ml, stream);
}

extern "C" size_t qw_attn_decode_workspace_bytes(int64_t B, int64_t nq, int64_t d, int64_t splits) {
  return (size_t)(B * nq * splits) * (size_t)(d + 2) * sizeof(float) + 256;
}

extern "C" int qw_attn_decode(const void* qkv, int64_t ldq, int64_t B, int64_t nq, int64_t nkv, int64_t d,
                              const void* k_cache, const void* v_cache, const int32_t* seq_len,
                              const int32_t* kv_base, int64_t max_len, int64_t splits, void* out, int64_t ldo,
                              float scale, void* workspace, size_t ws_bytes, qw_stream_t stream) {
  QW_CHECK_ARG(qkv && k_cache && v_cache && seq_len && kv_base && out && B > 0 && max_len > 0, QW_ERR_ARG);
  QW_CHECK_ARG(nq > 0 && nkv > 0 && nq % nkv == 0 && splits >= 1, QW_ERR_ARG);
  QW_CHECK_ARG(workspace && ws_bytes >= qw_attn_decode_workspace_bytes(B, nq, d, splits), QW_ERR_WORKSPACE);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int group = (int)(nq / nkv);
  const int kps = (int)(((max_len + splits - 1) / splits + 31) / 32 * 32);
  float* part_o = static_cast<float*>(workspace);
  float* part_ml = part_o + B * nq * splits * d;
  const float sl2 = scale * 1.4426950408889634f;
  dim3 grid((unsigned)(B * nkv), (unsigned)splits);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(attn_decode_kernel<256, 6>, cudaFuncAttributeMaxDynamicSharedMemorySize, DecodeSmem<256>::TOTAL);
    cudaFuncSetAttribute(attn_decode_kernel<256, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, DecodeSmem<256>::TOTAL);
    cudaFuncSetAttribute(attn_decode_kernel<64, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, DecodeSmem<64>::TOTAL);
    configured = true;
  }
  const auto* q = static_cast<const __nv_bfloat16*>(qkv);
  const auto* kc = static_cast<const __nv_bfloat16*>(k_cache);
  const auto* vc = static_cast<const __nv_bfloat16*>(v_cache);
  if (d == 256 && group == 6)
    launch_k(qw_pdl_small(), attn_decode_kernel<256, 6>, dim3(grid), dim3(32 * DecodeSmem<256>::NW), DecodeSmem<256>::TOTAL, s, q, ldq, (int)nq, (int)nkv, kc, vc, seq_len, kv_base, kps, sl2,
                                                    part_o, part_ml, (int)splits);
  else if (d == 256 && group == 3)  // 8-way tensor parallel: 3 query heads per replicated KV head
    launch_k(qw_pdl_small(), attn_decode_kernel<256, 3>, dim3(grid), dim3(32 * DecodeSmem<256>::NW), DecodeSmem<256>::TOTAL, s, q, ldq, (int)nq, (int)nkv, kc, vc, seq_len, kv_base, kps, sl2,
                                                    part_o, part_ml, (int)splits);
  else if (d == 64 && group == 2)
    launch_k(qw_pdl_small(), attn_decode_kernel<64, 2>, dim3(grid), dim3(32 * DecodeSmem<64>::NW), DecodeSmem<64>::TOTAL, s, q, ldq, (int)nq, (int)nkv, kc, vc, seq_len, kv_base, kps, sl2,
                                                   part_o, part_ml, (int)splits);
  else
    return QW_ERR_UNSUPPORTED;
  QW_LAUNCH_CHECK();
  if (d == 256)
    launch_k(qw_pdl_small(), attn_decode_combine_kernel<256>, dim3((unsigned)(B * nq)), dim3(128), 0, s, part_o, part_ml, (int)splits, q, ldq, (int)nq,
                                                                       static_cast<__nv_bfloat16*>(out), ldo);
  else
    launch_k(qw_pdl_small(), attn_decode_combine_kernel<64>, dim3((unsigned)(B * nq)), dim3(64), 0, s, part_o, part_ml, (int)splits, q, ldq, (int)nq,
                                                                     static_cast<__nv_bfloat16*>(out), ldo);
  QW_LAUNCH_CHECK();
  return QW_OK;
}
