// Dense bf16 projections on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the reference's cuBLAS F.linear calls (reference/qwen38_inference.py:5054,
// 5067, 5069, 5070, 5087, 5089, 5092, 5096) and fuses the SwiGLU of REF:5091.
//
// One persistent, warp-specialized kernel computes D[a_rows, b_rows] = A[a_rows,K] . B[b_rows,K]^T:
//   warp 0      TMA producer: 128 x 64 A tile and BN x 64 B tile per stage (SWIZZLE_128B)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16)
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator, rounding, stores
// The accumulator is double-buffered in TMEM so the epilogue of one tile overlaps the
// main loop of the next. Work units are (a_tile, b_tile, k_split) in a grouped raster.
//
// Prefill (M >= 65): A = activations, B = weights, BN = 256 (128 for SwiGLU halves).
// Decode  (M <= 64): A = weights (weight-streaming), B = the few activation rows,
//                    BN = M rounded up to 16, split over K to fill all SMs; fp32 partials
//                    are summed by a small deterministic reduction kernel.
// No TMA multicast is used (the same code runs in multi-GPU jobs).
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace qw {

__device__ int g_device_error_word = 0;

int* device_error_ptr() {
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) == cudaSuccess) ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

enum Epi : int {
  EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU = 2, EPI_PARTIAL = 3, EPI_F32RAW = 4, EPI_SWIGLU_SWAP = 5,
  EPI_QKV = 6  // the attention projection: q/k Gemma norm + RoPE, k/v into the cache (qkv_tile_row)
};

// fp32 outputs: EPI_F32 stores float(bf16(acc)) (F.linear().float()), EPI_F32RAW the accumulator itself
template <int EPI>
QW_DEV float f32_out(float acc) {
  if constexpr (EPI == EPI_F32) return bf16_round(acc);
  else return acc;
}

struct GemmParams {
  int a_rows, b_rows, K;
  int a_tiles, b_tiles, k_splits, kb_per_split, kb_total;
  int group;           // grouped raster width over a_tiles
  int swap;            // 0: out[a_row][b_row]; 1: out[b_row][a_row]
  int b_up_offset;     // SwiGLU: row offset of the "up" half inside B
  void* out;
  int64_t ldo;         // output row stride, elements
  int64_t part_stride; // EPI_PARTIAL: elements between split slices
  int* err;            // device error word
  int vec_ok;          // output rows 16-byte aligned: vector stores allowed
  int tma_out;         // CTA-pair bf16 / SwiGLU outputs: 32 x 64 boxes staged in shared memory, TMA stores
  // EPI_PARTIAL (weight streaming) with norm_rows > 0: the residual add-norm of the output
  // rows after the split-K product, by the last norm_rows CTAs to finish (partial_norm_finish)
  int norm_rows;
  int* norm_counter;  // [2], zero between launches
  __nv_bfloat16* resid;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* hidden;
  float eps;
  // tensor parallelism (norm_rows > 0, tp_world > 1): each row's local split sum is
  // exchanged through the ranks' peer buffers before the add-norm (partial_norm_finish)
  int tp_world, tp_rank;
  int tp_round_only;                    // 1: hidden = bf16(sum over ranks), no add-norm
  const unsigned long long* tp_bases;   // device array [tp_world]: every rank's buffer base
  int64_t tp_slot_off;                  // byte offset of this call's slot in every buffer
  // EPI_QKV: the output tile of 256 columns is one head segment of [q|gate per head, k, v]
  int qkv_nq, qkv_nkv;
  const __nv_bfloat16* q_w;
  const __nv_bfloat16* k_w;
  const float* rope;          // [rope_rows, 64] fp32: cos of 32 frequencies, then their sin
  int64_t rope_rows;
  const int32_t* positions;   // [M]
  const int32_t* locs;        // [M] cache row of each token
  __nv_bfloat16* kc;          // [cache_rows, nkv, 256]
  __nv_bfloat16* vc;
  int64_t cache_rows;
};

// The attention projection's epilogue for one token row of a 256-column output tile: tile bt
// is one head segment of the row [q_0 | gate_0 | ... | q_{nq-1} | gate_{nq-1} | k_0 .. | v_0 ..]
// (REF:4940), d = 256. x = bf16(acc) as F.linear rounds it; then, as REF:116-184 and
// REF:2656-2687 do (and qk_norm_rope_store_kernel):
//   gate: stored in place; v: stored at the token's cache row;
//   q, k: xn = bf16(x * rsqrt(mean x^2 + eps) * (1 + w)), NeoX RoPE on dims [0, 64) with the
//   pair (i, i + 32): o1 = xn1 cos - xn2 sin, o2 = xn2 cos + xn1 sin, rounded; q stored in
//   place, k at the token's cache row.
// t_row: TMEM address of this thread's row at the tile's first column. Every lane of the
// warp runs the whole function (tcgen05.ld is warp-collective); a lane whose row is past M
// (valid = false) reads along and touches no memory.
QW_DEV void qkv_tile_row(const GemmParams& p, uint32_t t_row, int a_row, int bt, bool valid) {
  constexpr int D = 256;
  const int nq = p.qkv_nq, nkv = p.qkv_nkv;
  __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)a_row * p.ldo;
  const bool is_q = bt < 2 * nq && (bt & 1) == 0;
  const bool is_gate = bt < 2 * nq && (bt & 1) == 1;
  const bool is_k = bt >= 2 * nq && bt < 2 * nq + nkv;
  const int kh = is_k ? bt - 2 * nq : bt - 2 * nq - nkv;  // kv head of a k or v segment
  __nv_bfloat16* dst = nullptr;
  if (!valid) {
  } else if (is_q || is_gate) {
    dst = row + (int64_t)bt * D;
  } else {
    const int64_t loc = p.locs[a_row];
    if (loc < 0 || loc >= p.cache_rows) {
      set_error(p.err, QW_DEV_ERR_INDEX);
      dst = nullptr;
    } else if (loc != 0) {  // row 0 is reserved and never written (REF:2683)
      dst = (is_k ? p.kc : p.vc) + (loc * nkv + kh) * D;
    }
  }
  if (is_gate || (!is_q && !is_k)) {
    // gate or v: the rounded projection as it is
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c, r);
      tmem_ld_wait();
      if (dst) {
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
#pragma unroll
        for (int j = 0; j < 32; j += 8) store_bf16x8(dst + c + j, f + j);
      }
    }
    return;
  }
  // q or k: sum of squares of the rounded row, then the norm and the rotation
  float ss = 0.f;
#pragma unroll 1
  for (int c = 0; c < D; c += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float x = bf16_round(__uint_as_float(r[j]));
      ss += x * x;
    }
  }
  const float inv = rsqrtf(ss / (float)D + p.eps);
  const __nv_bfloat16* wt = is_k ? p.k_w : p.q_w;
  int pos = valid ? p.positions[a_row] : 0;
  if (pos < 0 || pos >= p.rope_rows) {
    set_error(p.err, QW_DEV_ERR_INDEX);
    pos = 0;
  }
  const float* cs = p.rope + (int64_t)pos * 64;
  {
    uint32_t r1[32], r2[32];
    tmem_ld_32x32b_x32(t_row, r1);
    tmem_ld_32x32b_x32(t_row + 32, r2);
    tmem_ld_wait();
    float o[64];
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float w1[8], w2[8];
      load_bf16x8(wt + j, w1);
      load_bf16x8(wt + 32 + j, w2);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float x1 = bf16_round(bf16_round(__uint_as_float(r1[j + e])) * inv * (w1[e] + 1.0f));
        const float x2 = bf16_round(bf16_round(__uint_as_float(r2[j + e])) * inv * (w2[e] + 1.0f));
        const float c = cs[j + e], sn = cs[32 + j + e];
        o[j + e] = x1 * c + (-1.f * x2) * sn;
        o[32 + j + e] = x2 * c + (1.f * x1) * sn;
      }
    }
    if (dst) {
#pragma unroll
      for (int j = 0; j < 64; j += 8) store_bf16x8(dst + j, o + j);
    }
  }
#pragma unroll 1
  for (int c = 64; c < D; c += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c, r);
    tmem_ld_wait();
    float o[32];
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float w[8];
      load_bf16x8(wt + c + j, w);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[j + e] = bf16_round(bf16_round(__uint_as_float(r[j + e])) * inv * (w[e] + 1.0f));
    }
    if (dst) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) store_bf16x8(dst + c + j, o + j);
    }
  }
}

// Ticket counters of partial_norm_finish, one pair per device. Launches that use them must
// not overlap in time (calls ordered on one stream): two overlapping launches would draw
// tickets from the same pair. A launch that sees a ticket beyond its own grid knows the pair
// was left stale (an earlier launch gave up a wait) and records QW_DEV_ERR_GEMM_COUNTER
// instead of touching memory; qw_take_device_error() zeroes the pair after its synchronize.
__device__ int g_norm_counter[2];

static int* norm_counter_ptr() {
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_norm_counter) == cudaSuccess) ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

QW_DEV int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
QW_DEV unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
QW_DEV void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
QW_DEV float4 ld_volatile_f4(const float* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// The add-norm after a weight-streaming split-K product, inside the GEMM kernel. Every CTA,
// once its partial stores are issued, fences them and draws a ticket. The last norm_rows
// ticket holders wait (bounded) until every CTA of the grid holds a ticket, so all partials
// are in memory, then each takes one output row m:
//   x = bf16(sum_s partial[s][m][:]) (splits in order), v = x + resid (fp32),
//   resid = bf16(v), hidden = bf16(v * rsqrt(mean v^2 + eps) * (1 + w)).
// The waiters only wait for CTAs that are already running: the grid is at most one CTA per
// SM, and a CTA that has not drawn its ticket is either running or about to be placed on
// an SM that a finished CTA of this grid or of an earlier kernel gives back. The last waiter
// to finish resets both counters for the next launch.
template <int NT>
QW_DEV void partial_norm_finish(const GemmParams& p) {
  constexpr int MAXC = 6;  // 8-column chunks per thread: N <= 48 * NT
  __shared__ int s_ticket, s_ok;
  __shared__ float s_red[NT / 32];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_ticket = atomicAdd(p.norm_counter, 1);
  __syncthreads();
  const int first = (int)gridDim.x - p.norm_rows;
  const int t = s_ticket;
  if (t < 0 || t >= (int)gridDim.x) {
    // the pair did not start this launch at zero: no row index derived from it is valid
    if (threadIdx.x == 0) set_error(p.err, QW_DEV_ERR_GEMM_COUNTER);
    return;
  }
  if (t < first) return;
  // every exit from here on counts this finisher; the last one resets the pair for the next
  // launch (all CTAs of the grid hold a ticket by then, unless the ticket wait gave up)
  auto release = [&]() {
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(p.norm_counter + 1, 1) == p.norm_rows - 1) {
      p.norm_counter[0] = 0;
      p.norm_counter[1] = 0;
      __threadfence();
    }
  };
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_gpu(p.norm_counter) < (int)gridDim.x) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        set_error(p.err, QW_DEV_ERR_TIMEOUT_GEMM);
        ok = 0;
        break;
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;  // the pair stays stale: the next launch reports it (see above)
  const int m = t - first;  // 0 <= m < norm_rows by the ticket check
  const int N = p.a_rows;
  const float* ws = reinterpret_cast<const float*>(p.out) + (int64_t)m * p.ldo;
  // the row's residual and the norm weights do not depend on the partials: their loads go
  // out first and overlap the partial sums (round-only calls have neither)
  uint4 res_u[MAXC], w_u[MAXC];
  const bool norm = !(p.tp_world > 1 && p.tp_round_only);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (norm && c < N) {
      res_u[i] = *reinterpret_cast<const uint4*>(p.resid + (int64_t)m * N + c);
      w_u[i] = *reinterpret_cast<const uint4*>(p.norm_w + c);
    }
  }
  float v[MAXC][8];
#pragma unroll
  for (int i = 0; i < MAXC; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
  // splits in order, two at a time: the loads of both splits for every chunk are in flight
  // together, and each sum still adds split s before split s + 1
  auto add4 = [](float* d, const float4& a) {
    d[0] += a.x; d[1] += a.y; d[2] += a.z; d[3] += a.w;
  };
  int sp = 0;
  for (; sp + 1 < p.k_splits; sp += 2) {
    const float* s0 = ws + sp * p.part_stride;
    const float* s1 = s0 + p.part_stride;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = (threadIdx.x + i * NT) * 8;
      if (c < N) {
        const float4 a0 = __ldcg(reinterpret_cast<const float4*>(s0 + c));
        const float4 b0 = __ldcg(reinterpret_cast<const float4*>(s0 + c + 4));
        const float4 a1 = __ldcg(reinterpret_cast<const float4*>(s1 + c));
        const float4 b1 = __ldcg(reinterpret_cast<const float4*>(s1 + c + 4));
        add4(v[i], a0);
        add4(v[i] + 4, b0);
        add4(v[i], a1);
        add4(v[i] + 4, b1);
      }
    }
  }
  if (sp < p.k_splits) {
    const float* src = ws + sp * p.part_stride;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = (threadIdx.x + i * NT) * 8;
      if (c < N) {
        add4(v[i], __ldcg(reinterpret_cast<const float4*>(src + c)));
        add4(v[i] + 4, __ldcg(reinterpret_cast<const float4*>(src + c + 4)));
      }
    }
  }
  if (p.tp_world > 1) {
    // one-shot all-reduce of row m over the ranks: publish this rank's row in its own
    // buffer, raise this row's flag in every rank's buffer, wait (bounded) for every rank's
    // flag in this buffer, then sum the ranks' rows in rank order (the same bits on every
    // rank). The slot a call uses alternates with the caller's layer position, so a rank
    // writes a slot again only after every rank has passed the call that read it.
    uint8_t* mine = reinterpret_cast<uint8_t*>(p.tp_bases[p.tp_rank]);
    float* my_row = reinterpret_cast<float*>(mine + p.tp_slot_off) + (int64_t)m * N;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = (threadIdx.x + i * NT) * 8;
      if (c < N) {
        reinterpret_cast<float4*>(my_row + c)[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        reinterpret_cast<float4*>(my_row + c)[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
      }
    }
    __threadfence_system();
    __syncthreads();
    unsigned* my_flags = reinterpret_cast<unsigned*>(mine) + m * QW_TP_MAX_WORLD;
    unsigned* my_epoch = reinterpret_cast<unsigned*>(mine + 4096) + m;
    __shared__ unsigned s_ep;
    if (threadIdx.x == 0) s_ep = *my_epoch + 1;  // only this CTA touches row m's epoch in this launch
    __syncthreads();
    const unsigned ep = s_ep;
    if ((int)threadIdx.x < p.tp_world)
      st_release_sys(reinterpret_cast<unsigned*>(p.tp_bases[threadIdx.x]) + m * QW_TP_MAX_WORLD + p.tp_rank, ep);
    if (threadIdx.x == 0) {
      int ok = 1;
      const uint64_t t0 = globaltimer();
      for (int q = 0; q < p.tp_world && ok; ++q) {
        while (ld_acquire_sys(my_flags + q) < ep) {
          if (globaltimer() - t0 > kWaitLimitNs) {
            set_error(p.err, QW_DEV_ERR_TIMEOUT_TP);
            ok = 0;
            break;
          }
        }
      }
      *my_epoch = ep;
      s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) {  // every CTA of this grid holds a ticket: the reset stays exact
      release();
      return;
    }
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = (threadIdx.x + i * NT) * 8;
      if (c < N) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
        for (int q = 0; q < p.tp_world; ++q) {
          const float* row = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(p.tp_bases[q]) +
                                                            p.tp_slot_off) + (int64_t)m * N + c;
          const float4 a = ld_volatile_f4(row), b = ld_volatile_f4(row + 4);
          v[i][0] += a.x; v[i][1] += a.y; v[i][2] += a.z; v[i][3] += a.w;
          v[i][4] += b.x; v[i][5] += b.y; v[i][6] += b.z; v[i][7] += b.w;
        }
      }
    }
    if (p.tp_round_only) {
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = (threadIdx.x + i * NT) * 8;
        if (c < N) store_bf16x8(p.hidden + (int64_t)m * N + c, v[i]);
      }
      release();
      return;
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < N) {
      float r[8];
      unpack_bf16x2(res_u[i].x, r[0], r[1]);
      unpack_bf16x2(res_u[i].y, r[2], r[3]);
      unpack_bf16x2(res_u[i].z, r[4], r[5]);
      unpack_bf16x2(res_u[i].w, r[6], r[7]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i][j] = bf16_round(v[i][j]) + r[j];
        ss += v[i][j] * v[i][j];
      }
      store_bf16x8(p.resid + (int64_t)m * N + c, v[i]);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) tot += s_red[i];
  const float rstd = rsqrtf(tot / (float)N + p.eps);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = (threadIdx.x + i * NT) * 8;
    if (c < N) {
      float wf[8], o[8];
      unpack_bf16x2(w_u[i].x, wf[0], wf[1]);
      unpack_bf16x2(w_u[i].y, wf[2], wf[3]);
      unpack_bf16x2(w_u[i].z, wf[4], wf[5]);
      unpack_bf16x2(w_u[i].w, wf[6], wf[7]);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * rstd * (1.0f + wf[j]);
      store_bf16x8(p.hidden + (int64_t)m * N + c, o);
    }
  }
  release();  // every waiter is past its wait
}

constexpr int BM = 128;  // rows of one MMA (one TMEM accumulator)
constexpr int BK = 64;   // 64 bf16 = 128 bytes = one SWIZZLE_128B row

// MT = number of 128-row A sub-tiles per CTA sharing each B tile (1 or 2). MT = 2 gives a
// 256 x BN tile: a third fewer operand bytes per FLOP than 128 x BN, at the cost of a
// single-buffered accumulator when 2 * BN columns fill TMEM.
template <int MT>
constexpr int gemm_threads() { return 64 + 128 * MT; }

template <int BN, int STAGES, int MT = 1>
struct GemmSmem {
  static constexpr int A_BYTES = MT * BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFFSET + 256 + 1024;  // barriers + alignment slack
  // TMA-store epilogue (BN = 256 large-M tiles): per epilogue warp NBOX staging boxes of
  // 32 rows x 64 bf16 columns (4 KB, SWIZZLE_128B), two (used alternately) when they fit
  static constexpr int STG = BAR_OFFSET + 1024, STG_BOX = 32 * 64 * 2;
  static constexpr int NBOX = (STG + 4 * MT * 2 * STG_BOX + 1024 <= 232448) ? 2 : 1;
  static constexpr int TOTAL_TMA_OUT = STG + 4 * MT * NBOX * STG_BOX + 1024;
  // EPI_SWIGLU_SWAP: the up half of a tile handed from its TMEM lanes to the gate lanes,
  // [64 rows][33] fp32 (padded against bank conflicts), after the barriers
  static constexpr int XCH = BAR_OFFSET + 256;
  static constexpr int XCH_BYTES = 64 * 33 * 4;
};

QW_DEV void decode_unit(const GemmParams& p, int unit, int& at, int& bt, int& split) {
  split = unit % p.k_splits;
  int tile = unit / p.k_splits;
  int per_group = p.group * p.b_tiles;
  int g = tile / per_group;
  int first = g * p.group;
  int gsz = min(p.a_tiles - first, p.group);
  int r = tile - g * per_group;
  at = first + r % gsz;
  bt = r / gsz;
}

template <int BN, int STAGES, int EPI, int MT>
__global__ void __launch_bounds__(gemm_threads<MT>(), 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using L = GemmSmem<BN, STAGES, MT>;
  constexpr int NBUF = (2 * MT * BN <= 512) ? 2 : 1;  // TMEM accumulator buffers
  constexpr int ACC = MT * BN;                        // TMEM columns of one buffer
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2]
  uint64_t* tempty = tfull + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int units = p.a_tiles * p.b_tiles * p.k_splits;
  constexpr int NCOL = NBUF * ACC;
  constexpr uint32_t TMEM_COLS = (NCOL <= 32) ? 32 : (NCOL <= 64) ? 64 : (NCOL <= 128) ? 128 : (NCOL <= 256) ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4 * MT);  // one arrive per epilogue warp
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the tensor memory is held: the next kernel on the stream may start its prologue. Every
  // thread but the producer waits here for the previous kernels (the epilogue reads residuals
  // and writes outputs, partials and the add-norm tickets that earlier launches use)
  griddep_launch_dependents();
  if (warp != 0) griddep_wait();

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      auto load_a = [&](uint8_t* sa, int kb, int at, uint64_t* bar) {
        if constexpr (EPI == EPI_SWIGLU_SWAP) {
          // 64 gate rows, then the 64 up rows of the same output columns (64-row boxes)
          tma_load_2d(sa, &tmA, bar, kb * BK, at * 64);
          tma_load_2d(sa + 64 * BK * 2, &tmA, bar, kb * BK, p.b_up_offset + at * 64);
        } else {
          tma_load_2d(sa, &tmA, bar, kb * BK, at * (BM * MT));
        }
      };
      // swap form: A is the weight, which no earlier kernel writes, so the first unit's first
      // STAGES weight tiles are requested before waiting for the previous kernel (programmatic
      // dependent launch); the activations B follow the wait
      int npre = 0;
      if (p.swap && (int)blockIdx.x < units) {
        int at, bt, split;
        decode_unit(p, blockIdx.x, at, bt, split);
        const int kb0 = split * p.kb_per_split;
        npre = min(STAGES, min(p.kb_total, kb0 + p.kb_per_split) - kb0);
        for (int i = 0; i < npre; ++i) {
          mbar_arrive_expect_tx(&full[i], L::STAGE_BYTES);
          load_a(smem + i * L::STAGE_BYTES, kb0 + i, at, &full[i]);
        }
      }
      griddep_wait();
      int it = 0;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int at, bt, split;
        decode_unit(p, u, at, bt, split);
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          uint8_t* sa = smem + stage * L::STAGE_BYTES;
          uint8_t* sb = sa + L::A_BYTES;
          if (it >= npre) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.err, QW_DEV_ERR_TIMEOUT_GEMM)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], L::STAGE_BYTES);
            load_a(sa, kb, at, &full[stage]);
          }
          if constexpr (EPI == EPI_SWIGLU) {
            tma_load_2d(sb, &tmB, &full[stage], kb * BK, bt * (BN / 2));
            tma_load_2d(sb + (BN / 2) * BK * 2, &tmB, &full[stage], kb * BK, p.b_up_offset + bt * (BN / 2));
          } else {
            tma_load_2d(sb, &tmB, &full[stage], kb * BK, bt * BN);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    griddep_wait();  // the other lanes (they take part in the add-norm finisher)
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN);
    int stage = 0;
    uint32_t phase = 0;
    int tcount = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++tcount) {
      int at, bt, split;
      decode_unit(p, u, at, bt, split);
      const int kb0 = split * p.kb_per_split;
      const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
      const int buf = tcount % NBUF;
      const uint32_t tphase = ((tcount / NBUF) & 1) ^ 1;
      if (!mbar_wait(&tempty[buf], tphase, abort_flag, p.err, QW_DEV_ERR_TIMEOUT_GEMM)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * ACC;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, p.err, QW_DEV_ERR_TIMEOUT_GEMM)) { ok = false; break; }
        tc_fence_after();
        if (elect_one()) {
          const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
          const uint64_t da = umma_sdesc_sw128(sa);
          const uint64_t db = umma_sdesc_sw128(sb);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance the start address by 16 bf16 = 32 bytes inside the 128-byte swizzled row;
            // sub-tile mt of A starts 128 rows (16 KB, 1024 descriptor units) further
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
              umma_bf16(d_tmem + mt * BN, da + (uint64_t)(2 * k + mt * 1024), db + (uint64_t)(2 * k), IDESC,
                        (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&tfull[buf]);
      __syncwarp();
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..)
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int msub = (warp - 2) >> 2;   // which 128-row accumulator this warp drains
    const int row_in_tile = msub * BM + q * 32 + lane;
    uint8_t* stg = smem + L::STG + (warp - 2) * L::NBOX * L::STG_BOX;  // this warp's staging boxes
    int sbox = 0;
    int tcount = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++tcount) {
      int at, bt, split;
      decode_unit(p, u, at, bt, split);
      const int buf = tcount % NBUF;
      // warp-uniform: the tcgen05.ld below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (tcount / NBUF) & 1, abort_flag, p.err, QW_DEV_ERR_TIMEOUT_GEMM))) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + buf * ACC + msub * BN;
      const int a_row = at * (BM * MT) + row_in_tile;
      const bool a_ok = a_row < p.a_rows;
      if ((EPI == EPI_BF16 || EPI == EPI_SWIGLU) && BN == 256 && p.tma_out) {
        // 64 output columns at a time: the warp's 32 rows staged as bf16 (row = lane), then one
        // TMA store of the 32 x 64 box; rows past M and columns past N are not written
        const int row0 = at * (BM * MT) + msub * BM + q * 32;
        constexpr int NOUT = EPI == EPI_SWIGLU ? BN / 2 : BN;
#pragma unroll 1
        for (int c = 0; c < NOUT; c += 64) {
          uint8_t* box = stg + (sbox % L::NBOX) * L::STG_BOX;
          ++sbox;
          if (lane == 0) {  // the store issued from this box earlier has read it
            if constexpr (L::NBOX == 2) bulk_wait_read<1>();
            else bulk_wait_read<0>();
          }
          __syncwarp();
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float f[32];
            if constexpr (EPI == EPI_SWIGLU) {
              uint32_t g[32], v[32];
              tmem_ld_32x32b_x32(t_row + c + 32 * hf, g);
              tmem_ld_32x32b_x32(t_row + BN / 2 + c + 32 * hf, v);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float gg = bf16_round(__uint_as_float(g[j]));
                const float uu = bf16_round(__uint_as_float(v[j]));
                f[j] = gg / (1.0f + expf(-gg)) * uu;
              }
            } else {
              uint32_t r[32];
              tmem_ld_32x32b_x32(t_row + c + 32 * hf, r);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
            }
            stage_row_bf16_sw128(box, lane, hf, f);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0 && bt * NOUT + c < p.b_rows && row0 < p.a_rows) {  // a box wholly past the edge writes nothing
            tma_store_2d(&tmC, smem_u32(box), bt * NOUT + c, row0);
            bulk_commit();
          }
        }
      } else if constexpr (EPI == EPI_SWIGLU_SWAP) {
        // weight-streaming SwiGLU: TMEM lanes 0-63 hold gate rows at*64 + lane (warps with
        // q = 0, 1), lanes 64-127 the matching up rows (q = 2, 3). The up warps hand their
        // bf16-rounded values over in shared memory; the gate warps write
        // act[m][n] = bf16(silu(g) * u) (swap: n is the weight row, m the activation row).
        float* xch = reinterpret_cast<float*>(smem + L::XCH);
        const int n = at * 64 + (q & 1) * 32 + lane;  // output column of this lane's row pair
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          constexpr int CW = BN < 32 ? BN : 32;
          uint32_t r[32];
          if constexpr (BN >= 32) {
            tmem_ld_32x32b_x32(t_row + c, r);
          } else {
            tmem_ld_32x32b_x16(t_row + c, r);
          }
          tmem_ld_wait();
          if (q >= 2) {
#pragma unroll
            for (int j = 0; j < CW; ++j) xch[((q - 2) * 32 + lane) * 33 + j] = bf16_round(__uint_as_float(r[j]));
          }
          named_bar_sync(1, 128);
          if (q < 2 && n < p.a_rows) {
#pragma unroll
            for (int j = 0; j < CW; ++j) {
              const int m = bt * BN + c + j;
              if (m < p.b_rows) {
                const float gg = bf16_round(__uint_as_float(r[j]));
                const float uu = xch[(q * 32 + lane) * 33 + j];
                out[(int64_t)m * p.ldo + n] = f2bf(gg / (1.0f + expf(-gg)) * uu);
              }
            }
          }
          named_bar_sync(1, 128);  // the exchange buffer is rewritten by the next chunk
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
        // columns [0, BN/2) = gate, [BN/2, BN) = up of output columns bt*BN/2 ...
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          uint32_t g[32], v[32];
          tmem_ld_32x32b_x32(t_row + c, g);
          tmem_ld_32x32b_x32(t_row + BN / 2 + c, v);
          tmem_ld_wait();
          const int col0 = bt * (BN / 2) + c;
          if (a_ok) {
            float f[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float gg = bf16_round(__uint_as_float(g[j]));
              const float uu = bf16_round(__uint_as_float(v[j]));
              f[j] = gg / (1.0f + expf(-gg)) * uu;
            }
            const int ncols = p.b_rows - col0;  // b_rows = I (output columns)
            __nv_bfloat16* dst = out + (int64_t)a_row * p.ldo + col0;
            if (ncols >= 32 && p.vec_ok) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) store_bf16x8(dst + j, f + j);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncols) dst[j] = f2bf(f[j]);
            }
          }
        }
      } else if constexpr (EPI == EPI_QKV) {
        static_assert(BN == 256 && MT == 1, "the qkv epilogue takes one 256-column head segment per tile");
        qkv_tile_row(p, t_row, a_row, bt, a_ok);
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          if constexpr (BN >= 32) {
            tmem_ld_32x32b_x32(t_row + c, r);
          } else {
            tmem_ld_32x32b_x16(t_row + c, r);
          }
          tmem_ld_wait();
          if (!a_ok) continue;
          const int b0 = bt * BN + c;
          const int nb = min(32, p.b_rows - b0);
          if (nb <= 0) continue;
          if (!p.swap) {
            if constexpr (EPI == EPI_BF16) {
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)a_row * p.ldo + b0;
              float f[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
              if (nb == 32 && p.vec_ok) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) store_bf16x8(dst + j, f + j);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nb) dst[j] = f2bf(f[j]);
              }
            } else if constexpr (EPI == EPI_F32 || EPI == EPI_F32RAW || EPI == EPI_PARTIAL) {
              // EPI_PARTIAL: this split's fp32 slice of a split-K product, [M, ldo] per split
              float* dst = reinterpret_cast<float*>(p.out) + (EPI == EPI_PARTIAL ? (int64_t)split * p.part_stride : 0) +
                           (int64_t)a_row * p.ldo + b0;
              if (nb == 32 && p.vec_ok) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                  float4 v4 = make_float4(f32_out<EPI>(__uint_as_float(r[j])), f32_out<EPI>(__uint_as_float(r[j + 1])),
                                          f32_out<EPI>(__uint_as_float(r[j + 2])), f32_out<EPI>(__uint_as_float(r[j + 3])));
                  *reinterpret_cast<float4*>(dst + j) = v4;
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nb) dst[j] = f32_out<EPI>(__uint_as_float(r[j]));
              }
            }
          } else {
            // swap: out[b_row][a_row]; lanes of a warp write 32 consecutive a_rows
            if constexpr (EPI == EPI_BF16) {
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + a_row;
#pragma unroll
              for (int j = 0; j < (BN < 32 ? BN : 32); ++j)
                if (j < nb) dst[(int64_t)(b0 + j) * p.ldo] = f2bf(__uint_as_float(r[j]));
            } else if constexpr (EPI == EPI_F32 || EPI == EPI_F32RAW) {
              float* dst = reinterpret_cast<float*>(p.out) + a_row;
#pragma unroll
              for (int j = 0; j < (BN < 32 ? BN : 32); ++j)
                if (j < nb) dst[(int64_t)(b0 + j) * p.ldo] = f32_out<EPI>(__uint_as_float(r[j]));
            } else if constexpr (EPI == EPI_PARTIAL) {
              float* dst = reinterpret_cast<float*>(p.out) + (int64_t)split * p.part_stride + a_row;
#pragma unroll
              for (int j = 0; j < (BN < 32 ? BN : 32); ++j)
                if (j < nb) dst[(int64_t)(b0 + j) * p.ldo] = __uint_as_float(r[j]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (lane == 0) bulk_wait<0>();  // every store of this warp complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if constexpr (EPI == EPI_PARTIAL) {
    if (p.norm_rows > 0) partial_norm_finish<64 + 128 * MT>(p);  // gemm_threads<MT>()
  }
}

// ------------------------------------------------------------------ CTA-pair GEMM (cta_group::2)
// A cluster of 2 CTAs computes a 256 x 256 output tile with M=256 tcgen05.mma issued by the
// pair leader: CTA r stages A rows [128r, 128r+128) and B rows [128r, 128r+128) of the tile
// (32 KB per k-block instead of 48 KB for a 128 x 256 tile per CTA) and receives output rows
// [128r, 128r+128) x 256 in its own TMEM, double-buffered. Both CTAs' TMA loads complete on
// the leader's full barrier; the leader's MMA commits arrive on both CTAs' empty / tmem-full
// barriers; both epilogues release the accumulator on the leader's tmem-empty barrier.
// SwiGLU: CTA 0 stages the gate rows and CTA 1 the matching up rows, so accumulator columns
// [0,128) are gate and [128,256) up, exactly as in the single-CTA kernel.
// The wide form (NH = 2) computes a 256 x 512 tile per pair as two N-halves that share each
// staged A tile: two MMAs per k-step into accumulators at TMEM columns [0, 256) and [256, 512),
// which fill tensor memory, so the accumulator is single-buffered and the epilogue does not
// overlap the next tile's main loop. Per k-block a CTA stages 16 KB of A and 32 KB of B for
// twice the products of the 256 x 256 tile: 25 % fewer L2-to-SM bytes per FLOP.
constexpr int P_BN = 256;
constexpr int P_A_BYTES = BM * BK * 2, P_B_BOX = (P_BN / 2) * BK * 2;
// output staging of the TMA-store epilogue: per epilogue warp two 32-row x 64-column bf16 boxes
// (4 KB each, SWIZZLE_128B) used alternately, so a box is rewritten only after the store
// issued from it two boxes earlier has read it
constexpr int P_STG_BOX = 32 * 64 * 2;
template <int NH>
struct PairCfg {
  static constexpr int STAGES = NH == 1 ? 6 : 4;
  static constexpr int STAGE = P_A_BYTES + NH * P_B_BOX;  // per CTA and k-block
  static constexpr int BAR = STAGES * STAGE;
  static constexpr int STG = BAR + 1024;
  // epilogue warps: four per N-half (one per TMEM lane quarter), so the wide form drains its
  // two halves in parallel; staging boxes per epilogue warp: two (alternating) or one
  static constexpr int EW = 4 * NH, THREADS = 64 + 32 * EW, NBOX = NH == 1 ? 2 : 1;
  static constexpr int SMEM = STG + EW * NBOX * P_STG_BOX + 1024;
  static constexpr int NBUF = NH == 1 ? 2 : 1;  // accumulator buffers in the 512 TMEM columns
  static_assert(SMEM <= 232448, "CTA-pair GEMM shared memory above the sm_100 per-block limit");
};

template <int EPI, int NH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(64 + 128 * NH, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using C = PairCfg<NH>;
  static_assert(NH == 1 || EPI == EPI_BF16 || EPI == EPI_SWIGLU || EPI == EPI_QKV,
                "the wide form has bf16, SwiGLU and attention-projection epilogues");
  constexpr int P_STAGES = C::STAGES, NBUF = C::NBUF;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;  // [2]
  uint64_t* tempty = tfull + 2;        // [2], used in the leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int units = p.a_tiles * p.b_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * C::EW);  // every epilogue warp of both CTAs
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialized and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs) {
        int at, bt, split;
        decode_unit(p, u, at, bt, split);
        for (int kb = 0; kb < p.kb_total; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.err, QW_DEV_ERR_TIMEOUT_GEMM)) { ok = false; break; }
          uint8_t* sa = smem + stage * C::STAGE;
          uint8_t* sb = sa + P_A_BYTES;
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE);
          tma_load_2d_pair(sa, &tmA, bar, kb * BK, at * 256 + (int)rank * BM);
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            const int btx = bt * NH + h;  // the 256-column block of this N-half
            if constexpr (EPI == EPI_SWIGLU) {
              tma_load_2d_pair(sb + h * P_B_BOX, &tmB, bar, kb * BK, (rank ? p.b_up_offset : 0) + btx * (P_BN / 2));
            } else {
              tma_load_2d_pair(sb + h * P_B_BOX, &tmB, bar, kb * BK, btx * P_BN + (int)rank * (P_BN / 2));
            }
          }
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (leader) {
      constexpr uint32_t IDESC = umma_idesc_bf16(256, P_BN);
      int stage = 0;
      uint32_t phase = 0;
      int tcount = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs, ++tcount) {
        const int buf = tcount % NBUF;
        if (!mbar_wait(&tempty[buf], ((tcount / NBUF) & 1) ^ 1, abort_flag, p.err, QW_DEV_ERR_TIMEOUT_GEMM)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * P_BN;
        for (int kb = 0; kb < p.kb_total; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, QW_DEV_ERR_TIMEOUT_GEMM)) { ok = false; break; }
          tc_fence_after();
          if (elect_one()) {
            const uint32_t sa = smem_u32(smem + stage * C::STAGE);
            const uint64_t da = umma_sdesc_sw128(sa);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
#pragma unroll
              for (int h = 0; h < NH; ++h)
                umma_bf16_pair(d_tmem + h * P_BN, da + (uint64_t)(2 * k),
                               umma_sdesc_sw128(sa + P_A_BYTES + h * P_B_BOX) + (uint64_t)(2 * k), IDESC,
                               (kb > 0 || k > 0) ? 1u : 0u);
            umma_commit_pair(&empty[stage], 0x3);
          }
          __syncwarp();
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (elect_one()) umma_commit_pair(&tfull[buf], 0x3);
        __syncwarp();
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5, both CTAs)
    const int q = warp & 3;
    const int row_in_tile = (int)rank * BM + q * 32 + lane;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const int hw = (warp - 2) >> 2;  // the N-half this warp drains
    uint8_t* stg = smem + C::STG + (warp - 2) * C::NBOX * P_STG_BOX;  // this warp's staging boxes
    int sbox = 0;
    int tcount = 0;
    for (int u = pair; u < units; u += npairs, ++tcount) {
      int at, bt_unit, split;
      decode_unit(p, u, at, bt_unit, split);
      const int buf = tcount % NBUF;
      // warp-uniform: the tcgen05.ld below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (tcount / NBUF) & 1, abort_flag, p.err, QW_DEV_ERR_TIMEOUT_GEMM))) break;
      tc_fence_after();
      const int a_row = at * 256 + row_in_tile;
      const bool a_ok = a_row < p.a_rows;
      {
        // N-half h: accumulator columns (buf + h) * 256, output block bt = bt_unit * NH + h
        const int h = hw;
        const int bt = bt_unit * NH + h;
        const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (buf + h) * P_BN;
        if ((EPI == EPI_BF16 || EPI == EPI_SWIGLU) && p.tma_out) {
          // 64 output columns at a time: the warp's 32 rows staged as bf16 (row = lane), then one
          // TMA store of the 32 x 64 box; rows past M and columns past N are not written
          const int row0 = at * 256 + (int)rank * BM + q * 32;
          constexpr int NOUT = EPI == EPI_SWIGLU ? P_BN / 2 : P_BN;
#pragma unroll 1
          for (int c = 0; c < NOUT; c += 64) {
            uint8_t* box = stg + (sbox % C::NBOX) * P_STG_BOX;
            ++sbox;
            if (lane == 0) bulk_wait_read<C::NBOX - 1>();  // the store issued earlier from this box
            __syncwarp();
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              float f[32];
              if constexpr (EPI == EPI_SWIGLU) {
                uint32_t g[32], v[32];
                tmem_ld_32x32b_x32(t_row + c + 32 * hf, g);
                tmem_ld_32x32b_x32(t_row + P_BN / 2 + c + 32 * hf, v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  const float gg = bf16_round(__uint_as_float(g[j]));
                  const float uu = bf16_round(__uint_as_float(v[j]));
                  f[j] = gg / (1.0f + expf(-gg)) * uu;
                }
              } else {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + c + 32 * hf, r);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
              }
              stage_row_bf16_sw128(box, lane, hf, f);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0 && bt * NOUT + c < p.b_rows && row0 < p.a_rows) {  // a box wholly past the edge writes nothing
              tma_store_2d(&tmC, smem_u32(box), bt * NOUT + c, row0);
              bulk_commit();
            }
          }
        } else if constexpr (EPI == EPI_SWIGLU) {
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll 1
          for (int c = 0; c < P_BN / 2; c += 32) {
            uint32_t g[32], v[32];
            tmem_ld_32x32b_x32(t_row + c, g);
            tmem_ld_32x32b_x32(t_row + P_BN / 2 + c, v);
            tmem_ld_wait();
            const int col0 = bt * (P_BN / 2) + c;
            if (a_ok) {
              float f[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float gg = bf16_round(__uint_as_float(g[j]));
                const float uu = bf16_round(__uint_as_float(v[j]));
                f[j] = gg / (1.0f + expf(-gg)) * uu;
              }
              const int ncols = p.b_rows - col0;
              __nv_bfloat16* dst = out + (int64_t)a_row * p.ldo + col0;
              if (ncols >= 32 && p.vec_ok) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) store_bf16x8(dst + j, f + j);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < ncols) dst[j] = f2bf(f[j]);
              }
            }
          }
        } else if constexpr (EPI == EPI_QKV) {
          qkv_tile_row(p, t_row, a_row, bt, a_ok);
        } else {
#pragma unroll 1
          for (int c = 0; c < P_BN; c += 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_row + c, r);
            tmem_ld_wait();
            if (!a_ok) continue;
            const int b0 = bt * P_BN + c;
            const int nb = min(32, p.b_rows - b0);
            if (nb <= 0) continue;
            if constexpr (EPI == EPI_BF16) {
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)a_row * p.ldo + b0;
              float f[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
              if (nb == 32 && p.vec_ok) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) store_bf16x8(dst + j, f + j);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nb) dst[j] = f2bf(f[j]);
              }
            } else {
              float* dst = reinterpret_cast<float*>(p.out) + (int64_t)a_row * p.ldo + b0;
              if (nb == 32 && p.vec_ok) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                  *reinterpret_cast<float4*>(dst + j) =
                      make_float4(f32_out<EPI>(__uint_as_float(r[j])), f32_out<EPI>(__uint_as_float(r[j + 1])),
                                  f32_out<EPI>(__uint_as_float(r[j + 2])), f32_out<EPI>(__uint_as_float(r[j + 3])));
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nb) dst[j] = f32_out<EPI>(__uint_as_float(r[j]));
              }
            }
          }
        }
      }  // N-halves
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + buf * 8);  // the leader's tempty[buf]
    }
    if (lane == 0) bulk_wait<0>();  // every store of this warp complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no MMA or TMEM read in flight in either CTA
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

// Sum of split-K partials ws[s][m][n] (s = 0..splits-1 in order), then the output rounding.
template <int EPI>
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, void* out, int M, int N_out, int64_t ldo,
                                     int splits, int64_t part_stride, int64_t ldw, int up_offset) {
  griddep_launch_dependents();  // programmatic dependent launch (launch_k): see common.cuh
  griddep_wait();
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)M * N_out) return;
  const int m = (int)(idx / N_out);
  const int n = (int)(idx % N_out);
  float acc = 0.f;
  for (int s = 0; s < splits; ++s) acc += ws[s * part_stride + (int64_t)m * ldw + n];
  if constexpr (EPI == EPI_SWIGLU) {
    float up = 0.f;
    for (int s = 0; s < splits; ++s) up += ws[s * part_stride + (int64_t)m * ldw + up_offset + n];
    const float g = bf16_round(acc), u = bf16_round(up);
    reinterpret_cast<__nv_bfloat16*>(out)[(int64_t)m * ldo + n] = f2bf(g / (1.0f + expf(-g)) * u);
  } else if constexpr (EPI == EPI_F32 || EPI == EPI_F32RAW) {
    reinterpret_cast<float*>(out)[(int64_t)m * ldo + n] = f32_out<EPI>(acc);
  } else {
    reinterpret_cast<__nv_bfloat16*>(out)[(int64_t)m * ldo + n] = f2bf(acc);
  }
}

// Decode projection followed by the residual add-norm: row m of the output is
// x = bf16(sum_s ws[s][m][:]) (splits in order, as splitk_reduce_kernel), then
// v = x + resid (fp32), resid = bf16(v), hidden = bf16(v * rsqrt(mean v^2 + eps) * (1 + w)).
// One CTA per row, one thread per 8 columns (all split partials of a thread in flight at once).
constexpr int kAddNormMaxThreads = 1024;
__global__ void __launch_bounds__(kAddNormMaxThreads) splitk_add_rmsnorm_kernel(
    const float* __restrict__ ws, int splits, int64_t part_stride, int N, __nv_bfloat16* __restrict__ resid,
    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ hidden, float eps) {
  griddep_launch_dependents();  // programmatic dependent launch (launch_k): see common.cuh
  griddep_wait();
  __shared__ float red[32];
  const int m = blockIdx.x;
  const int c = threadIdx.x * 8;
  const bool on = c < N;
  float v[8];
  float ss = 0.f;
  if (on) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const float* src = ws + (int64_t)m * N + c;
#pragma unroll 4
    for (int sp = 0; sp < splits; ++sp) {
      const float4 a = reinterpret_cast<const float4*>(src + sp * part_stride)[0];
      const float4 b = reinterpret_cast<const float4*>(src + sp * part_stride)[1];
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
    float r[8];
    load_bf16x8(resid + (int64_t)m * N + c, r);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = bf16_round(acc[j]) + r[j];
      ss += v[j] * v[j];
    }
    store_bf16x8(resid + (int64_t)m * N + c, v);
  }
  ss = warp_sum(ss);
  const int nwarp = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < nwarp; ++i) tot += red[i];
  const float rstd = rsqrtf(tot / (float)N + eps);
  if (on) {
    float wf[8], o[8];
    load_bf16x8(w + c, wf);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = v[j] * rstd * (1.0f + wf[j]);
    store_bf16x8(hidden + (int64_t)m * N + c, o);
  }
}

// The attention projection after a split-K product (decode, or a chunk whose tiles leave SMs
// idle): one warp per (token, head segment of D columns), lane owning D/32 consecutive
// columns. x = bf16(sum of the split partials, in split order), then the epilogue of
// qkv_tile_row for any D and rotary width: gate stored in place, v at the token's cache row,
// q and k Gemma-normalized and rotated (pairs (i, i + rd/2)), q in place and k at the cache
// row (REF:116-184, REF:2656-2687).
template <int D>
__global__ void qkv_finish_kernel(const float* __restrict__ ws, int splits, int64_t part_stride, int N, int T,
                                  __nv_bfloat16* __restrict__ qkv, int64_t ldq, int nq, int nkv,
                                  const __nv_bfloat16* __restrict__ q_w, const __nv_bfloat16* __restrict__ k_w,
                                  const float* __restrict__ rope, int rd, int64_t rope_rows,
                                  const int32_t* __restrict__ positions, const int32_t* __restrict__ locs,
                                  __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, int64_t cache_rows,
                                  float eps, int* err) {
  griddep_launch_dependents();  // programmatic dependent launch (launch_k): see common.cuh
  griddep_wait();
  constexpr int E = D / 32;
  const int segs = 2 * nq + 2 * nkv;
  const int gw = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= T * segs) return;
  const int t = gw / segs, sg = gw % segs;
  const int c0 = lane * E;
  const int64_t col = (int64_t)sg * D + c0;
  float x[E];
#pragma unroll
  for (int j = 0; j < E; ++j) x[j] = 0.f;
  for (int sp = 0; sp < splits; ++sp) {
    const float* src = ws + sp * part_stride + (int64_t)t * N + col;
#pragma unroll
    for (int j = 0; j < E; ++j) x[j] += __ldcg(src + j);
  }
#pragma unroll
  for (int j = 0; j < E; ++j) x[j] = bf16_round(x[j]);
  const bool is_q = sg < 2 * nq && (sg & 1) == 0;
  const bool is_gate = sg < 2 * nq && (sg & 1) == 1;
  const bool is_k = sg >= 2 * nq && sg < 2 * nq + nkv;
  const int kh = is_k ? sg - 2 * nq : sg - 2 * nq - nkv;
  __nv_bfloat16* dst = nullptr;
  if (is_q || is_gate) {
    dst = qkv + (int64_t)t * ldq + col;
  } else {
    const int64_t loc = locs[t];
    if (loc < 0 || loc >= cache_rows) {
      if (lane == 0) set_error(err, QW_DEV_ERR_INDEX);
      return;
    }
    if (loc == 0) return;  // reserved row (REF:2683)
    dst = (is_k ? kc : vc) + (loc * nkv + kh) * D + c0;
  }
  if (is_gate || (!is_q && !is_k)) {
    for (int j = 0; j < E; j += 2) *reinterpret_cast<uint32_t*>(dst + j) = pack_bf16x2(x[j], x[j + 1]);
    return;
  }
  const __nv_bfloat16* wt = (is_k ? k_w : q_w) + c0;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < E; ++j) ss += x[j] * x[j];
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
  float xn[E];
#pragma unroll
  for (int j = 0; j < E; ++j) xn[j] = bf16_round(x[j] * inv * (bf2f(wt[j]) + 1.0f));
  const int half = rd / 2;
  const int off = half / E;
  int pos = positions[t];
  if (pos < 0 || pos >= rope_rows) {
    if (lane == 0) set_error(err, QW_DEV_ERR_INDEX);
    pos = 0;
  }
  float partner[E], o[E];
#pragma unroll
  for (int j = 0; j < E; ++j) partner[j] = __shfl_sync(0xffffffffu, xn[j], (c0 < half) ? lane + off : lane - off);
  if (c0 < rd) {
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
  for (int j = 0; j < E; j += 2) *reinterpret_cast<uint32_t*>(dst + j) = pack_bf16x2(o[j], o[j + 1]);
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 K-major operand [rows, K] with leading dimension ld (elements), box [box_rows, 64].
static int make_tmap(CUtensorMap* m, const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return QW_ERR_DRIVER;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QW_OK : QW_ERR_DRIVER;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN, int STAGES, int EPI, int MT = 1>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t s,
                       const CUtensorMap* tc = nullptr) {
  using L = GemmSmem<BN, STAGES, MT>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES, EPI, MT>;
  constexpr bool tma_epi = (EPI == EPI_BF16 || EPI == EPI_SWIGLU) && BN == 256;
  const int smem = tma_epi ? L::TOTAL_TMA_OUT : L::TOTAL + (EPI == EPI_SWIGLU_SWAP ? L::XCH_BYTES : 0);
  static bool configured = false;  // one flag per instantiation
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured = true;
  }
  const int units = p.a_tiles * p.b_tiles * p.k_splits;
  const int grid = units < num_sms() ? units : num_sms();
  GemmParams pp = p;
  pp.tma_out = tma_epi && tc != nullptr && !p.swap;
  // the weight-streaming (swap) form starts under programmatic dependent launch: its weight
  // tiles load while the previous kernel finishes
  launch_k(pp.swap != 0, kern, dim3(grid), dim3(gemm_threads<MT>()), smem, s, ta, tb, pp.tma_out ? *tc : ta, pp);
  QW_LAUNCH_CHECK();
  return QW_OK;
}

template <int EPI, int NH = 1>
static int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t s,
                       const CUtensorMap* tc = nullptr) {
  auto kern = gemm_pair_kernel<EPI, NH>;
  constexpr int P_SMEM = PairCfg<NH>::SMEM, P_THREADS = PairCfg<NH>::THREADS;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM);
    configured = true;
  }
  const int units = p.a_tiles * p.b_tiles;
  int grid = 2 * units;
  const int max_ctas = (num_sms() / 2) * 2;
  if (grid > max_ctas) grid = max_ctas;
  GemmParams pp = p;
  pp.tma_out = tc != nullptr;
  kern<<<grid, P_THREADS, P_SMEM, s>>>(ta, tb, tc ? *tc : ta, pp);
  QW_LAUNCH_CHECK();
  return QW_OK;
}

}  // namespace qw

bool qw_pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QW_PDL");
    v = (e && atoi(e) == 0) ? 0 : 1;
  }
  return v == 1;
}

bool qw_pdl_small() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QW_PDL_SMALL");
    v = (e && atoi(e) == 1) ? 1 : 0;
  }
  return v == 1;
}

namespace qw {

// bf16 outputs of the large-M kernels through shared-memory staging and TMA stores unless the
// environment variable QW_GEMM_TMA_STORE=0 selects the per-thread global stores (a tuning knob)
static bool gemm_tma_store() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QW_GEMM_TMA_STORE");
    v = (e && atoi(e) == 0) ? 0 : 1;
  }
  return v == 1;
}

// Wide CTA-pair tiles (256 x 512) for the pair kernel's outputs, bit flags: 1 bf16 outputs,
// 2 SwiGLU outputs, 4 the attention projection's q/k norm + RoPE + KV store; off unless the
// environment variable QW_GEMM_WIDE sets them (read at every call; a tuning knob). Measured
// in the power-capped B32 x L1024 step on B200: the wide tile draws less power per cycle
// (the SM clock rises 14-20 % with every shape on it) but its epilogue no longer overlaps the
// next tile's main loop; with the exact SwiGLU epilogue the gate_up loses more than the clock
// gives back, and the whole step is 3 % slower with QW_GEMM_WIDE=7 (bf16 outputs alone: the
// same as without).
static int gemm_wide_mode() {
  const char* e = getenv("QW_GEMM_WIDE");
  return e ? atoi(e) : 0;
}

// CTA-pair GEMM for large M: 0 (default) for none, 1 (the environment variable QW_GEMM_PAIR=1,
// read at every call) for plain outputs with K <= 6144 and the attention projection, 2
// (QW_GEMM_PAIR=2) for every large-M shape (tuning knobs). In the power-capped B32 x L1024 step on B200, with the raster
// groups of 16 (256-row tiles) and 24 (128-row tiles), three interleaved rounds each: pairs
// for the plain shapes and the SwiGLU gate_up 24,381 / 24,360 / 24,473 tok/s, pairs for the
// plain shapes only 24,835 / 24,859 / 24,716, no pairs 24,996 / 24,964 / 24,855. The pair
// kernel keeps its tensor pipe busier per cycle, but the single-CTA kernels leave the step a
// higher clock under the 1 kW cap (1383-1402 against 1282-1308 MHz).
static int gemm_pair_mode() {
  const char* e = getenv("QW_GEMM_PAIR");
  const int v = e ? atoi(e) : 0;
  return (v < 0 || v > 2) ? 0 : v;
}

struct SkinnyPlan {
  int bn, b_tiles, a_tiles, splits, kb_per_split, kb_total;
};

// Split-K plan for weight streaming (M <= 64). Cost of a plan in k-block times of the
// busiest SM: ceil(units / SMs) * (k-blocks per split + 2), the 2 standing for the unit's
// partial-tile epilogue, plus the split-K partials written and read back, spread over all
// SMs. The cheapest split count with at least 8 k-blocks per split wins (ties: fewer splits).
static SkinnyPlan plan_skinny(int64_t M, int64_t N, int64_t K) {
  SkinnyPlan pl;
  pl.bn = M <= 16 ? 16 : M <= 32 ? 32 : 64;
  pl.b_tiles = 1;
  pl.a_tiles = (int)((N + BM - 1) / BM);
  pl.kb_total = (int)((K + BK - 1) / BK);
  const int64_t sms = num_sms();
  const int64_t kb_bytes = (int64_t)BM * BK * 2;  // weight bytes of one k-block
  const int max_splits = pl.kb_total / 8 > 0 ? pl.kb_total / 8 : 1;
  int64_t best_cost = -1;
  int best_kbps = pl.kb_total;
  for (int s = 1; s <= max_splits; ++s) {
    const int kbps = (pl.kb_total + s - 1) / s;
    const int64_t splits = (pl.kb_total + kbps - 1) / kbps;
    const int64_t rounds = (pl.a_tiles * splits + sms - 1) / sms;
    int64_t cost = rounds * (kbps + 2);
    if (splits > 1) cost += (splits * M * N * 8 + kb_bytes * sms - 1) / (kb_bytes * sms);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_kbps = kbps;
    }
  }
  pl.kb_per_split = best_kbps;
  pl.splits = (pl.kb_total + pl.kb_per_split - 1) / pl.kb_per_split;
  return pl;
}

static bool use_skinny(int64_t M) { return M <= 64; }

// Split-K for large-M products whose 128 x 256 tiles leave SMs idle (e.g. a 512-token chunk
// times the 5120-wide down or output projection: 80 tiles for 148 SMs). Cost in k-block
// times of the busiest SM, as plan_skinny: ceil(units / SMs) * (k-blocks per split + 2), plus
// the fp32 partials written and read back (one k-block time moves ~3 MB from HBM over all
// SMs). Returns 1 (no split) when the tiles fill the SMs twice over.
static int plan_wide_splits(int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + 255) / 256);
  const int64_t sms = num_sms();
  if (tiles >= 2 * sms) return 1;
  const int kb = (int)((K + BK - 1) / BK);
  const int max_splits = kb / 8 > 0 ? kb / 8 : 1;
  const int64_t kblock_bytes = 3 << 20;
  int64_t best_cost = -1;
  int best = 1;
  for (int s = 1; s <= max_splits && s <= 16; ++s) {
    const int kbps = (kb + s - 1) / s;
    const int64_t splits = (kb + kbps - 1) / kbps;
    int64_t cost = ((tiles * splits + sms - 1) / sms) * (kbps + 2);
    if (splits > 1) cost += (splits * M * N * 8 + kblock_bytes - 1) / kblock_bytes;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = (int)splits;
    }
  }
  return best;
}

// The split-K partial GEMM of a large-M product: x [M, K] . w [N, K]^T as `splits` fp32
// slices [M, N] in ws (ldo N, slice stride M * N). 128 x 256 tiles, one CTA each.
static int launch_wide_partials(const void* x, const void* w, int64_t M, int64_t N, int64_t K, int64_t ldx,
                                int64_t ldw, int splits, void* ws, cudaStream_t s) {
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap(&ta, x, M, K, ldx, BM)) != QW_OK) return rc;
  if ((rc = make_tmap(&tb, w, N, K, ldw, 256)) != QW_OK) return rc;
  GemmParams p{};
  p.err = device_error_ptr();
  p.K = (int)K;
  p.kb_total = (int)((K + BK - 1) / BK);
  p.a_rows = (int)M;
  p.b_rows = (int)N;
  p.a_tiles = (int)((M + BM - 1) / BM);
  p.b_tiles = (int)((N + 255) / 256);
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.k_splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
  p.swap = 0;
  p.group = 16;
  p.out = ws;
  p.ldo = N;
  p.part_stride = M * N;
  p.vec_ok = ((uintptr_t)ws % 16) == 0 && (N % 4) == 0;
  return launch_gemm<256, 4, EPI_PARTIAL>(ta, tb, p, s);
}

// A tiles per raster group of the large-M kernels (a group's CTAs sweep the B tiles while
// its A tiles stay in L2): the per-kernel default unless the environment variable
// QW_GEMM_GROUP gives one for all of them (a tuning knob).
// Raster group of the kernels with 256-row tiles (CTA pair, and one CTA with two 128-row
// accumulators). Measured in the power-capped B32 x L1024 step on B200 (QW_GEMM_GROUP, two
// rounds each): 8: 23,115 / 22,859 tok/s, 12: 23,820 / 23,704, 16: 24,210 / 24,052,
// 24: 23,536 / 23,485, 32: 22,655 / 22,640 (SM clock 1207, 1260, 1271-1282, 1245-1260,
// 1144-1155 MHz: the group sets the DRAM traffic of the step's GEMMs and through it their
// share of the 1 kW power limit).
constexpr int kGroup256 = 16;
static int raster_group(int dflt) {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("QW_GEMM_GROUP");
    v = e ? atoi(e) : 0;
  }
  return v > 0 ? v : dflt;
}

// Rows of A per CTA for large-M GEMMs: 256 (two accumulators share each B tile) unless the
// environment variable QW_GEMM_TILE_ROWS=128 selects the double-buffered 128-row tile.
static int gemm_tile_rows() {
  static int rows = 0;
  if (rows == 0) {
    const char* e = getenv("QW_GEMM_TILE_ROWS");
    rows = (e && atoi(e) == 128) ? 128 : 256;
  }
  return rows;
}

}  // namespace qw

using namespace qw;

extern "C" size_t qw_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int out_kind) {
  if (!use_skinny(M)) {
    if (out_kind != QW_OUT_BF16 && out_kind != QW_OUT_F32) return 0;
    const int s = plan_wide_splits(M, N, K);
    return s > 1 ? (size_t)s * (size_t)M * (size_t)N * sizeof(float) : 0;
  }
  SkinnyPlan pl = plan_skinny(M, N, K);
  if (pl.splits == 1 && out_kind != QW_OUT_F32) return 0;  // SwiGLU without a split: in the epilogue
  return (size_t)pl.splits * (size_t)M * (size_t)N * sizeof(float);
}

extern "C" int qw_gemm_bf16(const void* x, const void* w, void* y, int64_t M, int64_t N, int64_t K, int64_t ldx,
                            int64_t ldw, int64_t ldy, int out_kind, void* workspace, size_t ws_bytes,
                            qw_stream_t stream) {
  QW_CHECK_ARG(x && w && y && M > 0 && N > 0 && K > 0, QW_ERR_ARG);
  QW_CHECK_ARG(ldx >= K && ldw >= K, QW_ERR_ARG);
  QW_CHECK_ARG(out_kind >= QW_OUT_BF16 && out_kind <= QW_OUT_F32, QW_ERR_ARG);
  QW_CHECK_ARG(M < (1 << 30) && N < (1 << 30), QW_ERR_ARG);
  QW_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)w % 16) == 0 && (ldx % 8) == 0 && (ldw % 8) == 0, QW_ERR_ALIGN);
  const int64_t n_out = out_kind == QW_OUT_SWIGLU ? N / 2 : N;
  QW_CHECK_ARG(out_kind != QW_OUT_SWIGLU || (N % 2 == 0), QW_ERR_ARG);
  QW_CHECK_ARG(ldy >= n_out, QW_ERR_ARG);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  CUtensorMap ta, tb;
  int rc;
  GemmParams p{};
  p.err = device_error_ptr();
  p.K = (int)K;
  p.kb_total = (int)((K + BK - 1) / BK);
  // 24 A tiles per group: measured on the SwiGLU gate_up GEMM under the power cap (sustained
  // 200-launch runs): 8: +8 %, 16: +1-2 %, 32: +0-2 %, 40: +6 %, 64: +13 % time against 24
  p.group = raster_group(24);

  if (!use_skinny(M) && (out_kind == QW_OUT_BF16 || out_kind == QW_OUT_F32)) {
    const int splits = plan_wide_splits(M, N, K);
    if (splits > 1) {
      // too few tiles for the SMs: split-K partials, then their sum in k order
      const size_t need = (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
      QW_CHECK_ARG(workspace != nullptr && ws_bytes >= need, QW_ERR_WORKSPACE);
      QW_CHECK_ARG(((uintptr_t)workspace % 16) == 0, QW_ERR_ALIGN);
      if ((rc = launch_wide_partials(x, w, M, N, K, ldx, ldw, splits, workspace, s)) != QW_OK) return rc;
      const int64_t total = M * N;
      const int threads = 256;
      const int blocks = (int)((total + threads - 1) / threads);
      const float* wsp = reinterpret_cast<const float*>(workspace);
      if (out_kind == QW_OUT_F32)
        launch_k(qw_pdl_small(), splitk_reduce_kernel<EPI_F32RAW>, dim3(blocks), dim3(threads), 0, s, wsp, y, (int)M, (int)N, ldy, splits, M * N, N, 0);
      else
        launch_k(qw_pdl_small(), splitk_reduce_kernel<EPI_BF16>, dim3(blocks), dim3(threads), 0, s, wsp, y, (int)M, (int)N, ldy, splits, M * N, N, 0);
      QW_LAUNCH_CHECK();
      return QW_OK;
    }
  }
  if (!use_skinny(M)) {
    // A = activations [M, K], B = weights [N, K]; out[m][n]
    const bool swiglu = out_kind == QW_OUT_SWIGLU;
    const int per16 = (out_kind == QW_OUT_F32_OF_BF16 || out_kind == QW_OUT_F32) ? 4 : 8;  // elements per 16 B
    p.vec_ok = ((uintptr_t)y % 16) == 0 && (ldy % per16) == 0;
    constexpr int BN = 256;
    // Kernel choice per shape (gemm_pair_mode): one CTA per tile by default; with
    // QW_GEMM_PAIR=1 CTA pairs for K <= 6144 plain outputs (qkvz, qkv, out_proj, o_proj),
    // with QW_GEMM_PAIR_SWIGLU=1 for the SwiGLU gate_up too (tuning knobs). K >= 8192 (the
    // down projection) does better on one CTA with 256-row tiles in every setting measured.
    const int pair_mode = gemm_pair_mode();
    const char* e_sw = getenv("QW_GEMM_PAIR_SWIGLU");
    const int pair_swiglu = e_sw ? atoi(e_sw) : 0;
    if (M >= 256 && ((!swiglu && K < 8192 && pair_mode == 1) || pair_mode == 2 || (swiglu && pair_swiglu == 1))) {
      if ((rc = make_tmap(&ta, x, M, K, ldx, BM)) != QW_OK) return rc;
      if ((rc = make_tmap(&tb, w, N, K, ldw, P_BN / 2)) != QW_OK) return rc;
      p.a_rows = (int)M;
      p.b_rows = (int)n_out;
      p.a_tiles = (int)((M + 255) / 256);
      p.b_tiles = swiglu ? (int)((n_out + P_BN / 2 - 1) / (P_BN / 2)) : (int)((N + P_BN - 1) / P_BN);
      p.k_splits = 1;
      p.kb_per_split = p.kb_total;
      p.swap = 0;
      p.group = raster_group(kGroup256);
      p.b_up_offset = (int)n_out;
      p.out = y;
      p.ldo = ldy;
      // bf16 outputs leave through TMA stores when their rows are 16-byte aligned
      CUtensorMap tc;
      const bool tma_out = (out_kind == QW_OUT_BF16 || swiglu) && p.vec_ok && gemm_tma_store() &&
                           make_tmap(&tc, y, M, n_out, ldy, 32) == QW_OK;
      const int wide = gemm_wide_mode();
      if (((wide & 1) && out_kind == QW_OUT_BF16) || ((wide & 2) && swiglu)) {
        // 256 x 512 tiles per pair: 256 SwiGLU or 512 plain output columns per unit
        p.b_tiles = swiglu ? (int)((n_out + P_BN - 1) / P_BN) : (int)((N + 2 * P_BN - 1) / (2 * P_BN));
        if (swiglu) return launch_pair<EPI_SWIGLU, 2>(ta, tb, p, s, tma_out ? &tc : nullptr);
        return launch_pair<EPI_BF16, 2>(ta, tb, p, s, tma_out ? &tc : nullptr);
      }
      if (swiglu) return launch_pair<EPI_SWIGLU>(ta, tb, p, s, tma_out ? &tc : nullptr);
      if (out_kind == QW_OUT_F32_OF_BF16) return launch_pair<EPI_F32>(ta, tb, p, s);
      if (out_kind == QW_OUT_F32) return launch_pair<EPI_F32RAW>(ta, tb, p, s);
      return launch_pair<EPI_BF16>(ta, tb, p, s, tma_out ? &tc : nullptr);
    }
    // 256-row tiles win when the main loop is long enough to hide their single-buffered
    // epilogue (measured on B200: K = 17408 +14%, N = 16384 +3%; SwiGLU, N = 5120 and
    // N = 14336 with K <= 6144 lose 3-5%)
    const bool big_tile = !swiglu && (K >= 8192 || N >= 16384);
    const int mt = (M >= 256 && big_tile && gemm_tile_rows() == 256) ? 2 : 1;
    if ((rc = make_tmap(&ta, x, M, K, ldx, BM * mt)) != QW_OK) return rc;
    if ((rc = make_tmap(&tb, w, N, K, ldw, swiglu ? BN / 2 : BN)) != QW_OK) return rc;
    p.a_rows = (int)M;
    p.b_rows = (int)n_out;
    p.a_tiles = (int)((M + BM * mt - 1) / (BM * mt));
    p.b_tiles = swiglu ? (int)((n_out + BN / 2 - 1) / (BN / 2)) : (int)((N + BN - 1) / BN);
    p.k_splits = 1;
    p.kb_per_split = p.kb_total;
    p.swap = 0;
    p.b_up_offset = (int)n_out;
    p.out = y;
    p.ldo = ldy;
    // bf16 outputs leave through TMA stores when their rows are 16-byte aligned
    CUtensorMap tc;
    const bool tma_out = (out_kind == QW_OUT_BF16 || swiglu) && p.vec_ok && gemm_tma_store() &&
                         make_tmap(&tc, y, M, n_out, ldy, 32) == QW_OK;
    const CUtensorMap* tcp = tma_out ? &tc : nullptr;
    if (mt == 2) {
      p.group = raster_group(kGroup256);
      if (swiglu) return launch_gemm<BN, 3, EPI_SWIGLU, 2>(ta, tb, p, s, tcp);
      if (out_kind == QW_OUT_F32_OF_BF16) return launch_gemm<BN, 3, EPI_F32, 2>(ta, tb, p, s);
      if (out_kind == QW_OUT_F32) return launch_gemm<BN, 3, EPI_F32RAW, 2>(ta, tb, p, s);
      return launch_gemm<BN, 3, EPI_BF16, 2>(ta, tb, p, s, tcp);
    }
    if (swiglu) return launch_gemm<BN, 4, EPI_SWIGLU>(ta, tb, p, s, tcp);
    if (out_kind == QW_OUT_F32_OF_BF16) return launch_gemm<BN, 4, EPI_F32>(ta, tb, p, s);
    if (out_kind == QW_OUT_F32) return launch_gemm<BN, 4, EPI_F32RAW>(ta, tb, p, s);
    return launch_gemm<BN, 4, EPI_BF16>(ta, tb, p, s, tcp);
  }

  // Skinny: A = weights [N, K] (streamed once), B = activations [M, K]
  SkinnyPlan pl = plan_skinny(M, N, K);
  if ((rc = make_tmap(&ta, w, N, K, ldw, BM)) != QW_OK) return rc;
  if ((rc = make_tmap(&tb, x, M, K, ldx, pl.bn)) != QW_OK) return rc;
  p.a_rows = (int)N;
  p.b_rows = (int)M;
  p.a_tiles = pl.a_tiles;
  p.b_tiles = 1;
  p.k_splits = pl.splits;
  p.kb_per_split = pl.kb_per_split;
  p.swap = 1;
  p.group = 1;
  if (out_kind == QW_OUT_SWIGLU && pl.splits == 1) {
    // gate and up rows of the same output columns in one tile: SwiGLU in the epilogue
    if ((rc = make_tmap(&ta, w, N, K, ldw, 64)) != QW_OK) return rc;
    p.a_rows = (int)n_out;
    p.a_tiles = (int)((n_out + 63) / 64);
    p.b_up_offset = (int)n_out;
    p.out = y;
    p.ldo = ldy;
    switch (pl.bn) {
      case 16: return launch_gemm<16, 8, EPI_SWIGLU_SWAP>(ta, tb, p, s);
      case 32: return launch_gemm<32, 8, EPI_SWIGLU_SWAP>(ta, tb, p, s);
      default: return launch_gemm<64, 8, EPI_SWIGLU_SWAP>(ta, tb, p, s);
    }
  }
  // raw fp32 outputs always take the partial + reduce route (one instantiation fewer per tile width)
  const bool partial = pl.splits > 1 || out_kind == QW_OUT_SWIGLU || out_kind == QW_OUT_F32;
  if (!partial) {
    p.out = y;
    p.ldo = ldy;
    const bool f32 = out_kind == QW_OUT_F32_OF_BF16;
    switch (pl.bn) {
      case 16: return f32 ? launch_gemm<16, 8, EPI_F32>(ta, tb, p, s) : launch_gemm<16, 8, EPI_BF16>(ta, tb, p, s);
      case 32: return f32 ? launch_gemm<32, 8, EPI_F32>(ta, tb, p, s) : launch_gemm<32, 8, EPI_BF16>(ta, tb, p, s);
      default: return f32 ? launch_gemm<64, 8, EPI_F32>(ta, tb, p, s) : launch_gemm<64, 8, EPI_BF16>(ta, tb, p, s);
    }
  }
  const size_t need = (size_t)pl.splits * (size_t)M * (size_t)N * sizeof(float);
  QW_CHECK_ARG(workspace != nullptr && ws_bytes >= need, QW_ERR_WORKSPACE);
  QW_CHECK_ARG(((uintptr_t)workspace % 16) == 0, QW_ERR_ALIGN);
  p.out = workspace;
  p.ldo = N;  // partial rows are [M][N] per split
  p.part_stride = (int64_t)M * N;
  switch (pl.bn) {
    case 16: rc = launch_gemm<16, 8, EPI_PARTIAL>(ta, tb, p, s); break;
    case 32: rc = launch_gemm<32, 8, EPI_PARTIAL>(ta, tb, p, s); break;
    default: rc = launch_gemm<64, 8, EPI_PARTIAL>(ta, tb, p, s); break;
  }
  if (rc != QW_OK) return rc;
  const int64_t total = M * n_out;
  const int threads = 256;
  const int blocks = (int)((total + threads - 1) / threads);
  const float* ws = reinterpret_cast<const float*>(workspace);
  if (out_kind == QW_OUT_SWIGLU)
    launch_k(qw_pdl_small(), splitk_reduce_kernel<EPI_SWIGLU>, dim3(blocks), dim3(threads), 0, s, ws, y, (int)M, (int)n_out, ldy, pl.splits, p.part_stride, N, (int)n_out);
  else if (out_kind == QW_OUT_F32_OF_BF16)
    launch_k(qw_pdl_small(), splitk_reduce_kernel<EPI_F32>, dim3(blocks), dim3(threads), 0, s, ws, y, (int)M, (int)n_out, ldy, pl.splits, p.part_stride, N, 0);
  else if (out_kind == QW_OUT_F32)
    launch_k(qw_pdl_small(), splitk_reduce_kernel<EPI_F32RAW>, dim3(blocks), dim3(threads), 0, s, ws, y, (int)M, (int)n_out, ldy, pl.splits, p.part_stride, N, 0);
  else
    launch_k(qw_pdl_small(), splitk_reduce_kernel<EPI_BF16>, dim3(blocks), dim3(threads), 0, s, ws, y, (int)M, (int)n_out, ldy, pl.splits, p.part_stride, N, 0);
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_add_rmsnorm(void* x, void* resid, const void* w, int64_t T, int64_t H, float eps,
                              qw_stream_t stream);  // norm.cu

extern "C" size_t qw_gemm_add_rmsnorm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (!use_skinny(M)) {
    const int s = plan_wide_splits(M, N, K);
    return s > 1 ? (size_t)s * (size_t)M * (size_t)N * sizeof(float) : 0;
  }
  const SkinnyPlan pl = plan_skinny(M, N, K);
  return (size_t)pl.splits * (size_t)M * (size_t)N * sizeof(float);
}

extern "C" int qw_gemm_add_rmsnorm_kernels(int64_t M, int64_t N, int64_t K) {
  if (!use_skinny(M)) return 2;
  const SkinnyPlan pl = plan_skinny(M, N, K);
  const int units = pl.a_tiles * pl.splits;
  const int grid = units < num_sms() ? units : num_sms();
  return (grid >= M && N <= 48 * gemm_threads<1>()) ? 1 : 2;
}

extern "C" int qw_gemm_add_rmsnorm(const void* x, const void* w, int64_t M, int64_t N, int64_t K, int64_t ldx,
                                   int64_t ldw, void* resid, const void* norm_w, void* hidden, float eps,
                                   void* workspace, size_t ws_bytes, qw_stream_t stream) {
  QW_CHECK_ARG(x && w && resid && norm_w && hidden && M > 0 && N > 0 && K > 0 && ldx >= K && ldw >= K, QW_ERR_ARG);
  QW_CHECK_ARG(N % 8 == 0 && N <= kAddNormMaxThreads * 8 && M <= 0x7fffffff, QW_ERR_UNSUPPORTED);
  QW_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)w % 16) == 0 && (ldx % 8) == 0 && (ldw % 8) == 0 &&
                   ((uintptr_t)resid % 16) == 0 && ((uintptr_t)hidden % 16) == 0 && ((uintptr_t)norm_w % 16) == 0,
               QW_ERR_ALIGN);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc;
  if (!use_skinny(M)) {
    const int splits = plan_wide_splits(M, N, K);
    if (splits == 1) {
      // enough tiles: bf16 product into hidden, then the in-place add-norm
      if ((rc = qw_gemm_bf16(x, w, hidden, M, N, K, ldx, ldw, N, QW_OUT_BF16, nullptr, 0, stream)) != QW_OK)
        return rc;
      return qw_add_rmsnorm(hidden, resid, norm_w, M, N, eps, stream);
    }
    const size_t need = (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
    QW_CHECK_ARG(workspace != nullptr && ws_bytes >= need, QW_ERR_WORKSPACE);
    QW_CHECK_ARG(((uintptr_t)workspace % 16) == 0, QW_ERR_ALIGN);
    if ((rc = launch_wide_partials(x, w, M, N, K, ldx, ldw, splits, workspace, s)) != QW_OK) return rc;
    const int threads = (int)((N / 8 + 31) / 32 * 32);
    launch_k(qw_pdl_small(), splitk_add_rmsnorm_kernel, dim3((unsigned)M), dim3(threads), 0, s, 
        static_cast<const float*>(workspace), splits, M * N, (int)N, static_cast<__nv_bfloat16*>(resid),
        static_cast<const __nv_bfloat16*>(norm_w), static_cast<__nv_bfloat16*>(hidden), eps);
    QW_LAUNCH_CHECK();
    return QW_OK;
  }
  const SkinnyPlan pl = plan_skinny(M, N, K);
  const size_t need = (size_t)pl.splits * (size_t)M * (size_t)N * sizeof(float);
  QW_CHECK_ARG(workspace != nullptr && ws_bytes >= need, QW_ERR_WORKSPACE);
  QW_CHECK_ARG(((uintptr_t)workspace % 16) == 0, QW_ERR_ALIGN);
  CUtensorMap ta, tb;
  if ((rc = make_tmap(&ta, w, N, K, ldw, BM)) != QW_OK) return rc;
  if ((rc = make_tmap(&tb, x, M, K, ldx, pl.bn)) != QW_OK) return rc;
  GemmParams p{};
  p.err = device_error_ptr();
  p.K = (int)K;
  p.kb_total = pl.kb_total;
  p.group = 1;
  p.a_rows = (int)N;
  p.b_rows = (int)M;
  p.a_tiles = pl.a_tiles;
  p.b_tiles = 1;
  p.k_splits = pl.splits;
  p.kb_per_split = pl.kb_per_split;
  p.swap = 1;
  p.out = workspace;
  p.ldo = N;
  p.part_stride = (int64_t)M * N;
  // the add-norm inside the GEMM when the grid has a CTA for every row (partial_norm_finish)
  const int units = p.a_tiles * p.b_tiles * p.k_splits;
  const int grid = units < num_sms() ? units : num_sms();
  int* counter = norm_counter_ptr();
  if (grid >= M && N <= 48 * gemm_threads<1>() && counter != nullptr) {
    p.norm_rows = (int)M;
    p.norm_counter = counter;
    p.resid = static_cast<__nv_bfloat16*>(resid);
    p.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
    p.hidden = static_cast<__nv_bfloat16*>(hidden);
    p.eps = eps;
  }
  switch (pl.bn) {
    case 16: rc = launch_gemm<16, 8, EPI_PARTIAL>(ta, tb, p, s); break;
    case 32: rc = launch_gemm<32, 8, EPI_PARTIAL>(ta, tb, p, s); break;
    default: rc = launch_gemm<64, 8, EPI_PARTIAL>(ta, tb, p, s); break;
  }
  if (rc != QW_OK || p.norm_rows > 0) return rc;
  const int threads = (int)((N / 8 + 31) / 32 * 32);
  launch_k(qw_pdl_small(), splitk_add_rmsnorm_kernel, dim3((unsigned)M), dim3(threads), 0, s, 
      static_cast<const float*>(workspace), pl.splits, p.part_stride, (int)N, static_cast<__nv_bfloat16*>(resid),
      static_cast<const __nv_bfloat16*>(norm_w), static_cast<__nv_bfloat16*>(hidden), eps);
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_gemm_add_rmsnorm_tp(const void* x, const void* w, int64_t M, int64_t N, int64_t K, int64_t ldx,
                                      int64_t ldw, void* resid, const void* norm_w, void* hidden, float eps,
                                      void* workspace, size_t ws_bytes, const void* peer_bases, int64_t world,
                                      int64_t rank, int64_t slot, int64_t round_only, qw_stream_t stream) {
  QW_CHECK_ARG(x && w && hidden && peer_bases && M > 0 && N > 0 && K > 0 && ldx >= K && ldw >= K, QW_ERR_ARG);
  QW_CHECK_ARG(round_only || (resid && norm_w), QW_ERR_ARG);
  QW_CHECK_ARG(world >= 2 && world <= QW_TP_MAX_WORLD && rank >= 0 && rank < world && slot >= 0 && slot < 3,
               QW_ERR_ARG);
  QW_CHECK_ARG(use_skinny(M) && M <= QW_TP_MAX_ROWS && N % 8 == 0 && N <= 48 * gemm_threads<1>(), QW_ERR_UNSUPPORTED);
  QW_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)w % 16) == 0 && (ldx % 8) == 0 && (ldw % 8) == 0 &&
                   ((uintptr_t)hidden % 16) == 0 && ((uintptr_t)resid % 16) == 0 && ((uintptr_t)norm_w % 16) == 0,
               QW_ERR_ALIGN);
  const SkinnyPlan pl = plan_skinny(M, N, K);
  const int units = pl.a_tiles * pl.splits;
  const int grid = units < num_sms() ? units : num_sms();
  int* counter = norm_counter_ptr();
  QW_CHECK_ARG(grid >= M && counter != nullptr, QW_ERR_UNSUPPORTED);
  const size_t need = (size_t)pl.splits * (size_t)M * (size_t)N * sizeof(float);
  QW_CHECK_ARG(workspace != nullptr && ws_bytes >= need, QW_ERR_WORKSPACE);
  QW_CHECK_ARG(((uintptr_t)workspace % 16) == 0, QW_ERR_ALIGN);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc;
  CUtensorMap ta, tb;
  if ((rc = make_tmap(&ta, w, N, K, ldw, BM)) != QW_OK) return rc;
  if ((rc = make_tmap(&tb, x, M, K, ldx, pl.bn)) != QW_OK) return rc;
  GemmParams p{};
  p.err = device_error_ptr();
  p.K = (int)K;
  p.kb_total = pl.kb_total;
  p.group = 1;
  p.a_rows = (int)N;
  p.b_rows = (int)M;
  p.a_tiles = pl.a_tiles;
  p.b_tiles = 1;
  p.k_splits = pl.splits;
  p.kb_per_split = pl.kb_per_split;
  p.swap = 1;
  p.out = workspace;
  p.ldo = N;
  p.part_stride = (int64_t)M * N;
  p.norm_rows = (int)M;
  p.norm_counter = counter;
  p.resid = static_cast<__nv_bfloat16*>(resid);
  p.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  p.hidden = static_cast<__nv_bfloat16*>(hidden);
  p.eps = eps;
  p.tp_world = (int)world;
  p.tp_rank = (int)rank;
  p.tp_round_only = round_only ? 1 : 0;
  p.tp_bases = static_cast<const unsigned long long*>(peer_bases);
  p.tp_slot_off = (int64_t)QW_TP_HEADER_BYTES + slot * (int64_t)QW_TP_MAX_ROWS * N * (int64_t)sizeof(float);
  switch (pl.bn) {
    case 16: return launch_gemm<16, 8, EPI_PARTIAL>(ta, tb, p, s);
    case 32: return launch_gemm<32, 8, EPI_PARTIAL>(ta, tb, p, s);
    default: return launch_gemm<64, 8, EPI_PARTIAL>(ta, tb, p, s);
  }
}

// ------------------------------------------------------------------ attention projection
// Whether qw_gemm_qkv_rope_store takes a split-K product (decode, a chunk whose tiles leave SMs
// idle) and its partial count; 0: the whole epilogue runs in the GEMM (one kernel).
static int qkv_splits(int64_t M, int64_t N, int64_t K, int64_t d, int64_t rd) {
  if (use_skinny(M)) return plan_skinny(M, N, K).splits;
  const int s = plan_wide_splits(M, N, K);
  if (s > 1) return s;
  return (d == 256 && rd == 64) ? 0 : -1;  // -1: GEMM, then qk_norm_rope_store (other head sizes)
}

extern "C" size_t qw_gemm_qkv_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t d, int64_t rotary_dim) {
  const int s = qkv_splits(M, N, K, d, rotary_dim);
  return s > 0 ? (size_t)s * (size_t)M * (size_t)N * sizeof(float) : 0;
}

extern "C" int qw_gemm_qkv_rope_store(const void* x, const void* w, void* qkv, int64_t M, int64_t N, int64_t K,
                                      int64_t ldx, int64_t ldw, int64_t ldq, int64_t nq, int64_t nkv, int64_t d,
                                      const void* q_w, const void* k_w, const float* rope, int64_t rotary_dim,
                                      int64_t rope_rows, const int32_t* positions, const int32_t* locations,
                                      void* k_cache, void* v_cache, int64_t cache_rows, float eps, void* workspace,
                                      size_t ws_bytes, qw_stream_t stream) {
  QW_CHECK_ARG(x && w && qkv && q_w && k_w && rope && positions && locations && k_cache && v_cache, QW_ERR_ARG);
  QW_CHECK_ARG(M > 0 && K > 0 && ldx >= K && ldw >= K && nq > 0 && nkv > 0 && nq % nkv == 0, QW_ERR_ARG);
  QW_CHECK_ARG(N == (2 * nq + 2 * nkv) * d && ldq >= N && M < (1 << 30) && N < (1 << 30), QW_ERR_ARG);
  QW_CHECK_ARG(rotary_dim > 0 && rotary_dim <= d && rotary_dim % 2 == 0 && rope_rows > 0 && cache_rows > 0, QW_ERR_ARG);
  QW_CHECK_ARG(d == 64 || d == 128 || d == 256, QW_ERR_UNSUPPORTED);
  QW_CHECK_ARG(((rotary_dim / 2) % (d / 32)) == 0, QW_ERR_UNSUPPORTED);
  QW_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)w % 16) == 0 && (ldx % 8) == 0 && (ldw % 8) == 0 &&
                   ((uintptr_t)qkv % 16) == 0 && (ldq % 8) == 0 && ((uintptr_t)k_cache % 16) == 0 &&
                   ((uintptr_t)v_cache % 16) == 0 && ((uintptr_t)q_w % 16) == 0 && ((uintptr_t)k_w % 16) == 0,
               QW_ERR_ALIGN);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int splits = qkv_splits(M, N, K, d, rotary_dim);
  if (splits < 0) {
    int rc = qw_gemm_bf16(x, w, qkv, M, N, K, ldx, ldw, ldq, QW_OUT_BF16, workspace, ws_bytes, stream);
    if (rc != QW_OK) return rc;
    return qw_qk_norm_rope_store(qkv, ldq, M, nq, nkv, d, q_w, k_w, rope, rotary_dim, rope_rows, positions, locations,
                                 k_cache, v_cache, cache_rows, eps, stream);
  }
  int rc;
  if (splits == 0) {
    // one kernel: 256-column tiles are head segments, the epilogue is qkv_tile_row
    CUtensorMap ta, tb;
    GemmParams p{};
    p.err = device_error_ptr();
    p.K = (int)K;
    p.kb_total = (int)((K + BK - 1) / BK);
    p.a_rows = (int)M;
    p.b_rows = (int)N;
    p.b_tiles = (int)(N / 256);
    p.k_splits = 1;
    p.kb_per_split = p.kb_total;
    p.swap = 0;
    p.out = qkv;
    p.ldo = ldq;
    p.vec_ok = 1;
    p.eps = eps;
    p.qkv_nq = (int)nq;
    p.qkv_nkv = (int)nkv;
    p.q_w = static_cast<const __nv_bfloat16*>(q_w);
    p.k_w = static_cast<const __nv_bfloat16*>(k_w);
    p.rope = rope;
    p.rope_rows = rope_rows;
    p.positions = positions;
    p.locs = locations;
    p.kc = static_cast<__nv_bfloat16*>(k_cache);
    p.vc = static_cast<__nv_bfloat16*>(v_cache);
    p.cache_rows = cache_rows;
    if (M >= 256 && gemm_pair_mode() != 0) {
      if ((rc = make_tmap(&ta, x, M, K, ldx, BM)) != QW_OK) return rc;
      if ((rc = make_tmap(&tb, w, N, K, ldw, P_BN / 2)) != QW_OK) return rc;
      p.a_tiles = (int)((M + 255) / 256);
      p.group = raster_group(kGroup256);
      if ((gemm_wide_mode() & 4) && (N / 256) % 2 == 0) {
        p.b_tiles = (int)(N / 512);  // two head segments per unit
        return launch_pair<EPI_QKV, 2>(ta, tb, p, s);
      }
      return launch_pair<EPI_QKV>(ta, tb, p, s);
    }
    if ((rc = make_tmap(&ta, x, M, K, ldx, BM)) != QW_OK) return rc;
    if ((rc = make_tmap(&tb, w, N, K, ldw, 256)) != QW_OK) return rc;
    p.a_tiles = (int)((M + BM - 1) / BM);
    p.group = raster_group(24);
    return launch_gemm<256, 4, EPI_QKV>(ta, tb, p, s);
  }
  const size_t need = (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
  QW_CHECK_ARG(workspace != nullptr && ws_bytes >= need, QW_ERR_WORKSPACE);
  QW_CHECK_ARG(((uintptr_t)workspace % 16) == 0, QW_ERR_ALIGN);
  if (use_skinny(M)) {
    const SkinnyPlan pl = plan_skinny(M, N, K);
    CUtensorMap ta, tb;
    if ((rc = make_tmap(&ta, w, N, K, ldw, BM)) != QW_OK) return rc;
    if ((rc = make_tmap(&tb, x, M, K, ldx, pl.bn)) != QW_OK) return rc;
    GemmParams p{};
    p.err = device_error_ptr();
    p.K = (int)K;
    p.kb_total = pl.kb_total;
    p.group = 1;
    p.a_rows = (int)N;
    p.b_rows = (int)M;
    p.a_tiles = pl.a_tiles;
    p.b_tiles = 1;
    p.k_splits = pl.splits;
    p.kb_per_split = pl.kb_per_split;
    p.swap = 1;
    p.out = workspace;
    p.ldo = N;
    p.part_stride = (int64_t)M * N;
    switch (pl.bn) {
      case 16: rc = launch_gemm<16, 8, EPI_PARTIAL>(ta, tb, p, s); break;
      case 32: rc = launch_gemm<32, 8, EPI_PARTIAL>(ta, tb, p, s); break;
      default: rc = launch_gemm<64, 8, EPI_PARTIAL>(ta, tb, p, s); break;
    }
  } else {
    rc = launch_wide_partials(x, w, M, N, K, ldx, ldw, splits, workspace, s);
  }
  if (rc != QW_OK) return rc;
  const int64_t warps = M * (2 * nq + 2 * nkv);
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  const float* ws = static_cast<const float*>(workspace);
  auto* q = static_cast<__nv_bfloat16*>(qkv);
  const auto* qw_ = static_cast<const __nv_bfloat16*>(q_w);
  const auto* kw_ = static_cast<const __nv_bfloat16*>(k_w);
  auto* kc = static_cast<__nv_bfloat16*>(k_cache);
  auto* vc = static_cast<__nv_bfloat16*>(v_cache);
  int* err = device_error_ptr();
  const int nsp = use_skinny(M) ? plan_skinny(M, N, K).splits : splits;
#define QW_QKV_FINISH(DD)                                                                                            \
  launch_k(qw_pdl_small(), qkv_finish_kernel<DD>, dim3(blocks), dim3(256), 0, s, ws, nsp, M * N, (int)N, (int)M, q, ldq, (int)nq, (int)nkv, qw_, kw_, \
                                               rope, (int)rotary_dim, rope_rows, positions, locations, kc, vc,     \
                                               cache_rows, eps, err)
  if (d == 256) QW_QKV_FINISH(256);
  else if (d == 128) QW_QKV_FINISH(128);
  else QW_QKV_FINISH(64);
#undef QW_QKV_FINISH
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_add_rmsnorm_f32(const float* x, int64_t n_parts, int64_t part_stride, int64_t T, int64_t H,
                                  void* resid, const void* norm_w, void* hidden, float eps, qw_stream_t stream) {
  QW_CHECK_ARG(x && resid && norm_w && hidden && T > 0 && n_parts >= 1 && part_stride >= 0, QW_ERR_ARG);
  QW_CHECK_ARG(n_parts == 1 || part_stride >= T * H, QW_ERR_ARG);
  QW_CHECK_ARG(H % 8 == 0 && H <= kAddNormMaxThreads * 8 && T <= 0x7fffffff, QW_ERR_UNSUPPORTED);
  QW_CHECK_ARG(((uintptr_t)x % 16) == 0 && (part_stride % 4) == 0 && ((uintptr_t)resid % 16) == 0 &&
                   ((uintptr_t)hidden % 16) == 0 && ((uintptr_t)norm_w % 16) == 0,
               QW_ERR_ALIGN);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int threads = (int)((H / 8 + 31) / 32 * 32);
  launch_k(qw_pdl_small(), splitk_add_rmsnorm_kernel, dim3((unsigned)T), dim3(threads), 0, s, x, (int)n_parts, part_stride, (int)H,
                                                            static_cast<__nv_bfloat16*>(resid),
                                                            static_cast<const __nv_bfloat16*>(norm_w),
                                                            static_cast<__nv_bfloat16*>(hidden), eps);
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_version(void) { return 1; }

extern "C" int qw_peek_device_error_async(int* host_dst, qw_stream_t stream) {
  if (!host_dst) return QW_ERR_ARG;
  int* word = qw::device_error_ptr();
  if (!word) return QW_ERR_CUDA_BASE + (int)cudaErrorInvalidSymbol;
  cudaError_t e = cudaMemcpyAsync(host_dst, word, sizeof(int), cudaMemcpyDeviceToHost,
                                  reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? QW_OK : QW_ERR_CUDA_BASE + (int)e;
}

extern "C" int qw_take_device_error(int* code) {
  if (!code) return QW_ERR_ARG;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return QW_ERR_CUDA_BASE + (int)e;
  int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, qw::g_device_error_word, sizeof(int));
  if (e != cudaSuccess) return QW_ERR_CUDA_BASE + (int)e;
  e = cudaMemcpyToSymbol(qw::g_device_error_word, &zero, sizeof(int));
  if (e != cudaSuccess) return QW_ERR_CUDA_BASE + (int)e;
  // nothing runs after the synchronize: a ticket pair left stale by a wait that gave up
  // starts from zero again
  const int zeros[2] = {0, 0};
  e = cudaMemcpyToSymbol(qw::g_norm_counter, zeros, sizeof(zeros));
  if (e != cudaSuccess) return QW_ERR_CUDA_BASE + (int)e;
  *code = v;
  return QW_OK;
}
