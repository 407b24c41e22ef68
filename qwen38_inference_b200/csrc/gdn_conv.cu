// Prefill causal depthwise conv1d (width 4) + SiLU over the q|k|v channels of the GDN
// projection, the split into token-major q, k, v, the L2 norm of q and k, and the conv
// state update (REF:704-1253 conv, REF:603-699 split, REF:1550-1638 l2norm).
//
// Grid (128-channel block, strip of 256 tokens, request), 256 threads; the channel block
// varies fastest so CTAs running together cover whole token rows (DRAM page locality). A CTA
// walks its strip in 64-token tiles: while it convolves and stores tile i, the 3 history
// rows + 64 token rows of tile i+1 (128 channels, 16-byte cp.async copies) land in the other
// of two shared buffers. Rows outside the request are zero-filled by the copy itself. The
// CTA convolves from shared memory, normalizes q/k heads per token (one warp per token) and
// writes 8-byte-aligned rows. Only the first strip of a request reads its previous conv
// state (when has_initial) and writes the new one (the last 3 raw inputs of
// [old state | x]), so no other CTA touches that request's state. Per channel:
// acc = sum_j bf16(x[t-3+j] * w[j]) for j = 0..3 in order, y = bf16(silu(acc)); q and k
// heads then become bf16(y / sqrt(sum y^2 + 1e-6)).
#include "common.cuh"

namespace qw {

struct ConvSmem {
  static constexpr int BT = 64, BC = 128, HIST = 3, TILES = 4;  // tokens per tile, channels, history, tiles per strip
  static constexpr int XROWS = BT + HIST;
  static constexpr int XBUF = XROWS * BC * 2;  // one staged tile, bytes
  static constexpr int Y = 2 * XBUF;           // sy [BT][BC] bf16 after the two x buffers
  static constexpr int TOTAL = Y + BT * BC * 2;
};

template <int HD>
__global__ void __launch_bounds__(256) conv_prefill_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ w,
    __nv_bfloat16* __restrict__ conv_state, const int32_t* __restrict__ cu, const int32_t* __restrict__ slots,
    const int32_t* __restrict__ has_initial, int n_slots, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out, int qk_dim, int v_dim, int* err) {
  using L = ConvSmem;
  constexpr int BT = L::BT, BC = L::BC, W = 4, HIST = L::HIST;
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16(*sy)[BC] = reinterpret_cast<__nv_bfloat16(*)[BC]>(smem + L::Y);
  const int cb = blockIdx.x, strip = blockIdx.y, seq = blockIdx.z;
  const int t0 = cu[seq], n = cu[seq + 1] - t0;
  const int sb = strip * BT * L::TILES;  // first token of the strip, within the request
  if (sb >= n) return;
  const int C = 2 * qk_dim + v_dim;
  const int tid = threadIdx.x;
  const int c0 = cb * BC;
  const int slot = slots[seq];
  if (slot < 0 || slot >= n_slots) {
    if (tid == 0) set_error(err, QW_DEV_ERR_INDEX);
    return;
  }
  const bool first = strip == 0;
  const bool hist = first && has_initial[seq];
  const int ntiles = min(L::TILES, (n - sb + BT - 1) / BT);

  // rows tb-3 .. tb+63 of tile `tile` into buffer `buf`; tokens outside [0, n) read as zero,
  // except the history rows of a request with a cached state (written from the state below)
  auto stage = [&](int tile, int buf) {
    const int tb = sb + tile * BT;
    const uint32_t base = smem_u32(smem + buf * L::XBUF);
    for (int i = tid; i < L::XROWS * 16; i += 256) {
      const int r = i >> 4, v = i & 15;
      const int tok = tb - HIST + r;
      if (tok < 0 && hist) continue;
      const bool ok = tok >= 0 && tok < n;
      cp_async16(base + (r * BC + v * 8) * 2, x + (int64_t)(t0 + (ok ? tok : 0)) * ldx + c0 + v * 8, ok);
    }
    cp_async_commit();
  };

  stage(0, 0);
  if (first && tid < BC) {
    __nv_bfloat16* st = conv_state + ((int64_t)slot * C + c0 + tid) * (W - 1);
    __nv_bfloat16 old[HIST];
#pragma unroll
    for (int j = 0; j < HIST; ++j) old[j] = hist ? st[j] : __float2bfloat16(0.f);
    if (hist) {
      __nv_bfloat16* sx0 = reinterpret_cast<__nv_bfloat16*>(smem);
#pragma unroll
      for (int j = 0; j < HIST; ++j) sx0[j * BC + tid] = old[j];
    }
    // new state = last 3 entries of [old state | x]
    __nv_bfloat16 ns[HIST];
#pragma unroll
    for (int i = 0; i < HIST; ++i) {
      const int pos = n - HIST + i;  // index within the request; negative = history
      ns[i] = pos >= 0 ? x[(int64_t)(t0 + pos) * ldx + c0 + tid] : old[pos + HIST];
    }
#pragma unroll
    for (int i = 0; i < HIST; ++i) st[i] = ns[i];
  }

  const int cp = tid & (BC / 2 - 1), quarter = tid >> 6;
  const int c = 2 * cp;
  __nv_bfloat162 wv[W];
#pragma unroll
  for (int j = 0; j < W; ++j)
    wv[j] = __halves2bfloat162(w[(int64_t)(c0 + c) * W + j], w[(int64_t)(c0 + c + 1) * W + j]);
  const int warp = tid >> 5, lane = tid & 31;
  const bool is_v = c0 >= 2 * qk_dim;

  for (int tile = 0; tile < ntiles; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < ntiles) {
      stage(tile + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int tb = sb + tile * BT;
    const int nt = min(BT, n - tb);
    const __nv_bfloat16(*sx)[BC] = reinterpret_cast<const __nv_bfloat16(*)[BC]>(smem + buf * L::XBUF);
    // ---- convolution: thread = (channel pair, quarter of the tokens), the 16 tokens fully
    // unrolled: rows past the request are zeros in sx and their sy rows are never stored.
    // Products are bf16 x bf16 rounded to bf16 (mul.rn.bf16x2, as the reference's bf16
    // multiply), summed in fp32 in tap order; silu(a) = a * rcp(1 + exp(-a)) with the
    // approximate exp2 and reciprocal (the reference's Triton kernel divides approximately;
    // a below about -88 gives -0 in both).
    {
      const int j0 = quarter * (BT / 4);
      __nv_bfloat162 h0 = *reinterpret_cast<const __nv_bfloat162*>(&sx[j0][c]);
      __nv_bfloat162 h1 = *reinterpret_cast<const __nv_bfloat162*>(&sx[j0 + 1][c]);
      __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&sx[j0 + 2][c]);
      // the channel pair's sums and silu run on fp32 pairs (sm_100 f32x2 arithmetic, each
      // lane rounded as its scalar operation); exp(-a) = 2^(-a log2 e)
      const unsigned long long neg_log2e = f2_pack(-1.4426950408889634f, -1.4426950408889634f);
      const unsigned long long one = f2_pack(1.0f, 1.0f);
#pragma unroll
      for (int jj = 0; jj < BT / 4; ++jj) {
        const int j = j0 + jj;
        const __nv_bfloat162 xv = *reinterpret_cast<const __nv_bfloat162*>(&sx[j + HIST][c]);
        const __nv_bfloat162 q0 = __hmul2(h0, wv[0]), q1 = __hmul2(h1, wv[1]);
        const __nv_bfloat162 q2 = __hmul2(h2, wv[2]), q3 = __hmul2(xv, wv[3]);
        unsigned long long a = bf16x2_to_f2(*reinterpret_cast<const uint32_t*>(&q0));
        a = f2_add(a, bf16x2_to_f2(*reinterpret_cast<const uint32_t*>(&q1)));
        a = f2_add(a, bf16x2_to_f2(*reinterpret_cast<const uint32_t*>(&q2)));
        a = f2_add(a, bf16x2_to_f2(*reinterpret_cast<const uint32_t*>(&q3)));
        const unsigned long long t = f2_mul(a, neg_log2e);
        const unsigned long long d = f2_add(f2_pack(ex2_ftz(f2_lo(t)), ex2_ftz(f2_hi(t))), one);
        const unsigned long long y = f2_mul(a, f2_pack(rcp_approx(f2_lo(d)), rcp_approx(f2_hi(d))));
        *reinterpret_cast<__nv_bfloat162*>(&sy[j][c]) = __floats2bfloat162_rn(f2_lo(y), f2_hi(y));
        h0 = h1;
        h1 = h2;
        h2 = xv;
      }
    }
    __syncthreads();
    // ---- outputs: one warp per token row; lane owns 4 channels of the 128-channel block
    for (int j = warp; j < nt; j += 8) {
      const int64_t t = t0 + tb + j;
      uint2 u = *reinterpret_cast<const uint2*>(&sy[j][lane * 4]);
      __nv_bfloat16* dst;
      if (is_v) {
        dst = v_out + t * v_dim + (c0 - 2 * qk_dim);  // v rows as computed
      } else {
        // q / k head: y * rsqrt(sum y^2 + 1e-6) (within 2 fp32 ulp of y / sqrt(...))
        const float2 ya = bf16x2_to_float2(u.x), yb = bf16x2_to_float2(u.y);
        float ss = ya.x * ya.x + ya.y * ya.y + yb.x * yb.x + yb.y * yb.y;
#pragma unroll
        for (int o = 1; o < HD / 4; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(ss + 1e-6f);
        u.x = pack_bf16x2(ya.x * inv, ya.y * inv);
        u.y = pack_bf16x2(yb.x * inv, yb.y * inv);
        dst = c0 < qk_dim ? q_out + t * qk_dim + c0 : k_out + t * qk_dim + (c0 - qk_dim);
      }
      *reinterpret_cast<uint2*>(dst + lane * 4) = u;
    }
    __syncthreads();  // sy and this tile's buffer are rewritten by the next iteration
  }
}

}  // namespace qw

using namespace qw;

extern "C" int qw_conv_prefill(const void* x, int64_t ldx, const void* conv_w, void* conv_state,
                               const int32_t* cu_seqlens, const int32_t* slots, const int32_t* has_initial,
                               int64_t B, int64_t n_slots, int64_t max_len, void* q_out, void* k_out, void* v_out,
                               int64_t qk_dim, int64_t v_dim, int64_t head_dim, qw_stream_t stream) {
  QW_CHECK_ARG(x && conv_w && conv_state && cu_seqlens && slots && has_initial && q_out && k_out && v_out, QW_ERR_ARG);
  QW_CHECK_ARG(B > 0 && max_len > 0 && n_slots > 0, QW_ERR_ARG);
  QW_CHECK_ARG(B <= 65535 && (max_len + 63) / 64 <= 65535, QW_ERR_UNSUPPORTED);  // grid y/z limits
  QW_CHECK_ARG(qk_dim % 128 == 0 && v_dim % 128 == 0, QW_ERR_UNSUPPORTED);
  QW_CHECK_ARG(((uintptr_t)x % 16) == 0 && (ldx % 8) == 0, QW_ERR_ALIGN);
  QW_CHECK_ARG(((uintptr_t)q_out % 8) == 0 && ((uintptr_t)k_out % 8) == 0 && ((uintptr_t)v_out % 8) == 0, QW_ERR_ALIGN);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int C = (int)(2 * qk_dim + v_dim);
  constexpr int STRIP = ConvSmem::BT * ConvSmem::TILES;
  dim3 grid((unsigned)(C / 128), (unsigned)((max_len + STRIP - 1) / STRIP), (unsigned)B);
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  const auto* wp = static_cast<const __nv_bfloat16*>(conv_w);
  auto* cs = static_cast<__nv_bfloat16*>(conv_state);
  auto* qo = static_cast<__nv_bfloat16*>(q_out);
  auto* ko = static_cast<__nv_bfloat16*>(k_out);
  auto* vo = static_cast<__nv_bfloat16*>(v_out);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(conv_prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, ConvSmem::TOTAL);
    cudaFuncSetAttribute(conv_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, ConvSmem::TOTAL);
    configured = true;
  }
  if (head_dim == 128)
    conv_prefill_kernel<128><<<grid, 256, ConvSmem::TOTAL, s>>>(xp, ldx, wp, cs, cu_seqlens, slots, has_initial, (int)n_slots, qo, ko,
                                                  vo, (int)qk_dim, (int)v_dim, device_error_ptr());
  else if (head_dim == 64)
    conv_prefill_kernel<64><<<grid, 256, ConvSmem::TOTAL, s>>>(xp, ldx, wp, cs, cu_seqlens, slots, has_initial, (int)n_slots, qo, ko,
                                                 vo, (int)qk_dim, (int)v_dim, device_error_ptr());
  else
    return QW_ERR_UNSUPPORTED;
  QW_LAUNCH_CHECK();
  return QW_OK;
}
