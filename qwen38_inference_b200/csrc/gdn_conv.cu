// Prefill causal depthwise conv1d (width 4) + SiLU over the q|k|v channels of the GDN
// projection, the split into token-major q, k, v, the L2 norm of q and k, and the conv
// state update (REF:704-1253 conv, REF:603-699 split, REF:1550-1638 l2norm).
//
// Grid (128-channel block, chunk of 64 tokens, request), 256 threads; the channel block
// varies fastest so CTAs running together cover whole token rows (DRAM page locality). The CTA stages the
// 3 history rows + 64 token rows of its 128 channels in shared memory with 16-byte loads
// (all in flight together), convolves from shared memory, normalizes q/k heads per token
// (one warp per token) and writes 16-byte-aligned rows. Only chunk 0 of a request reads
// its previous conv state (when has_initial) and writes the new one (the last 3 raw inputs
// of [old state | x]), so no other CTA touches that request's state. Per channel:
// acc = sum_j bf16(x[t-3+j] * w[j]) for j = 0..3 in order, y = bf16(silu(acc)); q and k
// heads then become bf16(y / sqrt(sum y^2 + 1e-6)).
#include "common.cuh"

namespace qw {

template <int HD>
__global__ void __launch_bounds__(256) conv_prefill_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ w,
    __nv_bfloat16* __restrict__ conv_state, const int32_t* __restrict__ cu, const int32_t* __restrict__ slots,
    const int32_t* __restrict__ has_initial, int n_slots, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out, int qk_dim, int v_dim, int* err) {
  constexpr int BT = 64, BC = 128, W = 4, HIST = W - 1;
  __shared__ __align__(16) __nv_bfloat16 sx[BT + HIST][BC];
  __shared__ __align__(16) __nv_bfloat16 sy[BT][BC];  // bf16(silu(conv)), exact
  const int cb = blockIdx.x, chunk = blockIdx.y, seq = blockIdx.z;
  const int t0 = cu[seq], n = cu[seq + 1] - t0;
  const int tb = chunk * BT;
  if (tb >= n) return;
  const int C = 2 * qk_dim + v_dim;
  const int tid = threadIdx.x;
  const int c0 = cb * BC;
  const int slot = slots[seq];
  if (slot < 0 || slot >= n_slots) {
    if (tid == 0) set_error(err, QW_DEV_ERR_INDEX);
    return;
  }
  const int nt = min(BT, n - tb);
  // ---- stage rows tb-3 .. tb+nt-1 (16-byte vectors; 16 per row)
  for (int i = tid; i < (BT + HIST) * 16; i += 256) {
    const int r = i >> 4, v = i & 15;
    const int tok = tb - HIST + r;  // index within the request
    uint4 val = make_uint4(0, 0, 0, 0);
    if (tok >= 0 && tok < tb + nt) val = *reinterpret_cast<const uint4*>(x + (int64_t)(t0 + tok) * ldx + c0 + v * 8);
    *reinterpret_cast<uint4*>(&sx[r][v * 8]) = val;
  }
  __nv_bfloat16* st = conv_state + ((int64_t)slot * C + c0) * (W - 1);
  if (chunk == 0) {
    // history rows from the old state when the request has one (zeros otherwise)
    if (has_initial[seq] && tid < BC) {
#pragma unroll
      for (int j = 0; j < HIST; ++j) sx[j][tid] = st[tid * (W - 1) + j];
    }
  }
  __syncthreads();
  if (chunk == 0 && tid < BC) {
    // new state = last 3 entries of [history | x] (history is in sx rows 0..2)
    __nv_bfloat16 ns[HIST];
#pragma unroll
    for (int i = 0; i < HIST; ++i) {
      const int pos = n - HIST + i;  // index within the request; negative = history row
      ns[i] = pos >= 0 ? x[(int64_t)(t0 + pos) * ldx + c0 + tid] : sx[pos + HIST][tid];
    }
#pragma unroll
    for (int i = 0; i < HIST; ++i) st[tid * (W - 1) + i] = ns[i];
  }
  // ---- convolution: thread = (channel pair, quarter of the tokens). Products are
  // bf16 x bf16 rounded to bf16 (mul.rn.bf16x2, as the reference's bf16 multiply), summed in
  // fp32 in tap order; silu uses the approximate divide of the reference's Triton kernels.
  {
    const int cp = tid & (BC / 2 - 1), quarter = tid >> 6;
    const int c = 2 * cp;
    __nv_bfloat162 wv[W];
#pragma unroll
    for (int j = 0; j < W; ++j)
      wv[j] = __halves2bfloat162(w[(int64_t)(c0 + c) * W + j], w[(int64_t)(c0 + c + 1) * W + j]);
    const int j0 = quarter * (BT / 4);
    __nv_bfloat162 h0 = *reinterpret_cast<const __nv_bfloat162*>(&sx[j0][c]);
    __nv_bfloat162 h1 = *reinterpret_cast<const __nv_bfloat162*>(&sx[j0 + 1][c]);
    __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&sx[j0 + 2][c]);
    for (int j = j0; j < j0 + BT / 4 && j < nt; ++j) {
      const __nv_bfloat162 xv = *reinterpret_cast<const __nv_bfloat162*>(&sx[j + HIST][c]);
      const float2 p0 = __bfloat1622float2(__hmul2(h0, wv[0]));
      const float2 p1 = __bfloat1622float2(__hmul2(h1, wv[1]));
      const float2 p2 = __bfloat1622float2(__hmul2(h2, wv[2]));
      const float2 p3 = __bfloat1622float2(__hmul2(xv, wv[3]));
      float a0 = 0.f, a1 = 0.f;
      a0 += p0.x; a1 += p0.y;
      a0 += p1.x; a1 += p1.y;
      a0 += p2.x; a1 += p2.y;
      a0 += p3.x; a1 += p3.y;
      *reinterpret_cast<__nv_bfloat162*>(&sy[j][c]) =
          __floats2bfloat162_rn(__fdividef(a0, 1.0f + __expf(-a0)), __fdividef(a1, 1.0f + __expf(-a1)));
      h0 = h1;
      h1 = h2;
      h2 = xv;
    }
  }
  __syncthreads();
  // ---- outputs: one warp per token row; lane owns 4 channels of the 128-channel block
  const int warp = tid >> 5, lane = tid & 31;
  const bool is_v = c0 >= 2 * qk_dim;
  for (int j = warp; j < nt; j += 8) {
    float y[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) y[e] = bf2f(sy[j][lane * 4 + e]);
    if (!is_v) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) ss += y[e] * y[e];
#pragma unroll
      for (int o = 1; o < HD / 4; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float den = sqrtf(ss + 1e-6f);
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = y[e] / den;
    }
    const int64_t t = t0 + tb + j;
    __nv_bfloat16* dst;
    if (c0 < qk_dim) dst = q_out + t * qk_dim + c0;
    else if (c0 < 2 * qk_dim) dst = k_out + t * qk_dim + (c0 - qk_dim);
    else dst = v_out + t * v_dim + (c0 - 2 * qk_dim);
    uint2 u;
    u.x = pack_bf16x2(y[0], y[1]);
    u.y = pack_bf16x2(y[2], y[3]);
    *reinterpret_cast<uint2*>(dst + lane * 4) = u;
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
  dim3 grid((unsigned)(C / 128), (unsigned)((max_len + 63) / 64), (unsigned)B);
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  const auto* wp = static_cast<const __nv_bfloat16*>(conv_w);
  auto* cs = static_cast<__nv_bfloat16*>(conv_state);
  auto* qo = static_cast<__nv_bfloat16*>(q_out);
  auto* ko = static_cast<__nv_bfloat16*>(k_out);
  auto* vo = static_cast<__nv_bfloat16*>(v_out);
  if (head_dim == 128)
    conv_prefill_kernel<128><<<grid, 256, 0, s>>>(xp, ldx, wp, cs, cu_seqlens, slots, has_initial, (int)n_slots, qo, ko,
                                                  vo, (int)qk_dim, (int)v_dim, device_error_ptr());
  else if (head_dim == 64)
    conv_prefill_kernel<64><<<grid, 256, 0, s>>>(xp, ldx, wp, cs, cu_seqlens, slots, has_initial, (int)n_slots, qo, ko,
                                                 vo, (int)qk_dim, (int)v_dim, device_error_ptr());
  else
    return QW_ERR_UNSUPPORTED;
  QW_LAUNCH_CHECK();
  return QW_OK;
}
