// Prefill causal depthwise conv1d (width 4) + SiLU over the q|k|v channels of the GDN
// projection, the split into token-major q, k, v, the L2 norm of q and k, and the conv
// state update (REF:704-1253 conv, REF:603-699 split, REF:1550-1638 l2norm).
//
// Grid (request, chunk of 64 tokens, 128-channel block). Only chunk 0 of a request reads
// its previous conv state (when has_initial) and writes the new one (the last W-1 raw
// inputs of [old state | x]), so no other CTA touches that request's state. Per channel:
// acc = sum_j bf16(x[t-3+j] * w[j]) for j = 0..3 in order, y = bf16(silu(acc)); q and k
// heads then become bf16(y / sqrt(sum y^2 + 1e-6)).
#include "common.cuh"

namespace qw {

template <int HD>
__global__ void __launch_bounds__(128) conv_prefill_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ w,
    __nv_bfloat16* __restrict__ conv_state, const int32_t* __restrict__ cu, const int32_t* __restrict__ slots,
    const int32_t* __restrict__ has_initial, int n_slots, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out, int qk_dim, int v_dim, int* err) {
  constexpr int BT = 64, BC = 128, W = 4;
  __shared__ float sy[BT][BC + 1];
  const int seq = blockIdx.x, chunk = blockIdx.y, cb = blockIdx.z;
  const int t0 = cu[seq], n = cu[seq + 1] - t0;
  const int tb = chunk * BT;
  if (tb >= n) return;
  const int C = 2 * qk_dim + v_dim;
  const int tid = threadIdx.x;
  const int c = cb * BC + tid;
  const int slot = slots[seq];
  if (slot < 0 || slot >= n_slots) {
    if (tid == 0) set_error(err, QW_DEV_ERR_INDEX);
    return;
  }
  const float w0 = bf2f(w[(int64_t)c * W + 0]), w1 = bf2f(w[(int64_t)c * W + 1]);
  const float w2 = bf2f(w[(int64_t)c * W + 2]), w3 = bf2f(w[(int64_t)c * W + 3]);
  float h0, h1, h2;  // x[t-3], x[t-2], x[t-1]
  __nv_bfloat16* st = conv_state + ((int64_t)slot * C + c) * (W - 1);
  if (chunk == 0) {
    if (has_initial[seq]) {
      h0 = bf2f(st[0]);
      h1 = bf2f(st[1]);
      h2 = bf2f(st[2]);
    } else {
      h0 = h1 = h2 = 0.f;
    }
    // new state = last 3 entries of [history | x]
    __nv_bfloat16 ns[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const int pos = n - 3 + i;  // index into x of this request; negative = history
      if (pos >= 0) ns[i] = x[(int64_t)(t0 + pos) * ldx + c];
      else ns[i] = f2bf(pos == -1 ? h2 : pos == -2 ? h1 : h0);
    }
    st[0] = ns[0];
    st[1] = ns[1];
    st[2] = ns[2];
  } else {
    h0 = bf2f(x[(int64_t)(t0 + tb - 3) * ldx + c]);
    h1 = bf2f(x[(int64_t)(t0 + tb - 2) * ldx + c]);
    h2 = bf2f(x[(int64_t)(t0 + tb - 1) * ldx + c]);
  }
  const int nt = min(BT, n - tb);
  for (int j = 0; j < nt; ++j) {
    const float xv = bf2f(x[(int64_t)(t0 + tb + j) * ldx + c]);
    float acc = 0.f;
    acc += bf16_round(h0 * w0);
    acc += bf16_round(h1 * w1);
    acc += bf16_round(h2 * w2);
    acc += bf16_round(xv * w3);
    sy[j][tid] = bf16_round(acc / (1.0f + __expf(-acc)));
    h0 = h1;
    h1 = h2;
    h2 = xv;
  }
  __syncthreads();
  // ---- outputs: 4 warps x 16 tokens; lane owns 4 channels of the 128-channel block
  const int warp = tid >> 5, lane = tid & 31;
  const int c0 = cb * BC;
  const bool is_v = c0 >= 2 * qk_dim;
  for (int j = warp; j < nt; j += 4) {
    float y[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) y[e] = sy[j][lane * 4 + e];
    if (!is_v) {
      // L2 norm per head of HD channels (HD = 128: whole warp; HD = 64: half warp)
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
  QW_CHECK_ARG(qk_dim % 128 == 0 && v_dim % 128 == 0, QW_ERR_UNSUPPORTED);
  QW_CHECK_ARG(((uintptr_t)q_out % 8) == 0 && ((uintptr_t)k_out % 8) == 0 && ((uintptr_t)v_out % 8) == 0, QW_ERR_ALIGN);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int C = (int)(2 * qk_dim + v_dim);
  dim3 grid((unsigned)B, (unsigned)((max_len + 63) / 64), (unsigned)(C / 128));
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  const auto* wp = static_cast<const __nv_bfloat16*>(conv_w);
  auto* cs = static_cast<__nv_bfloat16*>(conv_state);
  auto* qo = static_cast<__nv_bfloat16*>(q_out);
  auto* ko = static_cast<__nv_bfloat16*>(k_out);
  auto* vo = static_cast<__nv_bfloat16*>(v_out);
  if (head_dim == 128)
    conv_prefill_kernel<128><<<grid, 128, 0, s>>>(xp, ldx, wp, cs, cu_seqlens, slots, has_initial, (int)n_slots, qo, ko,
                                                  vo, (int)qk_dim, (int)v_dim, device_error_ptr());
  else if (head_dim == 64)
    conv_prefill_kernel<64><<<grid, 128, 0, s>>>(xp, ldx, wp, cs, cu_seqlens, slots, has_initial, (int)n_slots, qo, ko,
                                                 vo, (int)qk_dim, (int)v_dim, device_error_ptr());
  else
    return QW_ERR_UNSUPPORTED;
  QW_LAUNCH_CHECK();
  return QW_OK;
}
