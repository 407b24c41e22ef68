// Gated-DeltaNet decode step, one token per request, fully fused and HBM-bound:
//   causal conv update of the request's q/k/v channels + SiLU   (REF:334-414)
//   fp32 L2 norm of q and k, q scaled by dk^-0.5                  (REF:1385-1388)
//   gating g = -exp(A_log) softplus(a + dt_bias), beta = bf16(sigmoid(b))  (REF:1390-1397)
//   S <- exp(g) S;  v' = beta (v - S k);  S <- S + v' k^T;  o = S q      (REF:1399-1403)
//   o rounded to bf16, then the gated RMSNorm with z                     (REF:1804-1929)
// One CTA per (request, key head): it owns the conv channels of that key head and of its
// HV/H value heads (so every conv-state channel has exactly one writer), and streams the
// HV/H fp32 states [dv, dk] once each (read + write in place at the request's slot).
#include "common.cuh"

namespace qw {

template <int DK, int DV, int RATIO>
__global__ void __launch_bounds__(256) gdn_decode_kernel(
    const __nv_bfloat16* __restrict__ qkvz, int64_t ldx, const __nv_bfloat16* __restrict__ ba, int64_t ldba,
    const __nv_bfloat16* __restrict__ conv_w, __nv_bfloat16* __restrict__ conv_state, float* __restrict__ state,
    const int32_t* __restrict__ slots, int n_slots, const float* __restrict__ A_log,
    const __nv_bfloat16* __restrict__ dt_bias, const __nv_bfloat16* __restrict__ norm_w, __nv_bfloat16* __restrict__ y,
    int64_t ldy, int H, float scale, float eps, int* err) {
  constexpr int W = 4;  // conv width
  constexpr int NCH = 2 * DK + RATIO * DV;
  const int HV = H * RATIO;
  const int C = 2 * H * DK + HV * DV;  // conv channels
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  __shared__ float s_x[NCH];  // conv output (bf16-rounded) of q | k | v(RATIO heads)
  __shared__ float s_red[8][RATIO][2];
  const int slot = slots[b];
  const bool valid = slot >= 0 && slot < n_slots;
  const __nv_bfloat16* xrow = qkvz + (int64_t)b * ldx;

  // ---- conv update of this CTA's channels
  for (int i = tid; i < NCH; i += blockDim.x) {
    int c;
    if (i < DK) c = h * DK + i;
    else if (i < 2 * DK) c = H * DK + h * DK + (i - DK);
    else c = 2 * H * DK + h * RATIO * DV + (i - 2 * DK);
    const float x = bf2f(xrow[c]);
    if (!valid) {
      s_x[i] = x;
      continue;
    }
    __nv_bfloat16* st = conv_state + ((int64_t)slot * C + c) * (W - 1);
    const float s0 = bf2f(st[0]), s1 = bf2f(st[1]), s2 = bf2f(st[2]);
    const __nv_bfloat16* wc = conv_w + (int64_t)c * W;
    float acc = 0.f;
    acc += bf16_round(s0 * bf2f(wc[0]));
    acc += bf16_round(s1 * bf2f(wc[1]));
    acc += bf16_round(s2 * bf2f(wc[2]));
    acc += bf16_round(x * bf2f(wc[3]));
    s_x[i] = bf16_round(acc / (1.0f + __expf(-acc)));
    st[0] = st[1];
    st[1] = st[2];
    st[2] = xrow[c];
  }
  __syncthreads();
  if (!valid) {
    // the reference writes o = 0 for a padded slot; the gated norm of 0 is 0
    for (int i = tid; i < RATIO * DV; i += blockDim.x)
      y[(int64_t)b * ldy + (int64_t)(h * RATIO) * DV + i] = f2bf(0.f);
    if (tid == 0 && slot != -1) set_error(err, QW_DEV_ERR_INDEX);
    return;
  }
  // ---- L2 norms of q and k (fp32, unrounded), lane owns 4 consecutive dims
  static_assert(DK == 128, "decode kernel lane layout assumes dk = 128");
  float qv[4], kv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qv[j] = s_x[lane * 4 + j];
    kv[j] = s_x[DK + lane * 4 + j];
  }
  float qq = 0.f, kk = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qq += qv[j] * qv[j];
    kk += kv[j] * kv[j];
  }
  qq = warp_sum(qq);
  kk = warp_sum(kk);
  const float qden = sqrtf(qq + 1e-6f), kden = sqrtf(kk + 1e-6f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qv[j] = (qv[j] / qden) * scale;
    kv[j] = kv[j] / kden;
  }
  float kq = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) kq += kv[j] * qv[j];
  kq = warp_sum(kq);

  // ---- per value head: state update; warp w owns value rows [w*DV/8, (w+1)*DV/8)
  constexpr int ROWS = DV / 8;
  for (int r = 0; r < RATIO; ++r) {
    const int hv = h * RATIO + r;
    const float a = bf2f(ba[(int64_t)b * ldba + HV + hv]);
    const float bb = bf2f(ba[(int64_t)b * ldba + hv]);
    const float xg = a + bf2f(dt_bias[hv]);
    const float sp = xg <= 20.f ? logf(1.f + expf(xg)) : xg;
    const float g = -expf(A_log[hv]) * sp;
    const float alpha = expf(g);
    const float beta = bf16_round(1.f / (1.f + expf(-bb)));
    float* S = state + (((int64_t)slot * HV + hv) * DV) * DK;
    float4 sv[ROWS];
#pragma unroll
    for (int i = 0; i < ROWS; ++i)
      sv[i] = *reinterpret_cast<const float4*>(S + (int64_t)(warp * ROWS + i) * DK + lane * 4);
    float ov[ROWS];
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const float4 s4 = sv[i];
      float sk = s4.x * kv[0] + s4.y * kv[1] + s4.z * kv[2] + s4.w * kv[3];
      float sq = s4.x * qv[0] + s4.y * qv[1] + s4.z * qv[2] + s4.w * qv[3];
      sk = warp_sum(sk);
      sq = warp_sum(sq);
      const int row = warp * ROWS + i;
      const float vrow = s_x[2 * DK + r * DV + row];
      const float vp = beta * (vrow - alpha * sk);
      ov[i] = alpha * sq + vp * kq;
      float4 n4;
      n4.x = alpha * s4.x + vp * kv[0];
      n4.y = alpha * s4.y + vp * kv[1];
      n4.z = alpha * s4.z + vp * kv[2];
      n4.w = alpha * s4.w + vp * kv[3];
      *reinterpret_cast<float4*>(S + (int64_t)row * DK + lane * 4) = n4;
    }
    // ---- gated RMSNorm over the DV outputs of this head (o rounded to bf16 first)
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      ov[i] = bf16_round(ov[i]);
      ss += ov[i] * ov[i];
    }
    if (lane == 0) s_red[warp][r][0] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += s_red[w][r][0];
    const float rstd = rsqrtf(tot / (float)DV + eps);
    if (lane < ROWS) {
      // lane i of the warp writes row warp*ROWS + i
      float o_l = 0.f;
#pragma unroll
      for (int i = 0; i < ROWS; ++i)
        if (i == lane) o_l = ov[i];
      const int row = warp * ROWS + lane;
      const float z = bf2f(xrow[C + hv * DV + row]);
      const float gz = z / (1.f + __expf(-z));
      y[(int64_t)b * ldy + (int64_t)hv * DV + row] = f2bf(o_l * rstd * bf2f(norm_w[row]) * gz);
    }
  }
}

}  // namespace qw

using namespace qw;

extern "C" int qw_gdn_decode(const void* qkvz, int64_t ldx, const void* ba, int64_t ldba, const void* conv_w,
                             void* conv_state, float* state, const int32_t* slots, int64_t B, int64_t n_slots,
                             const float* A_log, const void* dt_bias, const void* norm_w, void* y, int64_t ldy,
                             int64_t H, int64_t HV, int64_t dk, int64_t dv, float eps, qw_stream_t stream) {
  QW_CHECK_ARG(qkvz && ba && conv_w && conv_state && state && slots && A_log && dt_bias && norm_w && y, QW_ERR_ARG);
  QW_CHECK_ARG(B > 0 && H > 0 && HV % H == 0 && n_slots > 0, QW_ERR_ARG);
  QW_CHECK_ARG(((uintptr_t)state % 16) == 0, QW_ERR_ALIGN);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int ratio = (int)(HV / H);
  const unsigned grid = (unsigned)(B * H);
  const auto* x = static_cast<const __nv_bfloat16*>(qkvz);
  const auto* bap = static_cast<const __nv_bfloat16*>(ba);
  const auto* cw = static_cast<const __nv_bfloat16*>(conv_w);
  auto* cs = static_cast<__nv_bfloat16*>(conv_state);
  const auto* dt = static_cast<const __nv_bfloat16*>(dt_bias);
  const auto* nw = static_cast<const __nv_bfloat16*>(norm_w);
  auto* yp = static_cast<__nv_bfloat16*>(y);
  int* err = device_error_ptr();
  if (dk == 128 && dv == 128 && ratio == 3)
    gdn_decode_kernel<128, 128, 3><<<grid, 256, 0, s>>>(x, ldx, bap, ldba, cw, cs, state, slots, (int)n_slots, A_log,
                                                        dt, nw, yp, ldy, (int)H, 1.0f / sqrtf((float)dk), eps, err);
  else if (dk == 128 && dv == 128 && ratio == 1)
    gdn_decode_kernel<128, 128, 1><<<grid, 256, 0, s>>>(x, ldx, bap, ldba, cw, cs, state, slots, (int)n_slots, A_log,
                                                        dt, nw, yp, ldy, (int)H, 1.0f / sqrtf((float)dk), eps, err);
  else
    return QW_ERR_UNSUPPORTED;
  QW_LAUNCH_CHECK();
  return QW_OK;
}
