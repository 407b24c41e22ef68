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

// v[i] = this lane's part of row i's sum (16 rows over a warp's 32 lanes). Halving exchange:
// at each step a lane keeps half of its rows and adds its partner's copy of them. Lanes
// 2i and 2i+1 return row i's full sum, summed in a fixed order on every lane.
QW_DEV float rows16_sum(const float (&v)[16], int lane) {
  float a[8];
  const bool h16 = lane & 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float send = h16 ? v[i] : v[i + 8], keep = h16 ? v[i + 8] : v[i];
    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float c[4];
  const bool h8 = lane & 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = h8 ? a[i] : a[i + 4], keep = h8 ? a[i + 4] : a[i];
    c[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float d[2];
  const bool h4 = lane & 4;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = h4 ? c[i] : c[i + 2], keep = h4 ? c[i + 2] : c[i];
    d[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  const bool h2 = lane & 2;
  const float e = (h2 ? d[1] : d[0]) + __shfl_xor_sync(0xffffffffu, h2 ? d[0] : d[1], 2);
  return e + __shfl_xor_sync(0xffffffffu, e, 1);
}

template <int DK, int DV, int RATIO>
__global__ void __launch_bounds__(256, 2) gdn_decode_kernel(
    const __nv_bfloat16* __restrict__ qkvz, int64_t ldx, const __nv_bfloat16* __restrict__ ba, int64_t ldba,
    const __nv_bfloat16* __restrict__ conv_w, __nv_bfloat16* __restrict__ conv_state, float* __restrict__ state,
    const int32_t* __restrict__ slots, int n_slots, const float* __restrict__ A_log,
    const __nv_bfloat16* __restrict__ dt_bias, const __nv_bfloat16* __restrict__ norm_w, __nv_bfloat16* __restrict__ y,
    int64_t ldy, int H, float scale, float eps, int* err) {
  griddep_launch_dependents();  // programmatic dependent launch (launch_k): see common.cuh
  griddep_wait();
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
  // warp w owns value rows [w*ROWS, (w+1)*ROWS) of every head, lane the dims 4*lane..+3;
  // the first head's rows are requested before the conv so their latency overlaps it
  constexpr int ROWS = DV / 8;
  static_assert(ROWS == 16 && DK == 128, "lane layout assumes dk = dv = 128, 8 warps");
  float* S0 = state + (((int64_t)(valid ? slot : 0) * HV + h * RATIO) * DV) * DK;
  float4 sv[ROWS];
  if (valid) {
#pragma unroll
    for (int i = 0; i < ROWS; ++i)
      sv[i] = *reinterpret_cast<const float4*>(S0 + (int64_t)(warp * ROWS + i) * DK + lane * 4);
  }

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

  // ---- per value head: state update. All 16 rows of a warp are requested before any is used
  // (16 loads in flight per thread). Row sums over the 32 lanes use a halving exchange:
  // after it, lanes 2i and 2i+1 hold row i's sum (16 shuffles for the warp's 16 rows
  // instead of 5 per row).
#pragma unroll
  for (int r = 0; r < RATIO; ++r) {
    const int hv = h * RATIO + r;
    if (r > 0) {
#pragma unroll
      for (int i = 0; i < ROWS; ++i)
        sv[i] = *reinterpret_cast<const float4*>(S0 + ((int64_t)r * DV + warp * ROWS + i) * DK + lane * 4);
    }
    const float a = bf2f(ba[(int64_t)b * ldba + HV + hv]);
    const float bb = bf2f(ba[(int64_t)b * ldba + hv]);
    const float xg = a + bf2f(dt_bias[hv]);
    const float sp = xg <= 20.f ? logf(1.f + expf(xg)) : xg;
    const float g = -expf(A_log[hv]) * sp;
    const float alpha = expf(g);
    const float beta = bf16_round(1.f / (1.f + expf(-bb)));
    float* S = S0 + (int64_t)r * DV * DK;
    float pk[ROWS], pq[ROWS];
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const float4 s4 = sv[i];
      pk[i] = s4.x * kv[0] + s4.y * kv[1] + s4.z * kv[2] + s4.w * kv[3];
      pq[i] = s4.x * qv[0] + s4.y * qv[1] + s4.z * qv[2] + s4.w * qv[3];
    }
    const float sk = rows16_sum(pk, lane), sq = rows16_sum(pq, lane);
    const int my_row = lane >> 1;  // the row whose sums this lane now holds
    const float vrow = s_x[2 * DK + r * DV + warp * ROWS + my_row];
    const float vp_mine = beta * (vrow - alpha * sk);
    const float o_mine = alpha * sq + vp_mine * kq;
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const float vp = __shfl_sync(0xffffffffu, vp_mine, 2 * i);
      const float4 s4 = sv[i];
      float4 n4;
      n4.x = alpha * s4.x + vp * kv[0];
      n4.y = alpha * s4.y + vp * kv[1];
      n4.z = alpha * s4.z + vp * kv[2];
      n4.w = alpha * s4.w + vp * kv[3];
      *reinterpret_cast<float4*>(S + (int64_t)(warp * ROWS + i) * DK + lane * 4) = n4;
    }
    // ---- gated RMSNorm over the DV outputs of this head (o rounded to bf16 first)
    const float o_r = bf16_round(o_mine);
    float ss = (lane & 1) ? 0.f : o_r * o_r;  // each row once (even lanes)
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp][r][0] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += s_red[w][r][0];
    const float rstd = rsqrtf(tot / (float)DV + eps);
    if ((lane & 1) == 0) {
      const int row = warp * ROWS + my_row;
      const float z = bf2f(xrow[C + hv * DV + row]);
      const float gz = z / (1.f + __expf(-z));
      y[(int64_t)b * ldy + (int64_t)hv * DV + row] = f2bf(o_r * rstd * bf2f(norm_w[row]) * gz);
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
    launch_k(qw_pdl_small(), gdn_decode_kernel<128, 128, 3>, dim3(grid), dim3(256), 0, s, x, ldx, bap, ldba, cw, cs, state, slots, (int)n_slots, A_log,
                                                        dt, nw, yp, ldy, (int)H, 1.0f / sqrtf((float)dk), eps, err);
  else if (dk == 128 && dv == 128 && ratio == 1)
    launch_k(qw_pdl_small(), gdn_decode_kernel<128, 128, 1>, dim3(grid), dim3(256), 0, s, x, ldx, bap, ldba, cw, cs, state, slots, (int)n_slots, A_log,
                                                        dt, nw, yp, ldy, (int)H, 1.0f / sqrtf((float)dk), eps, err);
  else
    return QW_ERR_UNSUPPORTED;
  QW_LAUNCH_CHECK();
  return QW_OK;
}
