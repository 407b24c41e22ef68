// Row normalizations of the hidden state (HBM-bound, one CTA per row).
//
//   qw_embed_rmsnorm      embedding gather + Gemma RMSNorm of layer 0
//                         (REF:5045 F.embedding, REF:5049-5050 sgl_kernel gemma_rmsnorm)
//   qw_add_rmsnorm        in-place fused residual add + Gemma RMSNorm
//                         (REF:5052/5088 sgl_kernel gemma_fused_add_rmsnorm)
//   qw_add_rmsnorm_rows   the final add + norm for selected rows only (REF:5093-5095)
//   qw_gated_rmsnorm      GDN output norm: x*rsqrt(mean x^2+eps)*w * z*sigmoid(z)
//                         (REF:1804-1929 with norm_before_gate=True, RMS mode)
//
// Gemma norm: y = bf16(h * rsqrt(mean(h^2) + eps) * (1 + w)); the fused add keeps
// residual = bf16(x + r) and normalizes the unrounded fp32 sum.
#include "common.cuh"

namespace qw {

constexpr int kNormThreads = 128;
constexpr int kMaxVec = 8;  // up to 128 * 8 * 8 = 8192 columns per row

QW_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x / 32) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  t = red[32];
  __syncthreads();
  return t;
}

// mode 0: embedding (src = table row), writes residual copy + normalized
// mode 1: in-place add-norm (x += r)
// VEC = 8-column vectors per thread (ceil(H / (8 * kNormThreads))): the row stays in VEC * 8
// registers, so a narrow row does not pay for the widest one in occupancy
template <int MODE, int VEC>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_rows_kernel(
    const __nv_bfloat16* __restrict__ src, int64_t ld_src, const int32_t* __restrict__ rows, int64_t n_table,
    __nv_bfloat16* x, __nv_bfloat16* resid, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* out, int H,
    float eps, int* err) {
  griddep_launch_dependents();  // programmatic dependent launch (launch_k): see common.cuh
  griddep_wait();
  __shared__ float red[33];
  const int row = blockIdx.x;
  const int nvec = H / 8;
  float v[VEC][8];
  float ss = 0.f;
  const __nv_bfloat16* in_row;
  if constexpr (MODE == 0) {
    int64_t tok = rows[row];
    if (tok < 0 || tok >= n_table) {
      set_error(err, QW_DEV_ERR_INDEX);
      tok = 0;
    }
    in_row = src + tok * ld_src;
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (threadIdx.x + i * kNormThreads) * 8;
    if (c < H) {
      if constexpr (MODE == 0) {
        load_bf16x8(in_row + c, v[i]);
        *reinterpret_cast<uint4*>(resid + (int64_t)row * H + c) = *reinterpret_cast<const uint4*>(in_row + c);
      } else {
        float r[8];
        load_bf16x8(x + (int64_t)row * H + c, v[i]);
        load_bf16x8(resid + (int64_t)row * H + c, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[j];
        store_bf16x8(resid + (int64_t)row * H + c, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  (void)nvec;
  const float tot = block_sum(ss, red);
  const float rstd = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (threadIdx.x + i * kNormThreads) * 8;
    if (c < H) {
      float wf[8], o[8];
      load_bf16x8(w + c, wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * rstd * (1.0f + wf[j]);
      store_bf16x8((MODE == 0 ? out : x) + (int64_t)row * H + c, o);
    }
  }
}

// Final norm on selected rows: out[i] = norm(x[rows[i]] + resid[rows[i]]); inputs unchanged.
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_select_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ resid, const int32_t* __restrict__ rows,
    int T, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int H, float eps, int* err) {
  griddep_launch_dependents();  // programmatic dependent launch (launch_k): see common.cuh
  griddep_wait();
  __shared__ float red[33];
  int r = rows ? rows[blockIdx.x] : blockIdx.x;
  if (r < 0 || r >= T) {
    set_error(err, QW_DEV_ERR_INDEX);
    r = 0;
  }
  float v[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = (threadIdx.x + i * kNormThreads) * 8;
    if (c < H) {
      float rr[8];
      load_bf16x8(x + (int64_t)r * H + c, v[i]);
      load_bf16x8(resid + (int64_t)r * H + c, rr);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i][j] += rr[j];
        ss += v[i][j] * v[i][j];
      }
    }
  }
  const float rstd = rsqrtf(block_sum(ss, red) / (float)H + eps);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = (threadIdx.x + i * kNormThreads) * 8;
    if (c < H) {
      float wf[8], o[8];
      load_bf16x8(w + c, wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * rstd * (1.0f + wf[j]);
      store_bf16x8(out + (int64_t)blockIdx.x * H + c, o);
    }
  }
}

// GDN gated RMSNorm over heads of D=dv columns; one warp per (token, head).
template <int D>
__global__ void gated_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                     const __nv_bfloat16* __restrict__ z, int64_t ldz,
                                     const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y, int64_t ldy,
                                     int T, int HV, float eps) {
  constexpr int E = D / 32;
  const int gw = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= T * HV) return;
  const int t = gw / HV, h = gw % HV;
  float xv[E], zv[E], wv[E];
  const int c0 = lane * E;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    xv[j] = bf2f(x[(int64_t)t * ldx + h * D + c0 + j]);
    zv[j] = bf2f(z[(int64_t)t * ldz + h * D + c0 + j]);
    wv[j] = bf2f(w[c0 + j]);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < E; ++j) ss += xv[j] * xv[j];
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const float g = zv[j] / (1.0f + __expf(-zv[j]));
    y[(int64_t)t * ldy + h * D + c0 + j] = f2bf(xv[j] * rstd * wv[j] * g);
  }
}

}  // namespace qw

using namespace qw;

extern "C" int qw_embed_rmsnorm(const int32_t* tokens, int64_t T, const void* table, int64_t vocab, int64_t H,
                                const void* w, void* resid_out, void* hidden_out, float eps, qw_stream_t stream) {
  QW_CHECK_ARG(tokens && table && w && resid_out && hidden_out && T > 0 && vocab > 0, QW_ERR_ARG);
  QW_CHECK_ARG(H % 8 == 0 && H <= kNormThreads * kMaxVec * 8, QW_ERR_UNSUPPORTED);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int vec = (int)((H + 8 * kNormThreads - 1) / (8 * kNormThreads));
#define QW_EMBED(V)                                                                                               \
  launch_k(qw_pdl_small(), rmsnorm_rows_kernel<0, V>, dim3((unsigned)T), dim3(kNormThreads), 0, s,                                                \
      static_cast<const __nv_bfloat16*>(table), H, tokens, vocab, nullptr, static_cast<__nv_bfloat16*>(resid_out), \
      static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(hidden_out), (int)H, eps, device_error_ptr())
  if (vec <= 1) QW_EMBED(1);
  else if (vec <= 5) QW_EMBED(5);
  else QW_EMBED(kMaxVec);
#undef QW_EMBED
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_add_rmsnorm(void* x, void* resid, const void* w, int64_t T, int64_t H, float eps,
                              qw_stream_t stream) {
  QW_CHECK_ARG(x && resid && w && T > 0, QW_ERR_ARG);
  QW_CHECK_ARG(H % 8 == 0 && H <= kNormThreads * kMaxVec * 8, QW_ERR_UNSUPPORTED);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int vec = (int)((H + 8 * kNormThreads - 1) / (8 * kNormThreads));
#define QW_ADDN(V)                                                                                                \
  launch_k(qw_pdl_small(), rmsnorm_rows_kernel<1, V>, dim3((unsigned)T), dim3(kNormThreads), 0, s,                                                \
      nullptr, 0, nullptr, 0, static_cast<__nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(resid),                \
      static_cast<const __nv_bfloat16*>(w), nullptr, (int)H, eps, nullptr)
  if (vec <= 1) QW_ADDN(1);
  else if (vec <= 5) QW_ADDN(5);
  else QW_ADDN(kMaxVec);
#undef QW_ADDN
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_add_rmsnorm_rows(const void* x, const void* resid, const int32_t* rows, int64_t n_rows, int64_t T,
                                   int64_t H, const void* w, void* out, float eps, qw_stream_t stream) {
  QW_CHECK_ARG(x && resid && w && out && n_rows > 0 && T > 0, QW_ERR_ARG);
  QW_CHECK_ARG(H % 8 == 0 && H <= kNormThreads * kMaxVec * 8, QW_ERR_UNSUPPORTED);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  launch_k(qw_pdl_small(), add_rmsnorm_select_kernel, dim3((unsigned)n_rows), dim3(kNormThreads), 0, s, 
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(resid), rows, (int)T,
      static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(out), (int)H, eps, device_error_ptr());
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_gated_rmsnorm(const void* x, int64_t ldx, const void* z, int64_t ldz, const void* w, void* y,
                                int64_t ldy, int64_t T, int64_t HV, int64_t D, float eps, qw_stream_t stream) {
  QW_CHECK_ARG(x && z && w && y && T > 0 && HV > 0, QW_ERR_ARG);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t warps = T * HV;
  const int threads = 256;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* zb = static_cast<const __nv_bfloat16*>(z);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  auto* yb = static_cast<__nv_bfloat16*>(y);
  if (D == 128)
    gated_rmsnorm_kernel<128><<<blocks, threads, 0, s>>>(xb, ldx, zb, ldz, wb, yb, ldy, (int)T, (int)HV, eps);
  else if (D == 64)
    gated_rmsnorm_kernel<64><<<blocks, threads, 0, s>>>(xb, ldx, zb, ldz, wb, yb, ldy, (int)T, (int)HV, eps);
  else
    return QW_ERR_UNSUPPORTED;
  QW_LAUNCH_CHECK();
  return QW_OK;
}
