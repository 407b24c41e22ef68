// Data movement around the collectives of head-wise tensor parallelism (one rank per GPU):
//   qw_round_f32_bf16       y = bf16(x): the all-reduced fp32 sum of a row-parallel projection
//                           becomes the bf16 F.linear output (REF:5092 for the last layer)
//   qw_gather_vocab_shards  [G, R, Vs] fp32 logits of G vocab shards (the rank-major result of
//                           an all-gather) -> [R, G * Vs] in vocabulary order (REF:5096)
// Both are plain HBM streams: 8-byte (bf16 x4) / 16-byte vector accesses, grid-stride loops.
// Also the peer buffers of the one-shot all-reduce fused into the decode projections
// (gemm.cu, partial_norm_finish): allocated here and shared between the ranks' processes
// with CUDA IPC handles.
#include <cstring>

#include "common.cuh"

namespace qw {

__global__ void round_f32_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n) {
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&lo);
    o.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(y)[i] = o;
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) y[i] = f2bf(x[i]);
}

// dst[r][g * Vs + v] = src[g][r][v]; Vs % 4 == 0 (checked on the host)
__global__ void gather_vocab_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t G, int64_t R,
                                    int64_t Vs) {
  const int64_t v4 = Vs / 4;
  const int64_t total = G * R * v4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t v = i % v4;
    const int64_t r = (i / v4) % R;
    const int64_t g = i / (v4 * R);
    const float4 val = reinterpret_cast<const float4*>(src)[i];
    reinterpret_cast<float4*>(dst + r * G * Vs + g * Vs)[v] = val;
  }
}

static unsigned stream_blocks(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  const int64_t cap = 148 * 8;  // a few waves of the 148 SMs; the loops stride over the rest
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace qw

using namespace qw;

// ---- peer buffers (CUDA IPC): the one allocation the library makes, on request
static_assert(sizeof(cudaIpcMemHandle_t) == QW_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" size_t qw_tp_buffer_bytes(int64_t H) {
  if (H <= 0) return 0;
  return (size_t)QW_TP_HEADER_BYTES + 3 * (size_t)QW_TP_MAX_ROWS * (size_t)H * sizeof(float);
}

extern "C" int qw_ipc_alloc(size_t bytes, void** dptr, void* handle) {
  QW_CHECK_ARG(bytes > 0 && dptr && handle, QW_ERR_ARG);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return QW_ERR_CUDA_BASE + (int)e;
  e = cudaMemset(p, 0, bytes);  // flags and epochs start at zero
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return QW_ERR_CUDA_BASE + (int)e;
  }
  *dptr = p;
  return QW_OK;
}

extern "C" int qw_ipc_open(const void* handle, void** dptr) {
  QW_CHECK_ARG(handle && dptr, QW_ERR_ARG);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return QW_ERR_CUDA_BASE + (int)e;
  *dptr = p;
  return QW_OK;
}

extern "C" int qw_ipc_close(void* dptr) {
  QW_CHECK_ARG(dptr, QW_ERR_ARG);
  const cudaError_t e = cudaIpcCloseMemHandle(dptr);
  return e == cudaSuccess ? QW_OK : QW_ERR_CUDA_BASE + (int)e;
}

extern "C" int qw_ipc_free(void* dptr) {
  QW_CHECK_ARG(dptr, QW_ERR_ARG);
  const cudaError_t e = cudaFree(dptr);
  return e == cudaSuccess ? QW_OK : QW_ERR_CUDA_BASE + (int)e;
}

extern "C" int qw_round_f32_bf16(const float* x, void* y, int64_t n, qw_stream_t stream) {
  QW_CHECK_ARG(x && y && n > 0, QW_ERR_ARG);
  QW_CHECK_ARG(((uintptr_t)x % 16) == 0 && ((uintptr_t)y % 8) == 0, QW_ERR_ALIGN);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  round_f32_bf16_kernel<<<stream_blocks((n + 3) / 4, 256), 256, 0, s>>>(x, static_cast<__nv_bfloat16*>(y), n);
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_gather_vocab_shards(const float* src, int64_t G, int64_t R, int64_t Vs, float* dst,
                                      qw_stream_t stream) {
  QW_CHECK_ARG(src && dst && G > 0 && R > 0 && Vs > 0, QW_ERR_ARG);
  QW_CHECK_ARG(Vs % 4 == 0 && ((uintptr_t)src % 16) == 0 && ((uintptr_t)dst % 16) == 0, QW_ERR_ALIGN);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  gather_vocab_kernel<<<stream_blocks(G * R * (Vs / 4), 256), 256, 0, s>>>(src, dst, G, R, Vs);
  QW_LAUNCH_CHECK();
  return QW_OK;
}
