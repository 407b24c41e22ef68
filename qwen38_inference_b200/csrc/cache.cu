// KV-cache growth: one pass that writes every row of the new K and V pools, copying each
// slot's live prefix to its new place and zero-filling the rest (reserved page, tails and
// stale rows past a slot's length). Replaces the per-slot zeros + copy_ loop of
// REF:4985-5001 (and the Triton kernel of solution/cache_growth.py:16-32).
#include "common.cuh"

namespace qw {

__global__ void kv_grow_kernel(const uint4* __restrict__ src_k, const uint4* __restrict__ src_v, uint4* __restrict__ dst_k,
                               uint4* __restrict__ dst_v, const int32_t* __restrict__ lengths, int S, int64_t old_cap,
                               int64_t new_cap, int64_t vec_per_row, int64_t total_vec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total_vec; i += stride) {
    const int64_t row = i / vec_per_row, v = i % vec_per_row;
    uint4 k = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    if (row >= 64) {
      const int64_t slot = (row - 64) / new_cap, j = (row - 64) % new_cap;
      if (slot < S && j < lengths[slot] && j < old_cap) {
        const int64_t srow = 64 + slot * old_cap + j;
        k = src_k[srow * vec_per_row + v];
        vv = src_v[srow * vec_per_row + v];
      }
    }
    dst_k[i] = k;
    dst_v[i] = vv;
  }
}

}  // namespace qw

using namespace qw;

extern "C" int qw_kv_grow(const void* src_k, const void* src_v, void* dst_k, void* dst_v, const int32_t* lengths,
                          int64_t S, int64_t old_cap, int64_t new_cap, int64_t row_elems, qw_stream_t stream) {
  QW_CHECK_ARG(src_k && src_v && dst_k && dst_v && lengths && S > 0 && old_cap > 0 && new_cap >= old_cap, QW_ERR_ARG);
  QW_CHECK_ARG((row_elems * 2) % 16 == 0, QW_ERR_ALIGN);
  QW_CHECK_ARG(((uintptr_t)src_k | (uintptr_t)src_v | (uintptr_t)dst_k | (uintptr_t)dst_v) % 16 == 0, QW_ERR_ALIGN);
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t vpr = row_elems * 2 / 16;
  const int64_t total = (S * new_cap + 64) * vpr;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  kv_grow_kernel<<<(unsigned)blocks, threads, 0, s>>>(
      static_cast<const uint4*>(src_k), static_cast<const uint4*>(src_v), static_cast<uint4*>(dst_k),
      static_cast<uint4*>(dst_v), lengths, (int)S, old_cap, new_cap, vpr, total);
  QW_LAUNCH_CHECK();
  return QW_OK;
}
