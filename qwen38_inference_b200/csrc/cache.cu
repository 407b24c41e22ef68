// KV-cache growth: one pass that writes every row of the new K and V pools, copying each
// slot's live prefix to its new place and zero-filling the rest (reserved page, tails and
// stale rows past a slot's length). Replaces the per-slot zeros + copy_ loop of
// REF:4985-5001 (and the Triton kernel of solution/cache_growth.py:16-32). One launch grows
// the pools of every attention layer (qw_kv_grow_layers); qw_kv_grow is the one-layer case.
//
// One warp per destination row: the row's source (or "zero") is found once per row with
// 64-bit index arithmetic, then the lanes move its 16-byte vectors of K and V, every load of
// the row issued before the stores.
#include "common.cuh"

namespace qw {

constexpr int kKvGrowMaxLayers = QW_KV_GROW_MAX_LAYERS;

struct KvGrowPtrs {
  const uint4* sk[kKvGrowMaxLayers];
  const uint4* sv[kKvGrowMaxLayers];
  uint4* dk[kKvGrowMaxLayers];
  uint4* dv[kKvGrowMaxLayers];
};

// PER = 16-byte vectors per lane when the row has 32 * PER of them; PER = 0: any row width
template <int PER>
__global__ void __launch_bounds__(256) kv_grow_rows_kernel(const __grid_constant__ KvGrowPtrs p, int n_layers,
                                                           const int32_t* __restrict__ lengths, int S,
                                                           int64_t old_cap, int64_t new_cap, int vpr, int64_t rows) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = rows * n_layers;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total; w += nwarps) {
    const int layer = (int)(w / rows);
    const int64_t row = w - (int64_t)layer * rows;
    int64_t srow = -1;
    if (row >= 64) {
      const int64_t slot = (row - 64) / new_cap, j = (row - 64) - slot * new_cap;
      if (slot < S && j < lengths[slot] && j < old_cap) srow = 64 + slot * old_cap + j;
    }
    uint4* dk = p.dk[layer] + row * vpr;
    uint4* dv = p.dv[layer] + row * vpr;
    const uint4 zero = make_uint4(0, 0, 0, 0);
    if constexpr (PER > 0) {
      uint4 k[PER], v[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) k[i] = v[i] = zero;
      if (srow >= 0) {
        const uint4* sk = p.sk[layer] + srow * vpr;
        const uint4* sv = p.sv[layer] + srow * vpr;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          k[i] = sk[lane + 32 * i];
          v[i] = sv[lane + 32 * i];
        }
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        dk[lane + 32 * i] = k[i];
        dv[lane + 32 * i] = v[i];
      }
    } else {
      for (int i = lane; i < vpr; i += 32) {
        uint4 k = zero, v = zero;
        if (srow >= 0) {
          k = p.sk[layer][srow * vpr + i];
          v = p.sv[layer][srow * vpr + i];
        }
        dk[i] = k;
        dv[i] = v;
      }
    }
  }
}

}  // namespace qw

using namespace qw;

extern "C" int qw_kv_grow_layers(const void* const* src_k, const void* const* src_v, void* const* dst_k,
                                 void* const* dst_v, int64_t n_layers, const int32_t* lengths, int64_t S,
                                 int64_t old_cap, int64_t new_cap, int64_t row_elems, qw_stream_t stream) {
  QW_CHECK_ARG(src_k && src_v && dst_k && dst_v && lengths && S > 0 && old_cap > 0 && new_cap >= old_cap, QW_ERR_ARG);
  QW_CHECK_ARG(n_layers >= 1 && n_layers <= kKvGrowMaxLayers, QW_ERR_ARG);
  QW_CHECK_ARG((row_elems * 2) % 16 == 0 && row_elems > 0, QW_ERR_ALIGN);
  QW_CHECK_ARG(S < (1 << 30), QW_ERR_ARG);
  KvGrowPtrs p = {};
  for (int64_t i = 0; i < n_layers; ++i) {
    QW_CHECK_ARG(src_k[i] && src_v[i] && dst_k[i] && dst_v[i], QW_ERR_ARG);
    QW_CHECK_ARG(((uintptr_t)src_k[i] | (uintptr_t)src_v[i] | (uintptr_t)dst_k[i] | (uintptr_t)dst_v[i]) % 16 == 0,
                 QW_ERR_ALIGN);
    p.sk[i] = static_cast<const uint4*>(src_k[i]);
    p.sv[i] = static_cast<const uint4*>(src_v[i]);
    p.dk[i] = static_cast<uint4*>(dst_k[i]);
    p.dv[i] = static_cast<uint4*>(dst_v[i]);
  }
  auto* s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t vpr = row_elems * 2 / 16;
  QW_CHECK_ARG(vpr < (1 << 30), QW_ERR_ARG);
  const int64_t rows = S * new_cap + 64;
  const int64_t warps = rows * n_layers;
  int64_t blocks = (warps + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  const int v = (int)vpr;
  if (vpr == 128)
    kv_grow_rows_kernel<4><<<(unsigned)blocks, 256, 0, s>>>(p, (int)n_layers, lengths, (int)S, old_cap, new_cap, v, rows);
  else if (vpr == 64)
    kv_grow_rows_kernel<2><<<(unsigned)blocks, 256, 0, s>>>(p, (int)n_layers, lengths, (int)S, old_cap, new_cap, v, rows);
  else if (vpr == 32)
    kv_grow_rows_kernel<1><<<(unsigned)blocks, 256, 0, s>>>(p, (int)n_layers, lengths, (int)S, old_cap, new_cap, v, rows);
  else
    kv_grow_rows_kernel<0><<<(unsigned)blocks, 256, 0, s>>>(p, (int)n_layers, lengths, (int)S, old_cap, new_cap, v, rows);
  QW_LAUNCH_CHECK();
  return QW_OK;
}

extern "C" int qw_kv_grow(const void* src_k, const void* src_v, void* dst_k, void* dst_v, const int32_t* lengths,
                          int64_t S, int64_t old_cap, int64_t new_cap, int64_t row_elems, qw_stream_t stream) {
  return qw_kv_grow_layers(&src_k, &src_v, &dst_k, &dst_v, 1, lengths, S, old_cap, new_cap, row_elems, stream);
}
