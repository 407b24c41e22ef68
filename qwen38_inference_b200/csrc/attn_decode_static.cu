// qw_attn_decode_static: qw_attn_decode with its split-KV scratch (per-split partial outputs
// and running max / sum) held in a file-scope device array instead of a caller workspace,
// so the call needs no allocation at all.
//
// The array is QW_ATTN_DECODE_STATIC_SCRATCH_BYTES long and is shared by every call on a
// device: two calls whose kernels overlap in time (different streams, or different host
// threads on one stream without ordering) race on it and may return wrong outputs. Calls
// ordered on one stream are safe. The first call on each device looks the array's address
// up with cudaGetSymbolAddress (which can load the module), so make that first call before
// any stream capture begins. Requests whose scratch would exceed the array return
// QW_ERR_WORKSPACE without launching anything.
#include <mutex>

#include "common.cuh"

extern "C" int qw_attn_decode(const void* qkv, int64_t ldq, int64_t B, int64_t nq, int64_t nkv, int64_t d,
                              const void* k_cache, const void* v_cache, const int32_t* seq_len,
                              const int32_t* kv_base, int64_t max_len, int64_t splits, void* out, int64_t ldo,
                              float scale, void* workspace, size_t ws_bytes, qw_stream_t stream);
extern "C" size_t qw_attn_decode_workspace_bytes(int64_t B, int64_t nq, int64_t d, int64_t splits);

namespace qw {

static __device__ __align__(256) unsigned char g_attn_decode_scratch[QW_ATTN_DECODE_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Address of the scratch array on the current device; looked up once per device while
// that device is current. Returns a QW_* status.
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return QW_ERR_CUDA_BASE + (int)e;
  if (dev < 0 || dev >= kMaxDevices) return QW_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_decode_scratch);
    if (e != cudaSuccess) return QW_ERR_CUDA_BASE + (int)e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return QW_OK;
}
}  // namespace

}  // namespace qw

extern "C" size_t qw_attn_decode_static_max_bytes(void) { return (size_t)QW_ATTN_DECODE_STATIC_SCRATCH_BYTES; }

extern "C" int qw_attn_decode_static(const void* qkv, int64_t ldq, int64_t B, int64_t nq, int64_t nkv, int64_t d,
                                     const void* k_cache, const void* v_cache, const int32_t* seq_len,
                                     const int32_t* kv_base, int64_t max_len, int64_t splits, void* out,
                                     int64_t ldo, float scale, qw_stream_t stream) {
  QW_CHECK_ARG(B > 0 && nq > 0 && d > 0 && splits >= 1, QW_ERR_ARG);
  QW_CHECK_ARG(qw_attn_decode_workspace_bytes(B, nq, d, splits) <= (size_t)QW_ATTN_DECODE_STATIC_SCRATCH_BYTES,
               QW_ERR_WORKSPACE);
  void* scratch = nullptr;
  const int rc = qw::scratch_address(&scratch);
  if (rc != QW_OK) return rc;
  return qw_attn_decode(qkv, ldq, B, nq, nkv, d, k_cache, v_cache, seq_len, kv_base, max_len, splits, out, ldo, scale,
                        scratch, (size_t)QW_ATTN_DECODE_STATIC_SCRATCH_BYTES, stream);
}
