/*
 * qw200.h - C ABI of the B200 (sm_100a) kernels behind the hybrid Gated-DeltaNet /
 * gated-GQA forward_step.
 *
 * Every entry point takes plain device pointers, sizes and strides (in elements), the
 * CUDA stream to launch on, and returns 0 or a QW_ERR_* code. No entry point allocates
 * device memory: callers pass every buffer, including workspaces. Kernels record
 * device-side failures (a bounded wait that gave up, an index outside its range) in one
 * library-wide error word that qw_take_device_error() reads and clears.
 *
 * Element types: "bf16" = __nv_bfloat16 bit patterns (uint16), "f32" = float,
 * "i32"/"i64" = int32_t/int64_t. Row-major unless stated.
 *
 * Each declaration names the reference interface it replaces, as
 * reference/qwen38_inference.py:<line> ("REF").
 */
#ifndef QW200_H
#define QW200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qw_stream_t;

/* ---- status codes ------------------------------------------------------------------ */
#define QW_OK 0
#define QW_ERR_ARG 1         /* bad size, count or null pointer                          */
#define QW_ERR_ALIGN 2       /* pointer or leading dimension not 16-byte aligned         */
#define QW_ERR_UNSUPPORTED 3 /* head size / width with no compiled kernel                */
#define QW_ERR_WORKSPACE 4   /* workspace smaller than qw_*_workspace_bytes()            */
#define QW_ERR_DRIVER 5      /* cuTensorMapEncodeTiled unavailable or failed             */
#define QW_ERR_CUDA_BASE 1000 /* + cudaError_t of a failed launch                       */

/* device error word values */
#define QW_DEV_ERR_TIMEOUT_GEMM 101
#define QW_DEV_ERR_INDEX 102
#define QW_DEV_ERR_TIMEOUT_GDN 103 /* a bounded wait of the chunked delta-rule pipeline gave up */
#define QW_DEV_ERR_TIMEOUT_ATTN 104 /* a bounded wait of the prefill attention pipeline gave up */
#define QW_DEV_ERR_TIMEOUT_TP 105 /* a peer rank's row did not arrive in the one-shot all-reduce */
#define QW_DEV_ERR_GEMM_COUNTER 106 /* the add-norm ticket pair of the weight-streaming GEMM did
                                       not start at zero (an earlier launch gave up a wait, or two
                                       launches overlapped); the launch skipped its add-norm rows */

/* ---- library ----------------------------------------------------------------------- */
int qw_version(void);
/* Synchronizes the device, stores the device error word in *code and clears it; also
 * zeroes the add-norm ticket pair of qw_gemm_add_rmsnorm (see there), so calls after a
 * reported error start clean. */
int qw_take_device_error(int* code);
/* Queues a 4-byte copy of the device error word (current device) into host_dst on `stream`
 * without synchronizing or clearing it: host_dst (pinned host memory) holds the word once
 * the stream's work up to this call has finished. Lets a caller check for device-side
 * failures at its own sync points; qw_take_device_error() then reads and clears the word. */
int qw_peek_device_error_async(int* host_dst, qw_stream_t stream);

/* ---- dense projections (REF:5054,5067,5069,5070,5087,5089,5092,5096: F.linear) ------ *
 * y = x[M,K] . w[N,K]^T with fp32 accumulation on tcgen05 tensor cores.
 *   out_kind QW_OUT_BF16:        y bf16 [M, ldy], N columns            (F.linear)
 *   out_kind QW_OUT_F32_OF_BF16: y f32  [M, ldy] = float(bf16(acc))     (F.linear().float(), REF:5096)
 *   out_kind QW_OUT_SWIGLU:      w = [gate; up] with N = 2*I rows, y bf16 [M, ldy] with I
 *                                columns = bf16(silu(bf16(g)) * bf16(u)) (REF:5089-5091 + REF:2238-2281)
 *   out_kind QW_OUT_F32:         y f32  [M, ldy] = acc, unrounded: the partial sum of one tensor-
 *                                parallel rank, rounded once after the all-reduce (qw_add_rmsnorm_f32)
 * Small M (decode) runs weight-streaming split-K tiles, and a large M whose 128 x 256 tiles
 * leave SMs idle splits K too (bf16 and fp32 outputs); both need a workspace of
 * qw_gemm_workspace_bytes(M, N, K, out_kind) bytes (0 when no split is taken).
 */
#define QW_OUT_BF16 0
#define QW_OUT_F32_OF_BF16 1
#define QW_OUT_SWIGLU 2
#define QW_OUT_F32 3
size_t qw_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int out_kind);
int qw_gemm_bf16(const void* x, const void* w, void* y, int64_t M, int64_t N, int64_t K, int64_t ldx,
                 int64_t ldw, int64_t ldy, int out_kind, void* workspace, size_t ws_bytes, qw_stream_t stream);

/* Projection fused with the residual add-norm that follows it:
 * x = bf16(x_in . w^T) [M, N]; v = x + resid (fp32); resid = bf16(v);
 * hidden = bf16(v * rsqrt(mean v^2 + eps) * (1 + norm_w)); resid and hidden are [M, N]
 * contiguous. Decode (M <= 64) streams the weights split over K; a large M whose tiles
 * leave SMs idle (a 512-token chunk) splits K as well. The split-K partials ([splits, M, N]
 * fp32, workspace of qw_gemm_add_rmsnorm_workspace_bytes) are summed in k order by the
 * norm kernel. When that size is 0 for a large M, the call is a bf16 GEMM into hidden and
 * then qw_add_rmsnorm (REF:5087-5088 / 5092 + 5052: F.linear then gemma_fused_add_rmsnorm).
 * When the add-norm runs inside the GEMM (qw_gemm_add_rmsnorm_kernels() == 1), its CTAs
 * take turns from one ticket pair per device: such calls (and qw_gemm_add_rmsnorm_tp) must
 * not overlap in time on one device, i.e. issue them on one stream. An overlap, or a pair
 * left stale by a wait that gave up, is reported as QW_DEV_ERR_GEMM_COUNTER; no row outside
 * [0, M) is ever touched.                                                                   */
size_t qw_gemm_add_rmsnorm_workspace_bytes(int64_t M, int64_t N, int64_t K);
/* Kernels one qw_gemm_add_rmsnorm call of this shape launches: 1 when the add-norm runs
 * inside the weight-streaming GEMM (its last M CTAs to finish each take one row), else 2. */
int qw_gemm_add_rmsnorm_kernels(int64_t M, int64_t N, int64_t K);
int qw_gemm_add_rmsnorm(const void* x, const void* w, int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                        void* resid, const void* norm_w, void* hidden, float eps, void* workspace, size_t ws_bytes,
                        qw_stream_t stream);

/* The residual add-norm of REF:5052/5088 (gemma_fused_add_rmsnorm) with the projection
 * output given as fp32 partial sums: x = bf16(sum_p parts[p]) over n_parts slices
 * part_stride floats apart (each [T, H] contiguous, summed in order p = 0, 1, ...);
 * v = x + resid (fp32); resid = bf16(v); hidden = bf16(v * rsqrt(mean v^2 + eps) * (1 + w)).
 * Tensor parallelism feeds it the all-reduced row-parallel projection (n_parts = 1).      */
int qw_add_rmsnorm_f32(const float* parts, int64_t n_parts, int64_t part_stride, int64_t T, int64_t H,
                       void* resid, const void* norm_w, void* hidden, float eps, qw_stream_t stream);

/* ---- hidden-state norms ------------------------------------------------------------ */
/* residual = table[tokens] (bf16 [T,H]); hidden = bf16(r * rsqrt(mean r^2 + eps) * (1 + w))
 * (REF:5045 F.embedding + REF:5049-5050 sgl_kernel gemma_rmsnorm)                          */
int qw_embed_rmsnorm(const int32_t* tokens, int64_t T, const void* table, int64_t vocab, int64_t H, const void* w,
                     void* resid_out, void* hidden_out, float eps, qw_stream_t stream);
/* in place: h = x + resid (fp32); resid = bf16(h); x = bf16(h * rsqrt(mean h^2 + eps) * (1 + w))
 * (REF:5052, 5088: sgl_kernel gemma_fused_add_rmsnorm)                                      */
int qw_add_rmsnorm(void* x, void* resid, const void* w, int64_t T, int64_t H, float eps, qw_stream_t stream);
/* out[i] = norm(x[rows[i]] + resid[rows[i]]) for n_rows selected rows (rows == NULL: all T);
 * inputs unchanged (REF:5093-5095: final add-norm + last-row select)                        */
int qw_add_rmsnorm_rows(const void* x, const void* resid, const int32_t* rows, int64_t n_rows, int64_t T, int64_t H,
                        const void* w, void* out, float eps, qw_stream_t stream);
/* y = bf16(x * rsqrt(mean x^2 + eps) * w * z * sigmoid(z)) per head of D columns
 * (REF:1804-2089 rms_norm_gated, norm_before_gate=True, swish)                             */
int qw_gated_rmsnorm(const void* x, int64_t ldx, const void* z, int64_t ldz, const void* w, void* y, int64_t ldy,
                     int64_t T, int64_t HV, int64_t D, float eps, qw_stream_t stream);

/* ---- gated GQA attention ---------------------------------------------------------- */
/* qkv bf16 [T, ldq] = per query head [q | gate] (2d), then k (nkv*d), then v (nkv*d).
 * Gemma RMSNorm of every q and k head, NeoX RoPE on the first rotary_dim dims with the
 * fp32 [cos | sin] table rope[rope_rows, rotary_dim] at positions[t]; q written back in
 * place; k and v stored at cache row locations[t] of k_cache/v_cache [cache_rows, nkv, d]
 * (REF:83-278 fused_qk_gemma_rmsnorm_rope_gate + REF:2656-2787 store_kvcache)              */
int qw_qk_norm_rope_store(void* qkv, int64_t ldq, int64_t T, int64_t nq, int64_t nkv, int64_t d, const void* q_w,
                          const void* k_w, const float* rope, int64_t rotary_dim, int64_t rope_rows,
                          const int32_t* positions, const int32_t* locations, void* k_cache, void* v_cache,
                          int64_t cache_rows, float eps, qw_stream_t stream);
/* The attention input projection with q/k norm, RoPE and the KV store in its epilogue:
 * qkv = bf16(x[M,K] . w[N,K]^T) with N = (2*nq + 2*nkv)*d (REF:5054 F.linear, REF:4940 row
 * layout), then exactly the arithmetic of qw_qk_norm_rope_store on that output (REF:5055-5058:
 * REF:83-190 + REF:2656-2687): q (normalized and rotated) and the gate are written to qkv;
 * k (normalized and rotated) and v go only to their cache rows locations[t] (the k and v
 * columns of qkv are left unwritten). For d = 256 and rotary_dim = 64 with tiles that fill the
 * SMs, this is one tcgen05 GEMM whose epilogue does all of it (one 256-column tile = one head
 * segment); decode (M <= 64) and chunks whose tiles leave SMs idle run the split-K product and
 * one finishing kernel (partials summed in split order, then the same epilogue). Workspace:
 * qw_gemm_qkv_workspace_bytes(M, N, K, d, rotary_dim) bytes.                                 */
size_t qw_gemm_qkv_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t d, int64_t rotary_dim);
int qw_gemm_qkv_rope_store(const void* x, const void* w, void* qkv, int64_t M, int64_t N, int64_t K, int64_t ldx,
                           int64_t ldw, int64_t ldq, int64_t nq, int64_t nkv, int64_t d, const void* q_w,
                           const void* k_w, const float* rope, int64_t rotary_dim, int64_t rope_rows,
                           const int32_t* positions, const int32_t* locations, void* k_cache, void* v_cache,
                           int64_t cache_rows, float eps, void* workspace, size_t ws_bytes, qw_stream_t stream);
/* Causal varlen attention for prefill/extend; tiles = int32 pairs (request, first query)
 * of 128-query tiles; request i owns query rows cu[i]..cu[i+1] of the T rows of qkv, has
 * prefix[i] cached tokens and its keys start at cache row kv_base[i] of the cache_rows rows
 * of k_cache / v_cache. out bf16 [T, ldo] = bf16(bf16(softmax(q k^T * scale) v) * sigmoid(gate))
 * (REF:5059-5066 trtllm_batch_context_with_kv_cache + fused_sigmoid_mul)                   */
int qw_attn_prefill(const void* qkv, int64_t ldq, int64_t nq, int64_t nkv, int64_t d, const void* k_cache,
                    const void* v_cache, const void* tiles, int64_t n_tiles, const int32_t* cu_seqlens,
                    const int32_t* prefix, const int32_t* kv_base, void* out, int64_t ldo, float scale, int64_t T,
                    int64_t cache_rows, qw_stream_t stream);
/* qw_attn_prefill with the keys of every tile split over `splits` CTAs (long prefixes, e.g.
 * chunked prefill of a 128k-token request, where heads x tiles alone leave SMs idle). Each
 * CTA writes an unnormalized partial (O, running max, sum) per query row to the workspace;
 * a merge kernel combines the splits and applies the gate. Same output as qw_attn_prefill up
 * to fp32 summation order. splits == 1 is qw_attn_prefill (no workspace needed).          */
size_t qw_attn_prefill_split_workspace_bytes(int64_t T, int64_t nq, int64_t d, int64_t splits);
int qw_attn_prefill_split(const void* qkv, int64_t ldq, int64_t nq, int64_t nkv, int64_t d, const void* k_cache,
                          const void* v_cache, const void* tiles, int64_t n_tiles, const int32_t* cu_seqlens,
                          const int32_t* prefix, const int32_t* kv_base, void* out, int64_t ldo, float scale,
                          int64_t T, int64_t cache_rows, int64_t splits, void* workspace, size_t ws_bytes,
                          qw_stream_t stream);
/* One query per request against seq_len[b] keys from row kv_base[b], split over `splits`
 * CTAs per (request, kv head) and combined (REF:5059-5062 trtllm_batch_decode_with_kv_cache
 * + REF:5066 fused_sigmoid_mul)                                                              */
size_t qw_attn_decode_workspace_bytes(int64_t B, int64_t nq, int64_t d, int64_t splits);
int qw_attn_decode(const void* qkv, int64_t ldq, int64_t B, int64_t nq, int64_t nkv, int64_t d, const void* k_cache,
                   const void* v_cache, const int32_t* seq_len, const int32_t* kv_base, int64_t max_len,
                   int64_t splits, void* out, int64_t ldo, float scale, void* workspace, size_t ws_bytes,
                   qw_stream_t stream);

/* qw_attn_decode with its split-KV scratch in a library-owned, file-scope device array of
 * QW_ATTN_DECODE_STATIC_SCRATCH_BYTES instead of a caller workspace: the call allocates
 * nothing. Returns QW_ERR_WORKSPACE when qw_attn_decode_workspace_bytes(B, nq, d, splits)
 * exceeds that size. Every call on a device shares the one array, so calls whose kernels
 * overlap in time race on it; calls ordered on one stream are safe. The first call on each
 * device looks up the array's address (cudaGetSymbolAddress, with that device current), so
 * make it before any stream capture. No counterpart in the reference.                        */
#define QW_ATTN_DECODE_STATIC_SCRATCH_BYTES (8u << 20)
size_t qw_attn_decode_static_max_bytes(void);
int qw_attn_decode_static(const void* qkv, int64_t ldq, int64_t B, int64_t nq, int64_t nkv, int64_t d,
                          const void* k_cache, const void* v_cache, const int32_t* seq_len, const int32_t* kv_base,
                          int64_t max_len, int64_t splits, void* out, int64_t ldo, float scale, qw_stream_t stream);

/* ---- Gated DeltaNet ------------------------------------------------------------------ */
/* Prefill causal conv (width 4) + SiLU over the first 2*qk_dim+v_dim columns of x [T, ldx],
 * L2 norm of q/k heads, token-major q,k [T, qk_dim], v [T, v_dim]; conv_state [S, C, 3]
 * read when has_initial[b] and rewritten for every request
 * (REF:704-1253 causal_conv1d_fn + REF:603-699 split + REF:1550-1638 l2norm)               */
int qw_conv_prefill(const void* x, int64_t ldx, const void* conv_w, void* conv_state, const int32_t* cu_seqlens,
                    const int32_t* slots, const int32_t* has_initial, int64_t B, int64_t n_slots, int64_t max_len,
                    void* q_out, void* k_out, void* v_out, int64_t qk_dim, int64_t v_dim, int64_t head_dim,
                    qw_stream_t stream);
/* Chunked gated delta rule over varlen requests with the gating folded in; state
 * [S, HV, dv, dk] fp32 read and written in place at slots[b]; the output o (rounded to
 * bf16) goes straight through the gated RMSNorm with z [T, ldz] and norm_w [dv]; q, k are
 * [T, H*dk] and v [T, HV*dv] (T = total tokens, read by TMA):
 * y bf16 [T, ldy] = bf16(o * rsqrt(mean o^2 + eps) * w * z * sigmoid(z))
 * (REF:5081-5086: fused_gdn_gating + flashinfer chunk_gated_delta_rule + index_copy_ +
 * rms_norm_gated)                                                                            */
int qw_gdn_prefill(const void* q, const void* k, const void* v, const void* ba, int64_t ldba, const float* A_log,
                   const void* dt_bias, const int32_t* cu_seqlens, const int32_t* slots, int64_t B, int64_t T,
                   int64_t n_slots, float* state, const void* z, int64_t ldz, const void* norm_w, void* y,
                   int64_t ldy, int64_t H, int64_t HV, int64_t dk, int64_t dv, float scale, float eps,
                   qw_stream_t stream);
/* Decode: conv update + L2 norm + gating + one recurrent step + gated RMSNorm, y bf16
 * [B, HV*dv] (REF:5072-5075 fused_qkvzba_causal_conv1d_update + recurrent packed decode,
 * REF:5086 rms_norm_gated)                                                                   */
int qw_gdn_decode(const void* qkvz, int64_t ldx, const void* ba, int64_t ldba, const void* conv_w, void* conv_state,
                  float* state, const int32_t* slots, int64_t B, int64_t n_slots, const float* A_log,
                  const void* dt_bias, const void* norm_w, void* y, int64_t ldy, int64_t H, int64_t HV, int64_t dk,
                  int64_t dv, float eps, qw_stream_t stream);

/* ---- cache growth ------------------------------------------------------------------- */
/* dst [S*new_cap + 64, row_elems] = live prefixes of src [S*old_cap + 64, row_elems]
 * (rows 64 + s*old_cap + j, j < lengths[s]) moved to rows 64 + s*new_cap + j; every other
 * row zero. Applied to K and V together (REF:4985-5001 _reserve; solution/cache_growth.py) */
int qw_kv_grow(const void* src_k, const void* src_v, void* dst_k, void* dst_v, const int32_t* lengths, int64_t S,
               int64_t old_cap, int64_t new_cap, int64_t row_elems, qw_stream_t stream);
/* The same growth for the (K, V) pools of n_layers attention layers in one launch: src_k,
 * src_v, dst_k, dst_v are host arrays of n_layers device pointers, n_layers at most
 * QW_KV_GROW_MAX_LAYERS (REF:4985-5001 applied to every layer, as solution/cache_growth.py
 * grow_fused does with one kernel)                                                          */
#define QW_KV_GROW_MAX_LAYERS 32
int qw_kv_grow_layers(const void* const* src_k, const void* const* src_v, void* const* dst_k, void* const* dst_v,
                      int64_t n_layers, const int32_t* lengths, int64_t S, int64_t old_cap, int64_t new_cap,
                      int64_t row_elems, qw_stream_t stream);

/* ---- head-wise tensor parallelism (new: the reference runs one GPU) ------------------ *
 * Peer buffers of the one-shot all-reduce fused into the decode projections
 * (qw_gemm_add_rmsnorm_tp). Each rank allocates one buffer of qw_tp_buffer_bytes(H) with
 * qw_ipc_alloc (the one allocation the library makes; zero-filled), publishes the
 * QW_IPC_HANDLE_BYTES handle to the other ranks of the node, and maps theirs with
 * qw_ipc_open. Layout: per-row arrival flags [QW_TP_MAX_ROWS][QW_TP_MAX_WORLD] u32 written
 * by the peers, then the row epochs of this rank, then (at QW_TP_HEADER_BYTES) three slots
 * of [QW_TP_MAX_ROWS, H] fp32 partial sums.                                                 */
#define QW_IPC_HANDLE_BYTES 64
#define QW_TP_MAX_WORLD 8
#define QW_TP_MAX_ROWS 64
#define QW_TP_HEADER_BYTES 65536
size_t qw_tp_buffer_bytes(int64_t H);
int qw_ipc_alloc(size_t bytes, void** dptr, void* handle);
int qw_ipc_open(const void* handle, void** dptr);
int qw_ipc_close(void* dptr);
int qw_ipc_free(void* dptr);
/* Decode (M <= QW_TP_MAX_ROWS) row-parallel projection of one tensor-parallel rank fused with
 * the all-reduce over the `world` ranks and the residual add-norm, in ONE kernel: the GEMM's
 * last M CTAs each sum one row's split-K partials, publish it in this rank's peer buffer
 * (slot `slot`), raise the row's flag in every rank's buffer, wait (bounded, else
 * QW_DEV_ERR_TIMEOUT_TP) for every rank's flag, sum the ranks' rows in rank order and apply
 * the add-norm of qw_gemm_add_rmsnorm (round_only: hidden = bf16(sum), resid untouched).
 * peer_bases: device array of the `world` buffer bases, this rank's own at index `rank`.
 * Every rank must make the same calls in the same order, and a rank must not reuse a slot
 * in two consecutive calls (alternate 0 and 1; 2 for an odd one out).
 * (REF:5087-5088 / 5092 + 5052 on one GPU; the all-reduce has no counterpart there)          */
int qw_gemm_add_rmsnorm_tp(const void* x, const void* w, int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                           void* resid, const void* norm_w, void* hidden, float eps, void* workspace,
                           size_t ws_bytes, const void* peer_bases, int64_t world, int64_t rank, int64_t slot,
                           int64_t round_only, qw_stream_t stream);

/* Prefill (and any call of more than QW_TP_MAX_ROWS rows) uses NCCL all-reduce / all-gather
 * calls made by the host; these move the data on either side of them.
 * y bf16 [n] = bf16(x fp32 [n]): the all-reduced row-parallel down projection of the last
 * layer becomes the bf16 F.linear output that the final norm reads (REF:5092-5093).        */
int qw_round_f32_bf16(const float* x, void* y, int64_t n, qw_stream_t stream);
/* dst fp32 [R, G*Vs] = src fp32 [G, R, Vs] with dst[r][g*Vs + v] = src[g][r][v]: the logits
 * of G vocabulary shards, all-gathered rank-major, in vocabulary order (REF:5096 lm_head). */
int qw_gather_vocab_shards(const float* src, int64_t G, int64_t R, int64_t Vs, float* dst, qw_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* QW200_H */
