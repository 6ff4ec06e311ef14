/*
 * unum_ops_b200 — C ABI of the B200 (sm_100a) InfLLM-v2 block-selection path.
 *
 * Every entry point takes raw device pointers, element counts and strides and
 * a CUDA stream (as `void *`, i.e. a cudaStream_t; NULL = legacy default
 * stream), enqueues its kernels on that stream and returns without
 * synchronising.  Return value: 0 on success, a negative UNUM_ERR_* code on
 * failure, with a message available from unum_last_error() (thread-local).
 * No C++ exception crosses this boundary, no entry point allocates device
 * memory, and all outputs are fully written by the kernels (callers may pass
 * uninitialised buffers).
 *
 * Reference interfaces replaced (Yanguan619/unum_ops, Python):
 *   unum_infllmv2_attn_stage1   <- src/unum_ops/infllm_v2/infllmv2_attn_stage1_triton_v2.py:153-228
 *                                  (public alias infllm_v2/__init__.py:3-5)
 *   unum_max_pooling_1d_varlen  <- src/unum_ops/infllm_v2/max_pooling_1d_varlen.py:127-183
 *                                  (public alias infllm_v2/__init__.py:7-9)
 *   unum_get_block_table        <- src/unum_ops/sparse_kernel_extension/get_table_torch.py:4-44
 *                                  and get_table_triton.py:218-369 (aliases __init__.py:1-12)
 *   unum_topk_blocks            <- no reference function: the reference's caller runs torch.topk
 *                                  on the pooled scores; the selection rule is stated below.
 */
#ifndef UNUM_OPS_B200_H
#define UNUM_OPS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UNUM_OK 0
#define UNUM_ERR_INVALID (-1)     /* bad argument (shape, size, alignment, null pointer) */
#define UNUM_ERR_UNSUPPORTED (-2) /* valid but not implemented on this path (e.g. head_dim != 128) */
#define UNUM_ERR_CUDA (-3)        /* a CUDA runtime/driver call failed */
#define UNUM_ERR_WORKSPACE (-4)   /* workspace missing or too small */

/* Element types of score tensors. */
#define UNUM_DTYPE_F32 0
#define UNUM_DTYPE_BF16 1
#define UNUM_DTYPE_F16 2

/* Message of the last failing call on this host thread ("" if none). */
const char *unum_last_error(void);

/* ABI version of this library (major * 100 + minor). */
int unum_abi_version(void);

/*
 * get_block_table — logical top-k blocks to physical KV slot ids.
 * Replaces get_block_table_ref_torch (get_table_torch.py:4-44) and the Triton
 * variants get_block_table_ref_triton{,_v2,_v3} (get_table_triton.py:218-369).
 *
 *   topk_idx       int32 [H, T, K], element strides (ts_h, ts_t, ts_k)
 *   block_table    int32 [B, L], row stride bt_stride (elements), column stride 1
 *   token_to_bs    int32 [T]
 *   token_pos_in_bs int32 [T], or one value broadcast when pos_is_scalar != 0
 *   seqlen_q       int32 [B], or one value broadcast when seqlen_is_scalar != 0
 *   out            int32 [T, H, K*64] contiguous, fully written
 *
 *   out[t,h,k*64+i] = head_group * block_table[bs, clamp(pos, 0, L-1)] + h
 *       if pos >= 0 && pos < seqlen_q[bs] && pos < token_pos_in_bs[t], else 0,
 *   with pos = topk_idx[h,t,k]*64 + i, bs = token_to_bs[t], int32 wrap-around.
 * head_group is 2 in the torch reference (get_table_torch.py:12) and H in the
 * Triton kernels (get_table_triton.py:252).  token_to_bs values must lie in
 * [0, B); the kernel checks and writes 0 for a token outside that range.
 */
int unum_get_block_table(const int32_t *topk_idx, int64_t H, int64_t T, int64_t K,
                         int64_t ts_h, int64_t ts_t, int64_t ts_k,
                         const int32_t *block_table, int64_t B, int64_t L, int64_t bt_stride,
                         const int32_t *token_to_bs, const int32_t *token_pos_in_bs,
                         int pos_is_scalar, const int32_t *seqlen_q, int seqlen_is_scalar,
                         int32_t head_group, int32_t *out, void *stream);

/*
 * get_block_table_shard — get_block_table for a shard of kv heads (and tokens),
 * for a rank that owns heads [head_offset, head_offset + H) of a token range.
 * No single reference function: the reference computes every head in one call.
 *
 *   topk_idx, token_to_bs, token_pos_in_bs: the shard's H heads and T tokens
 *   out[t * out_token_stride + h*K*64 + k*64 + i] for the shard's (t, h), with
 *       the value of get_block_table for head index head_offset + h;
 *   out_token_stride >= H*K*64, a multiple of 4 (H*K*64 for a dense shard, or the
 *       full model's Hk*K*64 with out pointing at head head_offset of token 0).
 */
int unum_get_block_table_shard(const int32_t *topk_idx, int64_t H, int64_t T, int64_t K,
                               int64_t ts_h, int64_t ts_t, int64_t ts_k,
                               const int32_t *block_table, int64_t B, int64_t L, int64_t bt_stride,
                               const int32_t *token_to_bs, const int32_t *token_pos_in_bs,
                               int pos_is_scalar, const int32_t *seqlen_q, int seqlen_is_scalar,
                               int32_t head_group, int64_t head_offset, int64_t out_token_stride,
                               int32_t *out, void *stream);

/*
 * max_pooling_1d_varlen — compressed scores to 64-token-block scores.
 * Replaces max_pooling_1d_varlen_ref_triton (max_pooling_1d_varlen.py:127-183).
 *
 *   input   dtype [H, T, *] read as the flat buffer in[h*T*fs + t*fs + c] with
 *           fs = max_seqlen_q / stride (the reference's flat_stride, :146);
 *           input_numel bounds every read (an element past it counts as
 *           masked — the reference reads out of bounds there).
 *   cu_seqlens_q/k int32 [n_seq+1], cache_lens int32 [n_seq]
 *   out     dtype [H, T, NB] contiguous, NB = ceil(max_context_len / block_size)
 *
 *   window of block j: c in [j*sp - 1, j*sp - 1 + sp + 1), sp = block_size/stride,
 *   clipped to [0, k_len) with k_len = cu_k[b+1]-cu_k[b]+cache_lens[b];
 *   out = +inf if j < init_blocks or j <= (t-cu_q[b])/block_size <= j+local_blocks,
 *   else the window max, or -inf for an empty window.  NaN inputs are ignored.
 */
int unum_max_pooling_1d_varlen(const void *input, int dtype, int64_t H, int64_t T,
                               int64_t input_numel, const int32_t *cu_seqlens_q,
                               const int32_t *cu_seqlens_k, const int32_t *cache_lens,
                               int64_t n_seq, int64_t max_seqlen_q, int64_t max_context_len,
                               int64_t local_blocks, int64_t init_blocks, int64_t block_size,
                               int64_t stride, void *out, void *stream);

/*
 * topk_blocks — top-K block selection per row of pooled scores.
 * No reference counterpart (the reference's caller uses torch.topk).
 *
 *   scores dtype [rows, NB] with row stride row_stride (elements)
 *   out    int32 [rows, K] contiguous
 *
 * Candidates are the entries that are neither -inf nor NaN; they are ranked by
 * (score descending, block index ascending); the first min(K, #candidates)
 * are written in ASCENDING block-index order, followed by -1 padding.
 * Supports NB <= 4096 and K <= 1024.
 */
int unum_topk_blocks(const void *scores, int dtype, int64_t rows, int64_t NB,
                     int64_t row_stride, int64_t K, int32_t *out, void *stream);

/*
 * topk_blocks_to_peers — topk_blocks whose rows also go, narrowed to int16, into the
 * buffers of every rank of a multi-GPU job (the top-k id exchange fused into the
 * kernel: plain stores over NVLink while the kernel selects, no separate collective).
 * No reference counterpart.
 *   peer_bufs  n_peers (1..8) int16 buffers, each mapped into this device's address
 *              space (e.g. the peers' pointers of a symmetric-memory allocation; this
 *              rank's own buffer among them); row r is stored at
 *              peer_bufs[i] + peer_offset + r*K for every i
 * Ids are below NB <= 32768, so int16 holds them (-1 stays -1).  K and peer_offset
 * must be even, the buffers 4-byte aligned.  The stores are complete on the peers
 * once unum_peer_signal_wait has passed on every rank.
 */
int unum_topk_blocks_to_peers(const void *scores, int dtype, int64_t rows, int64_t NB,
                              int64_t row_stride, int64_t K, int32_t *out, void *const *peer_bufs,
                              int32_t n_peers, int64_t peer_offset, void *stream);

/*
 * peer_signal_wait — cross-GPU step signal for such exchanges.  No reference
 * counterpart.  signal_bufs[i] = rank i's array of n_ranks int32 words (peer-mapped,
 * zeroed before the first step); epoch increases by one per step.  Each rank announces
 * the epoch to every peer (after a system-scope fence over its earlier stores) and
 * waits, on the stream, until every peer has announced it.  The wait is bounded (about
 * one second per peer); on expiry *status (if not NULL) becomes 40 and the kernel
 * returns, so a missing peer yields an error status rather than a hung GPU.
 */
int unum_peer_signal_wait(int32_t *const *signal_bufs, int32_t n_ranks, int32_t rank, int32_t epoch,
                          int32_t *status, void *stream);

/*
 * infllmv2_attn_stage1 — compressed-key GQA scores, softmax per head, summed
 * over each head group.  Replaces infllmv2_attn_stage1_triton_v2
 * (infllmv2_attn_stage1_triton_v2.py:153-228; kernel :19-150).
 *
 *   q    bf16 [T, Hq, D], strides (q_st, q_sh) elements for t and head, d contiguous
 *   k    bf16 [Tk, Hk, D], strides (k_st, k_sh), d contiguous
 *   cu_seqlens_q/k int32 [n_seq+1] (device)
 *   out  bf16 [Hk, T, out_stride] contiguous, fully written; out_stride is
 *        the reference's round-up-128 of max_seqlen_k.
 *
 *   out[g,t,j] = sum over the G = Hq/Hk heads h of group g of
 *                softmax_j(q[t,h] . k[k_start+j, g] * softmax_scale)
 *   over the keys j visible to t, 0 elsewhere (also 0 for a token whose
 *   softmax is empty, where the reference maps NaN to 0).  With causal != 0,
 *   key j is visible iff j < clamp((lq-15)/16 + k_len - (q_len-15)/16, 0, k_len)
 *   (C integer division, lq = t - cu_q[b]).
 *
 * Requirements: D == 128; G in {2, 4, 8, 16, 32} (the reference's Triton
 * kernel itself needs G >= 16 for its tl.dot); q, k 16-byte aligned with
 * 16-byte-multiple strides.  workspace: device memory of at least
 * unum_stage1_workspace_size(n_seq) bytes, 16-byte aligned; its contents on
 * entry do not matter.  Calls sharing a workspace must be stream-ordered.
 *
 * Two kernels compute this, with the same results: a tile kernel (256/G tokens x
 * one kv head per work item) and, for batches of at most 4 query tokens per
 * sequence with G in {16, 32} and out_stride <= 128*512/G, a decode kernel (one
 * token x one kv head per item, the token's key tiles all held in tensor memory).
 * A token with more visible keys than out_stride holds (a caller whose
 * max_seqlen_k is below a sequence's key count) gets the softmax over all its
 * visible keys with the first out_stride columns written, in both kernels.
 */
size_t unum_stage1_workspace_size(int64_t n_seq);

int unum_infllmv2_attn_stage1(const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st,
                              int64_t q_sh, const void *k, int64_t Tk, int64_t Hk, int64_t k_st,
                              int64_t k_sh, const int32_t *cu_seqlens_q,
                              const int32_t *cu_seqlens_k, int64_t n_seq, float softmax_scale,
                              int causal, void *out, int64_t out_stride, void *workspace,
                              size_t workspace_bytes, void *stream);

/*
 * infllmv2_attn_stage1_pooled — stage 1 with the block max-pooling fused in.
 * No single reference function: it computes, in one launch, exactly what the
 * reference's caller gets from infllmv2_attn_stage1 followed by
 * max_pooling_1d_varlen (max_pooling_1d_varlen.py:127-183) with block_size 64,
 * stride 16, zero cache_lens and max_seqlen_q = 16 * out_stride (the flat row
 * stride of the stage-1 output), so the pooling never re-reads the scores
 * from HBM.  `out` receives the stage-1 scores as above; `pooled` bf16
 * [Hk, T, NB] receives the block scores (+inf for the init blocks and the
 * local window, -inf for an empty window).  Requires G >= 16, and out_stride
 * must cover every sequence's compressed keys (max_seqlen_k >= each
 * cu_seqlens_k difference — the reference kernel writes past its rows
 * otherwise); with a smaller out_stride the pooled result may differ from the
 * separate pooling call, which then reads neighbouring rows.  `out` may be
 * NULL: the scores then stay on chip and only `pooled` is written (for a caller
 * that needs the selection and not the scores).
 */
int unum_infllmv2_attn_stage1_pooled(const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st,
                                     int64_t q_sh, const void *k, int64_t Tk, int64_t Hk,
                                     int64_t k_st, int64_t k_sh, const int32_t *cu_seqlens_q,
                                     const int32_t *cu_seqlens_k, int64_t n_seq,
                                     float softmax_scale, int causal, void *out,
                                     int64_t out_stride, void *pooled, int64_t NB,
                                     int64_t init_blocks, int64_t local_blocks, void *workspace,
                                     size_t workspace_bytes, void *stream);

/*
 * block_select_decode — the whole selection path of a decode batch in one launch:
 * stage 1 (the decode kernel: one CTA per (token, kv head) at a time, the token's
 * score row whole in tensor memory), then, from that row on chip, the block
 * max-pooling, the top-K and get_block_table.  No single reference function:
 * bit-identical to unum_infllmv2_attn_stage1 (out, row stride out_stride),
 * then max_pooling_1d_varlen (max_pooling_1d_varlen.py:127-183: block_size 64,
 * stride 16, max_seqlen_q = 16 * out_stride, cache_lens, NB, local_blocks,
 * init_blocks), then unum_topk_blocks (K), then unum_get_block_table
 * (get_table_torch.py:4-44 with the given head_group) — what block_select
 * runs as four kernels over HBM.
 *   out       bf16 [Hk, T, out_stride] scores, or NULL (kept on chip)
 *   pooled    bf16 [Hk, T, NB] block scores, or NULL
 *   topk_idx  int32 [Hk, T, K] (required)
 *   slots     int32 [T, Hk, K*64] physical slot ids, or NULL (then the block-table
 *             arguments are ignored)
 *   cache_lens int32 [n_seq], or NULL for zeros
 * Returns UNUM_ERR_UNSUPPORTED (nothing launched) unless G = Hq/Hk is 16 or 32,
 * D = 128, n_seq >= 1, Tk >= 1, out_stride <= 128*512/G, 0 < NB with
 * 4*NB <= out_stride (every pooling window inside the row) and 0 < K <= 1024.
 * Any T is accepted; the kernel takes one work item per (token, kv head), so it
 * is the fast path when sequences have one or a few query tokens.  Workspace and
 * status word as for unum_infllmv2_attn_stage1 (unum_stage1_status).
 */
int unum_block_select_decode(const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st,
                             int64_t q_sh, const void *k, int64_t Tk, int64_t Hk, int64_t k_st,
                             int64_t k_sh, const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                             const int32_t *cache_lens, int64_t n_seq, float softmax_scale,
                             int causal, void *out, int64_t out_stride, void *pooled, int64_t NB,
                             int64_t init_blocks, int64_t local_blocks, int32_t *topk_idx, int64_t K,
                             int32_t *slots, const int32_t *block_table, int64_t B, int64_t L,
                             int64_t bt_stride, const int32_t *token_to_bs,
                             const int32_t *token_pos_in_bs, int pos_is_scalar,
                             const int32_t *seqlen_q, int seqlen_is_scalar, int32_t head_group,
                             void *workspace, size_t workspace_bytes, void *stream);

/*
 * infllmv2_attn_stage1_window — stage 1 (optionally with fused pooling, pooled
 * may be NULL) restricted to a window of tokens: only query tiles whose tokens
 * intersect [t_begin, t_end) are computed and written; other rows of `out`
 * and `pooled` are left as they are.  No single reference function: it lets a
 * caller stream a long prefill through stage 1 chunk by chunk (for example
 * overlapping the host-to-device copy of the next chunk's queries), with the
 * same results as one full call when the chunks cover all tokens.  Tiles are
 * 256/G tokens of one sequence counted from the sequence start; a window edge
 * inside a tile computes (and rewrites) the whole tile.  `out` may be NULL when
 * `pooled` is given (scores kept on chip).
 */
int unum_infllmv2_attn_stage1_window(const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st,
                                     int64_t q_sh, const void *k, int64_t Tk, int64_t Hk,
                                     int64_t k_st, int64_t k_sh, const int32_t *cu_seqlens_q,
                                     const int32_t *cu_seqlens_k, int64_t n_seq,
                                     float softmax_scale, int causal, void *out,
                                     int64_t out_stride, void *pooled, int64_t NB,
                                     int64_t init_blocks, int64_t local_blocks, int64_t t_begin,
                                     int64_t t_end, void *workspace, size_t workspace_bytes,
                                     void *stream);

/*
 * Status word a stage-1 launch leaves in its workspace: 0 = ok; any nonzero
 * value = a bounded wait inside the kernel gave up (about one second without
 * progress; the output is then invalid, the kernel drained its in-flight work
 * and returned, and the context stays usable).  30 = that path taken on purpose:
 * with the environment variable UNUM_STAGE1_FORCE_EXPIRY=1 at call time every
 * wait reports expiry at once (a test hook).  Reads the word with a
 * stream-ordered copy and synchronises the stream.
 */
int unum_stage1_status(const void *workspace, void *stream, int32_t *status_out);

/*
 * infllmv2_attn_stage1_noalloc — unum_infllmv2_attn_stage1 without a workspace.
 * No counterpart in the reference: an addition of this library for callers
 * that cannot allocate device memory when they run stage 1 (an engine whose
 * allocator already owns all of HBM, a plugin host that forbids cudaMalloc in
 * its callbacks).  The schedule scratch is a fixed 64 KB array inside the
 * library, held by every GPU that loads the library until the process exits.
 *
 * Same arguments and results as unum_infllmv2_attn_stage1, minus the
 * workspace.  Limit: n_seq <= 16379 (larger batches fail with
 * UNUM_ERR_INVALID and a message).  Runs on the current device; the first
 * call on each device looks up the array's device address
 * (cudaGetSymbolAddress), so make that first call before any stream capture.
 * The call allocates nothing.  All calls on a device share the one array and
 * every call rewrites it fully, so calls that overlap on the GPU (different
 * streams, no ordering between them) race and must be avoided.  The array's
 * device address is cached per device for the life of the process: do not use
 * this entry point across cudaDeviceReset.
 */
int unum_infllmv2_attn_stage1_noalloc(const void *q, int64_t T, int64_t Hq, int64_t D,
                                      int64_t q_st, int64_t q_sh, const void *k, int64_t Tk,
                                      int64_t Hk, int64_t k_st, int64_t k_sh,
                                      const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                                      int64_t n_seq, float softmax_scale, int causal, void *out,
                                      int64_t out_stride, void *stream);

/*
 * stage1_noalloc_status — the status word (codes as in unum_stage1_status) that
 * the last unum_infllmv2_attn_stage1_noalloc call on the current device left in
 * the library's scratch array.  No counterpart in the reference.  Copies the
 * word on `stream` and synchronises that stream; allocates nothing.
 */
int unum_stage1_noalloc_status(void *stream, int32_t *status_out);

/*
 * sparse_attn_blocks — stage-2 sparse attention over the selected blocks, the
 * consumer of get_block_table with its gather fused in.  No reference function:
 * the reference's get_block_table (get_table_torch.py:4-44) emits the slot ids
 * such a kernel reads; here they are computed in the loader and never written.
 *
 *   q        bf16 [T, Hq, 128], strides (q_st, q_sh) elements, Hq = 16 * Hk
 *   k_cache, v_cache  bf16 [n_slots, 128] contiguous rows; row = head_group *
 *            physical token + kv head (get_block_table's slot numbering)
 *   topk_idx int32 [Hk, T, K] (element strides ts_h, ts_t; k contiguous), K <= 64
 *   block_table, token_to_bs, token_pos_in_bs, seqlen_q: as for unum_get_block_table
 *   out      bf16 [T, Hq, 128] contiguous, fully written
 *   status   optional device int32 (NULL: none): set to 0 on entry, nonzero when a
 *            bounded wait inside the kernel gave up (output then invalid)
 *
 *   out[t,h] = sum_p softmax_p(q[t,h] . k_cache[slot_p] * softmax_scale) v_cache[slot_p]
 *   over p = topk[g,t,k]*64 + i with topk >= 0, p < seqlen_q[bs], p < token_pos_in_bs[t],
 *   slot_p = head_group * block_table[bs, min(p, L-1)] + g (g = h / 16, bs = token_to_bs[t]);
 *   slots outside [0, n_slots) are skipped; 0 for a row with no valid position.
 */
int unum_sparse_attn_blocks(const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st, int64_t q_sh,
                            const void *k_cache, const void *v_cache, int64_t n_slots, int64_t Hk,
                            const int32_t *topk_idx, int64_t K, int64_t ts_h, int64_t ts_t,
                            const int32_t *block_table, int64_t B, int64_t L, int64_t bt_stride,
                            const int32_t *token_to_bs, const int32_t *token_pos_in_bs, int pos_is_scalar,
                            const int32_t *seqlen_q, int seqlen_is_scalar, int32_t head_group,
                            float softmax_scale, void *out, int32_t *status, void *stream);

/*
 * compress_keys — the producer of stage 1's compressed keys (no reference
 * function: the reference's caller builds k_cmp; the layout is the one its
 * stage-1 kernel assumes, the 16-token stride of infllmv2_attn_stage1_triton_v2.py:70).
 * Compressed key j of sequence b = bf16( sum_{t<kernel} k[cu_seqlens[b] + j*stride + t]
 * * (1/kernel) ), fp32 sums in token order, round to nearest even.
 *
 *   k        bf16 [T, Hk, D=128], strides (k_st, k_sh) elements, 16-byte aligned
 *   cu_out   int32 [n_seq+1]: cu_out[b+1]-cu_out[b] = (L_b - kernel)/stride + 1, or 0 when
 *            L_b < kernel; n_out = cu_out[n_seq]
 *   out      bf16 [n_out, Hk, 128] contiguous
 */
int unum_compress_keys(const void *k, int64_t T, int64_t Hk, int64_t D, int64_t k_st, int64_t k_sh,
                       const int32_t *cu_seqlens, const int32_t *cu_out, int64_t n_seq, int64_t n_out,
                       int64_t kernel, int64_t stride, void *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* UNUM_OPS_B200_H */
