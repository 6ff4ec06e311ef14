// get_block_table: logical top-k sparse blocks -> physical paged-KV slot ids.
//
// Semantics follow get_block_table_ref_torch
// (src/unum_ops/sparse_kernel_extension/get_table_torch.py:4-44): for every
// (token t, kv head h, selected block k) the 64 token positions
// pos = topk_idx[h,t,k]*64 + i map to head_group*block_table[bs, clamp(pos)] + h,
// or 0 when pos is negative, past seqlen_q[bs] or past token_pos_in_bs[t].
//
// B200 design: the path is a pure HBM write stream (T*H*K*256 bytes out, the
// table row of a sequence stays in L2).  One warp owns one (token, head) output
// row of K*64 ids; a half-warp covers one selected block, each lane producing 4
// consecutive ids with one 16-byte streaming store, so a warp writes 512
// contiguous bytes per step.  Index arithmetic is 32-bit and division-free
// inside a row; four steps are unrolled so their table loads are in flight
// together.  Table reads are 16-byte vector loads whenever the four positions
// are valid and inside the row.
#include "common.cuh"
#include "gbt_row.cuh"

namespace {

constexpr int kBlock = unum::kGbtBlock;
constexpr int kWarps = 8;

template <bool kSeg>  // false: one unit per whole row (span = the row)
__global__ void __launch_bounds__(kWarps * 32)
get_block_table_kernel(const int32_t *__restrict__ topk, int64_t H, int64_t T, int64_t K,
                       int64_t ts_h, int64_t ts_t, int64_t ts_k,
                       const int32_t *__restrict__ table, int64_t B, int64_t L, int64_t bt_stride,
                       const int32_t *__restrict__ token_to_bs, const int32_t *__restrict__ pos_in_bs,
                       int pos_scalar, const int32_t *__restrict__ seqlen, int seqlen_scalar,
                       uint32_t head_group, uint32_t h0, int64_t out_ts, bool vec_ok, int32_t span,
                       int32_t *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = T * H;
    const int32_t items = (int32_t)(K * (kBlock / 4));  // int4 items per row
    // work unit = (row, segment of `span` int4 items, a multiple of 128): few rows (decode
    // batches) still spread over the GPU
    const int32_t n_seg = kSeg ? (items + span - 1) / span : 1;
    const int64_t units = rows * n_seg;
    for (int64_t unit = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); unit < units;
         unit += (int64_t)gridDim.x * kWarps) {
        const int64_t row = kSeg ? unit / n_seg : unit;
        const int32_t eA = kSeg ? (int32_t)(unit - row * n_seg) * span : 0;
        const int32_t eB = kSeg ? (eA + span < items ? eA + span : items) : items;
        const int64_t t = row / H;
        const uint32_t hl = (uint32_t)(row - t * H);  // head within topk / out
        const uint32_t h = hl + h0;                    // head index in the block-table values
        const int32_t bs = __ldg(token_to_bs + t);
        const bool bs_ok = bs >= 0 && bs < B;
        const int32_t lim_pos = pos_scalar ? __ldg(pos_in_bs) : __ldg(pos_in_bs + t);
        const int32_t sl = seqlen_scalar ? __ldg(seqlen) : (bs_ok ? __ldg(seqlen + bs) : 0);
        const int32_t lim = bs_ok ? min(lim_pos, sl) : INT32_MIN;  // valid iff 0 <= pos < lim
        const int32_t *trow = table + (bs_ok ? (int64_t)bs * bt_stride : 0);
        const int32_t *tk = topk + (int64_t)hl * ts_h + t * ts_t;
        int4 *orow = reinterpret_cast<int4 *>(out + t * out_ts) + (int64_t)hl * items;
        unum::gbt_emit_row(tk, ts_k, (int32_t)K, trow, lim, (int32_t)L, head_group, h, vec_ok, orow, lane,
                           eA, eB);
    }
}

}  // namespace

namespace {
int launch_gbt(const int32_t *topk_idx, int64_t H, int64_t T, int64_t K, int64_t ts_h, int64_t ts_t,
               int64_t ts_k, const int32_t *block_table, int64_t B, int64_t L, int64_t bt_stride,
               const int32_t *token_to_bs, const int32_t *token_pos_in_bs, int pos_is_scalar,
               const int32_t *seqlen_q, int seqlen_is_scalar, int32_t head_group, int64_t h0,
               int64_t out_ts, int32_t *out, void *stream) {
    UNUM_CHECK_ARG(H >= 0 && T >= 0 && K >= 0 && B >= 0 && L >= 0, "negative size");
    if (H == 0 || T == 0 || K == 0) return UNUM_OK;
    UNUM_CHECK_ARG(topk_idx && token_to_bs && token_pos_in_bs && seqlen_q && out,
                   "null pointer argument");
    UNUM_CHECK_ARG(B > 0 && L > 0 && block_table, "block_table must be non-empty");
    UNUM_CHECK_ARG(unum::aligned16(out), "out must be 16-byte aligned");
    UNUM_CHECK_ARG(K * kBlock <= (int64_t)INT32_MAX / 4, "K too large");
    UNUM_CHECK_ARG(L <= (int64_t)INT32_MAX, "block_table row too long");
    UNUM_CHECK_ARG(h0 >= 0 && h0 <= (int64_t)INT32_MAX, "head offset out of range");
    UNUM_CHECK_ARG(out_ts >= H * K * kBlock && out_ts % 4 == 0,
                   "out token stride must cover H*K*64 ids and be a multiple of 4");
    const bool vec_ok = unum::aligned16(block_table) && (bt_stride % 4 == 0);
    const int64_t rows = T * H;
    // rows split into segments when there are fewer than ~64 warps' worth per SM (decode)
    const int64_t items = K * (kBlock / 4);
    const int64_t target = (int64_t)unum::sm_count() * 64;
    const int64_t ip = (items + 127) / 128;  // 128-item steps per row
    int64_t n_seg = rows >= target ? 1 : (target + rows - 1) / rows;
    if (n_seg > ip) n_seg = ip;
    const int32_t span = (int32_t)((ip + n_seg - 1) / n_seg * 128);
    const int64_t units = rows * ((items + span - 1) / span);
    const int64_t want = (units + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)unum::sm_count() * 32;
    const int grid = (int)(want < cap ? want : cap);
    auto kern = n_seg > 1 ? get_block_table_kernel<true> : get_block_table_kernel<false>;
    kern<<<grid, kWarps * 32, 0, (cudaStream_t)stream>>>(
        topk_idx, H, T, K, ts_h, ts_t, ts_k, block_table, B, L, bt_stride, token_to_bs,
        token_pos_in_bs, pos_is_scalar, seqlen_q, seqlen_is_scalar, (uint32_t)head_group,
        (uint32_t)h0, out_ts, vec_ok, span, out);
    return unum::check_launch("get_block_table_kernel");
}
}  // namespace

extern "C" int unum_get_block_table(const int32_t *topk_idx, int64_t H, int64_t T, int64_t K,
                                    int64_t ts_h, int64_t ts_t, int64_t ts_k,
                                    const int32_t *block_table, int64_t B, int64_t L,
                                    int64_t bt_stride, const int32_t *token_to_bs,
                                    const int32_t *token_pos_in_bs, int pos_is_scalar,
                                    const int32_t *seqlen_q, int seqlen_is_scalar,
                                    int32_t head_group, int32_t *out, void *stream) {
    unum::clear_error();
    return launch_gbt(topk_idx, H, T, K, ts_h, ts_t, ts_k, block_table, B, L, bt_stride, token_to_bs,
                      token_pos_in_bs, pos_is_scalar, seqlen_q, seqlen_is_scalar, head_group, 0,
                      H * K * kBlock, out, stream);
}

extern "C" int unum_get_block_table_shard(const int32_t *topk_idx, int64_t H, int64_t T, int64_t K,
                                          int64_t ts_h, int64_t ts_t, int64_t ts_k,
                                          const int32_t *block_table, int64_t B, int64_t L,
                                          int64_t bt_stride, const int32_t *token_to_bs,
                                          const int32_t *token_pos_in_bs, int pos_is_scalar,
                                          const int32_t *seqlen_q, int seqlen_is_scalar,
                                          int32_t head_group, int64_t head_offset,
                                          int64_t out_token_stride, int32_t *out, void *stream) {
    unum::clear_error();
    return launch_gbt(topk_idx, H, T, K, ts_h, ts_t, ts_k, block_table, B, L, bt_stride, token_to_bs,
                      token_pos_in_bs, pos_is_scalar, seqlen_q, seqlen_is_scalar, head_group,
                      head_offset, out_token_stride, out, stream);
}
