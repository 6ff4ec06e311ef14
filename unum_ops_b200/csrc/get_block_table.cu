// get_block_table: logical top-k sparse blocks -> physical paged-KV slot ids.
//
// Semantics follow get_block_table_ref_torch
// (src/unum_ops/sparse_kernel_extension/get_table_torch.py:4-44): for every
// (token t, kv head h, selected block k) the 64 token positions
// pos = topk_idx[h,t,k]*64 + i map to head_group*block_table[bs, clamp(pos)] + h,
// or 0 when pos is negative, past seqlen_q[bs] or past token_pos_in_bs[t].
//
// B200 design: the path is a pure HBM write stream (T*H*K*256 bytes out, the
// table row of a sequence stays in L2).  One CTA walks one token at a time
// (grid-stride over tokens); each thread produces 4 consecutive slot ids and
// writes them with one 16-byte streaming store, so a warp writes 512
// contiguous bytes.  Table reads are 16-byte vector loads whenever the four
// positions are valid and inside the row.
#include "common.cuh"

namespace {

constexpr int kBlock = 64;   // kSparseBlockSize (get_table_torch.py:13)
constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
get_block_table_kernel(const int32_t *__restrict__ topk, int64_t H, int64_t T, int64_t K,
                       int64_t ts_h, int64_t ts_t, int64_t ts_k,
                       const int32_t *__restrict__ table, int64_t B, int64_t L, int64_t bt_stride,
                       const int32_t *__restrict__ token_to_bs, const int32_t *__restrict__ pos_in_bs,
                       int pos_scalar, const int32_t *__restrict__ seqlen, int seqlen_scalar,
                       uint32_t head_group, bool vec_ok, int32_t *__restrict__ out) {
    const int64_t items = H * K * (kBlock / 4);  // int4 items per token
    for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
        const int32_t bs = __ldg(token_to_bs + t);
        const bool bs_ok = bs >= 0 && bs < B;
        const int32_t lim_pos = pos_scalar ? __ldg(pos_in_bs) : __ldg(pos_in_bs + t);
        const int32_t sl = seqlen_scalar ? __ldg(seqlen) : (bs_ok ? __ldg(seqlen + bs) : 0);
        const int32_t lim = bs_ok ? min(lim_pos, sl) : INT32_MIN;  // valid iff 0 <= pos < lim
        const int32_t *trow = table + (bs_ok ? (int64_t)bs * bt_stride : 0);
        int4 *orow = reinterpret_cast<int4 *>(out + t * H * K * kBlock);
        for (int64_t e = threadIdx.x; e < items; e += kThreads) {
            const int64_t slot = e >> 4;          // h*K + k
            const int q4 = (int)(e & 15) * 4;     // first of 4 positions inside the block
            const int64_t h = slot / K;
            const int64_t k = slot - h * K;
            const int32_t idx = __ldg(topk + h * ts_h + t * ts_t + k * ts_k);
            const int32_t p0 = (int32_t)((uint32_t)idx * (uint32_t)kBlock + (uint32_t)q4);
            const uint32_t hh = (uint32_t)h;
            int4 v;
            if (p0 >= 0 && p0 <= INT32_MAX - 3 && p0 + 3 < lim && p0 + 3 < L && vec_ok) {
                const int4 tv = __ldg(reinterpret_cast<const int4 *>(trow + p0));
                v.x = (int32_t)(head_group * (uint32_t)tv.x + hh);
                v.y = (int32_t)(head_group * (uint32_t)tv.y + hh);
                v.z = (int32_t)(head_group * (uint32_t)tv.z + hh);
                v.w = (int32_t)(head_group * (uint32_t)tv.w + hh);
            } else {
                int32_t r[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int32_t p = (int32_t)((uint32_t)p0 + (uint32_t)i);
                    const bool valid = p >= 0 && p < lim;
                    const int64_t sp = p < 0 ? 0 : (p > L - 1 ? L - 1 : p);  // clamp (get_table_torch.py:35)
                    r[i] = valid ? (int32_t)(head_group * (uint32_t)__ldg(trow + sp) + hh) : 0;
                }
                v = make_int4(r[0], r[1], r[2], r[3]);
            }
            __stcs(orow + e, v);
        }
    }
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
    UNUM_CHECK_ARG(H >= 0 && T >= 0 && K >= 0 && B >= 0 && L >= 0, "negative size");
    if (H == 0 || T == 0 || K == 0) return UNUM_OK;
    UNUM_CHECK_ARG(topk_idx && token_to_bs && token_pos_in_bs && seqlen_q && out,
                   "null pointer argument");
    UNUM_CHECK_ARG(B > 0 && L > 0 && block_table, "block_table must be non-empty");
    UNUM_CHECK_ARG(unum::aligned16(out), "out must be 16-byte aligned");
    UNUM_CHECK_ARG(H * K * kBlock <= (int64_t)INT32_MAX, "H*K*64 too large");
    const bool vec_ok = unum::aligned16(block_table) && (bt_stride % 4 == 0);
    const int64_t max_grid = (int64_t)unum::sm_count() * 16;
    const int grid = (int)(T < max_grid ? T : max_grid);
    get_block_table_kernel<<<grid, kThreads, 0, (cudaStream_t)stream>>>(
        topk_idx, H, T, K, ts_h, ts_t, ts_k, block_table, B, L, bt_stride, token_to_bs,
        token_pos_in_bs, pos_is_scalar, seqlen_q, seqlen_is_scalar, (uint32_t)head_group, vec_ok,
        out);
    return unum::check_launch("get_block_table_kernel");
}
