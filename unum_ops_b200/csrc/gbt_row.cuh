// One (token, head) row of get_block_table: the K selected blocks of that row to
// K*64 physical slot ids.  Semantics of get_block_table_ref_torch
// (src/unum_ops/sparse_kernel_extension/get_table_torch.py:4-44): position
// pos = topk[k]*64 + i maps to head_group*table[bs, clamp(pos, 0, L-1)] + h
// when 0 <= pos < lim (lim = min(token_pos_in_bs[t], seqlen_q[bs])), else 0.
// A half-warp covers one selected block, each lane producing 4 consecutive ids
// with one 16-byte streaming store (512 contiguous bytes per warp step); four
// steps are unrolled so their table loads are in flight together; table reads
// are 16-byte vector loads when the four positions are valid and inside the row.
#pragma once

#include <cstdint>

namespace unum {

constexpr int kGbtBlock = 64;   // kSparseBlockSize (get_table_torch.py:13)
constexpr int kGbtUnroll = 4;

// tk: the row's K block ids (stride ts_k); trow: the sequence's block-table row
// (L entries); orow: the row's K*64 output ids (16-byte aligned).  Writes the row's
// int4 items [e_begin, e_end) (of K*16; e_begin a multiple of 32*kGbtUnroll).
// kIdsWritten: tk was written by the calling kernel (shared memory, say), so it is
// read with plain loads rather than through the read-only cache.
template <bool kIdsWritten = false>
__device__ __forceinline__ void gbt_emit_row(const int32_t *__restrict__ tk, int64_t ts_k, int32_t K,
                                             const int32_t *__restrict__ trow, int32_t lim, int32_t L,
                                             uint32_t head_group, uint32_t h, bool vec_ok,
                                             int4 *__restrict__ orow, int lane, int32_t e_begin,
                                             int32_t e_end) {
    const int32_t items = e_end;
    const int32_t q4 = (lane & 15) * 4;         // first of this lane's 4 positions in a block
    const int32_t Lm1 = L - 1;
    for (int32_t e0 = e_begin; e0 < items; e0 += 32 * kGbtUnroll) {
        int32_t p0[kGbtUnroll];
#pragma unroll
        for (int u = 0; u < kGbtUnroll; ++u) {
            const int32_t e = e0 + u * 32 + lane;
            const int32_t *ip = tk + (int64_t)(e >> 4) * ts_k;
            const int32_t idx = e < items ? (kIdsWritten ? *ip : __ldg(ip)) : -1;
            p0[u] = (int32_t)((uint32_t)idx * (uint32_t)kGbtBlock + (uint32_t)q4);
        }
        int4 v[kGbtUnroll];
#pragma unroll
        for (int u = 0; u < kGbtUnroll; ++u) {
            const int32_t p = p0[u];
            if (vec_ok && p >= 0 && p <= INT32_MAX - 3 && p + 3 < lim && p + 3 <= Lm1) {
                const int4 tv = __ldg(reinterpret_cast<const int4 *>(trow + p));
                v[u].x = (int32_t)(head_group * (uint32_t)tv.x + h);
                v[u].y = (int32_t)(head_group * (uint32_t)tv.y + h);
                v[u].z = (int32_t)(head_group * (uint32_t)tv.z + h);
                v[u].w = (int32_t)(head_group * (uint32_t)tv.w + h);
            } else {
                int32_t r[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int32_t pi = (int32_t)((uint32_t)p + (uint32_t)i);
                    const bool valid = pi >= 0 && pi < lim;
                    const int32_t sp = pi < 0 ? 0 : (pi > Lm1 ? Lm1 : pi);  // clamp (get_table_torch.py:35)
                    r[i] = valid ? (int32_t)(head_group * (uint32_t)__ldg(trow + sp) + h) : 0;
                }
                v[u] = make_int4(r[0], r[1], r[2], r[3]);
            }
        }
#pragma unroll
        for (int u = 0; u < kGbtUnroll; ++u) {
            const int32_t e = e0 + u * 32 + lane;
            if (e < items) __stcs(orow + e, v[u]);
        }
    }
}

}  // namespace unum
