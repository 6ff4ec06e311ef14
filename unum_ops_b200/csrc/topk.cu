// topk_blocks: per row of pooled block scores, the K best blocks.
//
// The reference has no top-k kernel (its caller runs torch.topk on the pooled
// scores).  The rule implemented here: candidates are the entries that are
// neither -inf (a block past the sequence's compressed keys) nor NaN, ranked
// by (score desc, block index asc); the first min(K, #candidates) are written
// in ascending block order, then -1 padding.  The ascending, padded layout is
// the one the reference's block-table tests feed to get_block_table
// (test/test_sparse_kernel.py:80-87).
//
// B200 design: one warp per row.  The row is staged once in shared memory as
// order-preserving 32-bit keys (excluded entries get key 0).  A radix select
// (8-bit digits, a 256-bin warp-private histogram, a warp scan to locate the
// digit holding the K-th key) finds the threshold key in 2 passes for 16-bit
// score types and 4 for fp32.  A final ballot/popc sweep in index order emits
// the winners already sorted, taking only the lowest-index ties.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace {

constexpr int kWarps = 4;
constexpr int kMaxNB = 4096;
constexpr int kMaxK = 1024;

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

// Larger score -> larger key; -inf and NaN -> 0 (not a candidate).
__device__ __forceinline__ uint32_t score_key(float f) {
    if (f != f || f == -INFINITY) return 0u;
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T, int PASSES>
__global__ void __launch_bounds__(kWarps * 32)
topk_kernel(const T *__restrict__ scores, int64_t rows, int64_t NB, int64_t row_stride, int64_t K,
            int32_t *__restrict__ out) {
    extern __shared__ uint32_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t *keys = smem + warp * (NB + 256);
    uint32_t *hist = keys + NB;
    const uint32_t lt_mask = (1u << lane) - 1u;
    for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows;
         row += (int64_t)gridDim.x * kWarps) {
        const T *src = scores + row * row_stride;
        for (int64_t i = lane; i < NB; i += 32) keys[i] = score_key(to_f<T>(src[i]));
        uint32_t prefix = 0, pmask = 0;
        int64_t remaining = K;
        bool take_all = false;
#pragma unroll 1
        for (int p = 0; p < PASSES; ++p) {
            const int shift = 24 - 8 * p;
#pragma unroll
            for (int i = 0; i < 8; ++i) hist[lane * 8 + i] = 0;
            __syncwarp();
            for (int64_t i = lane; i < NB; i += 32) {
                const uint32_t k = keys[i];
                if (k != 0u && (k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
            }
            __syncwarp();
            // lane owns bins 255-8*lane-i, i = 0..7 (descending)
            uint32_t c[8];
            uint32_t s = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                c[i] = hist[255 - 8 * lane - i];
                s += c[i];
            }
            uint32_t incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
            if (p == 0 && total <= (uint32_t)K) {
                take_all = true;
                break;
            }
            const uint32_t excl = incl - s;
            const bool mine = excl < (uint32_t)remaining && (uint32_t)remaining <= incl;
            const uint32_t owner = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
            uint32_t digit = 0, above = 0;
            if (mine) {
                uint32_t run = excl;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (run + c[i] >= (uint32_t)remaining) {
                        digit = 255u - 8u * lane - i;
                        above = run;
                        break;
                    }
                    run += c[i];
                }
            }
            digit = __shfl_sync(0xffffffffu, digit, owner);
            above = __shfl_sync(0xffffffffu, above, owner);
            remaining -= above;
            prefix |= digit << shift;
            pmask |= 255u << shift;
            __syncwarp();
        }
        // emit winners in index order
        int32_t *orow = out + row * K;
        int64_t pos = 0;
        int64_t eq_seen = 0;
        for (int64_t b = 0; b < NB && pos < K; b += 32) {
            const int64_t i = b + lane;
            const uint32_t k = i < NB ? keys[i] : 0u;
            bool sel;
            if (take_all) {
                sel = k != 0u;
            } else {
                const bool eq = (k == prefix);
                const uint32_t em = __ballot_sync(0xffffffffu, eq);
                sel = (k > prefix) || (eq && eq_seen + __popc(em & lt_mask) < remaining);
                eq_seen += __popc(em);
            }
            const uint32_t sm = __ballot_sync(0xffffffffu, sel);
            if (sel) orow[pos + __popc(sm & lt_mask)] = (int32_t)i;
            pos += __popc(sm);
        }
        for (int64_t s2 = pos + lane; s2 < K; s2 += 32) orow[s2] = -1;
        __syncwarp();
    }
}

template <typename T, int PASSES>
int launch_topk(const void *scores, int64_t rows, int64_t NB, int64_t row_stride, int64_t K,
                int32_t *out, cudaStream_t s) {
    const size_t smem = (size_t)kWarps * (NB + 256) * sizeof(uint32_t);
    auto kern = topk_kernel<T, PASSES>;
    UNUM_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t want = (rows + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)unum::sm_count() * 64;
    const int grid = (int)(want < cap ? want : cap);
    kern<<<grid, kWarps * 32, smem, s>>>((const T *)scores, rows, NB, row_stride, K, out);
    return unum::check_launch("topk_kernel");
}

}  // namespace

extern "C" int unum_topk_blocks(const void *scores, int dtype, int64_t rows, int64_t NB,
                                int64_t row_stride, int64_t K, int32_t *out, void *stream) {
    unum::clear_error();
    UNUM_CHECK_ARG(rows >= 0 && NB >= 0 && K >= 0, "negative size");
    if (rows == 0 || K == 0) return UNUM_OK;
    UNUM_CHECK_ARG(out != nullptr, "null output");
    UNUM_CHECK_ARG(NB <= kMaxNB, "NB=%lld exceeds the supported maximum %d", (long long)NB, kMaxNB);
    UNUM_CHECK_ARG(K <= kMaxK, "K=%lld exceeds the supported maximum %d", (long long)K, kMaxK);
    UNUM_CHECK_ARG(NB == 0 || (scores != nullptr && row_stride >= NB), "bad scores / row_stride");
    cudaStream_t s = (cudaStream_t)stream;
    if (NB == 0) {
        UNUM_CHECK_CUDA(cudaMemsetAsync(out, 0xff, (size_t)rows * K * sizeof(int32_t), s));
        return UNUM_OK;
    }
    switch (dtype) {
        case UNUM_DTYPE_F32: return launch_topk<float, 4>(scores, rows, NB, row_stride, K, out, s);
        case UNUM_DTYPE_BF16: return launch_topk<__nv_bfloat16, 2>(scores, rows, NB, row_stride, K, out, s);
        case UNUM_DTYPE_F16: return launch_topk<__half, 2>(scores, rows, NB, row_stride, K, out, s);
        default:
            unum::set_error("unsupported dtype %d", dtype);
            return UNUM_ERR_UNSUPPORTED;
    }
}
