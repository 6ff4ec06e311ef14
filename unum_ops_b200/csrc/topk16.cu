// topk_blocks for 16-bit (bf16 / fp16) rows of pooled block scores.
//
// Selection rule (the reference has no top-k kernel; its caller runs
// torch.topk): candidates are the entries that are neither -inf nor NaN, ranked
// by (score descending, block index ascending); the first min(K, #candidates)
// are written in ascending block order, then -1 padding.  -0 ranks as +0.
//
// One warp per row, a run of consecutive rows per warp: neighbouring tokens'
// pooled rows are close, so the previous row's K-th key is a good hint.  The row
// is loaded once with coalesced 16-byte loads and staged in shared memory; lane
// l then owns the contiguous chunk [l*C, l*C + C) (C = padded NB / 32), so one
// warp scan of per-lane counts keeps block order (the staging pads each chunk
// by 16 bytes so that the lanes' chunk reads are free of bank conflicts).  Per row:
//   1. with a hint kp, every score is compared (packed bf16x2 / half2 compares)
//      with the bound t = kp - margin; when between K and kCap pass, their keys
//      go to a candidate list and one 256-bin histogram of (key - t) (bins
//      aggregated per warp with match.any) gives the K-th key k*;
//   2. otherwise (no hint, a miss) a 16-step bitwise search over the key range,
//      counting with the same packed compares on the staged row, gives k*;
//   3. a sweep compares the staged row with k* (greater / equal masks), takes
//      every score above k* and the lowest-index ties up to K, and writes the ids
//      in block order (one scan of per-lane counts).
// The margin adapts to the density of scores near the threshold.  Results never
// depend on which path ran.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace unum {
namespace topk16 {

constexpr int kWarps = 4;      // warps per block
constexpr int kCap = 384;      // candidate slots per warp
constexpr int kMaxVec = 16;    // 16-byte vectors per lane: NB <= 4096

template <typename T> struct Tr;
template <> struct Tr<__nv_bfloat16> {
    using T2 = __nv_bfloat162;
    static constexpr uint32_t kNegInf = 0xFF80u, kPosInf = 0x7F80u, kNanAbs = 0x7F80u;
    static constexpr uint32_t kMinKey = 0x0080u;  // key of the most negative finite value
    static constexpr uint32_t kMaxKey = 0xFF80u;  // key of +inf
};
template <> struct Tr<__half> {
    using T2 = __half2;
    static constexpr uint32_t kNegInf = 0xFC00u, kPosInf = 0x7C00u, kNanAbs = 0x7C00u;
    static constexpr uint32_t kMinKey = 0x0400u;
    static constexpr uint32_t kMaxKey = 0xFC00u;
};

template <typename T>
__device__ __forceinline__ uint32_t ge2(uint32_t x, uint32_t t2) {
    using T2 = typename Tr<T>::T2;
    return __hge2_mask(*reinterpret_cast<const T2 *>(&x), *reinterpret_cast<const T2 *>(&t2));
}
template <typename T>
__device__ __forceinline__ uint32_t gt2(uint32_t x, uint32_t t2) {
    using T2 = typename Tr<T>::T2;
    return __hgt2_mask(*reinterpret_cast<const T2 *>(&x), *reinterpret_cast<const T2 *>(&t2));
}
template <typename T>
__device__ __forceinline__ uint32_t eq2(uint32_t x, uint32_t t2) {
    using T2 = typename Tr<T>::T2;
    return __heq2_mask(*reinterpret_cast<const T2 *>(&x), *reinterpret_cast<const T2 *>(&t2));
}

// Order-preserving 16-bit key: larger score -> larger key; NaN, -inf -> 0; -0 -> +0.
template <typename T>
__device__ __forceinline__ uint32_t key_of(uint32_t u) {
    if ((u & 0x7FFFu) > Tr<T>::kNanAbs || u == Tr<T>::kNegInf) return 0u;
    if (u == 0x8000u) u = 0u;
    return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
}
// the score bits of key k (kMinKey <= k <= kMaxKey), twice (both halves)
__device__ __forceinline__ uint32_t bits2_of_key(uint32_t k) {
    const uint32_t b = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
    return b | (b << 16);
}

__device__ __forceinline__ uint32_t excl_scan(uint32_t x, int lane, uint32_t &total) {
    uint32_t v = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
    }
    total = __shfl_sync(0xffffffffu, v, 31);
    return v - x;
}

// 8-bit mask (bit e = score e of the 8) of the packed compare results of 4 words.
__device__ __forceinline__ uint32_t mask8(uint32_t m0, uint32_t m1, uint32_t m2, uint32_t m3) {
    const uint32_t a = (m0 & 0x00010001u) | ((m1 & 0x00010001u) << 2);
    const uint32_t b = (m2 & 0x00010001u) | ((m3 & 0x00010001u) << 2);
    const uint32_t c = a | (b << 4);
    return (c | (c >> 15)) & 0xFFu;
}

// Masks over the lane's chunk (bit 8v+e of m[v/4] = score 8v+e) of scores >= t2 (Ge),
// > t2 (Gt) or == t2 (Eq).
enum class Cmp { Ge, Gt, Eq };
template <typename T, Cmp kCmp>
__device__ __forceinline__ void chunk_mask(const uint16_t *chunk, int32_t nvec, uint32_t t2, uint32_t (&m)[4]) {
    m[0] = m[1] = m[2] = m[3] = 0u;
#pragma unroll
    for (int32_t v = 0; v < kMaxVec; ++v) {
        if (v >= nvec) break;
        const uint4 w = *reinterpret_cast<const uint4 *>(chunk + 8 * v);
        uint32_t r;
        if (kCmp == Cmp::Ge) r = mask8(ge2<T>(w.x, t2), ge2<T>(w.y, t2), ge2<T>(w.z, t2), ge2<T>(w.w, t2));
        else if (kCmp == Cmp::Gt) r = mask8(gt2<T>(w.x, t2), gt2<T>(w.y, t2), gt2<T>(w.z, t2), gt2<T>(w.w, t2));
        else r = mask8(eq2<T>(w.x, t2), eq2<T>(w.y, t2), eq2<T>(w.z, t2), eq2<T>(w.w, t2));
        m[v >> 2] |= r << (8 * (v & 3));
    }
}

__device__ __forceinline__ uint32_t popc4(const uint32_t (&m)[4]) {
    return __popc(m[0]) + __popc(m[1]) + __popc(m[2]) + __popc(m[3]);
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32, 8)  // 8 blocks of 4 warps per SM: <= 64 registers
topk16_kernel(const T *__restrict__ scores, int64_t rows, int32_t NB, int64_t row_stride, int32_t K,
              bool vec_ok, int64_t rows_per_warp, int32_t *__restrict__ out) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int32_t NBp = (NB + 255) & ~255;  // padded: C = NBp/32 is a multiple of 8
    const int32_t C = NBp >> 5;
    const int32_t nvec = C >> 3;
    // the staged row: lane l's chunk at 16-byte slots l*(nvec+1) .. (one slot of padding per
    // chunk, so the lanes' reads of their chunks hit distinct banks)
    uint8_t *wb = smem + (size_t)warp * (1024 + kCap * 4 + (size_t)NBp * 2 + 512);
    uint32_t *hist = reinterpret_cast<uint32_t *>(wb);
    uint32_t *cand = reinterpret_cast<uint32_t *>(wb + 1024);             // candidate keys
    uint16_t *rowb = reinterpret_cast<uint16_t *>(wb + 1024 + kCap * 4);  // the row's bits
    const uint16_t *chunk = rowb + lane * (C + 8);
    const int64_t gw = (int64_t)blockIdx.x * kWarps + warp;
    const int64_t r0 = gw * rows_per_warp;
    const int64_t r1 = r0 + rows_per_warp < rows ? r0 + rows_per_warp : rows;
    uint32_t hint = 0;     // K-th key of the previous row (0: none)
    uint32_t margin = 16;  // key steps below the hint
    for (int64_t row = r0; row < r1; ++row) {
        const T *src = scores + row * row_stride;
        int32_t *orow = out + row * K;
        // ---- coalesced loads (vector v of lane l = 16-byte chunk v*32 + l), staged in place
#pragma unroll
        for (int32_t v0 = 0; v0 < kMaxVec; v0 += 8) {
            if (v0 >= nvec) break;
            uint4 w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int32_t i0 = 8 * ((v0 + j) * 32 + lane);
                if (v0 + j >= nvec) {
                    w[j] = make_uint4(0u, 0u, 0u, 0u);
                } else if (vec_ok && i0 + 8 <= NB) {
                    w[j] = __ldg(reinterpret_cast<const uint4 *>(src + i0));
                } else {
                    uint32_t h[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        h[e] = i0 + e < NB ? (uint32_t)__ldg(reinterpret_cast<const unsigned short *>(src) + i0 + e)
                                           : Tr<T>::kNegInf;
                    w[j] = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16),
                                      h[6] | (h[7] << 16));
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (v0 + j < nvec) {
                    const int32_t g = (v0 + j) * 32 + lane;  // global vector: chunk g / nvec, slot g % nvec
                    *reinterpret_cast<uint4 *>(rowb + 8 * (g + g / nvec)) = w[j];
                }
        }
        __syncwarp();
        uint32_t kth = 0;   // K-th largest key; 0 with take_all
        bool take_all = false, found = false;
        if (hint != 0u) {
            // ---- 1. candidates >= t = hint - margin
            // a bound that misses (fewer than K or more than kCap above it) is moved and
            // retried a few times, bracketing the K-th key, before the bitwise search
            uint32_t t = hint > Tr<T>::kMinKey + margin ? hint - margin : Tr<T>::kMinKey;
            uint32_t t_few = 0u, t_many = 0u;  // bounds seen with too few / too many above
            uint32_t bm[4];
            uint32_t n = 0, slot = 0;
            bool ok = false;
#pragma unroll 1
            for (int attempt = 0; attempt < 5; ++attempt) {
                chunk_mask<T, Cmp::Ge>(chunk, nvec, bits2_of_key(t), bm);
                slot = excl_scan(popc4(bm), lane, n);
                if (n >= (uint32_t)K && n <= (uint32_t)kCap) {
                    ok = true;
                    break;
                }
                if (n < (uint32_t)K) {
                    t_few = t;
                    if (t <= Tr<T>::kMinKey) break;  // fewer than K candidates in all
                    const uint32_t lo = t_many ? t_many : (t > Tr<T>::kMinKey + 4 * margin ? t - 4 * margin
                                                                                          : Tr<T>::kMinKey);
                    t = t_many ? (t_many + t) / 2 : lo;
                    if (attempt == 0) margin = margin < 512u ? margin * 4 : 512u;
                } else {
                    t_many = t;
                    t = t_few ? (t + t_few + 1) / 2 : min(t + margin, Tr<T>::kMaxKey);
                    if (attempt == 0) margin = margin > 1u ? margin / 2 : 1u;
                }
                if (t_few && t_many && t_few <= t_many + 1) break;  // adjacent keys: a run of ties
            }
            if (ok) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    for (uint32_t m = bm[q]; m != 0u; m &= m - 1u)
                        cand[slot++] = key_of<T>(chunk[32 * q + __ffs(m) - 1]);
                reinterpret_cast<uint4 *>(hist)[2 * lane] = make_uint4(0u, 0u, 0u, 0u);
                reinterpret_cast<uint4 *>(hist)[2 * lane + 1] = make_uint4(0u, 0u, 0u, 0u);
                __syncwarp();
                // histogram of key - t (bin 255: t + 255 and above), aggregated per warp
                for (uint32_t base = 0; base < n; base += 32) {
                    const uint32_t i = base + lane;
                    const uint32_t bin = i < n ? min(cand[i] - t, 255u) : 256u;
                    const uint32_t peers = __match_any_sync(0xffffffffu, bin);
                    if (bin < 256u && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
                }
                __syncwarp();
                // lane owns bins 255-8*lane .. 248-8*lane (descending)
                const uint4 lo4 = reinterpret_cast<const uint4 *>(hist + 248 - 8 * lane)[0];
                const uint4 hi4 = reinterpret_cast<const uint4 *>(hist + 248 - 8 * lane)[1];
                const uint32_t c[8] = {hi4.w, hi4.z, hi4.y, hi4.x, lo4.w, lo4.z, lo4.y, lo4.x};
                uint32_t sum = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) sum += c[i];
                uint32_t tot;
                const uint32_t above = excl_scan(sum, lane, tot);
                const bool own = above < (uint32_t)K && (uint32_t)K <= above + sum;
                const uint32_t owner = __ffs(__ballot_sync(0xffffffffu, own)) - 1;
                uint32_t bin = 0;
                if (own) {
                    uint32_t run = above;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        if (run + c[i] >= (uint32_t)K) {
                            bin = 255u - 8u * lane - i;
                            break;
                        }
                        run += c[i];
                    }
                }
                bin = __shfl_sync(0xffffffffu, bin, owner);
                if (bin < 255u) {  // exact: the K-th key is t + bin
                    kth = t + bin;
                    found = true;
                }
                if (n > (uint32_t)kCap / 2) margin = margin > 1u ? margin / 2 : 1u;
            }
            __syncwarp();
        }
        if (!found) {
            // ---- 2. bitwise search for the largest key k with #{keys >= k} >= K
            uint32_t bm[4];
            chunk_mask<T, Cmp::Ge>(chunk, nvec, bits2_of_key(Tr<T>::kMinKey), bm);
            const uint32_t total = __reduce_add_sync(0xffffffffu, popc4(bm));
            if (total <= (uint32_t)K) {
                take_all = true;
            } else {
                uint32_t k = 0;
#pragma unroll 1
                for (int b = 15; b >= 0; --b) {
                    const uint32_t c2 = k | (1u << b);
                    uint32_t cnt;
                    if (c2 > Tr<T>::kMaxKey) cnt = 0u;  // above +inf: NaN keys, never counted
                    else if (c2 <= Tr<T>::kMinKey) cnt = total;
                    else {
                        chunk_mask<T, Cmp::Ge>(chunk, nvec, bits2_of_key(c2), bm);
                        cnt = __reduce_add_sync(0xffffffffu, popc4(bm));
                    }
                    if (cnt >= (uint32_t)K) k = c2;
                }
                kth = k;
            }
        }
        // ---- 3. sweep: every score above k*, the lowest-index ties up to K, in block order
        uint32_t gm[4], em[4] = {0u, 0u, 0u, 0u};
        if (take_all) {
            chunk_mask<T, Cmp::Ge>(chunk, nvec, bits2_of_key(Tr<T>::kMinKey), gm);
        } else {
            const uint32_t v2 = bits2_of_key(kth);
            chunk_mask<T, Cmp::Gt>(chunk, nvec, v2, gm);
            chunk_mask<T, Cmp::Eq>(chunk, nvec, v2, em);
        }
        uint32_t tot_gt, tot_eq;
        const uint32_t ngt = popc4(gm), neq = popc4(em);
        excl_scan(ngt, lane, tot_gt);
        const uint32_t eq_before = excl_scan(neq, lane, tot_eq);
        const int32_t need = take_all ? 0 : K - (int32_t)tot_gt;  // ties to take, lowest index first
        uint32_t quota = need > (int32_t)eq_before ? min(neq, (uint32_t)(need - (int32_t)eq_before)) : 0u;
        // keep the first `quota` tie bits of this lane
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t keep = 0u;
            for (uint32_t m = em[q]; m != 0u && quota > 0u; m &= m - 1u, --quota) keep |= m & (0u - m);
            gm[q] |= keep;
        }
        uint32_t written;
        uint32_t pos = excl_scan(popc4(gm), lane, written);
#pragma unroll
        for (int q = 0; q < 4; ++q)
            for (uint32_t m = gm[q]; m != 0u; m &= m - 1u) orow[pos++] = lane * C + 32 * q + __ffs(m) - 1;
        for (uint32_t i = written + lane; i < (uint32_t)K; i += 32) orow[i] = -1;
        hint = take_all ? 0u : kth;
        __syncwarp();
    }
}

template <typename T>
int launch(const void *scores, int64_t rows, int64_t NB, int64_t row_stride, int64_t K, int32_t *out,
           cudaStream_t s) {
    const int64_t NBp = (NB + 255) / 256 * 256;
    const size_t smem = (size_t)kWarps * (1024 + kCap * 4 + (size_t)NBp * 2 + 512);
    auto kern = topk16_kernel<T>;
    UNUM_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;  // one resident wave; runs of consecutive rows per warp reuse the hint
    UNUM_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarps * 32, smem));
    const int64_t want = (rows + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)unum::sm_count() * (per_sm > 0 ? per_sm : 1);
    const int grid = (int)(want < cap ? want : cap);
    const int64_t nwarps = (int64_t)grid * kWarps;
    const int64_t rows_per_warp = (rows + nwarps - 1) / nwarps;
    const bool vec_ok = unum::aligned16(scores) && ((row_stride * 2) % 16 == 0);
    kern<<<grid, kWarps * 32, smem, s>>>((const T *)scores, rows, (int32_t)NB, row_stride, (int32_t)K, vec_ok,
                                         rows_per_warp, out);
    return unum::check_launch("topk16_kernel");
}

}  // namespace topk16
}  // namespace unum

// Entry for the 16-bit score types, called by unum_topk_blocks (topk.cu).
int unum_topk16_launch(const void *scores, int dtype, int64_t rows, int64_t NB, int64_t row_stride, int64_t K,
                       int32_t *out, cudaStream_t s) {
    if (dtype == UNUM_DTYPE_BF16) return unum::topk16::launch<__nv_bfloat16>(scores, rows, NB, row_stride, K, out, s);
    return unum::topk16::launch<__half>(scores, rows, NB, row_stride, K, out, s);
}
