// max_pooling_1d_varlen: compressed attention scores -> 64-token block scores.
//
// Semantics follow max_pooling_1d_varlen_ref_triton and its kernel
// (src/unum_ops/infllm_v2/max_pooling_1d_varlen.py:33-183):
//   * the input is a flat buffer indexed h*T*fs + t*fs + c, fs = max_seqlen_q/stride (:82, :146);
//   * block j pools c in [j*sp-1, j*sp+sp) ∩ [0, k_len), sp = block_size/stride (:84-106);
//   * k_len = cu_k[b+1]-cu_k[b]+cache_lens[b] for the sequence b holding token t (:72-80);
//   * +inf for init blocks and the local window (:108-110), -inf for an empty window (:112-116).
//
// B200 design: an HBM stream (the whole score row is read once, the pooled
// row written once).  One warp owns one (head, token) row.  On the common
// layout (sp == 4, 16-byte aligned rows) each lane loads 16-byte vectors of
// scores (two in flight per step) and produces 16/sizeof(T)/4 pooled values
// per vector; the window's left element (c = 4j-1) is the previous lane's
// last element, fetched with a shuffle, so every score is read from HBM
// exactly once.  Only a row's last vector needs per-element masking.  Every other layout
// (odd flat strides as in the reference's own tests, other pooling ratios)
// takes a scalar path with the same results.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace {

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

constexpr int kWarps = 8;

// Sequence holding token t: the largest b with cu_q[b] <= t, if t < cu_q[b+1]
// (cu_seqlens are non-decreasing, so this is the reference's "last hit").
__device__ __forceinline__ int find_seq(const int32_t *__restrict__ cu_q, int64_t n_seq, int64_t t) {
    int64_t lo = 0, hi = n_seq;  // invariant: answer in [lo, hi)
    if (n_seq <= 0 || t < __ldg(cu_q) || t >= __ldg(cu_q + n_seq)) return -1;
    while (hi - lo > 1) {
        int64_t mid = (lo + hi) >> 1;
        if (__ldg(cu_q + mid) <= t) lo = mid; else hi = mid;
    }
    return (int)lo;
}

template <typename T> struct Pack2;  // two outputs stored as one word
template <> struct Pack2<float> { using type = float2; };
template <> struct Pack2<__nv_bfloat16> { using type = __nv_bfloat162; };
template <> struct Pack2<__half> { using type = __half2; };

template <typename T>
__device__ __forceinline__ void store2(T *p, float a, float b, bool paired) {
    if (paired) {
        typename Pack2<T>::type v;
        v.x = from_f<T>(a);
        v.y = from_f<T>(b);
        *reinterpret_cast<typename Pack2<T>::type *>(p) = v;
    } else {
        p[0] = from_f<T>(a);
        p[1] = from_f<T>(b);
    }
}

template <typename T, bool kSeg>  // kSeg false: one unit per whole row
__global__ void __launch_bounds__(kWarps * 32)
max_pool_kernel(const T *__restrict__ in, int64_t numel, int64_t H, int64_t T_, int64_t fs,
                const int32_t *__restrict__ cu_q, const int32_t *__restrict__ cu_k,
                const int32_t *__restrict__ cache_lens, int64_t n_seq, int64_t NB, int64_t sp,
                int64_t block_size, int64_t init_blocks, int64_t local_blocks, bool vec_ok,
                int32_t span, T *__restrict__ out) {
    constexpr int VEC = 16 / sizeof(T);  // scores per 16-byte load
    constexpr int OPV = VEC / 4;         // pooled outputs per load when sp == 4
    const int lane = threadIdx.x & 31;
    const int64_t rows = H * T_;
    const int64_t ksize = sp + 1;
    const int32_t nb = (int32_t)NB;
    const bool pair_ok = (NB % 2) == 0;  // 2 outputs per lane per vector: aligned word stores
    // work unit = (row, segment of `span` output blocks; span a multiple of 128, so the
    // 16-byte chunks of a segment never straddle its ends): few rows still fill the GPU
    const int32_t n_seg = kSeg ? (nb + span - 1) / span : 1;
    const int64_t units = rows * n_seg;
    for (int64_t unit = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); unit < units;
         unit += (int64_t)gridDim.x * kWarps) {
        const int64_t row = kSeg ? unit / n_seg : unit;
        const int32_t jA = kSeg ? (int32_t)(unit - row * n_seg) * span : 0;
        const int32_t jB = kSeg ? (jA + span < nb ? jA + span : nb) : nb;
        const int64_t h = row / T_, t = row - h * T_;
        const int b = find_seq(cu_q, n_seq, t);
        int32_t k_len = 0, off_bq = 0;
        if (b >= 0) {
            k_len = (__ldg(cu_k + b + 1) - __ldg(cu_k + b)) + __ldg(cache_lens + b);
            off_bq = (int32_t)((t - __ldg(cu_q + b)) / block_size);
        }
        const int64_t base = h * T_ * fs + t * fs;
        const T *src = in + base;
        // readable scores of this row: positions [0, avail)
        const int64_t room = numel - base;
        const int32_t avail = (int32_t)(room < (int64_t)k_len ? (room > 0 ? room : 0) : k_len);
        T *orow = out + row * NB;
        const int32_t init_b = (int32_t)init_blocks, local_b = (int32_t)local_blocks;
        // Blocks at or past j_end have an empty window (j*sp-1 >= k_len).
        int32_t j_end = k_len > 0 ? (int32_t)((k_len + sp) / sp) : 0;
        if (j_end > nb) j_end = nb;
        auto masked = [&](int32_t j) { return j < init_b || (off_bq >= j && off_bq <= j + local_b); };
        int32_t j_done = jA;
        // score 4*jA-1, the left end of the segment's first window
        const float carry0 = (jA > 0 && 4 * jA - 1 < avail) ? to_f<T>(src[4 * jA - 1]) : -INFINITY;
        const int32_t jE = j_end < jB ? j_end : jB;  // vector paths: blocks [jA, jE)
        if (vec_ok && sp == 4 && OPV == 2 && jE > jA) {
            // 16-bit scores: a 16-byte vector = 8 scores = the windows of 2 blocks
            const int32_t n_chunks = (jE + 1) / 2;
            float carry = carry0;  // score 8c-1 for lane 0 of the next step
            for (int32_t c0 = jA / 2; c0 < n_chunks; c0 += 64) {
                float e[2][8];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int32_t c = c0 + u * 32 + lane;
                    const int32_t p0 = c * 8;
                    if (c < n_chunks && p0 + 8 <= avail) {
                        const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(src + p0));
                        const T *tv = reinterpret_cast<const T *>(&raw);
#pragma unroll
                        for (int i = 0; i < 8; ++i) e[u][i] = to_f<T>(tv[i]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            e[u][i] = (c < n_chunks && p0 + i < avail) ? to_f<T>(src[p0 + i]) : -INFINITY;
                    }
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int32_t c = c0 + u * 32 + lane;
                    float prev = __shfl_up_sync(0xffffffffu, e[u][7], 1);
                    if (lane == 0) prev = carry;
                    carry = __shfl_sync(0xffffffffu, e[u][7], 31);
                    if (c < n_chunks) {
                        const int32_t j = 2 * c;  // outputs j and j+1
                        float m0 = fmaxf(fmaxf(j == 0 ? -INFINITY : prev, e[u][0]),
                                         fmaxf(fmaxf(e[u][1], e[u][2]), e[u][3]));
                        float m1 = fmaxf(fmaxf(e[u][3], e[u][4]), fmaxf(fmaxf(e[u][5], e[u][6]), e[u][7]));
                        m0 = masked(j) ? INFINITY : m0;          // j < j_end: window non-empty
                        if (j + 1 < jE) {
                            m1 = masked(j + 1) ? INFINITY : m1;
                            store2<T>(orow + j, m0, m1, pair_ok);
                        } else {
                            orow[j] = from_f<T>(m0);
                        }
                    }
                }
            }
            j_done = jE;
        } else if (vec_ok && sp == 4 && jE > jA) {
            // fp32 scores: a 16-byte vector = 4 scores = the window of 1 block
            float carry = carry0;
            for (int32_t c0 = jA; c0 < jE; c0 += 32) {
                const int32_t c = c0 + lane;
                const int32_t p0 = c * 4;
                float e[4];
                if (c < jE && p0 + 4 <= avail) {
                    const float4 v = __ldg(reinterpret_cast<const float4 *>(src + p0));
                    e[0] = v.x; e[1] = v.y; e[2] = v.z; e[3] = v.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        e[i] = (c < jE && p0 + i < avail) ? to_f<T>(src[p0 + i]) : -INFINITY;
                }
                float prev = __shfl_up_sync(0xffffffffu, e[3], 1);
                if (lane == 0) prev = carry;
                carry = __shfl_sync(0xffffffffu, e[3], 31);
                if (c < jE) {
                    float m = fmaxf(fmaxf(c == 0 ? -INFINITY : prev, e[0]), fmaxf(fmaxf(e[1], e[2]), e[3]));
                    orow[c] = from_f<T>(masked(c) ? INFINITY : m);
                }
            }
            j_done = jE;
        }
        // scalar path (general layouts) and the empty-window tail of the segment
        for (int32_t j = j_done + lane; j < jB; j += 32) {
            const int64_t ws = (int64_t)j * sp - 1;
            float mx = -INFINITY;
            for (int64_t ki = 0; ki < ksize; ++ki) {
                const int64_t kp = ws + ki;
                if (kp < 0 || kp >= avail) continue;
                mx = fmaxf(mx, to_f<T>(src[kp]));
            }
            const int64_t wlo = ws > 0 ? ws : 0;
            const int64_t whi = ws + ksize < k_len ? ws + ksize : k_len;
            orow[j] = from_f<T>(masked(j) ? INFINITY : (whi > wlo ? mx : -INFINITY));
        }
    }
}

}  // namespace

extern "C" int unum_max_pooling_1d_varlen(const void *input, int dtype, int64_t H, int64_t T,
                                          int64_t input_numel, const int32_t *cu_seqlens_q,
                                          const int32_t *cu_seqlens_k, const int32_t *cache_lens,
                                          int64_t n_seq, int64_t max_seqlen_q,
                                          int64_t max_context_len, int64_t local_blocks,
                                          int64_t init_blocks, int64_t block_size, int64_t stride,
                                          void *out, void *stream) {
    unum::clear_error();
    UNUM_CHECK_ARG(H >= 0 && T >= 0 && n_seq >= 0 && input_numel >= 0, "negative size");
    UNUM_CHECK_ARG(block_size > 0 && stride > 0, "block_size and stride must be positive");
    UNUM_CHECK_ARG(max_context_len >= 0 && max_seqlen_q >= 0, "negative max length");
    const int64_t NB = (max_context_len + block_size - 1) / block_size;
    const int64_t sp = block_size / stride;
    UNUM_CHECK_ARG(sp >= 1, "block_size must be >= stride");
    if (H == 0 || T == 0 || NB == 0) return UNUM_OK;
    UNUM_CHECK_ARG(input && out && cu_seqlens_q && cu_seqlens_k && cache_lens,
                   "null pointer argument");
    const int64_t fs = max_seqlen_q / stride;
    const int64_t rows = H * T;
    // rows split into segments when there are fewer than ~64 warps' worth per SM (decode)
    const int64_t target = (int64_t)unum::sm_count() * 64;
    const int64_t nbp = (NB + 127) / 128 * 128;
    int64_t n_seg = rows >= target ? 1 : (target + rows - 1) / rows;
    if (n_seg > nbp / 128) n_seg = nbp / 128;
    const int32_t span = (int32_t)((nbp / 128 + n_seg - 1) / n_seg * 128);
    const int64_t units = rows * ((NB + span - 1) / span);
    const int64_t want = (units + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)unum::sm_count() * 32;
    const int grid = (int)(want < cap ? want : cap);
    cudaStream_t s = (cudaStream_t)stream;
    const int vb = dtype == UNUM_DTYPE_F32 ? 4 : 8;  // elements per 16 bytes
    const bool vec_ok = unum::aligned16(input) && (fs % vb == 0);
    switch (dtype) {
        case UNUM_DTYPE_F32:
            (n_seg > 1 ? max_pool_kernel<float, true> : max_pool_kernel<float, false>)<<<grid, kWarps * 32, 0, s>>>(
                (const float *)input, input_numel, H, T, fs, cu_seqlens_q, cu_seqlens_k, cache_lens,
                n_seq, NB, sp, block_size, init_blocks, local_blocks, vec_ok, span, (float *)out);
            break;
        case UNUM_DTYPE_BF16:
            (n_seg > 1 ? max_pool_kernel<__nv_bfloat16, true> : max_pool_kernel<__nv_bfloat16, false>)<<<grid, kWarps * 32, 0, s>>>(
                (const __nv_bfloat16 *)input, input_numel, H, T, fs, cu_seqlens_q, cu_seqlens_k,
                cache_lens, n_seq, NB, sp, block_size, init_blocks, local_blocks, vec_ok, span,
                (__nv_bfloat16 *)out);
            break;
        case UNUM_DTYPE_F16:
            (n_seg > 1 ? max_pool_kernel<__half, true> : max_pool_kernel<__half, false>)<<<grid, kWarps * 32, 0, s>>>(
                (const __half *)input, input_numel, H, T, fs, cu_seqlens_q, cu_seqlens_k,
                cache_lens, n_seq, NB, sp, block_size, init_blocks, local_blocks, vec_ok, span,
                (__half *)out);
            break;
        default:
            unum::set_error("unsupported dtype %d", dtype);
            return UNUM_ERR_UNSUPPORTED;
    }
    return unum::check_launch("max_pool_kernel");
}
