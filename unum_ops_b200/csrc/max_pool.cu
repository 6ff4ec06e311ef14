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
// layout (sp == 4, 16-byte aligned rows) each lane loads one 16-byte vector of
// scores per step and produces 16/sizeof(T)/4 pooled values; the window's
// left element (c = 4j-1) is the previous lane's last element, fetched with a
// shuffle, so every score is read from HBM exactly once.  Every other layout
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

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
max_pool_kernel(const T *__restrict__ in, int64_t numel, int64_t H, int64_t T_, int64_t fs,
                const int32_t *__restrict__ cu_q, const int32_t *__restrict__ cu_k,
                const int32_t *__restrict__ cache_lens, int64_t n_seq, int64_t NB, int64_t sp,
                int64_t block_size, int64_t init_blocks, int64_t local_blocks, bool vec_ok,
                T *__restrict__ out) {
    constexpr int VEC = 16 / sizeof(T);  // scores per 16-byte load
    constexpr int OPV = VEC / 4;         // pooled outputs per load when sp == 4
    const int lane = threadIdx.x & 31;
    const int64_t rows = H * T_;
    const int64_t wid = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int64_t nw = (int64_t)gridDim.x * kWarps;
    const int64_t ksize = sp + 1;
    for (int64_t row = wid; row < rows; row += nw) {
        const int64_t h = row / T_, t = row - h * T_;
        const int b = find_seq(cu_q, n_seq, t);
        int64_t k_len = 0, off_bq = 0;
        if (b >= 0) {
            k_len = (int64_t)(__ldg(cu_k + b + 1) - __ldg(cu_k + b)) + __ldg(cache_lens + b);
            off_bq = (t - __ldg(cu_q + b)) / block_size;
        }
        const int64_t base = h * T_ * fs + t * fs;
        T *orow = out + row * NB;
        // Blocks at or past j_end have an empty window (4j-1 >= k_len).
        int64_t j_end = k_len > 0 ? (k_len + 1 + sp - 1) / sp : 0;  // first j with j*sp-1 >= k_len
        if (j_end > NB) j_end = NB;
        auto finish = [&](int64_t j, float mx, bool has) {
            const bool minf = (j < init_blocks) || (off_bq >= j && off_bq <= j + local_blocks);
            orow[j] = from_f<T>(minf ? INFINITY : (has ? mx : -INFINITY));
        };
        int64_t j_done = 0;
        if (vec_ok && sp == 4) {
            // vector path over outputs [0, j_end): chunk c covers scores [c*VEC, c*VEC+VEC)
            const int64_t n_chunks = (j_end + OPV - 1) / OPV;
            float carry = -INFINITY;  // score c*VEC-1 of the first lane of the next step
            for (int64_t c0 = 0; c0 < n_chunks; c0 += 32) {
                const int64_t c = c0 + lane;
                float e[VEC];
                const int64_t p0 = c * VEC;  // first score position of this chunk
                if (c < n_chunks && base + p0 + VEC <= numel) {
                    const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(in + base + p0));
                    const T *tv = reinterpret_cast<const T *>(&raw);
#pragma unroll
                    for (int i = 0; i < VEC; ++i) e[i] = to_f<T>(tv[i]);
                } else {
#pragma unroll
                    for (int i = 0; i < VEC; ++i) {
                        const int64_t off = base + p0 + i;
                        e[i] = (c < n_chunks && off < numel) ? to_f<T>(in[off]) : -INFINITY;
                    }
                }
                // mask positions at or past k_len (and the buffer end, handled above)
#pragma unroll
                for (int i = 0; i < VEC; ++i)
                    if (p0 + i >= k_len) e[i] = -INFINITY;
                float prev = __shfl_up_sync(0xffffffffu, e[VEC - 1], 1);
                if (lane == 0) prev = carry;
                carry = __shfl_sync(0xffffffffu, e[VEC - 1], 31);
                if (c < n_chunks) {
#pragma unroll
                    for (int o = 0; o < OPV; ++o) {
                        const int64_t j = c * OPV + o;
                        if (j < j_end) {
                            // window positions 4j-1 .. 4j+3 -> e[4o-1 .. 4o+3]
                            float mx = (o == 0) ? (j == 0 ? -INFINITY : prev) : e[4 * o - 1];
                            mx = fmaxf(mx, e[4 * o + 0]);
                            mx = fmaxf(mx, e[4 * o + 1]);
                            mx = fmaxf(mx, e[4 * o + 2]);
                            mx = fmaxf(mx, e[4 * o + 3]);
                            finish(j, mx, true);  // j < j_end: the window is non-empty
                        }
                    }
                }
            }
            j_done = j_end;
        }
        // scalar path (general layouts) and the empty-window tail
        for (int64_t j = j_done + lane; j < NB; j += 32) {
            const int64_t ws = j * sp - 1;
            float mx = -INFINITY;
            for (int64_t ki = 0; ki < ksize; ++ki) {
                const int64_t kp = ws + ki;
                if (kp < 0 || kp >= k_len) continue;
                const int64_t off = base + kp;
                if (off < 0 || off >= numel) continue;
                mx = fmaxf(mx, to_f<T>(in[off]));
            }
            const int64_t wlo = ws > 0 ? ws : 0;
            const int64_t whi = ws + ksize < k_len ? ws + ksize : k_len;
            finish(j, mx, whi > wlo);
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
    const int64_t want = (rows + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)unum::sm_count() * 32;
    const int grid = (int)(want < cap ? want : cap);
    cudaStream_t s = (cudaStream_t)stream;
    const int vb = dtype == UNUM_DTYPE_F32 ? 4 : 8;  // elements per 16 bytes
    const bool vec_ok = unum::aligned16(input) && (fs % vb == 0);
    switch (dtype) {
        case UNUM_DTYPE_F32:
            max_pool_kernel<float><<<grid, kWarps * 32, 0, s>>>(
                (const float *)input, input_numel, H, T, fs, cu_seqlens_q, cu_seqlens_k, cache_lens,
                n_seq, NB, sp, block_size, init_blocks, local_blocks, vec_ok, (float *)out);
            break;
        case UNUM_DTYPE_BF16:
            max_pool_kernel<__nv_bfloat16><<<grid, kWarps * 32, 0, s>>>(
                (const __nv_bfloat16 *)input, input_numel, H, T, fs, cu_seqlens_q, cu_seqlens_k,
                cache_lens, n_seq, NB, sp, block_size, init_blocks, local_blocks, vec_ok,
                (__nv_bfloat16 *)out);
            break;
        case UNUM_DTYPE_F16:
            max_pool_kernel<__half><<<grid, kWarps * 32, 0, s>>>(
                (const __half *)input, input_numel, H, T, fs, cu_seqlens_q, cu_seqlens_k,
                cache_lens, n_seq, NB, sp, block_size, init_blocks, local_blocks, vec_ok,
                (__half *)out);
            break;
        default:
            unum::set_error("unsupported dtype %d", dtype);
            return UNUM_ERR_UNSUPPORTED;
    }
    return unum::check_launch("max_pool_kernel");
}
