// compress_keys: the producer of stage 1's compressed keys.
//
// InfLLM-v2 stage 1 consumes k_cmp, one compressed key per `stride` tokens of a
// sequence's keys: the mean over a window of `kernel` tokens (32 tokens at stride
// 16, so compressed key j covers tokens [16j, 16j+32) and a sequence of L tokens
// has (L-32)/16+1 of them, 0 when L < 32) — the layout the reference's stage-1
// kernel assumes (src/unum_ops/infllm_v2/infllmv2_attn_stage1_triton_v2.py:70,
// the 16-token compression stride of its causal rule).  The reference builds
// k_cmp outside the repository; this kernel is the B200 producer for it.
//
// Arithmetic: the window's bf16 keys are summed in fp32 in token order, the sum
// is scaled by 1/kernel and rounded to bf16 (round to nearest even).
//
// B200 design: HBM-bound (each token row read once from HBM; the overlapping
// window re-reads hit L2).  One warp per (sequence, compressed key, kv head):
// lane l owns dims 4l..4l+3, so every load instruction reads one 256-byte head
// row; the 32 row loads of a window are independent and in flight together.
#include <cuda_bf16.h>

#include "common.cuh"

namespace {

constexpr int kWarps = 8;

template <int kKernel>  // > 0: the window length at compile time (loads all in flight); 0: runtime
__global__ void __launch_bounds__(kWarps * 32)
compress_keys_kernel(const __nv_bfloat16 *__restrict__ k, int64_t k_st, int64_t k_sh, int32_t Hk,
                     const int32_t *__restrict__ cu_in, const int32_t *__restrict__ cu_out,
                     int32_t n_seq, int32_t kernel, int32_t stride, float inv_kernel,
                     __nv_bfloat16 *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t units = (int64_t)__ldg(cu_out + n_seq) * Hk;  // (compressed key, head) pairs
    for (int64_t u = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); u < units;
         u += (int64_t)gridDim.x * kWarps) {
        const int64_t jg = u / Hk;  // global compressed-key row
        const int32_t h = (int32_t)(u - jg * Hk);
        int32_t lo = 0, hi = n_seq;  // largest b with cu_out[b] <= jg
        while (hi - lo > 1) {
            const int32_t mid = (lo + hi) >> 1;
            if (__ldg(cu_out + mid) <= jg) lo = mid; else hi = mid;
        }
        const int64_t j = jg - __ldg(cu_out + lo);
        const __nv_bfloat16 *src = k + ((int64_t)__ldg(cu_in + lo) + j * stride) * k_st + (int64_t)h * k_sh;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int32_t kn = kKernel > 0 ? kKernel : kernel;
#pragma unroll(kKernel > 0 ? kKernel : 1)
        for (int32_t t = 0; t < kn; ++t) {  // token order, as the definition states
            const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(src + (int64_t)t * k_st) + lane);
            const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162 *>(&raw.x);
            const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162 *>(&raw.y);
            acc[0] += __low2float(a);
            acc[1] += __high2float(a);
            acc[2] += __low2float(b);
            acc[3] += __high2float(b);
        }
        __nv_bfloat162 o0 = __floats2bfloat162_rn(acc[0] * inv_kernel, acc[1] * inv_kernel);
        __nv_bfloat162 o1 = __floats2bfloat162_rn(acc[2] * inv_kernel, acc[3] * inv_kernel);
        uint2 w;
        w.x = *reinterpret_cast<uint32_t *>(&o0);
        w.y = *reinterpret_cast<uint32_t *>(&o1);
        reinterpret_cast<uint2 *>(out + (jg * Hk + h) * 128)[lane] = w;
    }
}

}  // namespace

extern "C" int unum_compress_keys(const void *k, int64_t T, int64_t Hk, int64_t D, int64_t k_st,
                                  int64_t k_sh, const int32_t *cu_seqlens, const int32_t *cu_out,
                                  int64_t n_seq, int64_t n_out, int64_t kernel, int64_t stride,
                                  void *out, void *stream) {
    unum::clear_error();
    UNUM_CHECK_ARG(T >= 0 && Hk > 0 && n_seq >= 0 && n_out >= 0, "bad sizes");
    if (D != 128) {
        unum::set_error("head_dim %lld not supported (only 128)", (long long)D);
        return UNUM_ERR_UNSUPPORTED;
    }
    UNUM_CHECK_ARG(kernel > 0 && stride > 0 && kernel <= (int64_t)1 << 20, "bad kernel / stride");
    if (n_out == 0 || n_seq == 0) return UNUM_OK;
    UNUM_CHECK_ARG(k && cu_seqlens && cu_out && out, "null pointer argument");
    UNUM_CHECK_ARG(unum::aligned16(k) && unum::aligned16(out), "k and out must be 16-byte aligned");
    UNUM_CHECK_ARG(k_st % 4 == 0 && k_sh % 4 == 0, "k strides must be multiples of 4 elements");
    const int64_t units = n_out * Hk;
    const int64_t want = (units + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)unum::sm_count() * 16;
    const int grid = (int)(want < cap ? want : cap);
    auto kern = kernel == 32 ? compress_keys_kernel<32> : compress_keys_kernel<0>;
    kern<<<grid, kWarps * 32, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)k, k_st, k_sh, (int32_t)Hk, cu_seqlens, cu_out, (int32_t)n_seq,
        (int32_t)kernel, (int32_t)stride, 1.0f / (float)kernel, (__nv_bfloat16 *)out);
    return unum::check_launch("compress_keys_kernel");
}
