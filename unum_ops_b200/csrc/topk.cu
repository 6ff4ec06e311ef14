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
// B200 design: one warp per row at a time; each warp owns a run of
// consecutive rows.  The row is loaded once (16-byte vectors when aligned),
// turned into order-preserving keys — 16-bit for bf16/fp16 scores, 32-bit for
// fp32, excluded entries = key 0 — and staged in shared memory.  The same pass
// compacts the keys at or above the previous row's threshold minus a margin
// into a small candidate buffer (neighbouring rows of pooled scores are nearly
// identical); the exact selection — a radix select with 8-bit digits (2 passes
// for 16-bit keys, 4 for fp32), run-length aggregated shared-memory histogram
// atomics and warp scans — then runs on the candidates only, or on the whole
// staged row when the bound missed.  The emit sweep walks keys in index order
// with warp scans, so winners come out sorted and only the lowest-index ties
// are taken.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace {

constexpr int kWarps = 4;
constexpr int kMaxNB = 4096;
constexpr int kMaxK = 1024;
constexpr int kCandCap = 640;  // candidate buffer per warp (a multiple of 32)
constexpr int kShrink = 4;     // 16-bit path: narrow the margin once more than 1/kShrink of the slots fill
constexpr int kMinBlocks16 = 7;  // resident blocks per SM asked of the 16-bit instance

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }

// Order-preserving keys: larger score -> larger key; -inf and NaN -> 0.
template <typename T> struct KeyOf;
template <> struct KeyOf<float> {
    using K = uint32_t;
    static constexpr int kPasses = 4;
    __device__ static K key(float f) {
        if (f != f || f == -INFINITY) return 0u;
        const uint32_t u = __float_as_uint(f);
        return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    }
};
template <> struct KeyOf<__nv_bfloat16> {
    using K = uint16_t;
    static constexpr int kPasses = 2;
    __device__ static K key(__nv_bfloat16 v) {
        const uint16_t u = __bfloat16_as_ushort(v);
        if ((u & 0x7F80u) == 0x7F80u && (u & 0x7Fu) != 0) return 0;  // NaN
        if (u == 0xFF80u) return 0;                                    // -inf
        return (u & 0x8000u) ? (uint16_t)~u : (uint16_t)(u | 0x8000u);
    }
};
template <> struct KeyOf<__half> {
    using K = uint16_t;
    static constexpr int kPasses = 2;
    __device__ static K key(__half v) {
        const uint16_t u = __half_as_ushort(v);
        if ((u & 0x7C00u) == 0x7C00u && (u & 0x3FFu) != 0) return 0;  // NaN
        if (u == 0xFC00u) return 0;                                     // -inf
        return (u & 0x8000u) ? (uint16_t)~u : (uint16_t)(u | 0x8000u);
    }
};

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t x, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += v;
    }
    return x;
}

// key of a 16-bit score that is neither NaN nor -inf, from its bits, and back
__device__ __forceinline__ uint32_t key16_bits(uint32_t u) {
    return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
}
__device__ __forceinline__ uint32_t key_bits16(uint32_t k) {
    return (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
}

// 8 consecutive keys from shared memory (i0 a multiple of 8) with 16-byte loads.
template <typename Key>
__device__ __forceinline__ void load8(const Key *keys, int32_t i0, uint32_t (&k)[8]) {
    if constexpr (sizeof(Key) == 2) {
        const uint4 w = *reinterpret_cast<const uint4 *>(keys + i0);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            k[2 * e] = ws[e] & 0xFFFFu;
            k[2 * e + 1] = ws[e] >> 16;
        }
    } else {
        const uint4 a = *reinterpret_cast<const uint4 *>(keys + i0);
        const uint4 b = *reinterpret_cast<const uint4 *>(keys + i0 + 4);
        k[0] = a.x; k[1] = a.y; k[2] = a.z; k[3] = a.w;
        k[4] = b.x; k[5] = b.y; k[6] = b.z; k[7] = b.w;
    }
}

// Candidate keys (kCandCap slots) or, on the 16-bit path, three bitmaps over block ids.
template <typename Key>
__host__ __device__ constexpr size_t cand_region_bytes(size_t nbp) {
    return kCandCap * sizeof(Key) > 12 * nbp / 32 ? kCandCap * sizeof(Key) : 12 * nbp / 32;
}

// Shared memory of one warp: histogram, staged keys (16-bit path: the row's raw
// bits), candidate keys or, on the 16-bit path, three bitmaps over block ids, and
// candidate ids.
template <typename Key>
__host__ __device__ constexpr size_t warp_smem_bytes(int64_t NB) {
    const size_t nbp = (size_t)((NB + 255) / 256 * 256);
    return 1024 + nbp * sizeof(Key) + cand_region_bytes<Key>(nbp) + kCandCap * 2;
}

// Histogram of the staged keys[0, n_pad) whose bits under pmask equal prefix, by
// the digit at `shift`: run-length aggregated atomics (neighbouring keys of a
// lane often share a digit).
template <typename Key>
__device__ __forceinline__ void hist_staged(const Key *keys, int32_t n_pad, uint32_t *hist, int lane,
                                            uint32_t pmask, uint32_t prefix, int shift) {
    for (int32_t base = 0; base < n_pad; base += 256) {
        const int32_t i0 = base + 8 * lane;
        uint32_t kk[8];
        load8(keys, i0, kk);
        uint32_t run_d = 256u, run_c = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t k = kk[e];
            const bool m = k != 0u && (k & pmask) == prefix;
            const uint32_t d = m ? ((k >> shift) & 255u) : 256u;
            if (d != run_d) {
                if (run_c) atomicAdd(&hist[run_d], run_c);
                run_d = d;
                run_c = 0;
            }
            run_c += m ? 1u : 0u;
        }
        if (run_c) atomicAdd(&hist[run_d], run_c);
    }
}

// Radix select of the K-th largest among a warp's keys (key 0 = not a
// candidate), 8-bit digits from the top; fill(pmask, prefix, shift) adds the
// keys matching the prefix so far to the histogram.  Returns the threshold key
// in `prefix` and in `remaining` how many keys equal to it are taken (lowest
// index first); take_all when there are at most K candidates.
template <typename Key, int PASSES, typename Fill>
__device__ __forceinline__ void radix_select_with(Fill fill, int32_t K, uint32_t *hist, int lane,
                                                  uint32_t &prefix, int32_t &remaining, bool &take_all) {
    constexpr int KB = 8 * (int)sizeof(Key);
    prefix = 0;
    uint32_t pmask = 0;
    remaining = K;
    take_all = false;
#pragma unroll 1
    for (int p = 0; p < PASSES; ++p) {
        const int shift = KB - 8 - 8 * p;
        reinterpret_cast<uint4 *>(hist)[2 * lane] = make_uint4(0u, 0u, 0u, 0u);
        reinterpret_cast<uint4 *>(hist)[2 * lane + 1] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
        fill(pmask, prefix, shift);
        __syncwarp();
        uint32_t c[8];  // lane owns bins 255-8*lane-i (descending): two 16-byte loads
        {
            const uint4 lo4 = reinterpret_cast<const uint4 *>(hist + 248 - 8 * lane)[0];
            const uint4 hi4 = reinterpret_cast<const uint4 *>(hist + 248 - 8 * lane)[1];
            c[0] = hi4.w; c[1] = hi4.z; c[2] = hi4.y; c[3] = hi4.x;
            c[4] = lo4.w; c[5] = lo4.z; c[6] = lo4.y; c[7] = lo4.x;
        }
        uint32_t s = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) s += c[i];
        const uint32_t incl = warp_incl_scan(s, lane);
        const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
        if (p == 0 && total <= (uint32_t)K) {
            take_all = true;
            __syncwarp();
            return;
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
        remaining -= (int32_t)above;
        prefix |= digit << shift;
        pmask |= 255u << shift;
        __syncwarp();
    }
}

template <typename Key, int PASSES>
__device__ __forceinline__ void radix_select(const Key *keys, int32_t n_pad, int32_t K, uint32_t *hist,
                                             int lane, uint32_t &prefix, int32_t &remaining,
                                             bool &take_all) {
    radix_select_with<Key, PASSES>(
        [&](uint32_t pmask, uint32_t pre, int shift) { hist_staged(keys, n_pad, hist, lane, pmask, pre, shift); },
        K, hist, lane, prefix, remaining, take_all);
}

// K-th largest over one row of 16-bit scores, from the candidates of the
// loading pass: the stored ids (slot j of lane l at l + 32*j, `mine` slots this
// lane; their bits in rowb) plus E keys equal to hi, which were only counted.
// One histogram pass over keys offset from t0: bins 1..254 hold single keys
// (hi - t0 <= 128 is one of them and receives E), bin 0 everything <= t0, bin 255
// everything >= t0 + 255.  When the K-th largest lands in bins 1..254 it is
// exact; otherwise the 8-bit radix select over the stored keys settles it (the
// keys == hi then lie on one side of the threshold: taken if it is below, so the
// radix looks for the (K-E)-th largest, ignored if above).  Outputs as
// radix_select_with over stored and equal keys together, where take_all covers
// the stored keys only, plus eq_mode for the keys == hi: 0 not taken, 1 they are
// the threshold's ties, 2 all taken.
template <typename Key, int PASSES>
__device__ __forceinline__ void select_row16(const uint16_t *rowb, const uint16_t *cidx, uint32_t mine,
                                             uint32_t t0, uint32_t hi, int32_t E, int32_t K, uint32_t *hist,
                                             int lane, uint32_t &prefix, int32_t &remaining, bool &take_all,
                                             int &eq_mode) {
    reinterpret_cast<uint4 *>(hist)[2 * lane] = make_uint4(0u, 0u, 0u, 0u);
    reinterpret_cast<uint4 *>(hist)[2 * lane + 1] = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();
    for (uint32_t j = 0; j < mine; ++j) {
        const uint32_t k = key16_bits(rowb[cidx[lane + 32 * j]]);
        const uint32_t d = k <= t0 ? 0u : (k - t0 < 255u ? k - t0 : 255u);
        atomicAdd(&hist[d], 1u);
    }
    if (lane == 0 && E > 0) atomicAdd(&hist[hi - t0], (uint32_t)E);
    __syncwarp();
    uint32_t c[8];  // lane owns bins 255-8*lane-i (descending): two 16-byte loads
    {
        const uint4 lo4 = reinterpret_cast<const uint4 *>(hist + 248 - 8 * lane)[0];
        const uint4 hi4 = reinterpret_cast<const uint4 *>(hist + 248 - 8 * lane)[1];
        c[0] = hi4.w; c[1] = hi4.z; c[2] = hi4.y; c[3] = hi4.x;
        c[4] = lo4.w; c[5] = lo4.z; c[6] = lo4.y; c[7] = lo4.x;
    }
    uint32_t sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum += c[i];
    const uint32_t incl = warp_incl_scan(sum, lane);
    const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
    __syncwarp();
    if (total <= (uint32_t)K) {
        prefix = 0;
        remaining = K;
        take_all = true;
        eq_mode = 2;
        return;
    }
    const uint32_t excl = incl - sum;
    const bool own = excl < (uint32_t)K && (uint32_t)K <= incl;
    const uint32_t owner = __ffs(__ballot_sync(0xffffffffu, own)) - 1;
    uint32_t digit = 0, above = 0;
    if (own) {
        uint32_t run = excl;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (run + c[i] >= (uint32_t)K) {
                digit = 255u - 8u * lane - i;
                above = run;
                break;
            }
            run += c[i];
        }
    }
    digit = __shfl_sync(0xffffffffu, digit, owner);
    above = __shfl_sync(0xffffffffu, above, owner);
    if (digit != 0u && digit != 255u) {
        prefix = t0 + digit;
        remaining = K - (int32_t)above;
        take_all = false;
        eq_mode = prefix > hi ? 0 : (prefix == hi ? 1 : 2);
        return;
    }
    eq_mode = digit == 255u ? 0 : 2;
    radix_select_with<Key, PASSES>(
        [&](uint32_t pmask, uint32_t pre, int shift) {
            for (uint32_t j = 0; j < mine; ++j) {
                const uint32_t k = key16_bits(rowb[cidx[lane + 32 * j]]);
                if ((k & pmask) == pre) atomicAdd(&hist[(k >> shift) & 255u], 1u);
            }
        },
        digit == 255u ? K : K - E, hist, lane, prefix, remaining, take_all);
}

// Write the selected entries of keys[0, n) in index order to orow[0, K), then
// -1 padding.  idx(i) maps a key slot to its block index.
template <typename Key, typename IdxFn>
__device__ __forceinline__ void emit_selected(const Key *keys, int32_t n, int32_t K, uint32_t prefix,
                                              int32_t remaining, bool take_all, IdxFn idx, int lane,
                                              int32_t *orow) {
    int32_t pos = 0, eq_seen = 0;
    for (int32_t base = 0; base < n && pos < K; base += 256) {
        const int32_t i0 = base + 8 * lane;
        uint32_t kk[8];
        load8(keys, i0, kk);
        uint32_t gt = 0, eq = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t k = kk[e];
            if (take_all) {
                gt |= (k != 0u ? 1u : 0u) << e;
            } else {
                gt |= (k > prefix ? 1u : 0u) << e;
                eq |= (k == prefix ? 1u : 0u) << e;
            }
        }
        const uint32_t ne = (uint32_t)__popc(eq);
        const uint32_t eincl = warp_incl_scan(ne, lane);
        int32_t eq_budget = remaining - eq_seen - (int32_t)(eincl - ne);
        uint32_t sel = gt;
        for (uint32_t m = eq; m != 0u && eq_budget > 0; m &= m - 1u, --eq_budget)
            sel |= m & (0u - m);  // lowest remaining tie, in index order
        const uint32_t nsel = (uint32_t)__popc(sel);
        const uint32_t si = warp_incl_scan(nsel, lane);
        int32_t slot = pos + (int32_t)(si - nsel);
        for (uint32_t m = sel; m != 0u && slot < K; m &= m - 1u, ++slot) orow[slot] = idx(i0 + __ffs(m) - 1);
        pos += (int32_t)__shfl_sync(0xffffffffu, si, 31);
        eq_seen += (int32_t)__shfl_sync(0xffffffffu, eincl, 31);
    }
    for (int32_t s2 = (pos < K ? pos : K) + lane; s2 < K; s2 += 32) orow[s2] = -1;
}

// threshold margin in key steps: 32 bf16/fp16 steps (bf16: 2^(32/128) = 19 % in value);
// the same relative width for 32-bit keys
template <typename Key> constexpr uint32_t kMargin = sizeof(Key) == 2 ? 32u : (32u << 16);
// key of the most negative finite score (bf16 0xFF7F, fp16 0xFBFF, fp32
// 0xFF7FFFFF): the candidate bound never goes below it, so -inf (and NaN) scores
// are never counted as candidates
template <typename T> constexpr uint32_t kMinFinite = 0x00800000u;
template <> constexpr uint32_t kMinFinite<__nv_bfloat16> = 0x0080u;
template <> constexpr uint32_t kMinFinite<__half> = 0x0400u;

constexpr int kLaneCand = kCandCap / 32;  // candidate slots of one lane (16-bit path)

// "x >= t" on two packed 16-bit scores: 0xFFFF in each half where true (NaN: false).
template <typename T> __device__ __forceinline__ uint32_t ge2(uint32_t x, uint32_t t2);
template <> __device__ __forceinline__ uint32_t ge2<__nv_bfloat16>(uint32_t x, uint32_t t2) {
    return __hge2_mask(*reinterpret_cast<const __nv_bfloat162 *>(&x), *reinterpret_cast<const __nv_bfloat162 *>(&t2));
}
template <> __device__ __forceinline__ uint32_t ge2<__half>(uint32_t x, uint32_t t2) {
    return __hge2_mask(*reinterpret_cast<const __half2 *>(&x), *reinterpret_cast<const __half2 *>(&t2));
}
// "x == t" likewise (bit-pattern equality: keys are not NaN, and +0/-0 have distinct keys)
template <typename T> __device__ __forceinline__ uint32_t eq2(uint32_t x, uint32_t t2) {
    return __vcmpeq2(x, t2);
}
// -inf bit pattern: fill for positions past the row end
template <typename T> constexpr uint32_t kNegInf16 = 0xFF80u;
template <> constexpr uint32_t kNegInf16<__half> = 0xFC00u;
template <typename T> __device__ __forceinline__ uint32_t bits16(T v) {
    return (uint32_t)(*reinterpret_cast<const uint16_t *>(&v));
}

// 8 scores from i0 as packed bits, -inf past the row end (unaligned rows, row tail);
// kept out of line so the unrolled vector path stays small in the instruction cache.
template <typename T>
__device__ __noinline__ uint4 load8_bits_slow(const T *src, int32_t i0, int32_t NB) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint32_t lo = i0 + 2 * e < NB ? bits16(src[i0 + 2 * e]) : kNegInf16<T>;
        const uint32_t hv = i0 + 2 * e + 1 < NB ? bits16(src[i0 + 2 * e + 1]) : kNegInf16<T>;
        w[e] = lo | (hv << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Emit from bitmaps over block ids: sel = blocks taken outright, tie = blocks whose
// key equals the threshold, of which the `remaining` lowest ids are taken; a third
// bitmap eqw is ignored (eq_mode 0), replaces the ties (1) or is taken whole (2).
// Lane l sweeps a contiguous run of words, so ids come out ascending; then -1
// padding.
template <int kMaxW>  // bitmap words a lane sweeps at most: NBp / 32 / 32
__device__ __forceinline__ void emit_bitmap(const uint32_t *selw, const uint32_t *tiew, const uint32_t *eqw,
                                            int eq_mode, int32_t nw, int32_t K, int32_t remaining,
                                            int lane, int32_t *orow) {
    const int32_t wpl = (nw + 31) >> 5;
    const int32_t w0 = lane * wpl;
    uint32_t sw[kMaxW], tw[kMaxW];
    uint32_t tc = 0, sc = 0;
#pragma unroll
    for (int i = 0; i < kMaxW; ++i) {
        const bool in = i < wpl && w0 + i < nw;
        const uint32_t ew = in && eq_mode != 0 ? eqw[w0 + i] : 0u;
        sw[i] = (in ? selw[w0 + i] : 0u) | (eq_mode == 2 ? ew : 0u);
        tw[i] = eq_mode == 1 ? ew : (in ? tiew[w0 + i] : 0u);
        tc += (uint32_t)__popc(tw[i]);
        sc += (uint32_t)__popc(sw[i]);
    }
    // one scan for both counts (16 bits each: a row has at most 4096 blocks); ties are taken
    // in id order, so the lanes before this one take min(remaining, their ties) of them
    const uint32_t incl = warp_incl_scan((tc << 16) | sc, lane);
    const int32_t tie_excl = (int32_t)(incl >> 16) - (int32_t)tc;
    const int32_t sel_excl = (int32_t)(incl & 0xFFFFu) - (int32_t)sc;
    const int32_t rem = remaining > 0 ? remaining : 0;
    int32_t budget = rem - tie_excl;  // ties left for this lane, in id order
    int32_t slot = sel_excl + (tie_excl < rem ? tie_excl : rem);
#pragma unroll
    for (int i = 0; i < kMaxW; ++i)
        for (uint32_t m = tw[i]; m != 0u && budget > 0; m &= m - 1u, --budget) sw[i] |= m & (0u - m);
#pragma unroll
    for (int i = 0; i < kMaxW; ++i)
        for (uint32_t m = sw[i]; m != 0u && slot < K; m &= m - 1u, ++slot)
            orow[slot] = (w0 + i) * 32 + __ffs(m) - 1;
    const uint32_t tot = __shfl_sync(0xffffffffu, incl, 31);
    const int32_t tot_ties = (int32_t)(tot >> 16);
    const int32_t total = (int32_t)(tot & 0xFFFFu) + (tot_ties < rem ? tot_ties : rem);
    for (int32_t s2 = (total < K ? total : K) + lane; s2 < K; s2 += 32) orow[s2] = -1;
}

// 8 consecutive scores of a row as keys (vector loads when aligned).
template <typename T>
__device__ __forceinline__ void load8_keys(const T *src, int32_t i0, int32_t NB, bool vec_ok,
                                           uint32_t (&k)[8]) {
    constexpr int VT = 16 / (int)sizeof(T);
    if (vec_ok && i0 + 8 <= NB) {
#pragma unroll
        for (int h = 0; h < 8 / VT; ++h) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(src + i0 + h * VT));
            const T *tv = reinterpret_cast<const T *>(&raw);
#pragma unroll
            for (int e = 0; e < VT; ++e) k[h * VT + e] = KeyOf<T>::key(tv[e]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) k[e] = (i0 + e < NB) ? KeyOf<T>::key(src[i0 + e]) : 0u;
    }
}

// Buffers on other GPUs (peer-mapped into this device's address space) that also receive
// every row's ids, narrowed to int16: row r goes to p[i] + off + r*K for each i < n.
constexpr int kMaxPeers = 8;
struct Peers {
    int16_t *p[kMaxPeers];
    int32_t n;
    int64_t off;
};

// Score value whose key is k (inverse of KeyOf<T>::key for non-excluded keys).
template <typename T> __device__ __forceinline__ float key_value(uint32_t k);
template <> __device__ __forceinline__ float key_value<float>(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Each warp owns a contiguous run of rows.  Neighbouring rows of pooled block
// scores are nearly identical, so the previous row's threshold hi, lowered by an
// adaptive margin to t0, bounds this row's from below.
//   16-bit scores: the pass that loads the row compares packed pairs with t0 and
//   with hi; keys above t0 other than hi go to lane-private slots, keys equal to
//   hi only to a bitmap (rows whose threshold is shared by many entries, such as
//   the exact zeros of early causal tokens, store none of them).  Counting the
//   keys above hi (G) and equal to it (E) decides: G < K <= G+E means the
//   threshold is hi again and nothing is left to select; otherwise a histogram
//   over the stored keys finds it.  Winners and ties become bitmaps over block
//   ids that an in-order sweep turns into the sorted output.
//   fp32 scores: the loading pass compares floats with t0 and compacts the
//   candidates in index order; a radix select and an in-order emit follow.
// When the bound misses (no previous row, fewer than K entries above it, or
// more than the slots hold) the row is staged in shared memory as keys and the
// full radix select runs on it.  Results never depend on which path ran.
template <typename T, int kMaxW>  // kMaxW: 2 for rows of at most 2048 blocks, else 4
__global__ void __launch_bounds__(kWarps * 32, sizeof(T) == 2 ? kMinBlocks16 : 1)  // 16-bit: 7 blocks, <= 72 registers
topk_kernel(const T *__restrict__ scores, int64_t rows, int32_t NB, int64_t row_stride, int32_t K,
            bool vec_ok, int64_t rows_per_warp, int32_t *__restrict__ out, const __grid_constant__ Peers peers) {
    using Key = typename KeyOf<T>::K;
    constexpr int PASSES = KeyOf<T>::kPasses;
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int32_t NBp = (NB + 255) & ~255;  // padded to whole steps (8 keys x 32 lanes)
    uint8_t *wbase = smem + (size_t)warp * warp_smem_bytes<Key>(NB);
    uint32_t *hist = reinterpret_cast<uint32_t *>(wbase);
    Key *keys = reinterpret_cast<Key *>(wbase + 1024);
    Key *ckey = keys + NBp;
    uint16_t *cidx = reinterpret_cast<uint16_t *>(reinterpret_cast<uint8_t *>(ckey) +
                                                  cand_region_bytes<Key>((size_t)NBp));
    const int64_t gw = (int64_t)blockIdx.x * kWarps + warp;
    const int64_t r0 = gw * rows_per_warp;
    const int64_t r1 = r0 + rows_per_warp < rows ? r0 + rows_per_warp : rows;
    uint32_t tau_prev = 0;  // threshold key of the previous row (0: none)
    // margin below the previous threshold, in key steps (scaled for 32-bit keys); adapts to
    // the density of scores near the threshold: halved when the candidates overflowed the
    // buffer, doubled when they were fewer than K
    uint32_t margin = kMargin<Key>;
    constexpr uint32_t kMarginMin = sizeof(Key) == 2 ? 1u : (1u << 16);
    // 16-bit keys: at most 128 steps, so hi stays inside the exact bins of select_row16
    constexpr uint32_t kMarginMax = sizeof(Key) == 2 ? 128u : (1024u << 16);
    for (int64_t row = r0; row < r1; ++row) {
        const T *src = scores + row * row_stride;
        int32_t *orow = out + row * K;
        // the selection sets these warp-uniformly; tau_prev (from prefix) decides which path
        // the whole warp takes on the next row, and that path uses full-warp collectives
        uint32_t prefix = 0;
        int32_t remaining = K;
        bool take_all = true;
        bool done = false;
        if constexpr (sizeof(Key) == 2) {
            // a row whose threshold fell below the bound gets one more pass with a 4x wider margin
            for (int attempt = 0; attempt < 2 && tau_prev != 0u && !done; ++attempt) {
                // 16-bit scores.  hi = the previous row's threshold key, t0 = hi - margin.
                // One pass stages the row's bits in shared memory and compares packed
                // pairs with t0 and hi: ids of keys above t0 other than hi go to
                // lane-private slots (slot j of lane l at l + 32*j); keys == hi only set
                // bits in a bitmap over block ids, so a row with many ties at the
                // threshold (exact zeros of early causal tokens) stores none of them.
                const uint32_t hi = tau_prev;
                const uint32_t t0 = hi > kMinFinite<T> + margin ? hi - margin : kMinFinite<T>;
                const uint32_t tb = key_bits16(t0), hb = key_bits16(hi);
                const uint32_t t2 = tb | (tb << 16), h2 = hb | (hb << 16);
                const int32_t nw = NBp >> 5;
                uint32_t *eqw = reinterpret_cast<uint32_t *>(ckey);
                uint32_t *selw = eqw + nw;
                uint32_t *tiew = selw + nw;
                uint16_t *rowb = reinterpret_cast<uint16_t *>(keys);
                for (int32_t i = lane; i < 3 * nw; i += 32) eqw[i] = 0u;
                __syncwarp();
                uint32_t cnt = 0, neq = 0;
                constexpr int BATCH = 8;  // steps (256 scores each) whose loads are in flight together
                for (int32_t b0 = 0; b0 < NBp; b0 += 256 * BATCH) {
                    uint4 raw[BATCH];
#pragma unroll
                    for (int st = 0; st < BATCH; ++st) {
                        const int32_t i0 = b0 + st * 256 + 8 * lane;
                        if (vec_ok && i0 + 8 <= NB) raw[st] = __ldg(reinterpret_cast<const uint4 *>(src + i0));
                        else raw[st] = load8_bits_slow<T>(src, i0, NB);
                    }
#pragma unroll
                    for (int st = 0; st < BATCH; ++st) {
                        const int32_t i0 = b0 + st * 256 + 8 * lane;
                        if (b0 + st * 256 < NBp) *reinterpret_cast<uint4 *>(rowb + i0) = raw[st];
                        const uint32_t w[4] = {raw[st].x, raw[st].y, raw[st].z, raw[st].w};
                        const uint32_t a = __byte_perm(ge2<T>(w[0], t2), ge2<T>(w[1], t2), 0x6420);
                        const uint32_t b = __byte_perm(ge2<T>(w[2], t2), ge2<T>(w[3], t2), 0x6420);
                        if ((a | b) == 0u) continue;
                        // one 0xFF/0x00 byte per score -> 8-bit masks (the products sum disjoint bits)
                        const uint32_t ea = __byte_perm(eq2<T>(w[0], h2), eq2<T>(w[1], h2), 0x6420);
                        const uint32_t eb = __byte_perm(eq2<T>(w[2], h2), eq2<T>(w[3], h2), 0x6420);
                        const uint32_t eqm = (((ea & 0x08040201u) * 0x01010101u) >> 24) |
                                             (((eb & 0x80402010u) * 0x01010101u) >> 24);
                        uint32_t sel = ((((a & 0x08040201u) * 0x01010101u) >> 24) |
                                        (((b & 0x80402010u) * 0x01010101u) >> 24)) & ~eqm;
                        if (eqm) {
                            atomicOr(&eqw[i0 >> 5], eqm << (i0 & 31));
                            neq += (uint32_t)__popc(eqm);
                        }
                        for (; sel != 0u; sel &= sel - 1u, ++cnt)
                            if (cnt < (uint32_t)kLaneCand) cidx[lane + 32 * cnt] = (uint16_t)(i0 + __ffs(sel) - 1);
                    }
                }
                const int32_t n_st = (int32_t)__reduce_add_sync(0xffffffffu, cnt);  // stored
                const int32_t E = (int32_t)__reduce_add_sync(0xffffffffu, neq);     // == hi
                const bool ovf = __any_sync(0xffffffffu, cnt > (uint32_t)kLaneCand);
                const bool under = n_st + E < K;  // the threshold lies below t0
                if (ovf) margin = margin / 2 > kMarginMin ? margin / 2 : kMarginMin;
                else if (n_st > kCandCap / kShrink) margin = margin - margin / 4 > kMarginMin ? margin - margin / 4 : kMarginMin;
                else if (under && t0 > kMinFinite<T>) margin = margin * 2 < kMarginMax ? margin * 2 : kMarginMax;
                __syncwarp();
                if (!ovf && !under) {
                    const uint32_t mine = cnt;
                    int eq_mode;  // keys == hi: below the threshold (0), its ties (1) or all taken (2)
                    select_row16<Key, PASSES>(rowb, cidx, mine, t0, hi, E, K, hist, lane, prefix, remaining,
                                              take_all, eq_mode);
                    for (uint32_t j = 0; j < mine; ++j) {
                        const uint32_t id = cidx[lane + 32 * j];
                        const uint32_t k = key16_bits(rowb[id]);
                        if (take_all || k > prefix) atomicOr(&selw[id >> 5], 1u << (id & 31));
                        else if (k == prefix) atomicOr(&tiew[id >> 5], 1u << (id & 31));
                    }
                    __syncwarp();
                    emit_bitmap<kMaxW>(selw, tiew, eqw, eq_mode, nw, K, remaining, lane, orow);
                    done = true;
                }
                // overflow, or no finite bound left to lower: the staged radix select below
                if (!under || t0 <= kMinFinite<T>) break;
                margin = margin * 2 < kMarginMax ? margin * 2 : kMarginMax;  // x4 with the update above
            }
        } else if (tau_prev) {
            const uint32_t t0 = tau_prev > kMinFinite<T> + margin ? tau_prev - margin
                                                                    : kMinFinite<T>;
            const float tf = key_value<T>(t0);  // scores >= tf are candidates (NaN never is)
            int32_t n = 0;
            constexpr int VT = 16 / (int)sizeof(T);
            constexpr int BATCH = 8;  // steps (256 scores each) whose loads are in flight together
            for (int32_t b0 = 0; b0 < NBp; b0 += 256 * BATCH) {
                uint4 raw[BATCH][8 / VT];
#pragma unroll
                for (int st = 0; st < BATCH; ++st) {
                    const int32_t i0 = b0 + st * 256 + 8 * lane;
                    if (vec_ok && i0 + 8 <= NB) {
#pragma unroll
                        for (int h = 0; h < 8 / VT; ++h)
                            raw[st][h] = __ldg(reinterpret_cast<const uint4 *>(src + i0 + h * VT));
                    }
                }
#pragma unroll
                for (int st = 0; st < BATCH; ++st) {
                    const int32_t i0 = b0 + st * 256 + 8 * lane;
                    if (b0 + st * 256 >= NBp) break;
                    float x[8];
                    if (vec_ok && i0 + 8 <= NB) {
#pragma unroll
                        for (int h = 0; h < 8 / VT; ++h) {
                            const T *tv = reinterpret_cast<const T *>(&raw[st][h]);
#pragma unroll
                            for (int e = 0; e < VT; ++e) x[h * VT + e] = to_f<T>(tv[e]);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) x[e] = (i0 + e < NB) ? to_f<T>(src[i0 + e]) : -INFINITY;
                    }
                    uint32_t sel = 0;
#pragma unroll
                    for (int e = 0; e < 8; ++e) sel |= (x[e] >= tf ? 1u : 0u) << e;
                    if (__ballot_sync(0xffffffffu, sel != 0u) == 0u) continue;
                    const uint32_t ns = (uint32_t)__popc(sel);
                    const uint32_t si = warp_incl_scan(ns, lane);
                    int32_t slot = n + (int32_t)(si - ns);
                    for (uint32_t m = sel; m != 0u && slot < kCandCap; m &= m - 1u, ++slot) {
                        const int e = __ffs(m) - 1;  // only the set bits: 1-2 per lane typically
                        float xe = x[0];
#pragma unroll
                        for (int f = 1; f < 8; ++f) xe = (e == f) ? x[f] : xe;
                        ckey[slot] = (Key)KeyOf<T>::key(from_f<T>(xe));
                        cidx[slot] = (uint16_t)(i0 + e);
                    }
                    n += (int32_t)__shfl_sync(0xffffffffu, si, 31);
                }
            }
            __syncwarp();
            // the radix select pads the candidates to whole 256-key steps: at most kCand32 of them
            constexpr int32_t kCand32 = kCandCap / 256 * 256;
            if (n > kCand32) margin = margin / 2 > kMarginMin ? margin / 2 : kMarginMin;
            else if (n > kCand32 / 2) margin = margin - margin / 4 > kMarginMin ? margin - margin / 4 : kMarginMin;
            else if (n < K && t0 > kMinFinite<T>) margin = margin * 2 < kMarginMax ? margin * 2 : kMarginMax;
            if (n >= K && n <= kCand32) {
                const int32_t npad = (n + 255) & ~255;
                for (int32_t i = n + lane; i < npad; i += 32) ckey[i] = Key(0);
                __syncwarp();
                radix_select<Key, PASSES>(ckey, npad, K, hist, lane, prefix, remaining, take_all);
                emit_selected(ckey, npad, K, prefix, remaining, take_all,
                              [&](int32_t i) { return (int32_t)cidx[i]; }, lane, orow);
                done = true;
            }
        }
        if (!done) {
            for (int32_t base = 0; base < NBp; base += 256) {
                const int32_t i0 = base + 8 * lane;
                uint32_t kk[8];
                load8_keys<T>(src, i0, NB, vec_ok, kk);
                if constexpr (sizeof(Key) == 2) {
                    uint4 w;
                    w.x = kk[0] | (kk[1] << 16);
                    w.y = kk[2] | (kk[3] << 16);
                    w.z = kk[4] | (kk[5] << 16);
                    w.w = kk[6] | (kk[7] << 16);
                    *reinterpret_cast<uint4 *>(keys + i0) = w;
                } else {
                    *reinterpret_cast<uint4 *>(keys + i0) = make_uint4(kk[0], kk[1], kk[2], kk[3]);
                    *reinterpret_cast<uint4 *>(keys + i0 + 4) = make_uint4(kk[4], kk[5], kk[6], kk[7]);
                }
            }
            __syncwarp();
            radix_select<Key, PASSES>(keys, NBp, K, hist, lane, prefix, remaining, take_all);
            emit_selected(keys, NB, K, prefix, remaining, take_all, [](int32_t i) { return i; }, lane,
                          orow);
        }
        tau_prev = take_all ? 0u : prefix;
        __syncwarp();
        if (peers.n > 0) {
            // the row's ids (written by the lanes of this warp just above) as int16 pairs into
            // every peer's buffer: plain stores over NVLink, 2*K bytes per row per peer
            for (int32_t i = 2 * lane; i < K; i += 64) {
                const uint32_t pk = (uint32_t)(uint16_t)orow[i] | ((uint32_t)(uint16_t)orow[i + 1] << 16);
                const int64_t e = peers.off + row * K + i;
                for (int j = 0; j < peers.n; ++j) *reinterpret_cast<uint32_t *>(peers.p[j] + e) = pk;
            }
            __syncwarp();
        }
    }
}

template <typename T>
int launch_topk(const void *scores, int64_t rows, int64_t NB, int64_t row_stride, int64_t K,
                int32_t *out, cudaStream_t s, const Peers &peers) {
    using Key = typename KeyOf<T>::K;
    const size_t smem = (size_t)kWarps * warp_smem_bytes<Key>(NB);
    const int64_t NBp = (NB + 255) / 256 * 256;
    auto kern = NBp <= 2048 ? topk_kernel<T, 2> : topk_kernel<T, kMaxNB / 32 / 32>;
    UNUM_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // a few long runs of consecutive rows per warp, so most rows reuse a threshold
    const int64_t want = (rows + kWarps - 1) / kWarps;
    int per_sm = 0;  // one resident wave
    UNUM_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarps * 32, smem));
    const int64_t cap = (int64_t)unum::sm_count() * (per_sm > 0 ? per_sm : 1);
    const int grid = (int)(want < cap ? want : cap);
    const int64_t nwarps = (int64_t)grid * kWarps;
    const int64_t rows_per_warp = (rows + nwarps - 1) / nwarps;
    const bool vec_ok = unum::aligned16(scores) && ((row_stride * (int64_t)sizeof(T)) % 16 == 0);
    kern<<<grid, kWarps * 32, smem, s>>>((const T *)scores, rows, (int32_t)NB, row_stride, (int32_t)K,
                                         vec_ok, rows_per_warp, out, peers);
    return unum::check_launch("topk_kernel");
}

}  // namespace

namespace {
int topk_run(const void *scores, int dtype, int64_t rows, int64_t NB, int64_t row_stride, int64_t K,
             int32_t *out, void *stream, const Peers &peers) {
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
        case UNUM_DTYPE_F32: return launch_topk<float>(scores, rows, NB, row_stride, K, out, s, peers);
        case UNUM_DTYPE_BF16: return launch_topk<__nv_bfloat16>(scores, rows, NB, row_stride, K, out, s, peers);
        case UNUM_DTYPE_F16: return launch_topk<__half>(scores, rows, NB, row_stride, K, out, s, peers);
        default:
            unum::set_error("unsupported dtype %d", dtype);
            return UNUM_ERR_UNSUPPORTED;
    }
}
}  // namespace

extern "C" int unum_topk_blocks(const void *scores, int dtype, int64_t rows, int64_t NB,
                                int64_t row_stride, int64_t K, int32_t *out, void *stream) {
    unum::clear_error();
    Peers none{};
    return topk_run(scores, dtype, rows, NB, row_stride, K, out, stream, none);
}

extern "C" int unum_topk_blocks_to_peers(const void *scores, int dtype, int64_t rows, int64_t NB,
                                         int64_t row_stride, int64_t K, int32_t *out,
                                         void *const *peer_bufs, int32_t n_peers, int64_t peer_offset,
                                         void *stream) {
    unum::clear_error();
    UNUM_CHECK_ARG(n_peers >= 1 && n_peers <= kMaxPeers && peer_bufs != nullptr,
                   "1 to %d peer buffers needed", kMaxPeers);
    UNUM_CHECK_ARG(NB >= 1 && NB <= 32768, "ids travel as int16: 1 <= NB <= 32768 (got %lld)", (long long)NB);
    UNUM_CHECK_ARG(K % 2 == 0 && peer_offset >= 0 && peer_offset % 2 == 0,
                   "K and peer_offset must be even (ids travel in 4-byte pairs)");
    Peers peers{};
    peers.n = n_peers;
    peers.off = peer_offset;
    for (int i = 0; i < n_peers; ++i) {
        UNUM_CHECK_ARG(peer_bufs[i] != nullptr && ((uintptr_t)peer_bufs[i] & 3) == 0,
                       "peer buffer %d null or not 4-byte aligned", i);
        peers.p[i] = (int16_t *)peer_bufs[i];
    }
    return topk_run(scores, dtype, rows, NB, row_stride, K, out, stream, peers);
}
