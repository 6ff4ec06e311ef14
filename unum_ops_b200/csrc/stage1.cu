// infllmv2_attn_stage1 on B200: tcgen05 (TMEM) tensor-core kernel.
//
// Semantics follow the public Triton kernel of the reference
// (src/unum_ops/infllm_v2/infllmv2_attn_stage1_triton_v2.py:19-150, wrapper
// :153-228): for kv head g and token t,
//     out[g,t,j] = sum_{h in group g} softmax_j(q[t,h] . k[k_start+j,g] * scale)
// over the keys visible to t (causal rule :69-72), 0 elsewhere and 0 for an
// empty softmax (the reference's NaN -> 0, :227).
//
// Work decomposition.  A tile is QT = 256/G consecutive tokens of one sequence
// and one kv head: its 256 (token, head) rows of Q (64 KB bf16, loaded once by
// TMA) meet the sequence's compressed keys in 128-key tiles.  Two passes over
// the key tiles:
//   pass 1  S = Q K^T        (2 x UMMA 128x128x128, rows = (token, head)):
//           each epilogue thread owns one row and keeps its running max and
//           sum of exp2 — the per-head softmax statistics;
//   pass 2  S^T = K Q^T      (UMMA 128x256x128, rows = keys): each epilogue
//           thread owns one key and sums exp2(s*c - b[row]) over the G heads
//           of every token inside its own registers, so the head-group
//           reduction needs no shuffles and the per-head probabilities never
//           leave the SM.  Results go straight to HBM as bf16.
// The same Q/K shared-memory tiles serve both passes (operand roles swap).
//
// Warp roles (576 threads, one CTA per SM, persistent over tiles):
//   warps 0-15 epilogue (TMEM -> registers -> softmax math -> global), four
//              per scheduler so TMEM-load and MUFU latencies overlap
//   warp 16    TMA producer (Q tile, 4-stage ring of K tiles)
//   warp 17    TMEM allocator + single-thread UMMA issuer
// The epilogue issues packed f32x2 FMA/ADD (half the instructions of scalar
// code) and takes its exponentials on the MUFU pipe (ex2.approx).
// TMEM holds two 256-column accumulator buffers so the tensor core fills one
// while the epilogue drains the other.
//
// Every wait on an mbarrier is bounded (about one second of globaltimer);
// on expiry the kernel records a nonzero status word in the workspace, stops
// issuing TMA/UMMA work, runs its remaining loops without waiting, frees TMEM
// and returns, so the context stays usable and the host sees the status.
#include <cuda.h>
#include <cstdlib>
#include <cstring>

#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gbt_row.cuh"
#include "sm100.cuh"

namespace {

using namespace unum::sm100;

constexpr int kD = 128;            // head dim
constexpr int kRows = 256;         // (token, head) rows per tile
constexpr int kBN = 128;           // keys per key tile
constexpr int kStages = 4;         // K ring depth
constexpr int kEpiWarps = 16;      // 4 warpgroups, 64 accumulator columns each
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;
constexpr int kFillWarp = 18;       // writes what lies past each item's computed key tiles
constexpr int kThreads = (kEpiWarps + 3) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr int kEpiBarrier = 1;     // named barrier id for the 256 epilogue threads

constexpr uint32_t kQPanel = kRows * 128;          // one 64-column panel of Q: 32 KB
constexpr uint32_t kQBytes = 2 * kQPanel;          // 64 KB
constexpr uint32_t kKPanel = kBN * 128;            // 16 KB
constexpr uint32_t kKStage = 2 * kKPanel;          // 32 KB
constexpr uint32_t kOffK = kQBytes;
constexpr uint32_t kOffStats = kOffK + kStages * kKStage;
constexpr uint32_t kOffPart = kOffStats + kRows * 4;      // per-half (max, sum) of each row
constexpr uint32_t kOffLim = kOffPart + 2 * kRows * 8;
constexpr uint32_t kOffBar = kOffLim + kRows * 4;
constexpr uint32_t kNumBars = 2 + 2 * kStages + 4;
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;
constexpr uint32_t kOffStage = (kOffMisc + 64 + 1023) & ~1023u;  // pass-2 output staging (TMA needs 128-B alignment)
constexpr uint32_t kStageWg = 1024;                        // one [NQ=4 x 128] bf16 tile (G >= 16)
constexpr uint32_t kStageBytes = 4 * 2 * kStageWg;         // 4 warpgroups x 2 buffers
constexpr uint32_t kSmemBytes = kOffStage + kStageBytes + 1024;  // + slack for 1024-byte alignment
static_assert(kOffStage % 128 == 0 && kStageWg % 128 == 0, "TMA store sources must be 128-byte aligned");
static_assert(kSmemBytes <= 232448, "exceeds the 227 KB of shared memory a CTA may use");

constexpr uint32_t kIdescP1 = idesc_bf16_f32(128, 128);
constexpr uint32_t kIdescP2 = idesc_bf16_f32(128, 256);

constexpr float kLog2e = 1.4426950408889634f;
constexpr uint64_t kWaitNs = 1000000000ull;  // bounded wait: 1 s

// workspace layout (int32 words): [0] status, [1] decode work counter, [2..3] reserved,
// [4..4+n_seq] tile prefix
constexpr int kWsTiles = 4;

struct Params {
    const int32_t *cu_q;
    // compressed keys as plain memory (strides in elements), for the decode kernel's
    // keys beyond tensor-memory capacity
    const __nv_bfloat16 *k;
    int64_t k_st, k_sh;
    const int32_t *cu_k;
    int32_t *ws;
    __nv_bfloat16 *out;
    int64_t T;
    int64_t out_stride;
    int32_t n_seq;
    int32_t Hk;
    int32_t causal;
    float c;  // softmax_scale * log2(e)
    // optional fused max-pooling of the scores into 64-token blocks (G >= 16):
    // pooled[g][t][j] = max_pooling_1d_varlen(scores, max_seqlen_q = 16*W, cache 0)
    __nv_bfloat16 *pooled;  // [Hk, T, NB] or null
    int32_t NB, init_blocks, local_blocks;
    // token window: only tiles whose tokens intersect [t_begin, t_end) are computed
    int64_t t_begin, t_end;
    // nonzero: every bounded wait reports expiry at once (status 30) before any
    // TMA or UMMA work is issued, so the drain path can be tested without a fault
    int32_t force_expiry;
    // decode kernel in CTA pairs: items 0 .. joint_items-1 are shared by a pair, later ones
    // go to one CTA of a pair alone
    int64_t joint_items;
};

struct Item {
    int32_t g;
    int32_t nq;        // valid tokens in this tile
    int32_t nkt;       // key tiles to compute
    int32_t local0;    // position of the tile's first token inside its sequence
    int32_t q_len, k_len;
    int64_t t0, k_start;
};

// Visible compressed keys of a token (C integer division, like Triton's //).
__device__ __forceinline__ int32_t visible(int32_t lq, int32_t q_len, int32_t k_len, int causal) {
    if (k_len <= 0) return 0;
    if (!causal) return k_len;
    int32_t off = (lq - 15) / 16 + k_len - (q_len - 16 + 1) / 16;
    return off < 0 ? 0 : (off > k_len ? k_len : off);
}

__device__ __forceinline__ uint64_t exp2_mufu2(uint64_t x2) {
    float lo, hi;
    f2_unpack(x2, lo, hi);
    return f2_pack(ex2(lo), ex2(hi));
}

template <int QT>
__device__ __forceinline__ Item decode(int64_t w, const Params &p, const int32_t *cu_tiles,
                                       int32_t n_tiles) {
    Item it;
    it.g = (int32_t)(w % p.Hk);
    const int32_t tile = n_tiles - 1 - (int32_t)(w / p.Hk);  // last tiles (longest rows) first
    int32_t lo = 0, hi = p.n_seq;  // largest b with cu_tiles[b] <= tile
    while (hi - lo > 1) {
        const int32_t mid = (lo + hi) >> 1;
        if (cu_tiles[mid] <= tile) lo = mid; else hi = mid;
    }
    const int32_t b = lo;
    const int32_t chunk = tile - cu_tiles[b];
    const int32_t qs = __ldg(p.cu_q + b);
    it.q_len = __ldg(p.cu_q + b + 1) - qs;
    it.local0 = chunk * QT;
    it.t0 = (int64_t)qs + it.local0;
    const int32_t rest = it.q_len - it.local0;
    it.nq = rest < QT ? rest : QT;
    it.k_start = __ldg(p.cu_k + b);
    it.k_len = __ldg(p.cu_k + b + 1) - (int32_t)it.k_start;
    const int32_t lim = visible(it.local0 + it.nq - 1, it.q_len, it.k_len, p.causal);
    it.nkt = (lim + kBN - 1) / kBN;
    return it;
}

struct Sync {
    uint32_t q_full, q_empty, k_full, k_empty, s_full, s_empty;  // base addresses
    volatile int *abort;
    int32_t *status;
};

// Bounded wait: false once this CTA has given up (then callers stop issuing work).
// kCluster: the barrier is arrived on by another CTA of the cluster, whose writes before
// its arrive must be visible here (acquire at cluster scope).
template <bool kCluster = false>
__device__ __forceinline__ bool try_wait_scoped(uint32_t bar, uint32_t parity) {
    return kCluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
}

template <bool kCluster = false>
__device__ __forceinline__ bool wait_bar(const Sync &s, uint32_t bar, uint32_t parity, int code) {
    if (*s.abort) return false;
    if (try_wait_scoped<kCluster>(bar, parity)) return true;
    const uint64_t t_start = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (try_wait_scoped<kCluster>(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*s.abort) return false;
            if (globaltimer_ns() - t_start > kWaitNs) {
                *s.abort = 1;
                atomicCAS(s.status, 0, code);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- epilogue pieces
// Pass 1 on N (32 or 64) columns of row r: fold them into the running (max m, sum l).
template <int N>
__device__ __forceinline__ void p1_chunk(float (&v)[N], int32_t colbase, int32_t lim_r, float c,
                                         uint64_t c2, float &m, float &l) {
    if (colbase + N > lim_r) {
#pragma unroll
        for (int i = 0; i < N; ++i)
            if (colbase + i >= lim_r) v[i] = -INFINITY;
    }
    float mx[3] = {v[0], v[1], v[2]};
#pragma unroll
    for (int i = 3; i + 1 < N - 1; i += 2) mx[(i >> 1) % 3] = fmax3(mx[(i >> 1) % 3], v[i], v[i + 1]);
    const float mt = fmax3(fmax3(mx[0], mx[1], mx[2]), v[N - 1], m);  // new running max
    if (mt == -INFINITY) return;
    const uint64_t nmc = f2_pack(-mt * c, -mt * c);
    uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#define UNUM_P1(P) if ((P) < N / 2) acc[(P) & 3] = f2_add(acc[(P) & 3], exp2_mufu2(f2_fma(f2_pack(v[2 * (P)], v[2 * (P) + 1]), c2, nmc)));
#define UNUM_P1x4(P) UNUM_P1(P) UNUM_P1(P + 1) UNUM_P1(P + 2) UNUM_P1(P + 3)
    UNUM_P1x4(0) UNUM_P1x4(4) UNUM_P1x4(8) UNUM_P1x4(12)
    UNUM_P1x4(16) UNUM_P1x4(20) UNUM_P1x4(24) UNUM_P1x4(28)
#undef UNUM_P1x4
#undef UNUM_P1
    const uint64_t a2 = f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
    float alo, ahi;
    f2_unpack(a2, alo, ahi);
    if (mt != m) l = (m == -INFINITY ? 0.f : l * ex2((m - mt) * c));  // rescale only when the max moved
    l += alo + ahi;
    m = mt;
}

// Pass 2 on accumulator columns H*32..H*32+31 of this warpgroup (key = TMEM lane):
// add exp2(s*c - b) into the per-token head sums.
template <int G, int H>
__device__ __forceinline__ void p2_chunk(const float (&v)[32], uint64_t (&acc)[64 / G][2],
                                         const ulonglong2 *st4, uint64_t c2) {
#define UNUM_P2(P, SV)                                                                              \
    {                                                                                               \
        const uint64_t x2 = f2_fma(f2_pack(v[2 * (P)], v[2 * (P) + 1]), c2, SV);                    \
        const uint64_t e2 = exp2_mufu2(x2);                         \
        acc[(H * 32 + 2 * (P)) / G][(P) & 1] = f2_add(acc[(H * 32 + 2 * (P)) / G][(P) & 1], e2);                                         \
    }
#define UNUM_P2x2(P)                                                                                \
    {                                                                                               \
        const ulonglong2 sv = st4[H * 8 + ((P) >> 1)]; /* two pairs of -b per shared load */        \
        UNUM_P2(P, sv.x) UNUM_P2(P + 1, sv.y)                                                       \
    }
    UNUM_P2x2(0) UNUM_P2x2(2) UNUM_P2x2(4) UNUM_P2x2(6) UNUM_P2x2(8) UNUM_P2x2(10) UNUM_P2x2(12) UNUM_P2x2(14)
#undef UNUM_P2x2
#undef UNUM_P2
}

// Everything of an item past its computed key tiles: zero scores from column
// nkt*128 on, and the pooled blocks whose windows hold only those keys (zeros
// inside k_len, an empty window -inf past it, +inf on init/local blocks).  These
// regions are disjoint from every store of the epilogue warps, so this warp runs
// on its own, without barriers.
template <int QT>
__device__ __noinline__ void fill_tails(const Params &p, const int32_t *cu_tiles, int32_t n_tiles,
                                      int64_t n_items, int lane) {
    const bool vec_pool = p.pooled != nullptr && (p.NB & 7) == 0 &&
                          (reinterpret_cast<uintptr_t>(p.pooled) & 15) == 0;
    for (int64_t w = blockIdx.x; w < n_items; w += gridDim.x) {
        const Item it = decode<QT>(w, p, cu_tiles, n_tiles);
        if (it.t0 >= p.t_end || it.t0 + it.nq <= p.t_begin) continue;
        const int32_t c0 = it.nkt * kBN;
        const int32_t n16 = (int32_t)((p.out_stride - c0) >> 3);  // 16-byte chunks a row
        const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
        for (int32_t tq = 0; p.out != nullptr && tq < it.nq && n16 > 0; ++tq) {
            uint4 *dst = reinterpret_cast<uint4 *>(
                p.out + ((int64_t)it.g * p.T + it.t0 + tq) * p.out_stride + c0);
            for (int32_t e = lane; e < n16; e += 32) __stcs(dst + e, z4);
        }
        if (p.pooled == nullptr) continue;
        const int32_t jstart = it.nkt > 0 ? it.nkt * 32 + 1 : 0;
        const int32_t jhas = (it.k_len + 4) / 4;  // blocks jg < jhas have 4*jg-1 < k_len
        for (int32_t tq = 0; tq < it.nq && jstart < p.NB; ++tq) {
            const int32_t off_bq = (it.local0 + tq) / 64;
            __nv_bfloat16 *prow = p.pooled + ((int64_t)it.g * p.T + it.t0 + tq) * p.NB;
            auto value = [&](int32_t jg) -> uint16_t {
                const bool minf = jg < p.init_blocks || (off_bq >= jg && off_bq <= jg + p.local_blocks);
                return minf ? 0x7F80u : (jg < jhas ? 0x0000u : 0xFF80u);
            };
            int32_t jv = vec_pool ? ((jstart + 7) & ~7) : p.NB;  // first 8-aligned block
            if (jv > p.NB) jv = p.NB;
            for (int32_t jg = jstart + lane; jg < jv; jg += 32)
                reinterpret_cast<uint16_t *>(prow)[jg] = value(jg);
            for (int32_t j0 = jv + 8 * lane; j0 < p.NB; j0 += 256) {
                const bool no_mask = j0 >= p.init_blocks &&
                                     (p.local_blocks < 0 || off_bq < j0 || off_bq - p.local_blocks > j0 + 7);
                uint4 v;
                if (no_mask && j0 + 7 < jhas) {
                    v = z4;
                } else if (no_mask && j0 >= jhas) {
                    v = make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
                } else {
                    uint32_t h[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        h[i] = (uint32_t)value(j0 + 2 * i) | ((uint32_t)value(j0 + 2 * i + 1) << 16);
                    v = make_uint4(h[0], h[1], h[2], h[3]);
                }
                *reinterpret_cast<uint4 *>(prow + j0) = v;
            }
        }
    }
}

template <int G>
__global__ void __launch_bounds__(kThreads, 1)  // 19 warps, 5 on some schedulers: at most 96 registers a thread
stage1_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmO, const __grid_constant__ Params p) {
    constexpr int QT = kRows / G;  // tokens per tile
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t *sgen = smem_raw + (sbase - raw);

    float *stats = reinterpret_cast<float *>(sgen + kOffStats);
    int32_t *lim_s = reinterpret_cast<int32_t *>(sgen + kOffLim);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sgen + kOffMisc);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sgen + kOffMisc + 16);

    Sync sy;
    sy.q_full = sbase + kOffBar;
    sy.q_empty = sy.q_full + 8;
    sy.k_full = sy.q_full + 16;
    sy.k_empty = sy.k_full + 8 * kStages;
    sy.s_full = sy.k_empty + 8 * kStages;
    sy.s_empty = sy.s_full + 16;
    sy.abort = abort_flag;
    sy.status = p.ws;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(sy.q_full, 1);
        mbar_init(sy.q_empty, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(sy.k_full + 8 * s, 1);
            mbar_init(sy.k_empty + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(sy.s_full + 8 * b, 1);
            mbar_init(sy.s_empty + 8 * b, kEpiWarps);
        }
        *abort_flag = 0;
        if (p.force_expiry) {
            *abort_flag = 1;
            atomicCAS(p.ws, 0, 30);
        }
        fence_barrier_init();
    }
    if (warp == kProducerWarp && lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int32_t *cu_tiles = p.ws + kWsTiles;
    const int32_t n_tiles = cu_tiles[p.n_seq];
    const int64_t n_items = (int64_t)n_tiles * p.Hk;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            uint32_t kc = 0, qn = 0;
            for (int64_t w = blockIdx.x; w < n_items; w += gridDim.x) {
                const Item it = decode<QT>(w, p, cu_tiles, n_tiles);
                if (it.nkt == 0 || it.t0 >= p.t_end || it.t0 + it.nq <= p.t_begin) continue;
                if (wait_bar(sy, sy.q_empty, (qn & 1) ^ 1, 1)) {
                    mbar_arrive_expect_tx(sy.q_full, kQBytes);
                    tma_load_3d(sbase, &tmQ, 0, it.g * G, (int32_t)it.t0, sy.q_full);
                    tma_load_3d(sbase + kQPanel, &tmQ, 64, it.g * G, (int32_t)it.t0, sy.q_full);
                }
                ++qn;
                for (int pass = 0; pass < 2; ++pass) {
                    for (int32_t kt = 0; kt < it.nkt; ++kt, ++kc) {
                        const uint32_t s = kc % kStages, ph = (kc / kStages) & 1;
                        if (!wait_bar(sy, sy.k_empty + 8 * s, ph ^ 1, 2)) continue;
                        const uint32_t dst = sbase + kOffK + s * kKStage;
                        const int32_t krow = (int32_t)(it.k_start + (int64_t)kt * kBN);
                        mbar_arrive_expect_tx(sy.k_full + 8 * s, kKStage);
                        tma_load_3d(dst, &tmK, 0, it.g, krow, sy.k_full + 8 * s);
                        tma_load_3d(dst + kKPanel, &tmK, 64, it.g, krow, sy.k_full + 8 * s);
                    }
                }
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            uint32_t kc = 0, sc = 0, qn = 0;
            for (int64_t w = blockIdx.x; w < n_items; w += gridDim.x) {
                const Item it = decode<QT>(w, p, cu_tiles, n_tiles);
                if (it.nkt == 0 || it.t0 >= p.t_end || it.t0 + it.nq <= p.t_begin) continue;
                bool ok = wait_bar(sy, sy.q_full, qn & 1, 3);
                ++qn;
                tc_fence_after();
                for (int pass = 0; pass < 2; ++pass) {
                    for (int32_t kt = 0; kt < it.nkt; ++kt, ++kc, ++sc) {
                        const uint32_t s = kc % kStages;
                        const uint32_t buf = sc & 1;
                        ok = wait_bar(sy, sy.k_full + 8 * s, (kc / kStages) & 1, 4) && ok;
                        ok = wait_bar(sy, sy.s_empty + 8 * buf, ((sc >> 1) & 1) ^ 1, 5) && ok;
                        tc_fence_after();
                        if (!ok) continue;
                        const uint32_t d = tmem + buf * 256;
                        const uint32_t kb = sbase + kOffK + s * kKStage;
                        if (pass == 0) {
#pragma unroll
                            for (int kk = 0; kk < kD / 16; ++kk) {
                                const uint32_t koff = (kk >> 2) * kKPanel + (kk & 3) * 32;
                                const uint32_t qoff = (kk >> 2) * kQPanel + (kk & 3) * 32;
                                const uint64_t bdesc = desc_kmajor_sw128(kb + koff);
                                umma_bf16(d, desc_kmajor_sw128(sbase + qoff), bdesc, kIdescP1, kk > 0);
                                umma_bf16(d + 128, desc_kmajor_sw128(sbase + qoff + 128 * 128), bdesc,
                                          kIdescP1, kk > 0);
                            }
                        } else {
#pragma unroll
                            for (int kk = 0; kk < kD / 16; ++kk) {
                                const uint32_t koff = (kk >> 2) * kKPanel + (kk & 3) * 32;
                                const uint32_t qoff = (kk >> 2) * kQPanel + (kk & 3) * 32;
                                umma_bf16(d, desc_kmajor_sw128(kb + koff), desc_kmajor_sw128(sbase + qoff),
                                          kIdescP2, kk > 0);
                            }
                        }
                        umma_commit(sy.k_empty + 8 * s);
                        umma_commit(sy.s_full + 8 * buf);
                    }
                }
                if (ok) umma_commit(sy.q_empty);
            }
        }
    } else if (warp == kFillWarp) {
        fill_tails<QT>(p, cu_tiles, n_tiles, n_items, lane);
    } else {
        // ------------------------------------------------------------ epilogue
        // 16 warps = 4 warpgroups; warp w reads TMEM lanes 32*(w%4)..+31.
        //   pass 1: warpgroup wg owns accumulator rows (wg>>1)*128.. (one row per
        //           thread) and key columns (wg&1)*64..+63 of every key tile;
        //   pass 2: warpgroup wg owns tile rows (= accumulator columns) wg*64..+63,
        //           i.e. 64/G tokens, and one key per thread.
        const int tid = threadIdx.x;        // 0..511
        const int wg = warp >> 2;
        const int wq = warp & 3;
        const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
        const float c = p.c;
        const uint64_t c2 = f2_pack(c, c);
        float2 *part = reinterpret_cast<float2 *>(sgen + kOffPart);  // [2][kRows] (max, sum)
        uint32_t sc = 0, stc = 0;
        for (int64_t w = blockIdx.x; w < n_items; w += gridDim.x) {
            const Item it = decode<QT>(w, p, cu_tiles, n_tiles);
            // nothing to compute (the fill warp writes such rows) or outside the token window
            if (it.nkt == 0 || it.t0 >= p.t_end || it.t0 + it.nq <= p.t_begin) continue;
            named_bar_sync(kEpiBarrier, kEpiWarps * 32);  // previous tile done with lim_s/stats
            if (tid < QT)
                lim_s[tid] = tid < it.nq ? visible(it.local0 + tid, it.q_len, it.k_len, p.causal) : 0;
            named_bar_sync(kEpiBarrier, kEpiWarps * 32);
            __nv_bfloat16 *out_g = p.out + (int64_t)it.g * p.T * p.out_stride;

            if (it.nkt > 0) {
                // ---------------- pass 1: softmax statistics of row r over this half's keys
                const int r = (wg >> 1) * 128 + wq * 32 + lane;
                const int32_t lim_r = lim_s[r / G];
                const int colh = (wg & 1) * 64;
                float m = -INFINITY, l = 0.f;
                const uint32_t tcol = lane_base + (wg >> 1) * 128 + colh;
                // a warp whose rows all belong to tokens past the sequence end (decode tiles,
                // a sequence's last tile) only keeps the buffer handshake going
                const bool warp_idle1 = ((wg >> 1) * 128 + wq * 32) / G >= it.nq;
                for (int32_t kt = 0; warp_idle1 && kt < it.nkt; ++kt, ++sc) {
                    const uint32_t buf = sc & 1;
                    wait_bar(sy, sy.s_full + 8 * buf, (sc >> 1) & 1, 6);
                    tc_fence_after();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(sy.s_empty + 8 * buf);
                }
                for (int32_t kt = 0; !warp_idle1 && kt < it.nkt; ++kt, ++sc) {
                    const uint32_t buf = sc & 1;
                    wait_bar(sy, sy.s_full + 8 * buf, (sc >> 1) & 1, 6);
                    tc_fence_after();
                    float v64[64];
                    tmem_ld32(tmem + tcol + buf * 256, *reinterpret_cast<float(*)[32]>(&v64[0]));
                    tmem_ld32(tmem + tcol + buf * 256 + 32, *reinterpret_cast<float(*)[32]>(&v64[32]));
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(sy.s_empty + 8 * buf);  // values are in registers
                    p1_chunk<64>(v64, kt * kBN + colh, lim_r, c, c2, m, l);
                }
                part[(wg & 1) * kRows + r] = make_float2(m, l);
                named_bar_sync(kEpiBarrier, kEpiWarps * 32);
                if ((wg & 1) == 0) {  // merge the two column halves of row r
                    const float2 a = part[r], b2 = part[kRows + r];
                    const float mm = fmaxf(a.x, b2.x);
                    float ll = 0.f;
                    if (mm != -INFINITY) {
                        if (a.x != -INFINITY) ll += a.y * ex2((a.x - mm) * c);
                        if (b2.x != -INFINITY) ll += b2.y * ex2((b2.x - mm) * c);
                    }
                    stats[r] = (ll > 0.f) ? -fmaf(mm, c, log2f(ll)) : -INFINITY;  // -(m*c + log2 l)
                }
                named_bar_sync(kEpiBarrier, kEpiWarps * 32);

                // ---------------- pass 2: key j = this thread's TMEM lane
                constexpr int NQ = 64 / G;  // tokens of this warpgroup
                constexpr bool kTmaStore = (G >= 16);  // staging fits [NQ x 128] bf16 in kStageWg
                const int col0 = wg * 64;   // tile row index of v[0]
                const int tq0 = col0 / G;
                const ulonglong2 *st4 = reinterpret_cast<const ulonglong2 *>(stats + col0);  // -b, 4 at a time
                const uint32_t tcol2 = lane_base + col0;
                // fused pooling: warp wq pools token tq0 + wq (a pooled launch has G >= 16, so
                // NQ <= 4); the row pointer and the token's local-block window are per item
                const int32_t ptq = tq0 + wq;
                const bool pool_w = p.pooled != nullptr && wq < NQ && ptq < it.nq;
                __nv_bfloat16 *prow = p.pooled + ((int64_t)it.g * p.T + it.t0 + ptq) * p.NB;
                const int32_t off_bq = (it.local0 + ptq) / 64;
                float halo = -INFINITY;  // previous tile's last key (slow path)
                uint32_t halo_b = 0;     // the same as bf16 bits (fast path)
                const bool wg_idle2 = tq0 >= it.nq;  // every token of this warpgroup is past the end
                for (int32_t kt = 0; wg_idle2 && kt < it.nkt; ++kt, ++sc) {
                    const uint32_t buf = sc & 1;
                    wait_bar(sy, sy.s_full + 8 * buf, (sc >> 1) & 1, 7);
                    tc_fence_after();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(sy.s_empty + 8 * buf);
                }
                for (int32_t kt = 0; !wg_idle2 && kt < it.nkt; ++kt, ++sc) {
                    const uint32_t buf = sc & 1;
                    const int32_t j = kt * kBN + wq * 32 + lane;
                    wait_bar(sy, sy.s_full + 8 * buf, (sc >> 1) & 1, 7);
                    tc_fence_after();
                    float w64[64];
                    const float(&wa)[32] = *reinterpret_cast<const float(*)[32]>(&w64[0]);
                    const float(&wb)[32] = *reinterpret_cast<const float(*)[32]>(&w64[32]);
                    uint64_t acc[NQ][2];
#pragma unroll
                    for (int qi = 0; qi < NQ; ++qi) acc[qi][0] = acc[qi][1] = 0ull;
                    tmem_ld32(tmem + tcol2 + buf * 256, *reinterpret_cast<float(*)[32]>(&w64[0]));
                    tmem_ld32(tmem + tcol2 + buf * 256 + 32, *reinterpret_cast<float(*)[32]>(&w64[32]));
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(sy.s_empty + 8 * buf);
                    p2_chunk<G, 0>(wa, acc, st4, c2);
                    p2_chunk<G, 1>(wb, acc, st4, c2);
                    if (kTmaStore) {
                        // stage the warpgroup's [NQ tokens x 128 keys] tile in shared memory
                        const uint32_t buf_s = stc & 1;
                        __nv_bfloat16 *stg = reinterpret_cast<__nv_bfloat16 *>(
                            sgen + kOffStage + (wg * 2 + buf_s) * kStageWg);
#pragma unroll
                        for (int qi = 0; qi < NQ; ++qi) {
                            float a0, a1, b0, b1;
                            f2_unpack(acc[qi][0], a0, a1);
                            f2_unpack(acc[qi][1], b0, b1);
                            const float a = (a0 + a1) + (b0 + b1);
                            const float o = j < lim_s[tq0 + qi] ? fmaxf(a, 0.f) : 0.f;
                            stg[qi * kBN + wq * 32 + lane] = __float2bfloat16_rn(o);
                        }
                        fence_async_shared();
                        if (wq == 0 && lane == 0) bulk_wait_read_all();  // previous store left its buffer
                        named_bar_sync(2 + wg, 128);
                        const int t_idx = wq * 32 + lane;
                        if (p.out == nullptr) {
                            // scores not wanted (pooling only): nothing leaves the staging tile
                        } else if (tq0 + NQ <= it.nq) {  // whole tile belongs to this sequence: one TMA store
                            if (t_idx == 0) {
                                tma_store_2d(&tmO, smem_u32(stg), kt * kBN,
                                             (int32_t)((int64_t)it.g * p.T + it.t0 + tq0));
                                bulk_commit();
                            }
                        } else {  // sequence ends inside the tile: copy its rows only
                            for (int e = t_idx; e < NQ * kBN; e += 128) {
                                const int tq = tq0 + e / kBN;
                                const int64_t col = (int64_t)kt * kBN + (e % kBN);
                                if (tq < it.nq && col < p.out_stride)
                                    out_g[(it.t0 + tq) * p.out_stride + col] = stg[e];
                            }
                        }
                        if (pool_w) {
                            // lane = block jg of this tile; its window is keys [4*lane-1, 4*lane+3],
                            // key 4*lane-1 being the previous lane's last key (shuffle) or, for
                            // lane 0, the previous tile's last key (halo)
                            const uint2 raw = *reinterpret_cast<const uint2 *>(stg + wq * kBN + 4 * lane);
                            const int32_t jg = kt * 32 + lane;
                            const bool minf = jg < p.init_blocks || (off_bq >= jg && off_bq <= jg + p.local_blocks);
                            if (kt > 0 && kt + 1 < it.nkt && kt * kBN + kBN <= it.k_len) {
                                // interior tile: every window key exists and every staged score is
                                // finite and >= 0, so the max is the largest bf16 bit pattern
                                const uint32_t up = raw.y >> 16;
                                uint32_t left = __shfl_up_sync(0xffffffffu, up, 1);
                                if (lane == 0) left = halo_b;
                                halo_b = __shfl_sync(0xffffffffu, up, 31);
                                halo = __uint_as_float(halo_b << 16);
                                const uint32_t m2 = __vmaxu2(__vmaxu2(raw.x, raw.y), left | (left << 16));
                                const uint32_t mx = max(m2 & 0xffffu, m2 >> 16);
                                if (jg < p.NB)
                                    reinterpret_cast<uint16_t *>(prow)[jg] = minf ? (uint16_t)0x7F80u : (uint16_t)mx;
                            } else {
                                const __nv_bfloat162 lo2 = *reinterpret_cast<const __nv_bfloat162 *>(&raw.x);
                                const __nv_bfloat162 hi2 = *reinterpret_cast<const __nv_bfloat162 *>(&raw.y);
                                float x[4] = {__low2float(lo2), __high2float(lo2), __low2float(hi2), __high2float(hi2)};
                                float left = __shfl_up_sync(0xffffffffu, x[3], 1);
                                if (lane == 0) left = halo;
                                halo = __shfl_sync(0xffffffffu, x[3], 31);
                                halo_b = __float_as_uint(halo) >> 16;
                                const int32_t c0k = kt * kBN + 4 * lane;  // global key of x[0]
                                if (c0k + 3 >= it.k_len || c0k == 0) {
#pragma unroll
                                    for (int i = 0; i < 4; ++i)
                                        if (c0k + i >= it.k_len) x[i] = -INFINITY;
                                    if (c0k - 1 < 0 || c0k - 1 >= it.k_len) left = -INFINITY;
                                }
                                const float mx = fmaxf(fmax3(left, x[0], x[1]), fmaxf(x[2], x[3]));
                                if (jg < p.NB) {
                                    const bool has = 4 * jg - 1 < it.k_len;
                                    prow[jg] = __float2bfloat16_rn(minf ? INFINITY : (has ? mx : -INFINITY));
                                }
                                if (lane == 31 && kt + 1 == it.nkt && jg + 1 < p.NB) {
                                    // first block past the computed tiles: key 128*nkt-1 plus zeros
                                    const int32_t jn = jg + 1, cl = kt * kBN + kBN - 1;
                                    float m2 = -INFINITY;
                                    if (cl < it.k_len) m2 = x[3];
                                    if (cl + 1 < it.k_len) m2 = fmaxf(m2, 0.f);
                                    const bool minf2 = jn < p.init_blocks || (off_bq >= jn && off_bq <= jn + p.local_blocks);
                                    const bool has = 4 * jn - 1 < it.k_len;
                                    prow[jn] = __float2bfloat16_rn(minf2 ? INFINITY : (has ? m2 : -INFINITY));
                                }
                            }
                        }
                        ++stc;
                    } else if (j < p.out_stride) {
#pragma unroll
                        for (int qi = 0; qi < NQ; ++qi) {
                            const int tq = tq0 + qi;
                            if (tq < it.nq) {
                                float a0, a1, b0, b1;
                                f2_unpack(acc[qi][0], a0, a1);
                                f2_unpack(acc[qi][1], b0, b1);
                                const float a = (a0 + a1) + (b0 + b1);
                                const float o = j < lim_s[tq] ? fmaxf(a, 0.f) : 0.f;
                                out_g[(it.t0 + tq) * p.out_stride + j] = __float2bfloat16_rn(o);
                            }
                        }
                    }
                }
            }
        }
        if (wq == 0 && lane == 0) bulk_wait_all();  // output stores complete before exit
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        if (*abort_flag) {
            // give TMA/UMMA work already in flight time to land before TMEM is released
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < 2000000ull) {
            }
        }
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Prologue: per-sequence tile prefix into the workspace, status := 0, and
// zero rows of `out` that no sequence covers (tokens outside
// [cu_q[0], cu_q[n_seq]) keep the reference's torch.zeros value).
__global__ void __launch_bounds__(1024)
stage1_prologue(const int32_t *__restrict__ cu_q, int32_t n_seq, int32_t QT, int32_t *ws,
                __nv_bfloat16 *out, int64_t T, int32_t Hk, int64_t out_stride,
                __nv_bfloat16 *pooled, int32_t NB, int32_t init_blocks, int32_t local_blocks) {
    __shared__ int32_t warp_sums[32];
    __shared__ int32_t carry_s;
    // a decode kernel launched after this one with programmatic stream serialization
    // may start its set-up now; it waits (griddepcontrol.wait) for this grid to finish
    // before it touches the workspace
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        ws[0] = 0;
        ws[1] = 0;  // work counter of the decode kernel
        carry_s = 0;
    }
    __syncthreads();
    int32_t *cu_tiles = ws + kWsTiles;
    for (int32_t base = 0; base < n_seq; base += 1024) {
        const int32_t b = base + tid;
        int32_t cnt = 0;
        if (b < n_seq) {
            const int32_t len = cu_q[b + 1] - cu_q[b];
            cnt = len > 0 ? (len + QT - 1) / QT : 0;
        }
        int32_t x = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_sums[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int32_t s = warp_sums[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int32_t y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            warp_sums[lane] = s;  // inclusive over warps
        }
        __syncthreads();
        const int32_t carry = carry_s;
        const int32_t excl = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + x - cnt;
        if (b < n_seq) cu_tiles[b] = excl;
        __syncthreads();
        if (tid == 0) carry_s = carry + warp_sums[31];
        __syncthreads();
    }
    if (tid == 0) cu_tiles[n_seq] = carry_s;
    // rows outside every sequence
    const int64_t lo = n_seq > 0 ? cu_q[0] : T, hi = n_seq > 0 ? cu_q[n_seq] : T;
    const int64_t per_row = out_stride / 8;
    for (int32_t g = 0; g < Hk; ++g) {
        for (int64_t t = 0; t < T; ++t) {
            if (t >= lo && t < hi) {
                t = hi - 1;
                continue;
            }
            if (out) {
                uint4 *row = reinterpret_cast<uint4 *>(out + ((int64_t)g * T + t) * out_stride);
                for (int64_t e = tid; e < per_row; e += 1024) row[e] = make_uint4(0, 0, 0, 0);
            }
            if (pooled) {  // no sequence: k_len 0, local block 0 (max_pooling_1d_varlen.py:69-80)
                __nv_bfloat16 *prow = pooled + ((int64_t)g * T + t) * NB;
                for (int32_t j = tid; j < NB; j += 1024) {
                    const bool minf = j < init_blocks || (0 >= j && 0 <= j + local_blocks);
                    prow[j] = __float2bfloat16_rn(minf ? INFINITY : -INFINITY);
                }
            }
        }
    }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// 3-D bf16 map over [dim2][dim1][dim0] with a box of (64, box1, box2), 128-byte swizzle.
int make_map(CUtensorMap *m, const void *base, uint64_t dim0, uint64_t dim1, uint64_t dim2,
             uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box1, uint32_t box2) {
    auto enc = get_encode_fn();
    if (!enc) {
        unum::set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return UNUM_ERR_CUDA;
    }
    cuuint64_t gdim[3] = {dim0, dim1, dim2};
    cuuint64_t gstride[2] = {stride1_bytes, stride2_bytes};
    cuuint32_t box[3] = {64, box1, box2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), gdim, gstride,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        unum::set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return UNUM_ERR_CUDA;
    }
    return UNUM_OK;
}

template <int G>
int launch_main(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mo,
                const Params &p, int64_t T, cudaStream_t s) {
    auto kern = stage1_kernel<G>;
    UNUM_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    constexpr int QT = kRows / G;
    const int64_t items_ub = ((T + QT - 1) / QT + p.n_seq) * p.Hk;
    const int64_t sms = unum::sm_count();
    const int grid = (int)(items_ub < sms ? items_ub : sms);
    kern<<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mo, p);
    return unum::check_launch("stage1_kernel");
}

// ------------------------------------------------------------------ decode kernel
// Stage 1 with one work item per (query token, kv head): the path for decode
// batches (one or a few query tokens per sequence), where the tile kernel above
// would fill 1 of 256/G rows of each tile and re-read every key tile in its
// second pass.  Here each 128-key tile of the token's visible keys is one MMA
// M=128 (keys) x N=G (the token's query heads) x K=128, and all the item's tiles
// stay in TMEM side by side (G columns each, up to 512/G tiles), so the keys are
// read from HBM once and the softmax needs no second MMA pass: the epilogue reads
// the scores from TMEM three times (max, sum, output).  The path is HBM-bound on
// the compressed keys.  TMEM is a ring of 512/G tile slots released tile by
// tile, so consecutive items overlap.  Items are taken from a work counter (workspace word 1,
// zeroed by the prologue), so CTAs stay balanced although items differ in size.
#ifndef UNUM_DEC_STAGES
#define UNUM_DEC_STAGES 4
#endif
constexpr int kDecStages = UNUM_DEC_STAGES;  // K ring depth
constexpr int kDecSlots = 4;         // item queue depth (an item = its id + its q tile)
// 8 epilogue warps: warps w and w+4 read TMEM lane quarter w%4 (keys 32*(w%4)..+31 of a
// tile) and take alternate batches of tiles, so each scheduler has two of them
constexpr int kDecEpiWarps = 8;
constexpr int kDecProducerWarp = 8;
constexpr int kDecMmaWarp = 9;
constexpr int kDecThreads = 10 * 32;
constexpr int kDecEpiBarrier = 1;
constexpr uint32_t kDecQSlot = 2 * 32 * 128;                 // two 64-column panels of up to 32 heads
constexpr uint32_t kDecOffK = kDecSlots * kDecQSlot;          // 32 KB
constexpr uint32_t kDecOffRed = kDecOffK + kDecStages * kKStage;
constexpr uint32_t kDecOffBar = kDecOffRed + 2 * (kDecEpiWarps + 1) * 32 * 4;
// barriers: item_full, item_empty, q_full, tmem_full (per item slot), k_full, k_empty (per
// stage), and one per TMEM tile slot (free again)
constexpr int kDecTmemSlotsMax = 32;  // 512 columns / 16 heads
constexpr uint32_t kDecNumBars = 4 * kDecSlots + 2 * kDecStages + kDecTmemSlotsMax;
constexpr uint32_t kDecOffMisc = kDecOffBar + kDecNumBars * 8;  // item ids, abort flag, TMEM address
constexpr uint32_t kDecSmemBytes = kDecOffMisc + 64 + 1024;
static_assert(kDecOffK % 1024 == 0 && kDecQSlot % 1024 == 0, "SW128 operand tiles need 1024-byte alignment");
static_assert(kDecSmemBytes <= 232448, "exceeds the 227 KB of shared memory a CTA may use");

// Fused selection (unum_block_select_decode): a decode item's whole score row sits in
// one CTA, so the epilogue also pools it into 64-token blocks, picks the top-K blocks
// and writes their physical slot ids, the steps block_select otherwise runs as three
// more kernels over HBM.  Scratch: the row's bf16 scores, two 256-bin histograms, the
// selected ids and a few scan words.
struct DecSel {
    const int32_t *cache_lens;  // [n_seq] added to the pooling's key count, or null (0)
    __nv_bfloat16 *pooled;      // [Hk, T, NB] or null
    int32_t *topk;              // [Hk, T, K]
    int32_t *slots;             // [T, Hk, K*64] or null
    const int32_t *table;       // block table [B, L], row stride bt_stride
    const int32_t *tok_bs, *tok_pos, *seqlen;
    int64_t bt_stride;
    int32_t B, L, pos_scalar, seqlen_scalar;
    uint32_t head_group;
    int32_t NB, K, init_blocks, local_blocks;
    int32_t vec_ok;  // table rows may be read with 16-byte loads
};
constexpr uint32_t kSelRowMax = 4096;  // row columns: out_stride <= 128 * 512 / 16
constexpr int32_t kSelNBMax = 1024;    // pooled blocks: 4 * NB <= out_stride
constexpr int32_t kSelKMax = 1024;
constexpr uint32_t kSelOffRow = 0;
constexpr uint32_t kSelOffHist = kSelOffRow + kSelRowMax * 2;
constexpr uint32_t kSelOffIds = kSelOffHist + 2 * 256 * 4;
constexpr uint32_t kSelOffMisc = kSelOffIds + kSelKMax * 4;
constexpr uint32_t kSelBytes = kSelOffMisc + 32 * 4;
// CTA pairs (a cluster of two sharing each item): the peer's item mailbox, the
// exchanged per-head statistics and the barriers of the exchange
constexpr uint32_t kDecOffPair = (kDecOffMisc + 64 + 15) & ~15u;
constexpr uint32_t kPairInbox = 0;                        // int64 [kDecSlots]
constexpr uint32_t kPairX = kPairInbox + 8 * kDecSlots;   // float [2][32]: peer's max, sum
constexpr uint32_t kPairBars = kPairX + 2 * 32 * 4;       // item_in[slots], peer_empty[slots], x_full[2], row_full
constexpr uint32_t kPairBytes = kPairBars + (2 * kDecSlots + 3) * 8;
// each item slot's decoded item, written by the producer (the MMA warp and the epilogue
// read it instead of repeating the sequence search on their critical paths)
constexpr uint32_t kDecItemBytes = 96;  // the decoded item, then (fused selection) its SelPre
constexpr uint32_t kDecOffItems = (kDecOffPair + kPairBytes + 15) & ~15u;
constexpr uint32_t kDecOffSel = (kDecOffItems + kDecSlots * kDecItemBytes + 127) & ~127u;
constexpr uint32_t kDecSmemBytesSel = kDecOffSel + kSelBytes + 1024;
constexpr uint32_t kDecSmemBytesPair = kDecOffSel + 1024;
static_assert(kDecSmemBytesSel <= 232448, "exceeds the 227 KB of shared memory a CTA may use");

// N = 16 or 32 consecutive f32 columns of this thread's TMEM lane.
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld_cols<16>(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld_cols<32>(uint32_t taddr, float (&v)[32]) {
    tmem_ld32(taddr, v);
}

// What one decode item covers.
struct DecItem {
    int32_t g;        // kv head
    int64_t t;        // query token
    int32_t vis;      // visible compressed keys
    int32_t nkt;      // key tiles
    int64_t k_start;  // first compressed key of the token's sequence
    int32_t seq;      // the token's sequence
    int32_t lq;       // position of the token inside its sequence's queries
    int32_t k_len;    // the sequence's compressed keys
    bool active;      // false: token outside every sequence or outside the token window
};

// An item with more than max_tiles key tiles (more visible keys than tensor
// memory holds; only when the caller's out_stride is below a sequence's key
// count) keeps its full visible count in vis but only max_tiles tiles in nkt:
// the epilogue folds the keys past them into the softmax statistics on CUDA
// cores (dec_extra_scores).  Their columns lie past out_stride, so none is written.
__device__ __forceinline__ DecItem dec_decode(int64_t w, const Params &p, int32_t max_tiles) {
    DecItem it;
    it.g = (int32_t)(w % p.Hk);
    it.t = w / p.Hk;
    it.active = false;
    it.vis = 0;
    it.nkt = 0;
    it.k_start = 0;
    it.seq = 0;
    it.lq = 0;
    it.k_len = 0;
    if (p.n_seq <= 0 || it.t < p.t_begin || it.t >= p.t_end) return it;
    const int32_t t = (int32_t)it.t;
    if (t < __ldg(p.cu_q) || t >= __ldg(p.cu_q + p.n_seq)) return it;
    int32_t lo = 0, hi = p.n_seq;  // largest b with cu_q[b] <= t
    while (hi - lo > 1) {
        const int32_t mid = (lo + hi) >> 1;
        if (__ldg(p.cu_q + mid) <= t) lo = mid; else hi = mid;
    }
    const int32_t qs = __ldg(p.cu_q + lo);
    const int32_t q_len = __ldg(p.cu_q + lo + 1) - qs;
    it.k_start = __ldg(p.cu_k + lo);
    const int32_t k_len = __ldg(p.cu_k + lo + 1) - (int32_t)it.k_start;
    it.seq = lo;
    it.lq = t - qs;
    it.k_len = k_len;
    it.vis = visible(t - qs, q_len, k_len, p.causal);
    it.nkt = (it.vis + kBN - 1) / kBN;
    if (it.nkt > max_tiles) it.nkt = max_tiles;
    it.active = true;
    return it;
}

// Max (or sum) of each of N per-thread values (N = 16 or 32) over the 256 epilogue
// threads; every thread gets the N results.  In a warp, a reduce-scatter: at each step a
// lane keeps half of its values and receives its partner's copy of that half, so after
// log2(N) steps lane L holds value L % N reduced over N lanes (N - 1 shuffles instead of
// 5N); then across the 8 warps through shared memory `red` ([9][32] floats: the warps'
// partials, then the results).
template <int N, bool kMax>
__device__ __forceinline__ void dec_reduce(float (&v)[N], float *red, int warp, int lane) {
    static_assert(N == 16 || N == 32, "16 or 32 values");
#pragma unroll
    for (int h = N / 2; h >= 1; h >>= 1) {
        const bool upper = (lane & h) != 0;
#pragma unroll
        for (int i = 0; i < h; ++i) {
            const float send = upper ? v[i] : v[i + h];
            const float keep = upper ? v[i + h] : v[i];
            const float got = __shfl_xor_sync(0xffffffffu, send, h);
            v[i] = kMax ? fmaxf(keep, got) : keep + got;
        }
    }
    float x = v[0];  // value lane % N, over the N lanes that share lane / N
    if (N < 32) {
        const float y = __shfl_xor_sync(0xffffffffu, x, 16);
        x = kMax ? fmaxf(x, y) : x + y;
    }
    if (lane < N) red[warp * 32 + lane] = x;
    named_bar_sync(kDecEpiBarrier, kDecEpiWarps * 32);
    if (warp == 0 && lane < N) {
        float a = red[lane];
#pragma unroll
        for (int w2 = 1; w2 < kDecEpiWarps; ++w2) a = kMax ? fmaxf(a, red[w2 * 32 + lane]) : a + red[w2 * 32 + lane];
        red[kDecEpiWarps * 32 + lane] = a;
    }
    named_bar_sync(kDecEpiBarrier, kDecEpiWarps * 32);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = red[kDecEpiWarps * 32 + i];
}

// Named barrier over n threads that also ORs a predicate across them, so a
// decision taken after it (leave the loop) is the same in every thread.
__device__ __forceinline__ bool named_bar_or(int id, int n, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, %2, %3, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(n) : "memory");
    return r != 0;
}

// Raw scores q[t, h] . k[k_start + j, g] of heads h0..h0+7 of a decode item for
// one key j past the item's tensor-memory tiles, on CUDA cores: q from the
// item's shared-memory tile (two 64-column panels, 128-byte swizzle: 16-byte
// chunk c of row h sits at chunk c ^ (h & 7)), k from global memory.  Products
// of bf16 values are exact in f32, so these match the tensor-core scores up to
// the order of the sums.
template <int G>
__device__ __forceinline__ void dec_extra_scores8(const Params &p, const uint8_t *qtile, int32_t g,
                                                  int64_t k_start, int32_t j, int h0, float (&sc)[8]) {
    const uint4 *kr = reinterpret_cast<const uint4 *>(p.k + (k_start + j) * p.k_st + (int64_t)g * p.k_sh);
#pragma unroll
    for (int h = 0; h < 8; ++h) sc[h] = 0.f;
#pragma unroll 1
    for (int c = 0; c < 16; ++c) {
        const uint4 kv = __ldg(kr + c);
        const __nv_bfloat162 *k2 = reinterpret_cast<const __nv_bfloat162 *>(&kv);
        const uint8_t *panel = qtile + (c >> 3) * (G * 128);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
            const int hh = h0 + h;
            const uint4 qv = *reinterpret_cast<const uint4 *>(panel + hh * 128 + (((c & 7) ^ (hh & 7)) << 4));
            const __nv_bfloat162 *q2 = reinterpret_cast<const __nv_bfloat162 *>(&qv);
            float a = sc[h];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                a = fmaf(__low2float(q2[e]), __low2float(k2[e]), a);
                a = fmaf(__high2float(q2[e]), __high2float(k2[e]), a);
            }
            sc[h] = a;
        }
    }
}

// Inclusive sum of v over the 256 epilogue threads; scratch: 8 words.  Ends with the
// threads synchronised, so the scratch may be reused after the next barrier.
__device__ __forceinline__ int32_t epi_scan(int32_t v, int32_t *scratch, int warp, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
    }
    if (lane == 31) scratch[warp] = v;
    named_bar_sync(kDecEpiBarrier, kDecEpiWarps * 32);
    for (int w = 0; w < warp; ++w) v += scratch[w];
    return v;
}

// The bin of a 256-bin histogram (hist[b] = entries whose byte is b) that holds the
// need-th largest entry, counting from bin 255 down, and the count of entries in higher
// bins; bin -1 when the histogram holds fewer than `need` entries.  Computed by every
// warp that calls it (the same result in every lane), so no barrier is needed to share it.
struct BinPick {
    int32_t bin, above, total;
};

__device__ __forceinline__ BinPick sel_pick_bin(const int32_t *hist, int32_t need, int lane) {
    int32_t c[8], sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        c[i] = hist[255 - 8 * lane - i];
        sum += c[i];
    }
    int32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    BinPick r;
    r.total = __shfl_sync(0xffffffffu, incl, 31);
    r.bin = -1;
    r.above = 0;
    if (r.total < need) return r;
    const int32_t excl = incl - sum;
    const unsigned hit = __ballot_sync(0xffffffffu, excl < need && incl >= need);
    const int src = __ffs(hit) - 1;
    int32_t bin = -1, above = 0, run = excl;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (bin < 0 && run + c[i] >= need) {
            bin = 255 - 8 * lane - i;
            above = run;
        }
        run += c[i];
    }
    r.bin = __shfl_sync(0xffffffffu, bin, src);
    r.above = __shfl_sync(0xffffffffu, above, src);
    return r;
}

// Add one to hist[bin] for every lane with bin >= 0, one atomic per distinct bin of the warp.
__device__ __forceinline__ void hist_add_warp(int32_t *hist, int32_t bin, int lane) {
    const unsigned peers = __match_any_sync(0xffffffffu, bin);
    if (bin >= 0 && lane == __ffs(peers) - 1) atomicAdd(hist + bin, __popc(peers));
}

// A decode item as the pair's leader posts it: its id, plus kSoloBit when one CTA takes
// it alone rather than the pair sharing it; -1 ends the stream.  A CTA's share of the
// item: tiles cr, cr + cc, cr + 2cc, ... (joint: cr = rank, cc = 2; alone: 0, 1).
constexpr int64_t kSoloBit = (int64_t)1 << 40;

struct Role {
    int64_t w;     // item id, or -1
    bool joint;    // shared by the pair
    int32_t cr, cc, max_tiles;
};

template <int kC>
__device__ __forceinline__ Role role_of(int64_t v, uint32_t rank, int32_t tmem_tiles) {
    Role r;
    r.joint = kC == 2 && v >= 0 && (v & kSoloBit) == 0;
    r.w = v >= 0 ? (v & (kSoloBit - 1)) : -1;
    r.cr = r.joint ? (int32_t)rank : 0;
    r.cc = r.joint ? 2 : 1;
    r.max_tiles = tmem_tiles * r.cc;
    return r;
}

// Per-token values the selection needs from global memory, loaded by the producer with
// the item and handed over in its slot, so the epilogue never waits on them.
struct SelPre {
    int32_t k_len;   // the pooling's key count: compressed keys + cache_lens[b]
    int32_t off_bq;  // the token's local block
    int32_t lim;     // get_block_table: positions valid iff 0 <= pos < lim
    int64_t brow;    // offset of the token's block-table row
};

__device__ __forceinline__ SelPre dec_sel_pre(const DecSel &sel, const DecItem &it) {
    SelPre r;
    r.k_len = 0;  // a token outside every sequence: k_len 0, local block 0
    r.off_bq = 0;
    if (it.active) {
        r.k_len = it.k_len + (sel.cache_lens ? __ldg(sel.cache_lens + it.seq) : 0);
        r.off_bq = it.lq / 64;
    }
    r.lim = INT32_MIN;
    r.brow = 0;
    if (sel.slots) {
        const int32_t t = (int32_t)it.t;
        const int32_t bs = __ldg(sel.tok_bs + t);
        const bool bs_ok = bs >= 0 && bs < sel.B;
        const int32_t lim_pos = sel.pos_scalar ? __ldg(sel.tok_pos) : __ldg(sel.tok_pos + t);
        const int32_t sl = sel.seqlen_scalar ? __ldg(sel.seqlen) : (bs_ok ? __ldg(sel.seqlen + bs) : 0);
        r.lim = bs_ok ? min(lim_pos, sl) : INT32_MIN;
        r.brow = bs_ok ? (int64_t)bs * sel.bt_stride : 0;
    }
    return r;
}

// Pooling, top-k and get_block_table of one decode item, by the 256 epilogue threads,
// from the item's bf16 score row in shared memory (srow[j] = the value stage 1 writes at
// column j; zeros past the tensor-memory tiles, as the written row has).
//  - pooling: the window rule of max_pooling_1d_varlen (max_pooling_1d_varlen.py:69-116)
//    with kernel 5, stride 4, padding 1 over the row read as flat stride out_stride (the
//    caller's max_seqlen_q = 16 * out_stride), k_len = compressed keys + cache_lens[b],
//    blocks j < init_blocks or with j <= off_bq <= j + local_blocks forced to +inf;
//  - top-k: the rule of the top-k kernel: candidates are neither -inf nor NaN, ranked by
//    (score desc, block asc), the first min(K, candidates) emitted in ascending block
//    order, then -1;
//  - get_block_table_ref_torch (get_table_torch.py:4-44) on the selected blocks.
// Thread tid owns blocks 4*tid .. 4*tid+3, so a scan over threads orders blocks.
__device__ __forceinline__ void dec_select(const Params &p, const DecSel &sel, const DecItem &it,
                                           const SelPre &pre, uint8_t *smem, int tid, int warp, int lane) {
    const __nv_bfloat16 *srow = reinterpret_cast<const __nv_bfloat16 *>(smem + kSelOffRow);
    int32_t *hist = reinterpret_cast<int32_t *>(smem + kSelOffHist);  // [2][256], zeroed by the caller
    int32_t *sid = reinterpret_cast<int32_t *>(smem + kSelOffIds);
    int32_t *misc = reinterpret_cast<int32_t *>(smem + kSelOffMisc);
    const int32_t NB = sel.NB, K = sel.K;
    const int32_t k_len = pre.k_len, off_bq = pre.off_bq;
    const int64_t row = (int64_t)it.g * p.T + it.t;
    // the 17 row values the 4 windows of this thread read: columns 16*tid - 1 .. 16*tid + 15,
    // masked to -inf outside [0, k_len) (the reference's window bounds)
    float v[17];
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(srow) + 2 * tid;
        const uint4 a = src[0], b = src[1];
        const __nv_bfloat16 *pa = reinterpret_cast<const __nv_bfloat16 *>(&a);
        const __nv_bfloat16 *pb = reinterpret_cast<const __nv_bfloat16 *>(&b);
        const int32_t c0 = 16 * tid;
        v[0] = (c0 >= 1 && c0 - 1 < k_len) ? __bfloat162float(srow[c0 - 1]) : -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            v[1 + i] = c0 + i < k_len ? __bfloat162float(pa[i]) : -INFINITY;
            v[9 + i] = c0 + 8 + i < k_len ? __bfloat162float(pb[i]) : -INFINITY;
        }
    }
    uint32_t key[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int32_t j = 4 * tid + e;
        key[e] = 0;
        int32_t bin = -1;
        if (j < NB) {
            uint16_t bits;
            const bool minf = j < sel.init_blocks || (off_bq >= j && off_bq <= j + sel.local_blocks);
            if (minf) {
                bits = 0x7F80u;
            } else {  // window columns 4j-1 .. 4j+3 = v[4e .. 4e+4]; all masked: -inf
                const float m = fmaxf(fmaxf(fmaxf(v[4 * e], v[4 * e + 1]), fmaxf(v[4 * e + 2], v[4 * e + 3])),
                                      v[4 * e + 4]);
                bits = __bfloat16_as_ushort(__float2bfloat16_rn(m));
            }
            if (sel.pooled) sel.pooled[row * NB + j] = __ushort_as_bfloat16(bits);
            const bool nan = (bits & 0x7F80u) == 0x7F80u && (bits & 0x7Fu) != 0;
            if (bits != 0xFF80u && !nan) {
                key[e] = (bits & 0x8000u) ? (~bits & 0xFFFFu) : (bits | 0x8000u);  // order-preserving
                bin = (int32_t)(key[e] >> 8);
            }
        }
        hist_add_warp(hist, bin, lane);
    }
    named_bar_sync(kDecEpiBarrier, kDecEpiWarps * 32);
    const BinPick p1 = sel_pick_bin(hist, K, lane);
    const int32_t n_cand = p1.total;
    uint32_t thr = 0;  // selected: key > thr, and the first `need` keys == thr
    int32_t need = 0;
    if (p1.bin >= 0) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const bool in = key[e] != 0 && (int32_t)(key[e] >> 8) == p1.bin;
            hist_add_warp(hist + 256, in ? (int32_t)(key[e] & 255u) : -1, lane);
        }
        named_bar_sync(kDecEpiBarrier, kDecEpiWarps * 32);
        const BinPick p2 = sel_pick_bin(hist + 256, K - p1.above, lane);
        thr = ((uint32_t)p1.bin << 8) | (uint32_t)p2.bin;
        need = K - p1.above - p2.above;
    }
    int32_t gt = 0, eq = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        gt += key[e] > thr;
        eq += key[e] == thr && key[e] != 0;
    }
    const int32_t packed = (gt << 16) | eq;
    const int32_t excl = epi_scan(packed, misc, warp, lane) - packed;
    int32_t gt_before = excl >> 16, eq_before = excl & 0xFFFF;
    int32_t *trow = sel.topk + row * K;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int32_t j = 4 * tid + e;
        int32_t pos = -1;
        if (key[e] > thr) {
            pos = gt_before + (eq_before < need ? eq_before : need);
            ++gt_before;
        } else if (key[e] == thr && key[e] != 0) {
            if (eq_before < need) pos = gt_before + eq_before;
            ++eq_before;
        }
        if (pos >= 0) {
            sid[pos] = j;
            trow[pos] = j;
        }
    }
    const int32_t n_sel = n_cand < K ? n_cand : K;
    for (int32_t i = n_sel + tid; i < K; i += kDecEpiWarps * 32) {
        sid[i] = -1;
        trow[i] = -1;
    }
    named_bar_sync(kDecEpiBarrier, kDecEpiWarps * 32);
    if (sel.slots) {
        const int32_t lim = pre.lim;
        const int32_t *brow = sel.table + pre.brow;
        const int32_t items = K * 16;  // int4 items of the row
        const int32_t span = (items + kDecEpiWarps * 128 - 1) / (kDecEpiWarps * 128) * 128;
        const int32_t eA = warp * span, eB = eA + span < items ? eA + span : items;
        int4 *orow = reinterpret_cast<int4 *>(sel.slots + ((int64_t)it.t * p.Hk + it.g) * (int64_t)K * 64);
        if (eA < items)
            unum::gbt_emit_row<true>(sid, 1, K, brow, lim, sel.L, sel.head_group, (uint32_t)it.g,
                                     sel.vec_ok != 0, orow, lane, eA, eB);
    }
}

// kC = 2: the kernel runs as clusters of two CTAs, each pair working on one item at a
// time: the leader (rank 0) takes items and posts them to its peer, each CTA streams the
// key tiles of its own parity (tile kt goes to rank kt % 2), the per-head max and sum are
// exchanged through distributed shared memory, and the peer's bf16 outputs are written
// into the leader's row buffer, where the leader runs the fused selection.  Halves the
// time of an item: for batches with fewer items than SMs, where the longest item bounds
// the kernel (one SM streams keys at well below its share of HBM bandwidth).
template <int G, bool kSel, int kC>
__global__ void __launch_bounds__(kDecThreads, 1)
stage1_decode_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ Params p, const __grid_constant__ DecSel sel) {
    constexpr uint32_t kQPanelD = G * 128;        // one 64-column panel of the token's G heads
    constexpr uint32_t kQBytesD = 2 * kQPanelD;
    constexpr uint32_t kIdesc = idesc_bf16_f32(128, G);
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t *sgen = smem_raw + (sbase - raw);
    float *red = reinterpret_cast<float *>(sgen + kDecOffRed);  // [2][9][32]: max and sum reductions
    const uint32_t bar0 = sbase + kDecOffBar;
    const uint32_t item_full = bar0, item_empty = bar0 + 8 * kDecSlots, q_full = bar0 + 16 * kDecSlots;
    const uint32_t k_full = bar0 + 24 * kDecSlots, k_empty = k_full + 8 * kDecStages;
    // TMEM is a ring of kTs tile slots of G columns; tile i of this CTA's stream uses slot
    // i % kTs, so the next item's MMAs can start while the epilogue still reads this one
    constexpr uint32_t kTs = kTmemCols / G;
    // tmem_full per item slot: reusing a slot waits for item_empty, so no phase is overrun
    const uint32_t tmem_full = k_empty + 8 * kDecStages, slot_empty = tmem_full + 8 * kDecSlots;
    volatile int64_t *item_id = reinterpret_cast<volatile int64_t *>(sgen + kDecOffMisc);  // [kDecSlots]
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sgen + kDecOffMisc + 8 * kDecSlots);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sgen + kDecOffMisc + 8 * kDecSlots + 16);
    Sync sy;
    sy.abort = abort_flag;
    sy.status = p.ws;
    DecItem *slot_item = reinterpret_cast<DecItem *>(sgen + kDecOffItems);  // [kDecSlots]
    SelPre *slot_pre = reinterpret_cast<SelPre *>(sgen + kDecOffItems + kDecSlots * 64);  // [kDecSlots]
    static_assert(sizeof(DecItem) <= 64 && sizeof(SelPre) <= 32, "decoded item larger than its slot");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr bool kPair = kC == 2;
    const uint32_t rank = kPair ? cluster_ctarank() : 0u;
    const uint32_t pbase = sbase + kDecOffPair;
    volatile int64_t *inbox = reinterpret_cast<volatile int64_t *>(sgen + kDecOffPair + kPairInbox);
    volatile float *xbuf = reinterpret_cast<volatile float *>(sgen + kDecOffPair + kPairX);
    const uint32_t item_in = pbase + kPairBars, peer_empty = item_in + 8 * kDecSlots;
    const uint32_t x_full = peer_empty + 8 * kDecSlots, row_full = x_full + 16;
    if (threadIdx.x == 0) {
        if constexpr (kPair) {
            for (int i = 0; i < kDecSlots; ++i) {
                mbar_init(item_in + 8 * i, 1);     // the leader's post (peer)
                mbar_init(peer_empty + 8 * i, 1);  // the peer took the post (leader)
            }
            mbar_init(x_full, 1);                  // the other CTA's max
            mbar_init(x_full + 8, 1);              // the other CTA's sum
            mbar_init(row_full, kDecEpiWarps * 32);  // the peer's outputs are in srow (leader)
        }
        for (int i = 0; i < kDecSlots; ++i) {
            mbar_init(item_full + 8 * i, 1);
            mbar_init(item_empty + 8 * i, 2);  // the MMA warp's commit + the epilogue
            mbar_init(q_full + 8 * i, 1);
        }
        for (int i = 0; i < kDecStages; ++i) {
            mbar_init(k_full + 8 * i, 1);
            mbar_init(k_empty + 8 * i, 1);
        }
        for (int i = 0; i < kDecSlots; ++i) mbar_init(tmem_full + 8 * i, 1);
        for (uint32_t i = 0; i < kTs; ++i) mbar_init(slot_empty + 8 * i, 4);  // a tile's 4 reader warps
        *abort_flag = p.force_expiry ? 1 : 0;  // status 30 is set after the prologue
        fence_barrier_init();
    }
    if (warp == kDecProducerWarp && lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
    }
    if (warp == kDecMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync();  // both CTAs' barriers exist before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // set-up above overlaps the prologue's tail; the workspace (status, work counter) and
    // the rows the prologue zeroes are touched only after it has finished
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (threadIdx.x == 0 && p.force_expiry) atomicCAS(p.ws, 0, 30);
    const int64_t n_items = p.T * p.Hk;
    int32_t *counter = p.ws + 1;

    if (warp == kDecProducerWarp) {
        if (lane == 0) {
            uint32_t kc = 0;
            const int64_t n_groups = gridDim.x / kC;  // CTAs (pairs) taking items
            bool peer_done = false;                     // the peer was sent the end of the stream
            for (uint32_t n = 0;; ++n) {
                const uint32_t s = n % kDecSlots, eph = ((n / kDecSlots) & 1) ^ 1;
                if (!wait_bar(sy, item_empty + 8 * s, eph, 11)) break;
                int64_t v;  // this CTA's item as posted (id, solo bit)
                if (rank == 0) {
                    // first item static (no counter round trip on the critical path), then dynamic
                    int64_t w1 = n == 0 ? (int64_t)(blockIdx.x / kC) : atomicAdd(counter, 1) + n_groups;
                    if (w1 >= n_items) w1 = -1;
                    v = w1;
                    if constexpr (kPair) {
                        int64_t vp = w1;  // the peer's
                        if (w1 >= 0 && w1 >= p.joint_items) {  // one item each
                            v = w1 | kSoloBit;
                            const int64_t w2 = atomicAdd(counter, 1) + n_groups;
                            vp = w2 < n_items ? (w2 | kSoloBit) : -1;
                        }
                        if (!peer_done) {  // post it once the peer has taken the last post
                            if (!wait_bar<true>(sy, peer_empty + 8 * s, eph, 19)) break;
                            st_cluster_s64(mapa_shared(pbase + kPairInbox + 8 * s, 1), vp);
                            mbar_arrive_remote(mapa_shared(item_in + 8 * s, 1));
                            peer_done = vp < 0;  // the counter is spent: nothing more for either
                        }
                    }
                } else {
                    if (!wait_bar<true>(sy, item_in + 8 * s, (n / kDecSlots) & 1, 19)) break;
                    v = inbox[s];
                    mbar_arrive_remote(mapa_shared(peer_empty + 8 * s, 0));
                }
                const Role ro = role_of<kC>(v, rank, kTs);
                const int64_t w = ro.w;
                const DecItem it = w >= 0 ? dec_decode(w, p, ro.max_tiles) : DecItem{};
                slot_item[s] = it;  // published to the MMA warp and the epilogue by item_full
                if constexpr (kSel)
                    if (w >= 0) slot_pre[s] = dec_sel_pre(sel, it);
                const int32_t nl = (it.nkt - ro.cr + ro.cc - 1) / ro.cc;  // this CTA's tiles
                item_id[s] = v;
                if (w >= 0 && nl > 0) {
                    mbar_arrive_expect_tx(q_full + 8 * s, kQBytesD);
                    const uint32_t qd = sbase + s * kDecQSlot;
                    tma_load_3d(qd, &tmQ, 0, it.g * G, (int32_t)it.t, q_full + 8 * s);
                    tma_load_3d(qd + kQPanelD, &tmQ, 64, it.g * G, (int32_t)it.t, q_full + 8 * s);
                } else if (w >= 0) {
                    mbar_arrive(q_full + 8 * s);  // no keys: still one phase per use of the slot
                }
                mbar_arrive(item_full + 8 * s);
                if (w < 0) break;
                for (int32_t i = 0; i < nl; ++i, ++kc) {
                    const uint32_t st = kc % kDecStages, ph = (kc / kDecStages) & 1;
                    if (!wait_bar(sy, k_empty + 8 * st, ph ^ 1, 12)) break;
                    const uint32_t dst = sbase + kDecOffK + st * kKStage;
                    const int32_t kt = ro.cc * i + ro.cr;  // the item's tile
                    const int32_t krow = (int32_t)(it.k_start + (int64_t)kt * kBN);
                    mbar_arrive_expect_tx(k_full + 8 * st, kKStage);
                    tma_load_3d(dst, &tmK, 0, it.g, krow, k_full + 8 * st);
                    tma_load_3d(dst + kKPanel, &tmK, 64, it.g, krow, k_full + 8 * st);
                }
                if (*abort_flag) break;
            }
        }
    } else if (warp == kDecMmaWarp) {
        if (lane == 0) {
            uint32_t kc = 0, tc = 0;  // K stages used, TMEM tiles used
            for (uint32_t n = 0;; ++n) {
                const uint32_t s = n % kDecSlots, sph = (n / kDecSlots) & 1;
                if (!wait_bar(sy, item_full + 8 * s, sph, 13)) break;
                const Role ro = role_of<kC>(item_id[s], rank, kTs);
                if (ro.w < 0) break;
                const DecItem it = slot_item[s];
                const int32_t nl = (it.nkt - ro.cr + ro.cc - 1) / ro.cc;
                if (nl <= 0) {
                    mbar_arrive(tmem_full + 8 * s);  // one phase per use of the slot
                    mbar_arrive(item_empty + 8 * s);
                    continue;
                }
                bool ok = wait_bar(sy, q_full + 8 * s, sph, 15);
                tc_fence_after();
                const uint32_t qb = sbase + s * kDecQSlot;
                for (int32_t kt = 0; ok && kt < nl; ++kt, ++kc, ++tc) {
                    const uint32_t st = kc % kDecStages, slot = tc % kTs;
                    ok = wait_bar(sy, slot_empty + 8 * slot, ((tc / kTs) & 1) ^ 1, 14);
                    ok = ok && wait_bar(sy, k_full + 8 * st, (kc / kDecStages) & 1, 16);
                    tc_fence_after();
                    if (!ok) break;
                    const uint32_t kb = sbase + kDecOffK + st * kKStage;
#pragma unroll
                    for (int kk = 0; kk < kD / 16; ++kk) {
                        const uint32_t koff = (kk >> 2) * kKPanel + (kk & 3) * 32;
                        const uint32_t qoff = (kk >> 2) * kQPanelD + (kk & 3) * 32;
                        umma_bf16(tmem + slot * G, desc_kmajor_sw128(kb + koff), desc_kmajor_sw128(qb + qoff),
                                  kIdesc, kk > 0);
                    }
                    umma_commit(k_empty + 8 * st);
                }
                if (!ok) break;
                umma_commit(tmem_full + 8 * s);
                umma_commit(item_empty + 8 * s);  // the q tile is free once the MMAs are done
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        // thread tid = TMEM lane = key tid of every tile; tile kt of an item sits in ring slot
        // (tbase + kt) % kTs, columns slot*G..
        const int tid = threadIdx.x;    // 0..255
        const int key = tid & 127;      // TMEM lane = key within a tile
        const int par = warp >> 2;      // which batches of tiles this warp reads
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const float c = p.c;
        uint32_t tbase = 0;  // TMEM tiles consumed
        uint32_t xn = 0;     // items whose statistics were exchanged with the peer
        for (uint32_t n = 0;; ++n) {
            const uint32_t s = n % kDecSlots;
            const bool bad = !wait_bar(sy, item_full + 8 * s, (n / kDecSlots) & 1, 17);
            if (named_bar_or(kDecEpiBarrier, kDecEpiWarps * 32, bad)) break;  // gave up: all leave
            const Role ro = role_of<kC>(item_id[s], rank, kTs);
            if (ro.w < 0) break;
            const DecItem it = slot_item[s];
            const int32_t nl = (it.nkt - ro.cr + ro.cc - 1) / ro.cc;  // this CTA's tiles
            // the CTA that writes the row's tail and runs the selection: the leader of a
            // shared item, or the CTA that has the item alone
            const bool owner = !ro.joint || rank == 0;
            __nv_bfloat16 *orow = p.out + ((int64_t)it.g * p.T + it.t) * p.out_stride;
            int32_t zero_from = 0;  // first column of the row to zero-fill
            __nv_bfloat16 *srow = reinterpret_cast<__nv_bfloat16 *>(sgen + kDecOffSel + kSelOffRow);
            const uint32_t srow_leader = kPair ? mapa_shared(sbase + kDecOffSel + kSelOffRow, 0) : 0u;
            SelPre pre{};
            if (kSel && owner) {
                pre = slot_pre[s];
                // the histograms, and the row's columns past its tensor-memory tiles that
                // the pooling windows reach (4 * NB <= out_stride)
                int32_t *hist = reinterpret_cast<int32_t *>(sgen + kDecOffSel + kSelOffHist);
                for (int i = threadIdx.x; i < 512; i += kDecEpiWarps * 32) hist[i] = 0;
                if (it.active) {
                    const int32_t z0 = it.nkt * kBN, z1 = 4 * sel.NB;
                    for (int32_t j = z0 + (int32_t)threadIdx.x; j < z1; j += kDecEpiWarps * 32)
                        srow[j] = __float2bfloat16_rn(0.f);
                }
            }
            if (it.active && it.nkt > 0) {
                // TMEM reads in batches of kTB tiles (64 columns); local tile i of this CTA is
                // the item's tile kC*i + rank, key column col(i)
                constexpr int kTB = 64 / G;
                float vb[kTB][G], m[G], l[G];
                auto col = [&](int32_t i) { return (ro.cc * i + ro.cr) * kBN + key; };
                auto load_batch = [&](int32_t kt0) {
#pragma unroll
                    for (int b = 0; b < kTB; ++b)
                        if (kt0 + b < nl)
                            tmem_ld_cols<G>(tmem + lane_base + ((tbase + kt0 + b) % kTs) * G, vb[b]);
                    tmem_wait_ld();
                };
                const uint32_t xph = xn & 1;
                const bool bad2 = !wait_bar(sy, tmem_full + 8 * s, (n / kDecSlots) & 1, 18);
                if (named_bar_or(kDecEpiBarrier, kDecEpiWarps * 32, bad2)) break;
                tc_fence_after();
#pragma unroll
                for (int i = 0; i < G; ++i) m[i] = -INFINITY;
                for (int32_t kt0 = par * kTB; kt0 < nl; kt0 += 2 * kTB) {
                    load_batch(kt0);
#pragma unroll
                    for (int b = 0; b < kTB; ++b) {
                        if (col(kt0 + b) < it.vis) {
#pragma unroll
                            for (int i = 0; i < G; ++i) m[i] = fmaxf(m[i], vb[b][i]);
                        }
                    }
                }
                // keys past the tensor-memory tiles (an out_stride below the sequence's key
                // count): into the statistics only, on CUDA cores
                const uint8_t *qtile = sgen + s * kDecQSlot;
                for (int32_t j = it.nkt * kBN + tid; owner && j < it.vis; j += kDecEpiWarps * 32) {
#pragma unroll
                    for (int h0 = 0; h0 < G; h0 += 8) {
                        float sc[8];
                        dec_extra_scores8<G>(p, qtile, it.g, it.k_start, j, h0, sc);
#pragma unroll
                        for (int i = 0; i < 8; ++i) m[h0 + i] = fmaxf(m[h0 + i], sc[i]);
                    }
                }
                dec_reduce<G, true>(m, red, warp, lane);
                if (kPair && ro.joint) {  // the pair's max: this CTA's and the peer's
                    if (tid == 0) {
                        const uint32_t rx = mapa_shared(pbase + kPairX, rank ^ 1u);
#pragma unroll
                        for (int i = 0; i < G; ++i) st_cluster_f32(rx + 4 * i, m[i]);
                        mbar_arrive_remote(mapa_shared(x_full, rank ^ 1u));
                    }
                    const bool bx = !wait_bar<true>(sy, x_full, xph, 20);
                    if (named_bar_or(kDecEpiBarrier, kDecEpiWarps * 32, bx)) break;
#pragma unroll
                    for (int i = 0; i < G; ++i) m[i] = fmaxf(m[i], xbuf[i]);
                }
#pragma unroll
                for (int i = 0; i < G; ++i) l[i] = 0.f;
                for (int32_t kt0 = par * kTB; kt0 < nl; kt0 += 2 * kTB) {
                    load_batch(kt0);
#pragma unroll
                    for (int b = 0; b < kTB; ++b) {
                        if (col(kt0 + b) < it.vis) {
#pragma unroll
                            for (int i = 0; i < G; ++i) l[i] += ex2((vb[b][i] - m[i]) * c);
                        }
                    }
                }
                for (int32_t j = it.nkt * kBN + tid; owner && j < it.vis; j += kDecEpiWarps * 32) {
#pragma unroll
                    for (int h0 = 0; h0 < G; h0 += 8) {
                        float sc[8];
                        dec_extra_scores8<G>(p, qtile, it.g, it.k_start, j, h0, sc);
#pragma unroll
                        for (int i = 0; i < 8; ++i) l[h0 + i] += ex2((sc[i] - m[h0 + i]) * c);
                    }
                }
                dec_reduce<G, false>(l, red + (kDecEpiWarps + 1) * 32, warp, lane);
                if (kPair && ro.joint) {  // the pair's sum (both halves taken against the pair's max)
                    if (tid == 0) {
                        const uint32_t rx = mapa_shared(pbase + kPairX + 128, rank ^ 1u);
#pragma unroll
                        for (int i = 0; i < G; ++i) st_cluster_f32(rx + 4 * i, l[i]);
                        mbar_arrive_remote(mapa_shared(x_full + 8, rank ^ 1u));
                    }
                    const bool bx = !wait_bar<true>(sy, x_full + 8, xph, 21);
                    if (named_bar_or(kDecEpiBarrier, kDecEpiWarps * 32, bx)) break;
#pragma unroll
                    for (int i = 0; i < G; ++i) l[i] += xbuf[32 + i];
                }
#pragma unroll
                for (int i = 0; i < G; ++i) m[i] = fmaf(m[i], c, log2f(l[i]));  // b = m*c + log2(l)
                for (int32_t kt0 = par * kTB; kt0 < nl; kt0 += 2 * kTB) {
                    load_batch(kt0);
                    // this warp's last read of these tiles: their slots may take new tiles
                    tc_fence_before();
                    __syncwarp();
                    if (lane < kTB && kt0 + lane < nl) mbar_arrive(slot_empty + 8 * ((tbase + kt0 + lane) % kTs));
#pragma unroll
                    for (int b = 0; b < kTB; ++b) {
                        const int32_t j = col(kt0 + b);
                        if (kt0 + b >= nl) break;
                        float o = 0.f;
                        if (j < it.vis) {
#pragma unroll
                            for (int i = 0; i < G; ++i) o += ex2(fmaf(vb[b][i], c, -m[i]));
                            o = fmaxf(o, 0.f);  // NaN scores give 0, as in the tile kernel
                        }
                        if (j < p.out_stride) {
                            const __nv_bfloat16 ob = __float2bfloat16_rn(o);
                            if (p.out) orow[j] = ob;
                            if constexpr (kSel) {
                                if (owner) srow[j] = ob;
                                else st_cluster_u16(srow_leader + 2 * j, __bfloat16_as_ushort(ob));
                            }
                        }
                    }
                }
                if (kPair && kSel && !owner) mbar_arrive_remote(mapa_shared(row_full, 0));
                named_bar_sync(kDecEpiBarrier, kDecEpiWarps * 32);  // every thread has read item_id[s]
                tbase += (uint32_t)nl;
                zero_from = it.nkt * kBN;
            } else {
                named_bar_sync(kDecEpiBarrier, kDecEpiWarps * 32);  // every thread has read item_id[s]
            }
            if (tid == 0) mbar_arrive(item_empty + 8 * s);
            const bool exchanged = ro.joint && it.active && it.nkt > 0;
            if (exchanged) ++xn;
            if (!owner) continue;  // the leader writes the row's tail and runs the selection
            if (kPair && kSel && exchanged) {  // the peer's columns have landed in srow
                const bool br = !wait_bar<true>(sy, row_full, (xn - 1) & 1, 22);
                if (named_bar_or(kDecEpiBarrier, kDecEpiWarps * 32, br)) break;
            }
            if (p.out && it.active && zero_from < p.out_stride) {
                const int32_t n16 = (int32_t)((p.out_stride - zero_from) >> 3);
                uint4 *dst = reinterpret_cast<uint4 *>(orow + zero_from);
                for (int32_t e = tid; e < n16; e += kDecEpiWarps * 32) dst[e] = make_uint4(0u, 0u, 0u, 0u);
            }
            if constexpr (kSel) dec_select(p, sel, it, pre, sgen + kDecOffSel, tid, warp, lane);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kDecMmaWarp) {
        if (*abort_flag) {
            // give TMA/UMMA work already in flight time to land before TMEM is released
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < 2000000ull) {
            }
        }
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if constexpr (kPair) {
        __syncthreads();
        cluster_sync();  // neither CTA leaves while the other may still write into it
    }
}

template <int G, bool kSel, int kC>
int launch_decode(const CUtensorMap &mq, const CUtensorMap &mk, const Params &p, const DecSel &sel,
                  cudaStream_t s) {
    auto kern = stage1_decode_kernel<G, kSel, kC>;
    constexpr uint32_t smem = kSel ? kDecSmemBytesSel : (kC == 2 ? kDecSmemBytesPair : kDecSmemBytes);
    UNUM_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t items = p.T * p.Hk;
    const int64_t groups = unum::sm_count() / kC;  // CTAs (pairs) taking items
    const int grid = (int)(items < groups ? items : groups) * kC;
    // launched with programmatic stream serialization: its CTAs start while the
    // prologue (the previous launch on the stream) runs, and wait for it in-kernel
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kC;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    UNUM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, mq, mk, p, sel));
    return unum::check_launch("stage1_decode_kernel");
}

}  // namespace

extern "C" size_t unum_stage1_workspace_size(int64_t n_seq) {
    if (n_seq < 0) n_seq = 0;
    return (size_t)(((kWsTiles + n_seq + 1) * 4 + 15) / 16 * 16);
}

namespace {

// Which kernel computes stage 1: the decode kernel for batches of (nearly) one
// query token per sequence when its shape fits (no fused pooling, G of 16 or 32, a
// row's key tiles fit TMEM); otherwise the tile kernel.  UNUM_STAGE1_PATH=tile or
// =decode forces one (where the decode kernel can run), for testing.
bool use_decode_kernel(int64_t G, int64_t T, int64_t n_seq, int64_t out_stride, const void *pooled) {
    const bool fits = pooled == nullptr && (G == 16 || G == 32) &&
                      out_stride <= (int64_t)kBN * ((int64_t)kTmemCols / G);
    if (!fits) return false;
    const char *env = getenv("UNUM_STAGE1_PATH");
    if (env && strcmp(env, "tile") == 0) return false;
    if (env && strcmp(env, "decode") == 0) return true;
    return T <= 4 * n_seq;
}

// How the decode kernel spreads items over SMs: the first joint_items items are shared
// by a CTA pair (a cluster of two streams an item at about twice the rate of one SM),
// the rest get one CTA each; -1: no pairs.
//  - items <= SMs/2: every item shared;
//  - SMs/2 < items <= SMs: the first SMs - items items shared, so all items still start
//    in one round (shared ones take two SMs, the others one); a caller that orders its
//    batch longest first gets its longest items shared;
//  - more items: one CTA per item (pairs measured slower there: sharing costs SM time a
//    batch of many items needs).
// UNUM_DECODE_PAIRS=0|1 and UNUM_DECODE_JOINT_ITEMS=n force the choice, for testing.
int64_t decode_joint_items(int64_t items) {
    const char *env = getenv("UNUM_DECODE_PAIRS");
    const char *ji = getenv("UNUM_DECODE_JOINT_ITEMS");
    const int64_t forced = ji ? (int64_t)atoll(ji) : -1;
    if (env && env[0] == '0') return -1;
    if (env && env[0] == '1') return forced >= 0 ? forced : items;
    const int64_t sms = unum::sm_count();
    if (2 * items <= sms) return forced >= 0 ? forced : items;
    if (items <= sms) return forced >= 0 ? forced : sms - items;
    return -1;
}

int stage1_run(const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st, int64_t q_sh,
               const void *k, int64_t Tk, int64_t Hk, int64_t k_st, int64_t k_sh,
               const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k, int64_t n_seq,
               float softmax_scale, int causal, void *out, int64_t out_stride, void *workspace,
               size_t workspace_bytes, void *stream, void *pooled, int64_t NB, int64_t init_blocks,
               int64_t local_blocks, int64_t t_begin = 0, int64_t t_end = INT64_MAX,
               const DecSel *sel = nullptr) {
    UNUM_CHECK_ARG(T >= 0 && Tk >= 0 && Hq > 0 && Hk > 0 && n_seq >= 0 && out_stride >= 0,
                   "bad sizes");
    UNUM_CHECK_ARG(Hq % Hk == 0, "n_heads (%lld) must be a multiple of n_kv_heads (%lld)",
                   (long long)Hq, (long long)Hk);
    if (T == 0 || out_stride == 0) return UNUM_OK;
    if (D != kD) {
        unum::set_error("head_dim %lld not supported (only 128)", (long long)D);
        return UNUM_ERR_UNSUPPORTED;
    }
    const int64_t G = Hq / Hk;
    if (!(G == 2 || G == 4 || G == 8 || G == 16 || G == 32)) {
        unum::set_error("head group size %lld not supported (2,4,8,16,32)", (long long)G);
        return UNUM_ERR_UNSUPPORTED;
    }
    UNUM_CHECK_ARG(out_stride % 128 == 0, "out_stride must be a multiple of 128");
    UNUM_CHECK_ARG(q && (out || pooled || sel) && cu_seqlens_q && cu_seqlens_k, "null pointer argument");
    UNUM_CHECK_ARG(unum::aligned16(out), "out must be 16-byte aligned");
    UNUM_CHECK_ARG(T < (int64_t)1 << 31 && Tk < (int64_t)1 << 31, "too many tokens");
    if (!workspace || workspace_bytes < unum_stage1_workspace_size(n_seq)) {
        unum::set_error("workspace of %zu bytes needed", unum_stage1_workspace_size(n_seq));
        return UNUM_ERR_WORKSPACE;
    }
    cudaStream_t s = (cudaStream_t)stream;
    int32_t *ws = (int32_t *)workspace;
    const int QT = (int)(kRows / G);
    // test hook: UNUM_STAGE1_FORCE_EXPIRY=1 makes the main kernel take its expiry
    // path (status 30, output invalid) without waiting, to exercise the drain
    const char *fe = getenv("UNUM_STAGE1_FORCE_EXPIRY");
    const int32_t force_expiry = (fe && fe[0] == '1') ? 1 : 0;
    stage1_prologue<<<1, 1024, 0, s>>>(cu_seqlens_q, (int32_t)n_seq, QT, ws,
                                       (__nv_bfloat16 *)out, T, (int32_t)Hk, out_stride,
                                       (__nv_bfloat16 *)pooled, (int32_t)NB, (int32_t)init_blocks,
                                       (int32_t)local_blocks);
    if (int rc = unum::check_launch("stage1_prologue")) return rc;
    if (n_seq == 0) return UNUM_OK;
    if (Tk == 0 && pooled) {
        unum::set_error("fused pooling needs at least one compressed key");
        return UNUM_ERR_UNSUPPORTED;
    }
    if (Tk == 0 && out) {  // no compressed keys anywhere: every row is zero
        UNUM_CHECK_CUDA(cudaMemsetAsync(out, 0, (size_t)Hk * T * out_stride * 2, s));
        return UNUM_OK;
    }
    UNUM_CHECK_ARG(k != nullptr, "null k");
    UNUM_CHECK_ARG(unum::aligned16(q) && unum::aligned16(k), "q and k must be 16-byte aligned");
    UNUM_CHECK_ARG(q_st % 8 == 0 && q_sh % 8 == 0 && k_st % 8 == 0 && k_sh % 8 == 0,
                   "q/k strides must be multiples of 8 elements");
    CUtensorMap mq, mk;
    if (int rc = make_map(&mq, q, (uint64_t)D, (uint64_t)Hq, (uint64_t)T, (uint64_t)q_sh * 2,
                          (uint64_t)q_st * 2, (uint32_t)G, (uint32_t)QT))
        return rc;
    if (int rc = make_map(&mk, k, (uint64_t)D, (uint64_t)Hk, (uint64_t)Tk, (uint64_t)k_sh * 2,
                          (uint64_t)k_st * 2, 1, kBN))
        return rc;
    if (sel || use_decode_kernel(G, T, n_seq, out_stride, pooled)) {
        CUtensorMap mqd;  // q with one token's G heads per box
        if (int rc = make_map(&mqd, q, (uint64_t)D, (uint64_t)Hq, (uint64_t)T, (uint64_t)q_sh * 2,
                              (uint64_t)q_st * 2, (uint32_t)G, 1))
            return rc;
        Params p;
        p.cu_q = cu_seqlens_q;
        p.cu_k = cu_seqlens_k;
        p.ws = ws;
        p.out = (__nv_bfloat16 *)out;
        p.T = T;
        p.out_stride = out_stride;
        p.n_seq = (int32_t)n_seq;
        p.Hk = (int32_t)Hk;
        p.causal = causal ? 1 : 0;
        p.c = softmax_scale * kLog2e;
        p.pooled = nullptr;
        p.NB = 0;
        p.init_blocks = 0;
        p.local_blocks = 0;
        p.t_begin = t_begin;
        p.t_end = t_end;
        p.k = (const __nv_bfloat16 *)k;
        p.k_st = k_st;
        p.k_sh = k_sh;
        p.force_expiry = force_expiry;
        p.joint_items = decode_joint_items(T * Hk);
        const bool pair = p.joint_items >= 0;
        if (sel) {
            if (pair)
                return G == 16 ? launch_decode<16, true, 2>(mqd, mk, p, *sel, s)
                               : launch_decode<32, true, 2>(mqd, mk, p, *sel, s);
            return G == 16 ? launch_decode<16, true, 1>(mqd, mk, p, *sel, s)
                           : launch_decode<32, true, 1>(mqd, mk, p, *sel, s);
        }
        const DecSel none{};
        if (pair)
            return G == 16 ? launch_decode<16, false, 2>(mqd, mk, p, none, s)
                           : launch_decode<32, false, 2>(mqd, mk, p, none, s);
        return G == 16 ? launch_decode<16, false, 1>(mqd, mk, p, none, s)
                       : launch_decode<32, false, 1>(mqd, mk, p, none, s);
    }
    CUtensorMap mo;  // out as a 2-D [Hk*T, out_stride] bf16 tensor, [64/G x 128] store boxes
    memset(&mo, 0, sizeof(mo));
    if (out) {
        auto enc = get_encode_fn();
        cuuint64_t gdim[2] = {(cuuint64_t)out_stride, (cuuint64_t)(Hk * T)};
        cuuint64_t gstride[1] = {(cuuint64_t)out_stride * 2};
        cuuint32_t box[2] = {kBN, (cuuint32_t)(64 / G)};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&mo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, gdim, gstride, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            unum::set_error("cuTensorMapEncodeTiled (out) failed (%d)", (int)r);
            return UNUM_ERR_CUDA;
        }
    }
    Params p;
    p.cu_q = cu_seqlens_q;
    p.cu_k = cu_seqlens_k;
    p.ws = ws;
    p.out = (__nv_bfloat16 *)out;
    p.T = T;
    p.out_stride = out_stride;
    p.n_seq = (int32_t)n_seq;
    p.Hk = (int32_t)Hk;
    p.causal = causal ? 1 : 0;
    p.c = softmax_scale * kLog2e;
    p.pooled = (__nv_bfloat16 *)pooled;
    p.NB = (int32_t)NB;
    p.init_blocks = (int32_t)init_blocks;
    p.local_blocks = (int32_t)local_blocks;
    p.t_begin = t_begin;
    p.t_end = t_end;
    p.k = (const __nv_bfloat16 *)k;
    p.k_st = k_st;
    p.k_sh = k_sh;
    p.force_expiry = force_expiry;
    p.joint_items = 0;
    switch (G) {
        case 2: return launch_main<2>(mq, mk, mo, p, T, s);
        case 4: return launch_main<4>(mq, mk, mo, p, T, s);
        case 8: return launch_main<8>(mq, mk, mo, p, T, s);
        case 16: return launch_main<16>(mq, mk, mo, p, T, s);
        default: return launch_main<32>(mq, mk, mo, p, T, s);
    }
}

}  // namespace

extern "C" int unum_infllmv2_attn_stage1(const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st,
                                         int64_t q_sh, const void *k, int64_t Tk, int64_t Hk,
                                         int64_t k_st, int64_t k_sh, const int32_t *cu_seqlens_q,
                                         const int32_t *cu_seqlens_k, int64_t n_seq,
                                         float softmax_scale, int causal, void *out,
                                         int64_t out_stride, void *workspace,
                                         size_t workspace_bytes, void *stream) {
    unum::clear_error();
    return stage1_run(q, T, Hq, D, q_st, q_sh, k, Tk, Hk, k_st, k_sh, cu_seqlens_q, cu_seqlens_k,
                      n_seq, softmax_scale, causal, out, out_stride, workspace, workspace_bytes,
                      stream, nullptr, 0, 0, 0);
}

extern "C" int unum_infllmv2_attn_stage1_pooled(
    const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st, int64_t q_sh, const void *k,
    int64_t Tk, int64_t Hk, int64_t k_st, int64_t k_sh, const int32_t *cu_seqlens_q,
    const int32_t *cu_seqlens_k, int64_t n_seq, float softmax_scale, int causal, void *out,
    int64_t out_stride, void *pooled, int64_t NB, int64_t init_blocks, int64_t local_blocks,
    void *workspace, size_t workspace_bytes, void *stream) {
    unum::clear_error();
    UNUM_CHECK_ARG(pooled != nullptr && NB > 0, "pooled output required");
    UNUM_CHECK_ARG(NB < (int64_t)1 << 30 && init_blocks >= -(1 << 30) && init_blocks < (1 << 30) &&
                       local_blocks >= -(1 << 30) && local_blocks < (1 << 30),
                   "pooling parameters out of range");
    if (Hk <= 0 || Hq % Hk != 0 || Hq / Hk < 16) {
        unum::set_error("fused pooling needs a head group of at least 16 (got %lld/%lld)",
                        (long long)Hq, (long long)Hk);
        return UNUM_ERR_UNSUPPORTED;
    }
    return stage1_run(q, T, Hq, D, q_st, q_sh, k, Tk, Hk, k_st, k_sh, cu_seqlens_q, cu_seqlens_k,
                      n_seq, softmax_scale, causal, out, out_stride, workspace, workspace_bytes,
                      stream, pooled, NB, init_blocks, local_blocks);
}

extern "C" int unum_block_select_decode(
    const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st, int64_t q_sh, const void *k,
    int64_t Tk, int64_t Hk, int64_t k_st, int64_t k_sh, const int32_t *cu_seqlens_q,
    const int32_t *cu_seqlens_k, const int32_t *cache_lens, int64_t n_seq, float softmax_scale,
    int causal, void *out, int64_t out_stride, void *pooled, int64_t NB, int64_t init_blocks,
    int64_t local_blocks, int32_t *topk_idx, int64_t K, int32_t *slots, const int32_t *block_table,
    int64_t B, int64_t L, int64_t bt_stride, const int32_t *token_to_bs, const int32_t *token_pos_in_bs,
    int pos_is_scalar, const int32_t *seqlen_q, int seqlen_is_scalar, int32_t head_group,
    void *workspace, size_t workspace_bytes, void *stream) {
    unum::clear_error();
    UNUM_CHECK_ARG(Hk > 0 && Hq > 0 && Hq % Hk == 0, "n_heads must be a multiple of n_kv_heads");
    const int64_t G = Hq / Hk;
    if (!(G == 16 || G == 32) || D != kD || n_seq <= 0 || Tk <= 0 ||
        out_stride > (int64_t)kBN * ((int64_t)kTmemCols / G)) {
        unum::set_error("fused decode selection needs G in {16, 32}, head_dim 128, at least one "
                        "sequence and compressed key, and out_stride <= %lld",
                        (long long)(kBN * (kTmemCols / (G > 0 ? G : 1))));
        return UNUM_ERR_UNSUPPORTED;
    }
    if (NB <= 0 || NB > kSelNBMax || 4 * NB > out_stride || K <= 0 || K > kSelKMax) {
        unum::set_error("fused decode selection needs 0 < NB, 4 * NB <= out_stride (the pooling "
                        "windows inside the row) and 0 < K <= %d", (int)kSelKMax);
        return UNUM_ERR_UNSUPPORTED;
    }
    UNUM_CHECK_ARG(init_blocks >= -(1 << 30) && init_blocks < (1 << 30) && local_blocks >= -(1 << 30) &&
                       local_blocks < (1 << 30),
                   "pooling parameters out of range");
    UNUM_CHECK_ARG(topk_idx != nullptr, "topk_idx output required");
    if (slots) {
        UNUM_CHECK_ARG(block_table && token_to_bs && token_pos_in_bs && seqlen_q && B > 0 && L > 0 &&
                           L <= (int64_t)INT32_MAX && B <= (int64_t)INT32_MAX && bt_stride >= L,
                       "slots need a non-empty block table and the token maps");
        UNUM_CHECK_ARG(unum::aligned16(slots), "slots must be 16-byte aligned");
    }
    DecSel sel{};
    sel.cache_lens = cache_lens;
    sel.pooled = (__nv_bfloat16 *)pooled;
    sel.topk = topk_idx;
    sel.slots = slots;
    sel.table = block_table;
    sel.tok_bs = token_to_bs;
    sel.tok_pos = token_pos_in_bs;
    sel.seqlen = seqlen_q;
    sel.bt_stride = bt_stride;
    sel.B = (int32_t)B;
    sel.L = (int32_t)L;
    sel.pos_scalar = pos_is_scalar ? 1 : 0;
    sel.seqlen_scalar = seqlen_is_scalar ? 1 : 0;
    sel.head_group = (uint32_t)head_group;
    sel.NB = (int32_t)NB;
    sel.K = (int32_t)K;
    sel.init_blocks = (int32_t)init_blocks;
    sel.local_blocks = (int32_t)local_blocks;
    sel.vec_ok = unum::aligned16(block_table) && (bt_stride % 4 == 0);
    return stage1_run(q, T, Hq, D, q_st, q_sh, k, Tk, Hk, k_st, k_sh, cu_seqlens_q, cu_seqlens_k,
                      n_seq, softmax_scale, causal, out, out_stride, workspace, workspace_bytes,
                      stream, nullptr, 0, 0, 0, 0, INT64_MAX, &sel);
}

extern "C" int unum_stage1_status(const void *workspace, void *stream, int32_t *status_out) {
    unum::clear_error();
    UNUM_CHECK_ARG(workspace && status_out, "null pointer argument");
    cudaStream_t s = (cudaStream_t)stream;
    UNUM_CHECK_CUDA(cudaMemcpyAsync(status_out, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    UNUM_CHECK_CUDA(cudaStreamSynchronize(s));
    return UNUM_OK;
}

extern "C" int unum_infllmv2_attn_stage1_window(
    const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st, int64_t q_sh, const void *k,
    int64_t Tk, int64_t Hk, int64_t k_st, int64_t k_sh, const int32_t *cu_seqlens_q,
    const int32_t *cu_seqlens_k, int64_t n_seq, float softmax_scale, int causal, void *out,
    int64_t out_stride, void *pooled, int64_t NB, int64_t init_blocks, int64_t local_blocks,
    int64_t t_begin, int64_t t_end, void *workspace, size_t workspace_bytes, void *stream) {
    unum::clear_error();
    UNUM_CHECK_ARG(t_begin >= 0 && t_end >= t_begin, "bad token window [%lld, %lld)",
                   (long long)t_begin, (long long)t_end);
    if (pooled) {
        UNUM_CHECK_ARG(NB > 0 && NB < (int64_t)1 << 30, "pooled output needs 0 < NB < 2^30");
        if (Hk <= 0 || Hq % Hk != 0 || Hq / Hk < 16) {
            unum::set_error("fused pooling needs a head group of at least 16");
            return UNUM_ERR_UNSUPPORTED;
        }
    }
    return stage1_run(q, T, Hq, D, q_st, q_sh, k, Tk, Hk, k_st, k_sh, cu_seqlens_q, cu_seqlens_k,
                      n_seq, softmax_scale, causal, out, out_stride, workspace, workspace_bytes,
                      stream, pooled, pooled ? NB : 0, init_blocks, local_blocks, t_begin, t_end);
}

// ------------------------------------------------------------------ allocation-free variant
// Some callers cannot allocate device memory at the point where they run
// stage 1: an inference engine whose allocator has carved up all of HBM up
// front, a plugin host that forbids cudaMalloc inside its callbacks, or code
// running where an allocation would synchronise the device.  For them the
// schedule scratch lives in this fixed, library-owned array instead of a
// caller-supplied workspace.  Every GPU that loads the library keeps it
// (64 KB) until the process exits.
#include <mutex>

namespace {

constexpr int64_t kNoAllocMaxSeqs = 16379;  // (4 + 16379 + 1) * 4 bytes = the whole array
constexpr size_t kNoAllocBytes = 65536;
static __device__ __align__(256) int32_t g_stage1_scratch[kNoAllocBytes / 4];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_stage1_scratch on the current device (looked up once per
// device; host code cannot use the symbol itself as a device pointer).  The
// address is cached for the life of the process: after cudaDeviceReset (or
// any other teardown of the device's primary context) the module may load at
// another address, so these entry points must not be used across a reset.
int scratch_for_current_device(void **out) {
    int dev = 0;
    UNUM_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        unum::set_error("device index %d out of range", dev);
        return UNUM_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        UNUM_CHECK_CUDA(cudaGetSymbolAddress(&p, g_stage1_scratch));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return UNUM_OK;
}

}  // namespace

extern "C" int unum_infllmv2_attn_stage1_noalloc(const void *q, int64_t T, int64_t Hq, int64_t D,
                                                 int64_t q_st, int64_t q_sh, const void *k,
                                                 int64_t Tk, int64_t Hk, int64_t k_st, int64_t k_sh,
                                                 const int32_t *cu_seqlens_q,
                                                 const int32_t *cu_seqlens_k, int64_t n_seq,
                                                 float softmax_scale, int causal, void *out,
                                                 int64_t out_stride, void *stream) {
    unum::clear_error();
    if (n_seq < 0 || n_seq > kNoAllocMaxSeqs) {
        unum::set_error("unum_infllmv2_attn_stage1_noalloc supports at most %lld sequences per "
                        "call (got %lld); use unum_infllmv2_attn_stage1 with a workspace",
                        (long long)kNoAllocMaxSeqs, (long long)n_seq);
        return UNUM_ERR_INVALID;
    }
    void *scratch = nullptr;
    if (int rc = scratch_for_current_device(&scratch)) return rc;
    // The prologue kernel rewrites the status word and the whole tile prefix
    // on every call, so nothing left from an earlier call is read.
    return unum_infllmv2_attn_stage1(q, T, Hq, D, q_st, q_sh, k, Tk, Hk, k_st, k_sh, cu_seqlens_q,
                                     cu_seqlens_k, n_seq, softmax_scale, causal, out, out_stride,
                                     scratch, kNoAllocBytes, stream);
}

// Status word of the last unum_infllmv2_attn_stage1_noalloc call on the current
// device (word 0 of the library's scratch array): the same codes as
// unum_stage1_status.  Reads it with a stream-ordered copy and synchronises the
// stream, so pass the stream the stage-1 call was made on.
extern "C" int unum_stage1_noalloc_status(void *stream, int32_t *status_out) {
    unum::clear_error();
    UNUM_CHECK_ARG(status_out != nullptr, "null pointer argument");
    void *scratch = nullptr;
    if (int rc = scratch_for_current_device(&scratch)) return rc;
    return unum_stage1_status(scratch, stream, status_out);
}
