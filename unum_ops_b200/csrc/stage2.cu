// Stage-2 sparse attention over the selected blocks, with get_block_table's
// gather fused into its loader: the consumer of the block-selection path.
//
// The reference repository has no stage-2 kernel; its get_block_table
// (src/unum_ops/sparse_kernel_extension/get_table_torch.py:4-44) produces the
// per-(token, kv head) physical slot ids such a kernel reads.  Here the slot
// ids are never written: the loader computes them from the top-k block ids and
// the block table (the same rule, get_table_torch.py:29-44) and gathers the key
// and value rows directly.  For token t, kv head g and each of its G = 16
// query heads h:
//     positions p = topk[g,t,k]*64 + i (k < K, i < 64), valid iff topk >= 0,
//     p < seqlen_q[bs] and p < token_pos_in_bs[t] (bs = token_to_bs[t]);
//     slot_p = head_group * block_table[bs, clamp(p, 0, L-1)] + g;
//     out[t,h] = sum_p softmax_p(q[t,h] . k_cache[slot_p] * scale) v_cache[slot_p]
// (0 when no position is valid).
//
// One work item = (token, kv head): up to K*64 = 4096 keys in 128-key tiles.
//   phase 1  the loader warps look up the item's slots once (shared memory),
//            then one thread gathers the key rows with TMA row gathers
//            (tile::gather4: four rows of one 64-column panel per instruction,
//            written in the 128-byte-swizzled UMMA layout; an invalid position
//            reads a row past the cache, which TMA fills with zeros), and the
//            MMA warp computes S^T = K Q^T per
//            tile (M = 128 keys, N = 16 heads) into its own 16 TMEM columns, so
//            all of the item's scores stay in tensor memory (32 tiles x 16 = 512
//            columns);
//   softmax  the epilogue warps (TMEM lane = key) read the scores twice for the
//            per-head max and sum (one cross-lane reduction each per item), then
//            a third time to write P = exp(s - max) / sum as bf16 into shared
//            memory, tile by tile;
//   phase 2  the loaders gather the value rows of each tile and the MMA warp
//            accumulates O^T += V^T P^T (M = 128 dims, A = V MN-major, N = 16
//            heads) into the first tile's TMEM columns, free by then;
//   output   the epilogue reads O^T (lane = dim) and stores bf16 rows.
// Keys and values each cross HBM once; the kernel is bound by that gather
// (2 * 4096 * 256 bytes per item at K = 64).
// Every wait is bounded (about one second); on expiry the kernel records a
// status in `status` (if given), stops issuing work, drains and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "sm100.cuh"

namespace {

using namespace unum::sm100;

// TMA gather of four rows (y0..y3) of a 2-D tensor, columns x..x+63, into four
// consecutive 128-byte rows of shared memory (128-byte swizzle), completion
// counted on `bar`.  No multicast.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const void *tmap, int32_t x, int32_t y0, int32_t y1,
                                            int32_t y2, int32_t y3, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(bar)
        : "memory");
}

constexpr int kD = 128;
constexpr int kG = 16;               // query heads per kv head
constexpr int kTileKeys = 128;
constexpr int kMaxTiles = 32;        // K <= 64 blocks of 64 positions
constexpr int kStages = 5;           // key/value tile ring
constexpr int kLoadWarps = 4;        // one loader thread per key of a tile
constexpr int kEpiWarps = 8;         // two per TMEM lane quarter, alternating tiles
constexpr int kEpi0 = kLoadWarps;    // first epilogue warp
constexpr int kMmaWarp = kEpi0 + kEpiWarps;
constexpr int kThreads = (kMmaWarp + 1) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr int kEpiBar = 1;           // named barrier of the epilogue warps

constexpr uint32_t kPanelKV = kTileKeys * 128;      // one 64-column panel of a K/V tile: 16 KB
constexpr uint32_t kStageKV = 2 * kPanelKV;          // 32 KB
constexpr uint32_t kPanelQ = kG * 128;               // 2 KB
constexpr uint32_t kSlotQ = 2 * kPanelQ;             // 4 KB
constexpr uint32_t kPanelP = kG * 128;               // P^T: 16 heads x 64 keys
constexpr uint32_t kStageP = 2 * kPanelP;            // 4 KB
constexpr uint32_t kOffQ = 0;                        // 2 Q slots
constexpr uint32_t kOffKV = 2 * kSlotQ;              // 8 KB (1024-aligned)
constexpr uint32_t kOffP = kOffKV + kStages * kStageKV;
constexpr uint32_t kOffRed = kOffP + 2 * kStageP;
constexpr uint32_t kOffSlots = kOffRed + 2 * kEpiWarps * 32 * 4;  // [2][32 tiles x 128 keys] int32
constexpr uint32_t kOffBar = kOffSlots + 2 * kMaxTiles * kTileKeys * 4;
// barriers: q_full[2], q_empty[2], kv_full[S], kv_empty[S], s_full, p_full[2], p_empty[2],
// o_full, tmem_free, slot_full[2], slot_free[2]
constexpr uint32_t kNumBars = 4 + 2 * kStages + 1 + 4 + 2 + 4;
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 64 + 1024;
static_assert(kOffKV % 1024 == 0 && kOffP % 1024 == 0, "SW128 tiles need 1024-byte alignment");
static_assert(kSmemBytes <= 232448, "exceeds the 227 KB of shared memory a CTA may use");

constexpr uint32_t kIdescS = idesc_bf16_f32(128, kG);
constexpr uint32_t kIdescO = idesc_bf16_f32_amn(128, kG);
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint64_t kWaitNs = 1000000000ull;

struct Params {
    const __nv_bfloat16 *q;
    int64_t q_st, q_sh;
    const __nv_bfloat16 *kc, *vc;
    int64_t n_slots;
    const int32_t *topk;
    int64_t ts_h, ts_t;
    int32_t K;
    const int32_t *table;
    int64_t bt_stride;
    int32_t L;
    const int32_t *tb, *pos, *seqlen;
    int32_t pos_scalar, seqlen_scalar, head_group;
    int64_t T;
    int32_t Hk;
    float c;  // scale * log2(e)
    __nv_bfloat16 *out;
    int32_t *status;
};

// Slot of key j (0..127) of tile i of item (t, g), or -1 when the position is not valid.
__device__ __forceinline__ int64_t key_slot(const Params &p, int64_t t, int32_t g, int32_t i, int32_t j,
                                            int32_t bs, int32_t lim) {
    const int32_t k = 2 * i + (j >> 6);
    if (k >= p.K) return -1;
    const int32_t blk = __ldg(p.topk + (int64_t)g * p.ts_h + t * p.ts_t + k);
    if (blk < 0) return -1;
    const int64_t pos = (int64_t)blk * 64 + (j & 63);
    if (pos >= lim) return -1;
    const int64_t col = pos > p.L - 1 ? p.L - 1 : pos;
    const int64_t slot = (int64_t)p.head_group * __ldg(p.table + (int64_t)bs * p.bt_stride + col) + g;
    return (slot >= 0 && slot < p.n_slots) ? slot : -1;
}

struct ItemInfo {
    int64_t t;
    int32_t g, bs, lim, nt;
};

__device__ __forceinline__ ItemInfo item_info(const Params &p, int64_t w) {
    ItemInfo it;
    it.t = w / p.Hk;
    it.g = (int32_t)(w % p.Hk);
    it.bs = __ldg(p.tb + it.t);
    const int32_t sl = __ldg(p.seqlen + (p.seqlen_scalar ? 0 : it.bs));
    const int32_t ps = __ldg(p.pos + (p.pos_scalar ? 0 : it.t));
    it.lim = sl < ps ? sl : ps;
    it.nt = (p.K + 1) / 2;
    return it;
}

struct Waits {
    volatile int *abort;
    int32_t *status;
};

__device__ __forceinline__ bool wait_bar(const Waits &s, uint32_t bar, uint32_t parity, int code) {
    if (*s.abort) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*s.abort) return false;
            if (globaltimer_ns() - t0 > kWaitNs) {
                *s.abort = 1;
                if (s.status) atomicCAS(s.status, 0, code);
                return false;
            }
        }
    }
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

// Max (kMax) or sum of each of the 16 per-head values over the 128 keys of the
// epilogue warps (8 warps: each key quarter twice), broadcast to every thread.
template <bool kMax>
__device__ __forceinline__ void reduce16(float (&v)[kG], float *red, int ew, int lane) {
#pragma unroll
    for (int h = 0; h < kG; ++h) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float y = __shfl_xor_sync(0xffffffffu, v[h], o);
            v[h] = kMax ? fmaxf(v[h], y) : v[h] + y;
        }
    }
    if (lane < kG) {
        float x = v[0];
#pragma unroll
        for (int h = 1; h < kG; ++h) x = lane == h ? v[h] : x;
        red[ew * 32 + lane] = x;
    }
    named_bar_sync(kEpiBar, kEpiWarps * 32);
#pragma unroll
    for (int h = 0; h < kG; ++h) {
        float a = red[h];
#pragma unroll
        for (int w = 1; w < kEpiWarps; ++w) a = kMax ? fmaxf(a, red[w * 32 + h]) : a + red[w * 32 + h];
        v[h] = a;
    }
    named_bar_sync(kEpiBar, kEpiWarps * 32);  // red is reused by the next reduction
}

__global__ void __launch_bounds__(kThreads, 1)
stage2_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
              const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t *sgen = smem_raw + (sbase - raw);
    const uint32_t bar0 = sbase + kOffBar;
    const uint32_t q_full = bar0, q_empty = bar0 + 16, kv_full = bar0 + 32, kv_empty = kv_full + 8 * kStages;
    const uint32_t s_full = kv_empty + 8 * kStages, p_full = s_full + 8, p_empty = p_full + 16;
    const uint32_t o_full = p_empty + 16, tmem_free = o_full + 8;
    const uint32_t slot_full = tmem_free + 8, slot_free = slot_full + 16;
    int32_t *slots_s = reinterpret_cast<int32_t *>(sgen + kOffSlots);  // [2][kMaxTiles * 128]
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sgen + kOffMisc);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sgen + kOffMisc + 16);
    float *red = reinterpret_cast<float *>(sgen + kOffRed);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Waits sy{abort_flag, p.status};

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(q_full + 8 * i, kLoadWarps * 32);
            mbar_init(q_empty + 8 * i, 1);
            mbar_init(p_full + 8 * i, 4);  // the 4 epilogue warps that write a tile's P
            mbar_init(p_empty + 8 * i, 1);
            mbar_init(slot_full + 8 * i, kLoadWarps * 32);
            mbar_init(slot_free + 8 * i, kEpiWarps);
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(kv_full + 8 * s, 64);  // the 64 gathering threads' expect_tx
            mbar_init(kv_empty + 8 * s, 1);
        }
        mbar_init(s_full, 1);
        mbar_init(o_full, 1);
        mbar_init(tmem_free, 4);  // the 4 warps that read O
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int64_t n_items = p.T * p.Hk;

    if (warp < kLoadWarps) {
        // ---------------------------------------------------------------- loaders
        const int j = threadIdx.x;  // 0..127
        uint32_t kc_cnt = 0;
        // q and the slots of item w into buffer qn & 1; false when a wait gave up (decided by
        // all loader threads together: one leaving alone would strand the others at a barrier)
        auto prepare = [&](int64_t w, uint32_t qn) -> bool {
            const ItemInfo it = item_info(p, w);
            const uint32_t qs = qn & 1;
            bool bad = !wait_bar(sy, q_empty + 8 * qs, ((qn >> 1) & 1) ^ 1, 41);
            bad = !wait_bar(sy, slot_free + 8 * qs, ((qn >> 1) & 1) ^ 1, 40) || bad;
            if (named_bar_or(2, kLoadWarps * 32, bad)) return false;
            // the token's 16 query heads: 256 chunks of 16 bytes, two per thread
            const uint32_t qdst = sbase + kOffQ + qs * kSlotQ;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int h = j >> 3, ch = (j & 7) * 2 + e;  // head, 16-byte chunk of its 256-byte row
                const __nv_bfloat16 *src = p.q + it.t * p.q_st + (int64_t)(it.g * kG + h) * p.q_sh + ch * 8;
                cp_async16(qdst + (ch >> 3) * kPanelQ + h * 128 + (((ch & 7) ^ (h & 7)) << 4), src, 16);
            }
            cp_async_arrive(q_full + 8 * qs);
            // the slot of key j of every tile, all looked up at once (independent loads) and
            // kept in shared memory for the gathers and the epilogue's masks
            int32_t *my_slots = slots_s + qs * (kMaxTiles * kTileKeys);
#pragma unroll
            for (int32_t i = 0; i < kMaxTiles; ++i)
                if (i < it.nt) my_slots[i * kTileKeys + j] = (int32_t)key_slot(p, it.t, it.g, i, j, it.bs, it.lim);
            mbar_arrive(slot_full + 8 * qs);
            named_bar_sync(2, kLoadWarps * 32);  // every slot of the item is in shared memory
            return true;
        };
        // the key (phase 0) or value (phase 1) tiles of an item: threads 0..63 each gather four
        // rows (row quad j % 32) of one panel (j / 32) per tile
        auto gather = [&](const ItemInfo &it, uint32_t qs, int phase) {
            if (j >= 64) {
                kc_cnt += (uint32_t)it.nt;
                return;
            }
            const int rq = j & 31, panel = j >> 5;
            const int32_t oob = (int32_t)p.n_slots;  // a row past the cache: read as zeros
            const int32_t *my_slots = slots_s + qs * (kMaxTiles * kTileKeys);
            const void *tm = phase == 0 ? (const void *)&tmK : (const void *)&tmV;
            for (int32_t i = 0; i < it.nt; ++i, ++kc_cnt) {
                const uint32_t s = kc_cnt % kStages;
                if (!wait_bar(sy, kv_empty + 8 * s, ((kc_cnt / kStages) & 1) ^ 1, 42)) continue;
                const int4 r = reinterpret_cast<const int4 *>(my_slots + i * kTileKeys)[rq];
                const int32_t y0 = r.x < 0 ? oob : r.x, y1 = r.y < 0 ? oob : r.y;
                const int32_t y2 = r.z < 0 ? oob : r.z, y3 = r.w < 0 ? oob : r.w;
                mbar_arrive_expect_tx(kv_full + 8 * s, 4 * 128);
                tma_gather4(sbase + kOffKV + s * kStageKV + panel * kPanelKV + rq * 512, tm, 64 * panel, y0, y1,
                            y2, y3, kv_full + 8 * s);
            }
        };
        // item n's keys, then the next item's q and slots (their lookups overlap item n's
        // softmax), then item n's values
        uint32_t qn = 0;
        int64_t w = blockIdx.x;
        if (w < n_items && prepare(w, 0)) {
            for (; w < n_items; w += gridDim.x, ++qn) {
                const ItemInfo it = item_info(p, w);
                gather(it, qn & 1, 0);
                const bool ok = w + gridDim.x >= n_items || prepare(w + gridDim.x, qn + 1);
                gather(it, qn & 1, 1);
                if (!ok) break;
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t kc_cnt = 0, qn = 0, pc = 0;
            bool ok = true;
            for (int64_t w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++qn) {
                const ItemInfo it = item_info(p, w);
                const uint32_t qs = qn & 1;
                // the previous item's O has been read: every TMEM column is free
                ok = ok && (qn == 0 || wait_bar(sy, tmem_free, (qn - 1) & 1, 43));
                ok = ok && wait_bar(sy, q_full + 8 * qs, (qn >> 1) & 1, 44);
                tc_fence_after();
                const uint32_t qb = sbase + kOffQ + qs * kSlotQ;
                for (int32_t i = 0; ok && i < it.nt; ++i, ++kc_cnt) {
                    const uint32_t s = kc_cnt % kStages;
                    ok = wait_bar(sy, kv_full + 8 * s, (kc_cnt / kStages) & 1, 45);
                    tc_fence_after();
                    if (!ok) break;
                    const uint32_t kb = sbase + kOffKV + s * kStageKV;
#pragma unroll
                    for (int kk = 0; kk < kD / 16; ++kk) {
                        const uint32_t koff = (kk >> 2) * kPanelKV + (kk & 3) * 32;
                        const uint32_t qoff = (kk >> 2) * kPanelQ + (kk & 3) * 32;
                        umma_bf16(tmem + i * kG, desc_kmajor_sw128(kb + koff), desc_kmajor_sw128(qb + qoff),
                                  kIdescS, kk > 0);
                    }
                    umma_commit(kv_empty + 8 * s);
                }
                if (!ok) break;
                umma_commit(s_full);
                umma_commit(q_empty + 8 * qs);
                // phase 2: O^T (TMEM columns 0..15) += V^T P^T, tile by tile
                for (int32_t i = 0; ok && i < it.nt; ++i, ++kc_cnt, ++pc) {
                    const uint32_t s = kc_cnt % kStages, ps = pc & 1;
                    ok = wait_bar(sy, kv_full + 8 * s, (kc_cnt / kStages) & 1, 46);
                    ok = ok && wait_bar(sy, p_full + 8 * ps, (pc >> 1) & 1, 47);
                    tc_fence_after();
                    if (!ok) break;
                    const uint32_t vb = sbase + kOffKV + s * kStageKV;
                    const uint32_t pb = sbase + kOffP + ps * kStageP;
#pragma unroll
                    for (int kk = 0; kk < kTileKeys / 16; ++kk) {
                        // A = V^T: 16 keys (K) x 128 dims (M), rows of 64 dims, dims 64.. one panel on
                        const uint64_t adesc = desc_mnmajor_sw128(vb + kk * 16 * 128, kPanelKV, 1024);
                        const uint32_t poff = (kk >> 2) * kPanelP + (kk & 3) * 32;
                        umma_bf16(tmem, adesc, desc_kmajor_sw128(pb + poff), kIdescO, (i > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(kv_empty + 8 * s);
                    umma_commit(p_empty + 8 * ps);
                }
                if (!ok) break;
                umma_commit(o_full);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int ew = warp - kEpi0;       // 0..7
        const int par = ew >> 2;            // tiles of this parity
        const int qtr = ew & 3;             // TMEM lane quarter = keys 32*qtr.. of a tile
        const int key = qtr * 32 + lane;
        const uint32_t lane_base = (uint32_t)(qtr * 32) << 16;
        const float c = p.c;
        uint32_t qn = 0, pc0 = 0;
        for (int64_t w = blockIdx.x; w < n_items; w += gridDim.x, ++qn) {
            const ItemInfo it = item_info(p, w);
            const bool bad = !wait_bar(sy, s_full, qn & 1, 48);
            const bool bad1 = !wait_bar(sy, slot_full + 8 * (qn & 1), (qn >> 1) & 1, 51);
            if (named_bar_or(kEpiBar, kEpiWarps * 32, bad || bad1)) break;  // gave up: all epilogue warps leave
            tc_fence_after();
            const int32_t *islots = slots_s + (qn & 1) * (kMaxTiles * kTileKeys);
            float m[kG], l[kG];
#pragma unroll
            for (int h = 0; h < kG; ++h) {
                m[h] = -INFINITY;
                l[h] = 0.f;
            }
            // read 1: per-head maximum over this thread's keys
            for (int32_t i = par; i < it.nt; i += 2) {
                const bool valid = islots[i * kTileKeys + key] >= 0;
                float v[kG];
                tmem_ld16(tmem + lane_base + i * kG, v);  // warp-collective: every lane loads
                tmem_wait_ld();
                if (valid) {
#pragma unroll
                    for (int h = 0; h < kG; ++h) m[h] = fmaxf(m[h], v[h]);
                }
            }
            reduce16<true>(m, red, ew, lane);
            // read 2: per-head sum of exp2((s - max) * c)
            for (int32_t i = par; i < it.nt; i += 2) {
                const bool valid = islots[i * kTileKeys + key] >= 0;
                float v[kG];
                tmem_ld16(tmem + lane_base + i * kG, v);
                tmem_wait_ld();
                if (valid) {
#pragma unroll
                    for (int h = 0; h < kG; ++h) l[h] += ex2((v[h] - m[h]) * c);
                }
            }
            reduce16<false>(l, red + kEpiWarps * 32, ew, lane);
            // b = max*c + log2(sum): P = exp2(s*c - b); no valid key: P = 0
#pragma unroll
            for (int h = 0; h < kG; ++h) m[h] = l[h] > 0.f ? fmaf(m[h], c, log2f(l[h])) : INFINITY;
            // read 3: P^T of each tile as bf16 into its shared-memory stage
            uint32_t pc = pc0 + (uint32_t)par;  // this CTA's running tile count picks the P stage
            for (int32_t i = par; i < it.nt; i += 2, pc += 2) {
                const uint32_t ps = pc & 1;
                const bool bad2 = !wait_bar(sy, p_empty + 8 * ps, ((pc >> 1) & 1) ^ 1, 49);
                if (__any_sync(0xffffffffu, bad2)) break;
                const bool valid = islots[i * kTileKeys + key] >= 0;
                float v[kG];
                tmem_ld16(tmem + lane_base + i * kG, v);
                tmem_wait_ld();
                uint8_t *pt = sgen + kOffP + ps * kStageP + (key >> 6) * kPanelP;
                const int kc16 = (key & 63) >> 3, kin = (key & 7) * 2;
#pragma unroll
                for (int h = 0; h < kG; ++h) {
                    const float pv = valid ? ex2(fmaf(v[h], c, -m[h])) : 0.f;
                    *reinterpret_cast<__nv_bfloat16 *>(pt + h * 128 + ((kc16 ^ (h & 7)) << 4) + kin) =
                        __float2bfloat16_rn(pv);
                }
                fence_async_shared();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full + 8 * ps);
            }
            pc0 += (uint32_t)it.nt;
            // output: O^T in TMEM columns 0..15, lane = dim
            if (par == 0) {
                const bool bad3 = !wait_bar(sy, o_full, qn & 1, 50);
                if (!__any_sync(0xffffffffu, bad3)) {
                    tc_fence_after();
                    float o[kG];
                    tmem_ld16(tmem + lane_base, o);
                    tmem_wait_ld();
                    __nv_bfloat16 *orow = p.out + (it.t * (int64_t)p.Hk * kG + (int64_t)it.g * kG) * kD + key;
#pragma unroll
                    for (int h = 0; h < kG; ++h) orow[h * kD] = __float2bfloat16_rn(o[h]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tmem_free);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(slot_free + 8 * (qn & 1));  // this item's masks are no longer read
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        if (*abort_flag) {
            // give copies and UMMA work already in flight time to land before TMEM is released
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < 2000000ull) {
            }
        }
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// [n_slots, 128] bf16 rows, 256-byte row stride, gathered one 64-column panel x one
// row per box (the box of a tile::gather4 load is one row high), 128-byte swizzle.
int make_rows_map(CUtensorMap *m, const void *base, int64_t n_slots) {
    auto enc = encode_fn();
    if (!enc) {
        unum::set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return UNUM_ERR_CUDA;
    }
    cuuint64_t gdim[2] = {(cuuint64_t)kD, (cuuint64_t)n_slots};
    cuuint64_t gstride[1] = {(cuuint64_t)kD * 2};
    cuuint32_t box[2] = {64, 1};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), gdim, gstride, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        unum::set_error("cuTensorMapEncodeTiled (kv cache) failed (%d)", (int)r);
        return UNUM_ERR_CUDA;
    }
    return UNUM_OK;
}

}  // namespace

extern "C" int unum_sparse_attn_blocks(const void *q, int64_t T, int64_t Hq, int64_t D, int64_t q_st,
                                       int64_t q_sh, const void *k_cache, const void *v_cache,
                                       int64_t n_slots, int64_t Hk, const int32_t *topk_idx, int64_t K,
                                       int64_t ts_h, int64_t ts_t, const int32_t *block_table, int64_t B,
                                       int64_t L, int64_t bt_stride, const int32_t *token_to_bs,
                                       const int32_t *token_pos_in_bs, int pos_is_scalar,
                                       const int32_t *seqlen_q, int seqlen_is_scalar, int32_t head_group,
                                       float softmax_scale, void *out, int32_t *status, void *stream) {
    unum::clear_error();
    UNUM_CHECK_ARG(T >= 0 && Hq > 0 && Hk > 0 && K >= 0 && B >= 0 && L > 0 && n_slots >= 0, "bad sizes");
    if (T == 0) return UNUM_OK;
    if (D != kD || Hq != Hk * kG) {
        unum::set_error("sparse attention supports head_dim 128 and 16 query heads per kv head "
                        "(got head_dim %lld, %lld/%lld heads)", (long long)D, (long long)Hq, (long long)Hk);
        return UNUM_ERR_UNSUPPORTED;
    }
    UNUM_CHECK_ARG(K <= 2 * kMaxTiles, "at most %d selected blocks per token (got %lld)", 2 * kMaxTiles,
                   (long long)K);
    UNUM_CHECK_ARG(q && k_cache && v_cache && topk_idx && block_table && token_to_bs && token_pos_in_bs &&
                       seqlen_q && out,
                   "null pointer argument");
    UNUM_CHECK_ARG(unum::aligned16(q) && unum::aligned16(k_cache) && unum::aligned16(v_cache) &&
                       q_st % 8 == 0 && q_sh % 8 == 0,
                   "q, k_cache and v_cache must be 16-byte aligned with strides that are multiples of 8");
    UNUM_CHECK_ARG(T < ((int64_t)1 << 31) / Hk && L < ((int64_t)1 << 31), "too many tokens");
    Params p;
    p.q = (const __nv_bfloat16 *)q;
    p.q_st = q_st;
    p.q_sh = q_sh;
    p.kc = (const __nv_bfloat16 *)k_cache;
    p.vc = (const __nv_bfloat16 *)v_cache;
    p.n_slots = n_slots;
    p.topk = topk_idx;
    p.ts_h = ts_h;
    p.ts_t = ts_t;
    p.K = (int32_t)K;
    p.table = block_table;
    p.bt_stride = bt_stride;
    p.L = (int32_t)L;
    p.tb = token_to_bs;
    p.pos = token_pos_in_bs;
    p.seqlen = seqlen_q;
    p.pos_scalar = pos_is_scalar ? 1 : 0;
    p.seqlen_scalar = seqlen_is_scalar ? 1 : 0;
    p.head_group = head_group;
    p.T = T;
    p.Hk = (int32_t)Hk;
    p.c = softmax_scale * kLog2e;
    p.out = (__nv_bfloat16 *)out;
    p.status = status;
    UNUM_CHECK_ARG(n_slots > 0 && n_slots < ((int64_t)1 << 31), "n_slots must be in [1, 2^31)");
    CUtensorMap mk, mv;
    if (int rc = make_rows_map(&mk, k_cache, n_slots)) return rc;
    if (int rc = make_rows_map(&mv, v_cache, n_slots)) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    if (status) UNUM_CHECK_CUDA(cudaMemsetAsync(status, 0, sizeof(int32_t), s));
    UNUM_CHECK_CUDA(cudaFuncSetAttribute(stage2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSmemBytes));
    const int64_t items = T * Hk;
    const int64_t sms = unum::sm_count();
    const int grid = (int)(items < sms ? items : sms);
    stage2_kernel<<<grid, kThreads, kSmemBytes, s>>>(mk, mv, p);
    return unum::check_launch("stage2_kernel");
}
