// Cross-GPU step signal for exchanges whose data a kernel stored straight into the
// peers' buffers over NVLink (unum_topk_blocks_to_peers): a rank may read its buffer
// once every peer has announced that its stores for this step are done.
//
// Each rank r owns an array of n int32 signal words in peer-mapped memory; word q of
// rank r's array holds the last step (epoch) rank q announced to r.  One thread per
// peer q: a system-scope fence (so this GPU's earlier stores, from earlier kernels on
// the stream included, are visible before the announcement), a release store of the
// epoch into word [rank] of q's array, then an acquire poll of word [q] of this
// rank's own array until q has announced this epoch.  The poll is bounded (about one
// second of %globaltimer); on expiry the kernel records status 40 and returns, and
// the host reads the status instead of the GPU hanging.  No multicast.
#include <cstdint>

#include "common.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr uint64_t kWaitNs = 1000000000ull;

struct Signals {
    int32_t *buf[kMaxRanks];  // rank i's signal array, mapped into this device
    int32_t n, rank, epoch;
    int32_t *status;          // nonzero after a poll gave up (or null)
};

__device__ __forceinline__ uint64_t timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(int32_t *p, int32_t v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t *p) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(32) peer_signal_wait_kernel(const __grid_constant__ Signals s) {
    const int q = threadIdx.x;
    if (q >= s.n) return;
    __threadfence_system();
    st_release_sys(s.buf[q] + s.rank, s.epoch);
    const int32_t *mine = s.buf[s.rank] + q;
    if (ld_acquire_sys(mine) - s.epoch >= 0) return;
    const uint64_t t0 = timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (ld_acquire_sys(mine) - s.epoch >= 0) return;
        if ((i & 255) == 0 && timer_ns() - t0 > kWaitNs) {
            if (s.status) atomicCAS(s.status, 0, 40);
            return;
        }
    }
}

}  // namespace

extern "C" int unum_peer_signal_wait(int32_t *const *signal_bufs, int32_t n_ranks, int32_t rank,
                                     int32_t epoch, int32_t *status, void *stream) {
    unum::clear_error();
    UNUM_CHECK_ARG(signal_bufs != nullptr && n_ranks >= 1 && n_ranks <= kMaxRanks, "1 to %d ranks", kMaxRanks);
    UNUM_CHECK_ARG(rank >= 0 && rank < n_ranks, "rank %d outside [0, %d)", (int)rank, (int)n_ranks);
    Signals s{};
    for (int i = 0; i < n_ranks; ++i) {
        UNUM_CHECK_ARG(signal_bufs[i] != nullptr && ((uintptr_t)signal_bufs[i] & 3) == 0,
                       "signal buffer %d null or misaligned", i);
        s.buf[i] = signal_bufs[i];
    }
    s.n = n_ranks;
    s.rank = rank;
    s.epoch = epoch;
    s.status = status;
    peer_signal_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(s);
    return unum::check_launch("peer_signal_wait_kernel");
}
