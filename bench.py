"""Benchmark: InfLLM-v2 block selection at 128k prefill on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: one 131072-token sequence, q [131072, 32, 128]
bf16 ~ N(0,1), compressed keys k_cmp [8191, 2, 128] bf16 ~ N(0,1), causal.
One step is the whole path as unum_ops_b200.block_select runs it: stage 1
with max_pooling_1d_varlen (block 64, stride 16, 1 init + 2 local blocks)
fused into its epilogue -> top-64 -> get_block_table with a per-token block
table [1, 131072] (a random permutation).  The four separate reference-API
calls are also timed, as context (`kernels_api_path`).  Inputs and
outputs (q 1.07 GB, scores 4.3 GB, slots 4.3 GB) are far larger than the
126 MB L2, so no explicit flush is needed between steps.

Multi-GPU (torchrun, one process per GPU), config 3's sharding: the one
128k sequence is split into kv head x query range shards (ranges of equal
stage-1 plus per-token work); each rank computes its shard with no exchange,
then the top-k ids are all-gathered (NCCL) inside the step.  The step time is
the max over ranks, value = 131072 tokens / step time (strong scaling).
--scaling weak gives every rank its own sequence instead.

--impl reference times the reference's CPU path on this host, with all host
threads, on a bounded sample of the same workload (an early and a late token
range): stage 1 and pooling by the C restatement of the reference's kernels,
top-k by torch.topk, get_block_table by the restatement of the reference's
torch function (oracle/, "port").
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L_SEQ = 131072  # tokens of the prefill sequence (--seqlen overrides, for small profiling cases)
HQ, HK, D = 32, 2, 128
NKC = (L_SEQ - 32) // 16 + 1  # 8191 compressed keys
TOPK = 64
INIT_BLOCKS, LOCAL_BLOCKS = 1, 2
METRIC = "block-selection tokens/s at 128k prefill (stage1+pool+topk+get_block_table)"


def visible_counts(L=None, k_len=None):
    L = L_SEQ if L is None else L
    k_len = NKC if k_len is None else k_len
    lq = np.arange(L, dtype=np.int64)
    off = np.trunc((lq - 15) / 16).astype(np.int64) + k_len - (L - 15) // 16
    return np.clip(off, 0, k_len)


def stage1_flops(t_begin=0, t_end=None):
    """Algorithmic work of stage 1 over query rows [t_begin, t_end), all q heads: one
    QK^T pass over the visible pairs."""
    return float(2 * D * HQ * visible_counts()[t_begin:t_end].sum())


def algorithmic_bytes(T=None, nh=HK):
    """Per-kernel algorithmic HBM bytes of one step over T query rows of nh kv heads
    (bf16 scores, int32 ids)."""
    W = (NKC + 127) // 128 * 128
    NB = (L_SEQ + 63) // 64
    T = L_SEQ if T is None else T
    return {
        "pool": nh * T * W * 2 + nh * T * NB * 2,
        "topk": nh * T * NB * 2 + nh * T * TOPK * 4,
        "get_block_table": T * nh * TOPK * 64 * 4 + nh * T * TOPK * 4 + 8 * T + 4 * T,
        "stage1_out": nh * T * W * 2,
    }


MUFU_EX2_PER_CLK_SM = 16  # ex2.approx results per clock per SM, measured on this B200 pool


def mufu_roofline(flops, ms, clocks):
    """Stage 1's second ceiling: its softmax takes two exponentials per visible
    (query head, key) pair (one per pass), flops / D of them, on the MUFU unit."""
    exps = flops / D
    mhz = clocks.get("sm_mhz") or 1965.0
    floor_ms = exps / (MUFU_EX2_PER_CLK_SM * 148 * mhz * 1e6) * 1e3
    return {"exp2_per_launch": exps, "sm_mhz": mhz, "floor_ms": floor_ms, "frac": floor_ms / ms}


def workload_name():
    tag = "C3: 128k-token" if L_SEQ == 131072 else f"{L_SEQ}-token (reduced C3)"
    return (f"{tag} causal prefill, 32 q-heads / 2 kv-heads, d=128, k_cmp {NKC}, "
            f"NB {(L_SEQ + 63) // 64}, top-64, per-token block table [1,{L_SEQ}]")


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), d.get(
            "bf16_tflops_sustained", 1400.0), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def load_traffic():
    """Per-launch DRAM bytes of each kernel from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "traffic_c3.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi clock / throttle sampling (every 50 ms).  Started before the warm-up
    so it is running when the timed region begins; summary() keeps only the samples
    whose timestamps fall inside the timed window [t0, t1] (host wall clock taken
    after the synchronisations that bracket the region)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        out_dir = os.environ.get("UNUM_BENCH_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = os.path.join(out_dir, f"unum_bench_clocks_rank{index}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.fh,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self, t0=None, t1=None):
        import datetime

        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons, kept = [], None, set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                mhz, mx = float(f[2]), float(f[3])
            except ValueError:
                continue
            if t0 is not None and not (t0 - 0.05 <= ts <= t1 + 0.05):
                continue
            kept += 1
            sm.append(mhz)
            smax = mx
            for n, v in zip(names, f[6:10]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": kept}


_JSON_FD = None


def quiet_stdout():
    """Route fd 1 (where NCCL and other libraries print banners) to stderr, keeping
    the original stdout for the one JSON result line."""
    global _JSON_FD
    if _JSON_FD is None:
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)


def emit(line: dict):
    text = json.dumps(line) + "\n"
    if _JSON_FD is not None:
        os.write(_JSON_FD, text.encode())
    else:
        sys.stdout.write(text)
        sys.stdout.flush()


def make_inputs(seed, device):
    import torch

    gdev = device if device is not None else "cpu"
    g = torch.Generator(device=gdev).manual_seed(seed)
    q = torch.randn(L_SEQ, HQ, D, generator=g, dtype=torch.float32, device=gdev).to(torch.bfloat16)
    k = torch.randn(NKC, HK, D, generator=g, dtype=torch.float32, device=gdev).to(torch.bfloat16)
    table = torch.randperm(L_SEQ, generator=g, dtype=torch.int64, device=gdev).to(
        torch.int32).reshape(1, L_SEQ)
    q, k, table = q.cpu(), k.cpu(), table.cpu()
    cu_q = torch.tensor([0, L_SEQ], dtype=torch.int32)
    cu_k = torch.tensor([0, NKC], dtype=torch.int32)
    tb = torch.zeros(L_SEQ, dtype=torch.int32)
    pos = torch.arange(1, L_SEQ + 1, dtype=torch.int32)
    seqlen = torch.tensor([L_SEQ], dtype=torch.int32)
    host = dict(q=q, k=k, table=table, cu_q=cu_q, cu_k=cu_k, tb=tb, pos=pos, seqlen=seqlen)
    return host


def parse_cpulist(text):
    """CPU ids of a Linux cpulist string ("0-3,8,10-11")."""
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        a, _, b = part.partition("-")
        cpus.update(range(int(a), int(b or a) + 1))
    return cpus


def bind_to_gpu_numa(dev_index):
    """Run this process on the CPUs of its GPU's NUMA node (from sysfs, via the GPU's PCI
    address), so the pinned host buffers it allocates are placed on that node (first
    touch) and its host-to-device copies stay on the local socket.  Returns what was done,
    for the JSON line; leaves the affinity unchanged when sysfs does not say."""
    import torch

    try:
        pr = torch.cuda.get_device_properties(dev_index)
        base = f"/sys/bus/pci/devices/{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        with open(base + "/numa_node") as f:
            node = int(f.read())
        with open(base + "/local_cpulist") as f:
            cpus = parse_cpulist(f.read()) & os.sched_getaffinity(0)
        if node < 0 or not cpus:
            return {"numa_node": node, "bound": False}
        os.sched_setaffinity(0, cpus)
        return {"numa_node": node, "bound": True, "cpus": len(cpus)}
    except (OSError, ValueError, AttributeError) as e:
        return {"bound": False, "why": type(e).__name__}


# ------------------------------------------------------------------ our arm
# Per-token work of pooling, top-k and get_block_table, in units of one visible
# compressed key of stage 1 (both per kv head), from the kernel times at 128k:
# stage 1 ~1.0e-11 s per key, top-k + block table ~5.6e-9 s per (token, head).
TOKEN_COST = 560.0
# End to end the query rows cross PCIe first: one token's 16 query heads (4 KB) take
# ~1e-7 s at ~40 GB/s per GPU, ~1e4 visible keys of stage-1 time, so the end-to-end
# shards are near-equal token ranges (compute, smaller, is hidden under the copies).
E2E_TOKEN_COST = 1.0e4


def shard_of(world, rank, strong, token_cost=TOKEN_COST):
    """(first kv head, kv heads, t_begin, t_end) this rank computes: config 3's kv head x
    query range shard with strong scaling, the whole sequence with weak scaling."""
    from unum_ops_b200.sharding import prefill_shard

    if world == 1 or not strong:
        return 0, HK, 0, L_SEQ
    return prefill_shard(world, rank, L_SEQ, NKC, HK, token_cost=token_cost)


def run_ours(args):
    import torch
    import torch.distributed as dist

    import unum_ops_b200
    from unum_ops_b200 import block_select_streamed, get_block_table_shard
    from unum_ops_b200.block_select import stage1_pooled
    from unum_ops_b200.infllm_v2 import (_workspace, infllmv2_attn_stage1, max_pooling_1d_varlen,
                                         stage1_status)
    from unum_ops_b200.sharding import exchange_shards

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    host_binding = bind_to_gpu_numa(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    unum_ops_b200.load()
    L = unum_ops_b200.load()
    strong = args.scaling == "strong"
    # the top-k ids are gathered across ranks only when they share one sequence (strong
    # scaling); with weak scaling every rank's result is its own
    gather = world > 1 and strong
    g0, nh, ta, tb_ = shard_of(world, rank, strong)
    nrows = tb_ - ta
    G = HQ // HK

    # strong scaling: every rank holds the same global input (one seed) and computes
    # its shard; weak scaling: every rank its own sequence
    host = make_inputs(1234 + 3 + (0 if strong else rank), dev)
    d = {k: v.to(dev) for k, v in host.items()}
    q_s = d["q"][:, g0 * G:(g0 + nh) * G]   # this rank's query heads (a strided view)
    k_s = d["k"][:, g0:g0 + nh]
    stream = torch.cuda.current_stream(dev)
    W = (NKC + 127) // 128 * 128
    NB = (L_SEQ + 63) // 64
    zeros_cache = torch.zeros(1, dtype=torch.int32, device=dev)
    scores = torch.empty(nh, L_SEQ, W, dtype=torch.bfloat16, device=dev)
    pooled = torch.empty(nh, L_SEQ, NB, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(nh, nrows, TOPK, dtype=torch.int32, device=dev)
    slots = torch.empty(nrows, nh, TOPK * 64, dtype=torch.int32, device=dev)
    ws = _workspace(dev, int(L.unum_stage1_workspace_size(1)))
    # topk_idx of all ranks in one place: every rank's exact shard sent straight into
    # each rank's full [Hk, T, K] buffer (NCCL point-to-point, no padding)
    ranges = [shard_of(world, r, strong) for r in range(world)]
    full_idx = torch.empty(HK, L_SEQ, TOPK, dtype=torch.int32, device=dev)
    # the ids travel as int16 (block ids < NB <= 2^15, -1 padding kept): half the bytes
    wire_idx = torch.empty(HK, L_SEQ, TOPK, dtype=torch.int16, device=dev)

    def gather_idx(local_idx, shards):
        exchange_shards(local_idx, full_idx, shards, rank, wire=wire_idx)

    # the exchange runs on a side stream once top-k is done, overlapping get_block_table
    # (an HBM-bound kernel, while the exchange is NVLink traffic); the step ends when both do
    xstream = torch.cuda.Stream(dev) if gather else None
    topk_done = torch.cuda.Event()
    # --exchange peer: the top-k kernel itself stores the ids into every rank's gathered
    # buffer over NVLink (symmetric memory), then one bounded cross-GPU signal
    from unum_ops_b200.sharding import PeerIdExchange
    xch = PeerIdExchange((HK, L_SEQ, TOPK), dev) if gather and args.exchange == "peer" else None

    def step(ev=None):
        """One block-selection pass over this rank's shard: stage 1 with the pooling
        fused in (token window [ta, tb_) of kv heads g0..g0+nh-1), top-k, get_block_table;
        with several ranks, the top-k ids are gathered on every rank meanwhile."""
        if ev is not None:
            ev[0].record(stream)
        unum_ops_b200._lib.check(L.unum_infllmv2_attn_stage1_window(
            q_s.data_ptr(), L_SEQ, nh * G, D, q_s.stride(0), q_s.stride(1), k_s.data_ptr(), NKC, nh,
            k_s.stride(0), k_s.stride(1), d["cu_q"].data_ptr(), d["cu_k"].data_ptr(), 1, D ** -0.5, 1,
            scores.data_ptr(), W, pooled.data_ptr(), NB, INIT_BLOCKS, LOCAL_BLOCKS, ta, tb_,
            ws.data_ptr(), ws.numel(), stream.cuda_stream))
        if ev is not None:
            ev[1].record(stream)
        if xch is not None:
            xch.begin()
            if nrows == L_SEQ:
                xch.topk(pooled.view(nh * nrows, NB), TOPK, idx.view(nh * nrows, TOPK), g0 * L_SEQ * TOPK)
            else:
                for h in range(nh):
                    xch.topk(pooled[h, ta:tb_], TOPK, idx[h], ((g0 + h) * L_SEQ + ta) * TOPK)
        elif nrows == L_SEQ:  # every row: one launch over the heads' rows together
            unum_ops_b200._lib.check(L.unum_topk_blocks(
                pooled.data_ptr(), 1, nh * nrows, NB, NB, TOPK, idx.data_ptr(), stream.cuda_stream))
        else:
            for h in range(nh):
                unum_ops_b200._lib.check(L.unum_topk_blocks(
                    pooled[h, ta:tb_].data_ptr(), 1, nrows, NB, NB, TOPK, idx[h].data_ptr(),
                    stream.cuda_stream))
        if ev is not None:
            ev[2].record(stream)
        if gather and xch is None:
            topk_done.record(stream)
            xstream.wait_event(topk_done)
            with torch.cuda.stream(xstream):
                if ev is not None:
                    ev[5].record(xstream)
                gather_idx(idx, ranges)
                if ev is not None:
                    ev[6].record(xstream)
        get_block_table_shard(idx, d["table"], d["tb"][ta:tb_], d["pos"][ta:tb_], d["seqlen"],
                              head_offset=g0, out=slots)
        if ev is not None:
            ev[3].record(stream)
        if xch is not None:
            if ev is not None:
                ev[5].record(stream)
            xch.finish(full_idx)
            if ev is not None:
                ev[6].record(stream)
        elif gather:
            stream.wait_stream(xstream)
        if ev is not None:
            ev[4].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    clk = ClockSampler(local).start()
    for _ in range(args.warmup):
        step()
    barrier()
    if stage1_status(dev) != 0:
        raise RuntimeError("stage-1 kernel reported a timeout")

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    barrier()
    wall0 = time.time()
    t_start.record(stream)
    for i in range(args.steps):
        step(evs[i])
    t_end.record(stream)
    barrier()
    wall1 = time.time()
    clk.stop()
    total_ms = t_start.elapsed_time(t_end)
    if xch is not None:
        xch.check()
    if gather:
        # the exchange delivered the ids: this rank's own shard is in place, and
        # every rank holds the same gathered tensor
        torch.cuda.synchronize(dev)
        assert torch.equal(full_idx[g0:g0 + nh, ta:tb_], idx), "own top-k shard missing after the exchange"
        w = torch.arange(1, full_idx.numel() + 1, device=dev, dtype=torch.int64).view(full_idx.shape)
        sums = torch.stack([(full_idx.to(torch.int64) * w).sum()] * 2)
        lo, hi = sums.clone(), sums.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        assert int(lo[0]) == int(hi[0]), "ranks hold different gathered top-k ids"
    per = {"stage1": [], "topk": [], "get_block_table": [], "gather": [], "tail": []}
    for e in evs:
        per["stage1"].append(e[0].elapsed_time(e[1]))
        per["topk"].append(e[1].elapsed_time(e[2]))
        per["get_block_table"].append(e[2].elapsed_time(e[3]))
        if gather:
            per["gather"].append(e[5].elapsed_time(e[6]))
            per["tail"].append(e[2].elapsed_time(e[4]))
    ms_step = total_ms / args.steps
    if world > 1:
        t = torch.tensor([ms_step], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step = float(t.item())
    api = None
    if world == 1:
        # context: the separate reference-API calls for stage 1 and pooling
        api = {"stage1": [], "pool": []}
        for _ in range(3):
            a0, a1, a2 = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            a0.record(stream)
            sc = infllmv2_attn_stage1(d["q"], d["k"], None, d["cu_q"], d["cu_k"], max_seqlen_k=NKC,
                                      causal=True)
            a1.record(stream)
            max_pooling_1d_varlen(sc, d["cu_q"], d["cu_k"], zeros_cache, 16 * W, L_SEQ, LOCAL_BLOCKS,
                                  INIT_BLOCKS)
            a2.record(stream)
            torch.cuda.synchronize(dev)
            api["stage1"].append(a0.elapsed_time(a1))
            api["pool"].append(a1.elapsed_time(a2))
            del sc
        # context: stage 1 + fused pooling with the scores kept on chip (out = NULL), for a
        # caller that needs only the selection
        api["stage1_pooled_no_scores"] = []
        for _ in range(4):
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            unum_ops_b200._lib.check(L.unum_infllmv2_attn_stage1_window(
                q_s.data_ptr(), L_SEQ, nh * G, D, q_s.stride(0), q_s.stride(1), k_s.data_ptr(), NKC, nh,
                k_s.stride(0), k_s.stride(1), d["cu_q"].data_ptr(), d["cu_k"].data_ptr(), 1, D ** -0.5, 1,
                None, W, pooled.data_ptr(), NB, INIT_BLOCKS, LOCAL_BLOCKS, ta, tb_,
                ws.data_ptr(), ws.numel(), stream.cuda_stream))
            a1.record(stream)
            torch.cuda.synchronize(dev)
            api["stage1_pooled_no_scores"].append(a0.elapsed_time(a1))
    del scores, pooled, slots
    producer = None
    if world == 1:
        # context: the producer of k_cmp — mean-pool the sequence's keys over 32-token
        # windows at stride 16 (k [131072, 2, 128] bf16 -> k_cmp [8191, 2, 128])
        from unum_ops_b200 import compress_keys

        gk = torch.Generator(device=dev).manual_seed(99)
        k_full = torch.randn(L_SEQ, HK, D, generator=gk, device=dev).to(torch.bfloat16)
        cu_full = torch.tensor([0, L_SEQ], dtype=torch.int32, device=dev)
        cu_host = cu_full.cpu()
        kc, cu_out = compress_keys(k_full, cu_full, cu_seqlens_host=cu_host)

        def produce():  # the kernel alone: sizes precomputed, as a decode loop would hold them
            unum_ops_b200._lib.check(L.unum_compress_keys(
                k_full.data_ptr(), L_SEQ, HK, D, k_full.stride(0), k_full.stride(1), cu_full.data_ptr(),
                cu_out.data_ptr(), 1, kc.shape[0], 32, 16, kc.data_ptr(), stream.cuda_stream))

        for _ in range(3):
            produce()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        for _ in range(20):
            produce()
        p1.record(stream)
        torch.cuda.synchronize(dev)
        pms = p0.elapsed_time(p1) / 20
        pbytes = L_SEQ * HK * D * 2 + NKC * HK * D * 2
        producer = {"kernel": "compress_keys (k -> k_cmp, not part of the timed step)", "ms": pms,
                    "gbs": pbytes / (pms * 1e-3) / 1e9, "bytes": pbytes}
        del k_full

    # ---- the config-4 decode batch (and the stage-2 consumer on it) at the same N, as
    # context in the same line
    decode = None
    if args.decode_batch > 0:
        torch.cuda.empty_cache()
        decode = measure_decode(args, world, rank, dev, steps=max(args.steps, 20), warmup=max(args.warmup, 3))
        torch.cuda.empty_cache()
        decode["stage2"] = measure_stage2(args, world, rank, dev)
        torch.cuda.empty_cache()

    # ---- end to end through the public API with host buffers (pinned), copies timed:
    # this rank's query rows of its kv heads stream in, its top-k ids go back to the host
    # (end to end the shards balance the host-to-device copy: near-equal token ranges)
    eg0, enh, ea, eb = shard_of(world, rank, strong, E2E_TOKEN_COST)
    q_pin = host["q"][ea:eb, eg0 * G:(eg0 + enh) * G].contiguous().pin_memory()
    pin = {k: v.pin_memory() for k, v in host.items() if k != "q"}
    res_host = torch.empty(enh, eb - ea, TOPK, dtype=torch.int32).pin_memory()

    def e2e_step():
        """Through the public streamed API: host-resident queries copied in chunk by chunk
        while the previous chunk computes; the top-k ids come back to pinned host memory."""
        kk = pin["k"][:, eg0:eg0 + enh].to(dev, non_blocking=True)
        small = {n: pin[n].to(dev, non_blocking=True) for n in ("cu_q", "cu_k", "table", "tb", "pos",
                                                                 "seqlen")}
        block_select_streamed(
            q_pin, kk, small["cu_q"], small["cu_k"], NKC, small["table"], small["tb"],
            small["pos"], small["seqlen"], max_context_len=L_SEQ, init_blocks=INIT_BLOCKS,
            local_blocks=LOCAL_BLOCKS, topk=TOPK, chunk_tokens=16384, result_host=res_host,
            t_begin=ea, head_offset=eg0)

    e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, 5))
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = q_pin.numel() * 2 + pin["k"][:, eg0:eg0 + enh].numel() * 2 + sum(
        pin[n].numel() * pin[n].element_size() for n in ("cu_q", "cu_k", "table", "tb", "pos", "seqlen"))
    d2h = res_host.numel() * 4
    if world > 1:  # whole-job bytes: every rank's copies
        t = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        h2d, d2h = int(t[0].item()), int(t[1].item())

    if rank == 0:
        clocks = clk.summary(wall0, wall1)
        hbm, tf_burst, tf_sus, src = load_peaks()
        mean = {k: statistics.mean(v) for k, v in per.items() if v}
        flops = stage1_flops(ta, tb_) * nh / HK
        ab = algorithmic_bytes(nrows, nh)
        traffic = load_traffic()
        s1_tf = flops / (mean["stage1"] * 1e-3) / 1e12
        kernels = {
            "stage1": {"ms": mean["stage1"], "tflops": s1_tf, "frac": s1_tf / tf_burst,
                       "bound": "tensor", "fused": "max_pooling_1d_varlen",
                       "out_gbs": ab["stage1_out"] / (mean["stage1"] * 1e-3) / 1e9},
        }
        for kname in ("topk", "get_block_table"):
            gbs = ab[kname] / (mean[kname] * 1e-3) / 1e9
            kernels[kname] = {"ms": mean[kname], "gbs": gbs, "frac": gbs / hbm, "bound": "hbm"}
        if gather:
            kernels["topk_idx_gather"] = {"ms": mean["gather"], "bytes": full_idx.numel() * 2,
                                          "how": ("fused into the top-k kernel: int16 ids stored into "
                                                  "every rank's gathered buffer over NVLink (symmetric "
                                                  "memory), then a bounded cross-GPU signal and the "
                                                  "int32 widening (ms = signal + widening)")
                                                 if xch is not None else
                                                 ("NCCL send/recv of each rank's exact shard, int16 "
                                                  "on the wire, widened to int32 once; on a side "
                                                  "stream, overlapping get_block_table"),
                                          "after_topk_ms": mean["tail"]}
        cpu = None
        if args.cpu_sample > 0 and world == 1:
            hf = {k: v.numpy() for k, v in host.items() if k not in ("q", "k")}
            hf["q"] = host["q"].float().numpy()
            hf["k"] = host["k"].float().numpy()
            cpu = cpu_baseline(args, sample_tokens=args.cpu_sample, host=hf)
        if strong and world > 1:
            par = (f"{world} ranks: kv head x query range ({HK} x {world // HK})" if world % HK == 0
                   else f"{world} query ranges") + ", ranges of equal stage-1 + per-token work"
        else:
            par = f"dp{world} (one sequence per GPU)"
        tokens = L_SEQ if strong else world * L_SEQ
        line = {
            "metric": METRIC,
            "value": tokens / (ms_step * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k_cmp, random-permutation block table)",
            "config": {"workload": workload_name(),
                       "tokens_total": tokens, "parallelism": par,
                       "rank0_shard": {"kv_heads": [g0, g0 + nh], "tokens": [ta, tb_]},
                       "l2": "inputs larger than L2 (q 1.07 GB, scores 4.3 GB, slots 4.3 GB)"},
            "roofline": {"bound": "tensor", "kernel": "stage1", "achieved": s1_tf,
                         "peak": tf_burst, "unit": "TFLOP/s", "frac": s1_tf / tf_burst,
                         "peak_source": f"{src} bf16_tflops (burst: the timed region is a fraction of a second)",
                         "frac_of_sustained": s1_tf / tf_sus,
                         "algorithmic": "2*D*G*sum_t visible(t) over rank 0's shard = %.4g flop "
                                        "per launch" % flops,
                         "traffic": traffic.get("stage1") if world == 1 else None,
                         "traffic_source": "profiles/traffic_c3.json (ncu dram bytes at 32k and 64k, "
                                           "derived per term for 128k)" if world == 1 else None,
                         "mufu": mufu_roofline(flops, mean["stage1"], clocks)},
            "kernels": kernels,
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "result": "top-64 block ids int32 of every rank's shard copied to host",
                    "api": "block_select_streamed (query chunks of 16384 tokens copied while the "
                           "previous chunk computes)",
                    "shards": "kv head x query range, ranges of near-equal host-to-device bytes"
                              if strong and world > 1 else "as the device step",
                    "host_binding": host_binding},
            "gpu_launches": (2 + (1 if nrows == L_SEQ else nh)) * args.steps,
            "clocks": clocks,
        }
        if producer is not None:
            line["producer"] = producer
        if decode is not None:
            line["decode"] = decode
        if api is not None:
            am = {k2: statistics.mean(v) for k2, v in api.items()}
            pool_gbs = ab["pool"] / (am["pool"] * 1e-3) / 1e9
            line["kernels_api_path"] = {
                "stage1": {"ms": am["stage1"]},
                "stage1_pooled_no_scores": {
                    "ms": am["stage1_pooled_no_scores"],
                    "note": "stage 1 + fused pooling with out = NULL: the 4.3 GB of scores stay on chip"},
                "pool": {"ms": am["pool"], "gbs": pool_gbs, "frac": pool_gbs / hbm, "bound": "hbm"},
                "note": "separate max_pooling_1d_varlen call; the step fuses it into stage1"}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        emit(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ decode batch (config 4)
def measure_decode(args, world, rank, dev, steps=None, warmup=None):
    """512 sequences x 1 query token, contexts U[4096, 65536].  A step is
    block_select on the batch (one CUDA-graph replay).  With N ranks the batch is split by
    longest-processing-time packing of the sequences' compressed-key counts (strong
    scaling; --scaling weak gives every rank its own batch); a rank's ids and slots stay
    on that rank (no exchange step: the sequences are independent).  Returns the measurement as a dict (max over ranks)."""
    import torch
    import torch.distributed as dist

    from unum_ops_b200 import BlockSelectGraph, block_select
    from unum_ops_b200.sharding import plan_sequences, sequence_cost

    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    strong = args.scaling == "strong"
    B_all = args.decode_batch
    seed = 4 + (0 if strong else rank)
    rng = np.random.default_rng(seed)
    ctx_all = rng.integers(4096, 65537, size=B_all)
    k_lens_all = (ctx_all - 32) // 16 + 1
    table_all = rng.integers(0, 1 << 20, size=(B_all, 1024)).astype(np.int32)
    g = torch.Generator(device=dev).manual_seed(seed)
    q_all = torch.randn(B_all, HQ, D, generator=g, device=dev).to(torch.bfloat16)
    k_all = torch.randn(int(k_lens_all.sum()), HK, D, generator=g, device=dev).to(torch.bfloat16)
    if strong and world > 1:
        plan = plan_sequences(sequence_cost([1] * B_all, k_lens_all), world)
    else:
        plan = [list(range(B_all))] * world
    mine = np.array(plan[rank], np.int64)
    # longest sequences first: the decode kernel takes (token, kv head) items in order, so
    # the longest start first and the shorter ones fill in behind them (the order a decode
    # scheduler can give its batch; the work is the same)
    mine = mine[np.argsort(-k_lens_all[mine], kind="stable")]
    B = len(mine)
    starts = np.concatenate([[0], np.cumsum(k_lens_all)])
    k_rows = np.concatenate([np.arange(starts[i], starts[i + 1]) for i in mine])
    k_lens = k_lens_all[mine]
    ctx = ctx_all[mine]
    q = q_all[torch.from_numpy(mine).to(dev)].contiguous()
    k = k_all[torch.from_numpy(k_rows).to(dev)].contiguous()
    del q_all, k_all
    cu_q = torch.arange(B + 1, dtype=torch.int32, device=dev)
    cu_k = torch.from_numpy(np.concatenate([[0], np.cumsum(k_lens)]).astype(np.int32)).to(dev)
    table = torch.from_numpy(table_all[mine]).to(dev)
    tb = torch.arange(B, dtype=torch.int32, device=dev)
    pos = torch.from_numpy(ctx.astype(np.int32)).to(dev)
    cache = torch.from_numpy((ctx - 1).astype(np.int32)).to(dev)
    stream = torch.cuda.current_stream(dev)

    sel_args = (q, k, cu_q, cu_k, int(k_lens.max()), table, tb, pos, pos)
    sel_kw = dict(max_context_len=65536, cache_lens=cache)
    graph = BlockSelectGraph(*sel_args, **sel_kw)  # the decode loop's form: one graph replay

    def step(eager=False):
        # no collective: decode sequences are independent, and each rank keeps its own
        # sequences' ids and slots, which its own stage 2 consumes
        return block_select(*sel_args, **sel_kw) if eager else graph()

    def timed(eager):
        for _ in range(warmup):
            step(eager)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step(eager)
        e1.record(stream)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    ms_eager = timed(True)
    ms = timed(False)
    # the graph replays the same kernels as the eager call: same top-k ids
    assert torch.equal(block_select(*sel_args, **sel_kw)[2], graph()[2])
    kbytes = int(k_lens.sum()) * HK * D * 2
    hbm = load_peaks()[0]
    seqs = B_all if strong else world * B_all
    del graph
    return {"ms_per_step": ms, "eager_ms_per_step": ms_eager, "sequences_per_s": seqs / (ms * 1e-3),
            "sequences": seqs, "rank0_sequences": B, "shard_sizes": [len(p_) for p_ in plan],
            "rank0_k_cmp_bytes": kbytes, "k_cmp_stream_gbs": kbytes / (ms * 1e-3) / 1e9,
            "k_cmp_stream_frac": kbytes / (ms * 1e-3) / 1e9 / hbm,
            "parallelism": (f"{world} ranks, sequences by LPT on compressed-key counts"
                            if strong and world > 1 else f"dp{world}"),
            "api": ("BlockSelectGraph (block_select captured once in a CUDA graph, replayed per step): "
                    "the fused decode kernel (stage 1, pooling, top-k, get_block_table in one launch)")}


def measure_stage2(args, world, rank, dev, steps=20, warmup=3):
    """The stage-2 consumer on the config-4 decode batch: each of the 512 tokens attends
    (16 query heads per kv head) over its 64 selected 64-token blocks of a paged KV cache
    (per-token block table [512, 65536] of random physical slots, 2^20 physical tokens),
    the gather fused into the kernel (no slot tensor).  Sequences are split as in the
    decode measurement.  HBM-bound: algorithmic bytes = K and V rows of the valid
    positions + q + out + top-k ids + the table entries read."""
    import torch
    import torch.distributed as dist

    from unum_ops_b200 import sparse_attention
    from unum_ops_b200.sharding import plan_sequences, sequence_cost

    strong = args.scaling == "strong"
    B_all = args.decode_batch
    rng = np.random.default_rng(40 + (0 if strong else rank))
    ctx_all = rng.integers(4096, 65537, size=B_all)
    if strong and world > 1:
        plan = plan_sequences(sequence_cost([1] * B_all, (ctx_all - 32) // 16 + 1), world)
    else:
        plan = [list(range(B_all))] * world
    mine = np.array(plan[rank], np.int64)
    B = len(mine)
    ctx = ctx_all[mine]
    n_phys = 1 << 20
    g = torch.Generator(device=dev).manual_seed(41 + rank)
    table = torch.randint(0, n_phys, (B, 65536), generator=g, device=dev, dtype=torch.int32)
    kc = torch.randn(n_phys * HK, D, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(n_phys * HK, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(B, HQ, D, generator=g, device=dev).to(torch.bfloat16)
    topk = np.empty((HK, B, TOPK), np.int32)
    for h in range(HK):
        for b in range(B):
            nblk = (int(ctx[b]) + 63) // 64
            topk[h, b] = np.sort(rng.choice(nblk, TOPK, replace=False))
    topk_d = torch.from_numpy(topk).to(dev)
    tb = torch.arange(B, dtype=torch.int32, device=dev)
    pos = torch.from_numpy(ctx.astype(np.int32)).to(dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def run():
        return sparse_attention(q, kc, vc, topk_d, table, tb, pos, pos, status=st)

    for _ in range(warmup):
        run()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        run()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    if int(st.item()) != 0:
        raise RuntimeError("stage-2 kernel reported a timeout")
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    valid = 0  # valid positions: p < ctx (the last selected block may be partial)
    for b in range(B):
        blocks = topk[:, b, :].astype(np.int64)
        valid += int(np.minimum(64, np.maximum(0, int(ctx[b]) - blocks * 64)).sum())
    nbytes = valid * D * 2 * 2 + B * HQ * D * 2 * 2 + topk.size * 4 + valid * 4
    hbm = load_peaks()[0]
    del kc, vc, table
    return {"ms_per_step": ms, "kernel": "stage2_kernel (unum_sparse_attn_blocks)",
            "tokens": B, "valid_positions": valid, "bytes": nbytes,
            "gbs": nbytes / (ms * 1e-3) / 1e9, "frac": nbytes / (ms * 1e-3) / 1e9 / hbm, "bound": "hbm",
            "workload": "C4 decode batch x top-64 blocks, paged KV cache (per-token table [B, 65536], "
                        "2^20 physical tokens), 16 query heads per kv head"}


def run_decode(args):
    """--workload decode: the config-4 decode batch as the bench line itself."""
    import torch
    import torch.distributed as dist

    import unum_ops_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    host_binding = bind_to_gpu_numa(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    unum_ops_b200.load()
    d = measure_decode(args, world, rank, dev)
    d["stage2"] = measure_stage2(args, world, rank, dev)
    if rank == 0:
        emit({
            "metric": f"decode block selection, sequences/s ({args.decode_batch} x 1 query, contexts U[4096,65536])",
            "value": d["sequences_per_s"], "unit": "sequences/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": d["ms_per_step"],
            "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {"workload": "C4 decode batch", "parallelism": d["parallelism"]},
            "decode": d})
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ CPU baseline
def cpu_baseline(args, sample_tokens=2048, repeats=1, host=None):
    """Time the reference path on the host cores, all threads, on two samples of
    `sample_tokens` // 2 consecutive tokens each (one early in the 128k sequence, one
    late, so that short and long causal rows are both timed): stage 1 and pooling by
    the C restatement of the reference's kernels (oracle/oracle.c), top-k by torch.topk
    (the reference's caller) and get_block_table by the restatement of the reference's
    own torch function (oracle/torch_ref.py).  The full step is extrapolated by
    visible-pair count (stage 1) and token count (the other steps); the measured seconds
    and the sample sizes are returned beside the extrapolation."""
    import torch

    import oracle
    from oracle import torch_ref

    nthreads = oracle.set_num_threads(0)
    torch.set_num_threads(nthreads)
    if host is None:
        host = host_inputs_f32()
    q = host["q"]
    k = host["k"]
    cu_q = host["cu_q"]
    cu_k = host["cu_k"]
    vis = visible_counts()
    half = max(1, sample_tokens // 2)
    ranges = [(L_SEQ // 8, L_SEQ // 8 + half), (L_SEQ - L_SEQ // 8 - half, L_SEQ - L_SEQ // 8)]
    W = (NKC + 127) // 128 * 128
    times = []
    for _ in range(repeats):
        t_s1 = t_rest = 0.0
        per_step = {"stage1": 0.0, "pool": 0.0, "topk": 0.0, "get_block_table": 0.0}
        for a, b in ranges:
            t0 = time.perf_counter()
            sc = oracle.stage1(q, k, cu_q, cu_k, True, t_range=(a, b))
            t1 = time.perf_counter()
            cu_qs = np.array([-a, b - a], np.int32)  # sampled rows keep their positions
            pooled = oracle.max_pool(sc, cu_qs, cu_k, np.zeros(1, np.int32), 16 * W, L_SEQ,
                                     LOCAL_BLOCKS, INIT_BLOCKS)
            t2 = time.perf_counter()
            idx = torch_ref.topk(torch.from_numpy(pooled), TOPK)
            t3 = time.perf_counter()
            torch_ref.get_block_table(idx, torch.from_numpy(host["table"]),
                                      torch.from_numpy(host["tb"][a:b]),
                                      torch.from_numpy(host["pos"][a:b]),
                                      torch.from_numpy(host["seqlen"]))
            t4 = time.perf_counter()
            t_s1 += t1 - t0
            t_rest += t4 - t1
            for kname, dt in zip(per_step, (t1 - t0, t2 - t1, t3 - t2, t4 - t3)):
                per_step[kname] += dt
        vis_s = sum(int(vis[a:b].sum()) for a, b in ranges)
        tok_s = sum(b - a for a, b in ranges)
        full_s = t_s1 * vis.sum() / vis_s + t_rest * L_SEQ / tok_s
        times.append((full_s, t_s1 + t_rest, per_step))
    full_s, measured_s, per_step = sorted(times, key=lambda t: t[0])[len(times) // 2]
    desc = ", ".join(f"[{a},{b})" for a, b in ranges)
    return {"value": L_SEQ / full_s, "unit": "tokens/s", "cores": nthreads, "kind": "port",
            "measured_s": measured_s, "sample_tokens": tok_s,
            "measured_s_by_step": per_step,
            "extrapolated_full_step_s": full_s,
            "sample": f"tokens {desc} of the {L_SEQ}-token sequence, {tok_s} tokens measured in "
                      f"{measured_s:.2f} s; stage 1 (C port) scaled by visible pairs "
                      f"({vis_s / vis.sum():.4f} of the total), pooling (C port), top-k "
                      f"(torch.topk) and get_block_table (the reference's torch function, "
                      f"restated) by token count; extrapolated full step {full_s:.1f} s"}


def host_inputs_f32():
    host = make_inputs(1234 + 3, None)
    out = {k: v.numpy() for k, v in host.items() if k not in ("q", "k")}
    out["q"] = host["q"].float().numpy()
    out["k"] = host["k"].float().numpy()
    return out


def run_reference(args):
    """The reference arm: the reference path on the host cores (cpu_baseline), one
    bounded sample per step.  `value` is the extrapolated full-step throughput;
    `ms_per_step` is the measured time of one timed sample step (what actually ran)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    host = host_inputs_f32()
    steps = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        cb = cpu_baseline(args, sample_tokens=args.ref_sample, host=host)
        cb["wall_s"] = time.perf_counter() - t0
        if i >= args.warmup:
            steps.append(cb)
    steps.sort(key=lambda c: c["value"])
    med = steps[len(steps) // 2]
    v = med["value"]
    line = {
        "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": statistics.median(c["wall_s"] for c in steps) * 1e3,
        "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32", "impl": "reference",
        "data": "synthetic (seeded N(0,1) q/k_cmp, random-permutation block table)",
        "config": {"workload": workload_name()},
        "step": "one bounded sample of the workload (ms_per_step is its measured time); value "
                "is the full 128k step extrapolated from it",
        "extrapolated_ms_per_full_step": med["extrapolated_full_step_s"] * 1e3,
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": med["cores"], "kind": "port",
                         "sample": med["sample"], "measured_s_by_step": med["measured_s_by_step"]},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


def main():
    quiet_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-sample", type=int, default=8192,
                    help="tokens of the CPU-baseline sample (0: skip)")
    ap.add_argument("--ref-sample", type=int, default=2048)
    ap.add_argument("--workload", default="prefill", choices=["prefill", "decode"],
                    help="prefill: the 128k headline (config 3); decode: config 4")
    ap.add_argument("--seqlen", type=int, default=131072,
                    help="prefill length (default: the 128k headline workload)")
    ap.add_argument("--decode-batch", type=int, default=512,
                    help="decode batch (config 4: 512 sequences); the prefill line also carries "
                         "its measurement under 'decode' (0: skip)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="N>1 top-k id exchange: fused into the top-k kernel over NVLink (peer), "
                         "or NCCL send/recv after it (nccl)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="N>1: strong = one sequence sharded by kv head x query range "
                         "(config 3); weak = every rank its own sequence")
    args = ap.parse_args()
    global L_SEQ, NKC
    L_SEQ = args.seqlen
    NKC = (L_SEQ - 32) // 16 + 1
    args.cpu_sample = min(args.cpu_sample, L_SEQ)
    args.ref_sample = min(args.ref_sample, L_SEQ)
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "decode":
        run_decode(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
