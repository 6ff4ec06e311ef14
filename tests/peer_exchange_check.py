"""Checker for the top-k id exchange fused into the top-k kernel (PeerIdExchange), run by
tests/test_peer_exchange.py under torch.distributed.run with one process per GPU.

Every rank holds the same pooled scores [2, T, NB]; rank r selects the rows of a token
range of both heads with unum_topk_blocks_to_peers (ids stored into every rank's
gathered buffer), then the bounded signal and the widening; the gathered [2, T, K] ids
must equal a local unum_topk_blocks over all rows, on every rank, for several steps in
a row (the two alternating buffers) with new scores each step.  Exit code 0 = pass."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from unum_ops_b200 import topk_blocks  # noqa: E402
from unum_ops_b200.sharding import PeerIdExchange  # noqa: E402


def main():
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    H, T, NB, K = 2, 4096 + 17, 512, 64
    bounds = [T * r // world for r in range(world + 1)]
    a, b = bounds[rank], bounds[rank + 1]
    xch = PeerIdExchange((H, T, K), dev)
    full = torch.empty(H, T, K, dtype=torch.int32, device=dev)
    idx = torch.empty(H, b - a, K, dtype=torch.int32, device=dev)
    for step in range(5):
        g = torch.Generator(device=dev).manual_seed(100 + step)
        pooled = torch.randn(H, T, NB, generator=g, device=dev).to(torch.bfloat16)
        pooled[:, :, :3] = float("inf")           # forced blocks, as the pooling writes them
        pooled[:, : T // 8, NB // 2:] = float("-inf")  # rows with fewer candidates than K
        xch.begin()
        for h in range(H):
            xch.topk(pooled[h, a:b], K, idx[h], (h * T + a) * K)
        xch.finish(full)
        ref = topk_blocks(pooled, K)
        torch.cuda.synchronize(dev)
        assert torch.equal(idx, ref[:, a:b]), f"rank {rank} step {step}: local ids differ"
        assert torch.equal(full, ref), f"rank {rank} step {step}: gathered ids differ at {int((full != ref).sum())}"
    xch.check()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}/{world}: ok")


if __name__ == "__main__":
    main()
