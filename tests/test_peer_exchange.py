"""The top-k id exchange fused into the top-k kernel (unum_topk_blocks_to_peers +
unum_peer_signal_wait, driven by sharding.PeerIdExchange): one process per GPU, the
gathered ids equal to a local top-k over all rows on every rank.  On a one-GPU box the
single rank stores into its own buffer through the same path."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_topk_ids_exchanged_through_peer_stores():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import unum_ops_b200

    unum_ops_b200.build()
    n = min(torch.cuda.device_count(), 4)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
                        "--master-addr", "127.0.0.1", "--master-port", "29547",
                        os.path.join(ROOT, "tests", "peer_exchange_check.py")],
                       capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-4000:])
    assert r.stdout.count(": ok") == n
