"""Key compression (the producer of stage 1's k_cmp): the oracle against a plain
restatement on CPU, the CUDA kernel against the oracle bit for bit on the GPU."""
import numpy as np
import pytest
import torch

import cases


def _restated(k, lens, kernel=32, stride=16):
    out, starts = [], np.concatenate([[0], np.cumsum(lens)])
    for b, L in enumerate(lens):
        for j in range(max(0, (L - kernel) // stride + 1) if L >= kernel else 0):
            acc = np.zeros(k.shape[1:], np.float32)
            for t in range(kernel):  # fp32, token order
                acc += k[starts[b] + j * stride + t]
            out.append(acc * np.float32(1.0 / kernel))
    if not out:
        return np.zeros((0,) + k.shape[1:], np.uint16)
    x = torch.from_numpy(np.stack(out)).to(torch.bfloat16)
    return x.view(torch.int16).numpy().view(np.uint16)


def test_oracle_compress_matches_restatement(oracle_lib):
    rng = np.random.default_rng(61)
    lens = [31, 32, 33, 47, 48, 200, 0, 64]
    k = cases.bf16_round(rng.standard_normal((sum(lens), 2, 128), dtype=np.float32))
    got, cu_out = oracle_lib.compress_keys(k, cases.cu(lens))
    assert list(np.diff(cu_out)) == [0, 1, 1, 1, 2, 11, 0, 3]
    np.testing.assert_array_equal(got, _restated(k, lens))


@pytest.mark.gpu
@pytest.mark.parametrize("lens", [[31, 32, 33, 47, 48, 200, 0, 64], [131072]],
                         ids=["varlen_edges", "one_128k_sequence"])
def test_compress_keys_kernel_bit_exact(lens, oracle_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from unum_ops_b200 import compress_keys

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(62)
    k = torch.randn(sum(lens), 2, 128, generator=g, device=dev).to(torch.bfloat16)
    cu = torch.from_numpy(cases.cu(lens)).to(dev)
    kc, cu_out = compress_keys(k, cu)
    ref, ref_cu = oracle_lib.compress_keys(k.float().cpu().numpy(), cases.cu(lens))
    assert np.array_equal(cu_out.cpu().numpy(), ref_cu)
    np.testing.assert_array_equal(kc.view(torch.int16).cpu().numpy().view(np.uint16), ref)
    # one kv head of the two, as a strided view
    kc1, _ = compress_keys(k[:, 1:2], cu)
    assert torch.equal(kc1[:, 0], kc[:, 1])
