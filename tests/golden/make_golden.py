"""Generate the golden fixtures by running the REFERENCE implementation.

Run in the build container (the reference checkout is not present on GPU
machines):

    python tests/golden/make_golden.py --ref /path/to/unum_ops/checkout   (or UNUM_OPS_REF=...)

It imports the reference's own Python modules straight from its source tree
(``src/unum_ops/...``) and runs them on CPU:

* ``get_block_table_ref_torch`` (torch) and the three Triton block-table
  kernels under the Triton interpreter (``TRITON_INTERPRET=1``);
* the Triton pooling kernel ``_max_pooling_1d_varlen_kernel`` under the
  interpreter, on float32 input (the max is exact, so this equals the bf16
  result widened);
* the public stage-1 kernel ``_infllmv2_attn_stage1_kernel`` (Triton v2) under
  the interpreter, plus ``infllmv2_attn_stage1_ref_torch`` for the
  non-causal 32/2-head cases it supports.

Two shims make the reference importable on stock torch without an NPU:
``torch.npu.is_available`` is stubbed to False (the pooling module calls it
at import time), and the modules are loaded by file path so the package
``__init__`` (which imports an absent ``spconv``) is skipped.  The Triton
interpreter of triton 3.6 multiplies bf16 operands of ``tl.dot`` as raw
uint16 bit patterns; the script widens them to float32 first, which is what
the compiled kernel's bf16 MMA computes exactly (products of bf16 values are
exact in fp32).  Autotune lists are cut to their first entry because the
interpreter cannot benchmark; the autotuned parameters are tile sizes only
and do not change results.

Outputs: ``stage1.npz``, ``pool.npz``, ``gbt.npz`` next to this script, each
holding per-case outputs and the SHA-256 of the case's inputs.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def _shim_triton():
    import triton.language as tl
    from triton.runtime import interpreter as I

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        ad, bd = a.data, b.data
        if a.dtype.scalar == tl.bfloat16:
            ad = I._convert_float(ad, tl.bfloat16, tl.float32, None).view(np.float32)
        if b.dtype.scalar == tl.bfloat16:
            bd = I._convert_float(bd, tl.bfloat16, tl.float32, None).view(np.float32)
        return I.TensorHandle(np.matmul(ad, bd, dtype=d.data.dtype) + d.data, d.dtype.scalar)

    I.InterpreterBuilder.create_dot = create_dot


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _one_config(kernel):
    kernel.configs = kernel.configs[:1]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("UNUM_OPS_REF"),
                    help="checkout of the reference repository (or set UNUM_OPS_REF)")
    ap.add_argument("--only", default="", help="comma list of stage1,pool,gbt")
    args = ap.parse_args()
    if not args.ref:
        ap.error("pass --ref <reference checkout> or set UNUM_OPS_REF")
    src = os.path.join(args.ref, "src", "unum_ops")
    torch.npu = types.SimpleNamespace(is_available=lambda: False)
    _shim_triton()
    only = set(filter(None, args.only.split(",")))

    if not only or "gbt" in only:
        gt = _load("ref_get_table_torch", os.path.join(src, "sparse_kernel_extension/get_table_torch.py"))
        gtr = _load("ref_get_table_triton", os.path.join(src, "sparse_kernel_extension/get_table_triton.py"))
        _one_config(gtr.get_block_table_kernel_v3)
        out = {}
        for c in cases.gbt_cases():
            args_t = [torch.from_numpy(c[k]) for k in ("topk", "table", "token_to_bs", "pos", "seqlen")]
            ref = gt.get_block_table_ref_torch(*args_t, topk=c["K"]).numpy()
            T = c["topk"].shape[1]
            L = c["table"].shape[1]
            # The Triton kernels do not clamp the table column; run them only
            # where every valid position lies inside the table row.
            lim = np.minimum(c["seqlen"].max(), c["pos"].max())
            if lim <= L:
                for fn in (gtr.get_block_table_ref_triton, gtr.get_block_table_ref_triton_v2,
                           gtr.get_block_table_ref_triton_v3):
                    o = fn(*args_t, topk=c["K"]).numpy()
                    assert np.array_equal(o, ref), (c["name"], fn.__name__)
            out[c["name"] + "/out"] = ref
            out[c["name"] + "/digest"] = np.array(cases.digest(c["topk"], c["table"], c["token_to_bs"],
                                                               c["pos"], c["seqlen"]))
            print("gbt", c["name"], ref.shape, "T=", T)
        np.savez_compressed(os.path.join(HERE, "gbt.npz"), **out)

    if not only or "pool" in only:
        mp = _load("ref_max_pool", os.path.join(src, "infllm_v2/max_pooling_1d_varlen.py"))
        _one_config(mp._max_pooling_1d_varlen_kernel)
        out = {}
        for c in cases.pool_cases():
            x = c["x"]
            H, T, W = x.shape
            fs = c["max_seqlen_q"] // c["stride"]
            kl = (c["cu_k"][1:] - c["cu_k"][:-1]) + c["cache_lens"]
            # every read of the reference must stay inside the buffer
            for b in range(len(kl)):
                t_last = int(c["cu_q"][b + 1]) - 1
                if t_last >= int(c["cu_q"][b]):
                    assert (H - 1) * T * fs + t_last * fs + int(kl[b]) <= x.size, c["name"]
            o = mp.max_pooling_1d_varlen_ref_triton(
                torch.from_numpy(x), torch.from_numpy(c["cu_q"]), torch.from_numpy(c["cu_k"]),
                torch.from_numpy(c["cache_lens"]), c["max_seqlen_q"], c["max_context_len"],
                c["local_blocks"], c["init_blocks"], c["block_size"], c["stride"]).numpy()
            out[c["name"] + "/out"] = o
            out[c["name"] + "/digest"] = np.array(cases.digest(x, c["cu_q"], c["cu_k"], c["cache_lens"]))
            print("pool", c["name"], o.shape)
        np.savez_compressed(os.path.join(HERE, "pool.npz"), **out)

    if not only or "stage1" in only:
        s1 = _load("ref_stage1_v2", os.path.join(src, "infllm_v2/infllmv2_attn_stage1_triton_v2.py"))
        s1r = _load("ref_stage1_torch", os.path.join(src, "infllm_v2/infllmv2_attn_stage1.py"))
        _one_config(s1._infllmv2_attn_stage1_kernel)
        out = {}
        for c in cases.stage1_cases():
            q = torch.from_numpy(c["q"]).bfloat16()
            k = torch.from_numpy(c["k"]).bfloat16()
            cq, ck = torch.from_numpy(c["cu_q"]), torch.from_numpy(c["cu_k"])
            o = s1.infllmv2_attn_stage1_triton_v2(q, k, k, cq, ck, max_seqlen_q=c["max_seqlen_q"],
                                                  max_seqlen_k=c["max_seqlen_k"], causal=c["causal"])
            out[c["name"] + "/out_bf16"] = o.view(torch.int16).numpy().view(np.uint16)
            if not c["causal"] and q.shape[1] == 32 and k.shape[1] == 2 and len(c["cu_q"]) == 2:
                r = s1r.infllmv2_attn_stage1_ref_torch(q, k, k, cq, ck, causal=False)
                out[c["name"] + "/torchref_bf16"] = r.view(torch.int16).numpy().view(np.uint16)
            out[c["name"] + "/digest"] = np.array(cases.digest(c["q"], c["k"], c["cu_q"], c["cu_k"]))
            print("stage1", c["name"], tuple(o.shape))
        np.savez_compressed(os.path.join(HERE, "stage1.npz"), **out)


if __name__ == "__main__":
    main()
