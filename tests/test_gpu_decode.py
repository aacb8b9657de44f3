"""The decode-step kernels (one query per (b,h)) against the prefill kernels
and the oracle.

Both paths implement the same rounding points and the same logit MMA
accumulation order, so the importance and every selection must agree bit for
bit, and the outputs to 1e-5 normwise (the correction's fp32 sums differ in
order).  Shapes cover parent counts that are not a multiple of the 128-parent
logit tile, batches that are not a multiple of the 64-query tile, D = 64 and
128, one to eight children, bf16 and fp16, a budget equal to M0, and the
budget floor below the budget.  The incremental append of new keys is checked
by the cache tests (state equal to the oracle's full re-quantization).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from avqa_b200 import _lib, ops
from avqa_b200.codebook import codebook_from_keys
from avqa_b200.workloads import TORCH_DTYPE, Workload, make_inputs
from oracle import avq_oracle as O
from parity import (OUT_TOL, check_quantization, check_routing_single_query, heads_view, normrel, oracle_config,
                    quant_arrays, to_dev)

pytestmark = pytest.mark.gpu

CASES = [
    Workload("dec_c3like_bf16", B=70, T=1, S=2048, H=3, D=128, M0=1024, C=8, P=64, dtype="bf16", keys="aniso", seed=71),
    Workload("dec_d64_f16", B=5, T=1, S=900, H=2, D=64, M0=200, C=4, P=24, dtype="f16", keys="mixture", seed=72),
    Workload("dec_c1_bf16", B=3, T=1, S=300, H=2, D=64, M0=40, C=1, P=40, dtype="bf16", keys="mixture", seed=73),
    Workload("dec_sparse_bf16", B=2, T=1, S=20, H=2, D=128, M0=300, C=3, P=32, dtype="bf16", keys="mixture", seed=74),
    Workload("dec_m4096_bf16", B=2, T=1, S=6000, H=1, D=128, M0=4096, C=8, P=128, dtype="bf16", keys="mixture",
             seed=75),
    # a budget above 256: the routing sorts every key instead of the radix select
    Workload("dec_wide_budget_bf16", B=3, T=1, S=4096, H=2, D=64, M0=1024, C=2, P=320, dtype="bf16", keys="mixture",
             seed=76),
]


def _forward(w: Workload, q, st, cb, decode: bool):
    os.environ["AVQ_DISABLE_DECODE"] = "0" if decode else "1"
    try:
        out, diag = ops.forward(heads_view(q, w.H), cb, st, min(w.P, w.M0), diagnostics=True)
        torch.cuda.synchronize()
    finally:
        os.environ.pop("AVQ_DISABLE_DECODE", None)
    code = ctypes.c_int(-1)
    _lib.check(_lib.load().avq_device_fault(ctypes.byref(code), None), "avq_device_fault")
    assert code.value == 0
    return out.clone(), diag


@pytest.mark.parametrize("w", CASES, ids=lambda w: w.name)
def test_decode_matches_prefill_kernels_and_oracle(w: Workload) -> None:
    dt = w.dtype
    q, k, v = make_inputs(w)
    qn, kn, vn = (O.rnd(x.numpy(), dt) for x in (q, k, v))
    kh0 = torch.from_numpy(kn).view(w.B, w.S, w.H, w.D).transpose(1, 2)[0]
    cbk = codebook_from_keys(kh0, w.M0, w.C, w.seed)
    cb = ops.prepare_codebook(cbk.parents, cbk.children, TORCH_DTYPE[dt], torch.device("cuda"))
    st = ops.quantize(heads_view(to_dev(kn, dt), w.H), heads_view(to_dev(vn, dt), w.H), cb)
    qd = to_dev(qn, dt)
    out_d, d_d = _forward(w, qd, st, cb, True)
    out_p, d_p = _forward(w, qd, st, cb, False)
    assert torch.equal(d_d.importance, d_p.importance)
    assert torch.equal(d_d.selected, d_p.selected)
    assert torch.equal(d_d.pass_counts, d_p.pass_counts)
    assert normrel(out_d.cpu().numpy(), out_p.cpu().numpy()) < 1e-4  # fp32 sums in different orders
    pd, cd = O.cast_codebook(cbk.parents.numpy(), cbk.children.numpy(), dt)
    cfg = oracle_config(dict(w.__dict__), "entropy", 1.0)
    res = O.forward(qn, kn, vn, pd, cd, cfg)
    quant = check_quantization(quant_arrays(st, w.B, w.H), O.split_heads(kn, w.H), O.split_heads(vn, w.H), pd, cd,
                               dt, res["quant"], tag=w.name)
    if quant is not res["quant"]:
        res = O.forward(qn, kn, vn, pd, cd, cfg, quant=quant)
    nrows = check_routing_single_query(d_d, res, O.split_heads(qn, w.H), pd, w.H, dt, w.name)
    print(f"{w.name}: {nrows} of {w.B * w.H} rows with a certified logit near-tie")
    got = out_d.cpu().numpy().transpose(0, 2, 1, 3).reshape(w.B, w.T, w.E)
    err = normrel(got, res["out_bte"])
    assert err <= OUT_TOL[dt], f"{w.name}: output normrel {err}"
