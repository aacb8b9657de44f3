"""The tcgen05 parent-attention kernel against the mma.sync kernel and the oracle.

Both kernels implement the first routing pass with the same rounding points,
so the forward output, the importance and every selection must agree bit for
bit.  The shapes cover the kernel's edges: query counts that leave dead rows
in the last 128-query tile (and a last 64-query tile beyond T), parent counts
that are not a multiple of the 64-parent chunk, empty parents, D = 64 and
128, bf16 and fp16, several routing passes.  ``avq_device_fault`` must stay 0
(no bounded wait gave up).
"""
from __future__ import annotations

import ctypes
import os

import pytest
import torch

from avqa_b200 import _lib, ops
from avqa_b200.codebook import codebook_from_keys
from avqa_b200.workloads import TORCH_DTYPE, Workload, make_inputs
from oracle import avq_oracle as O
from parity import (OUT_TOL, check_quantization, check_routing, heads_view, normrel, oracle_config, quant_arrays,
                    to_dev)

pytestmark = pytest.mark.gpu

CASES = [
    Workload("tail_bf16", B=1, T=200, S=1024, H=2, D=128, M0=128, C=4, P=16, dtype="bf16", keys="mixture", seed=41),
    Workload("short_bf16", B=2, T=40, S=600, H=2, D=128, M0=72, C=4, P=8, dtype="bf16", keys="mixture", seed=42),
    Workload("d64_f16", B=2, T=300, S=768, H=2, D=64, M0=96, C=4, P=12, dtype="f16", keys="mixture", seed=43),
    Workload("empty_bf16", B=1, T=256, S=40, H=2, D=64, M0=256, C=2, P=16, dtype="bf16", keys="mixture", seed=44),
    Workload("mp_bf16", B=1, T=384, S=2048, H=2, D=128, M0=192, C=8, P=24, dtype="bf16", keys="aniso", seed=45,
             passes=3, pass_decay=0.5),
]


def _forward(w: Workload, q, st, cb, tc: bool):
    os.environ["AVQ_DISABLE_TCGEN05"] = "0" if tc else "1"
    try:
        out, diag = ops.forward(heads_view(q, w.H), cb, st, min(w.P, w.M0), w.passes, w.pass_decay,
                                diagnostics=True)
        torch.cuda.synchronize()
    finally:
        os.environ.pop("AVQ_DISABLE_TCGEN05", None)
    code = ctypes.c_int(-1)
    _lib.check(_lib.load().avq_device_fault(ctypes.byref(code), None), "avq_device_fault")
    assert code.value == 0, f"device fault record {code.value}"
    return out.clone(), diag


@pytest.mark.parametrize("w", CASES, ids=lambda w: w.name)
def test_tcgen05_matches_mma_and_oracle(w: Workload) -> None:
    dt = w.dtype
    q, k, v = make_inputs(w)
    qn, kn, vn = (O.rnd(x.numpy(), dt) for x in (q, k, v))
    kh0 = torch.from_numpy(kn).view(w.B, w.S, w.H, w.D).transpose(1, 2)[0]
    cbk = codebook_from_keys(kh0, w.M0, w.C, w.seed)
    cb = ops.prepare_codebook(cbk.parents, cbk.children, TORCH_DTYPE[dt], torch.device("cuda"))
    st = ops.quantize(heads_view(to_dev(kn, dt), w.H), heads_view(to_dev(vn, dt), w.H), cb)
    qd = to_dev(qn, dt)
    out_tc, d_tc = _forward(w, qd, st, cb, True)
    out_mma, d_mma = _forward(w, qd, st, cb, False)
    assert torch.equal(out_tc, out_mma)
    assert torch.equal(d_tc.importance, d_mma.importance)
    assert torch.equal(d_tc.selected, d_mma.selected)
    assert torch.equal(d_tc.pass_counts, d_mma.pass_counts)
    # and the oracle, as for every forward
    pd, cd = O.cast_codebook(cbk.parents.numpy(), cbk.children.numpy(), dt)
    cfg = oracle_config(dict(w.__dict__), "entropy", 1.0)
    res = O.forward(qn, kn, vn, pd, cd, cfg)
    quant = check_quantization(quant_arrays(st, w.B, w.H), O.split_heads(kn, w.H), O.split_heads(vn, w.H), pd, cd,
                               dt, res["quant"], tag=w.name)
    if quant is not res["quant"]:
        res = O.forward(qn, kn, vn, pd, cd, cfg, quant=quant)
    check_routing(d_tc, res, dt, w.name)
    got = out_tc.cpu().numpy().transpose(0, 2, 1, 3).reshape(w.B, w.T, w.E)
    err = normrel(got, res["out_bte"])
    assert err <= OUT_TOL[dt], f"{w.name}: output normrel {err}"


def test_device_fault_record_starts_clear() -> None:
    code = ctypes.c_int(-1)
    _lib.check(_lib.load().avq_device_fault(ctypes.byref(code), None), "avq_device_fault")
    assert code.value == 0
