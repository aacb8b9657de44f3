"""The tcgen05 kernels against the mma.sync kernels and the oracle.

The parent-attention and assignment kernels implement the same rounding
points as their mma.sync counterparts, so the importance, every selection
and every assignment must agree bit for bit; the correction kernels differ
only in the order of fp32 additions, so the outputs agree to 1e-5 normwise.  The shapes cover the kernel's edges: query counts that leave dead rows
in the last 128-query tile (and a last 64-query tile beyond T), parent counts
that are not a multiple of the 64-parent chunk, empty parents, D = 64 and
128, bf16 and fp16, several routing passes.  ``avq_device_fault`` must stay 0
(no bounded wait gave up).
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
    Workload("hvaq_bf16", B=2, T=160, S=900, H=2, D=64, M0=64, C=4, P=12, dtype="bf16", keys="mixture", seed=46,
             hvaq=True),
    Workload("quirk_bf16", B=1, T=64, S=200, H=2, D=64, M0=8, C=4, P=8, dtype="bf16", keys="mixture", seed=47,
             passes=2, pass_decay=1.0),
    # 5 and 7 parent chunks (the last one partial): the first pass's four logit slots run
    # out at different chunks and the second pass starts on an odd chunk
    Workload("m320_bf16", B=1, T=200, S=2048, H=2, D=128, M0=320, C=4, P=16, dtype="bf16", keys="mixture",
             seed=49),
    Workload("m440_d64_bf16", B=1, T=130, S=2048, H=2, D=64, M0=440, C=4, P=16, dtype="bf16", keys="aniso",
             seed=50),
    # one CTA per SM: 32 and 64 parent chunks
    Workload("m2048_bf16", B=1, T=160, S=4096, H=1, D=128, M0=2048, C=4, P=64, dtype="bf16", keys="mixture",
             seed=48),
    Workload("m4096_bf16", B=1, T=130, S=8192, H=1, D=128, M0=4096, C=8, P=128, dtype="bf16", keys="mixture",
             seed=59),
    # the HVAQ rescaling pass on tcgen05: fp16 with three routing passes (the
    # long-context multi-pass shape, reduced), D = 128 (one CTA per SM), a
    # budget filling the gathered 64-row tile, and one above it (both passes
    # then run on the mma.sync kernels)
    Workload("mp_hvaq_f16", B=2, T=300, S=2048, H=2, D=64, M0=256, C=4, P=48, dtype="f16", keys="student_t",
             seed=60, passes=3, pass_decay=0.5, hvaq=True),
    Workload("hvaq_d128_bf16", B=1, T=200, S=1500, H=2, D=128, M0=192, C=4, P=24, dtype="bf16", keys="mixture",
             seed=61, hvaq=True),
    Workload("hvaq_p64_f16", B=1, T=129, S=1200, H=2, D=64, M0=128, C=8, P=64, dtype="f16", keys="aniso", seed=62,
             hvaq=True, passes=2, pass_decay=0.5),
    Workload("hvaq_p80_bf16", B=1, T=100, S=1200, H=2, D=64, M0=128, C=4, P=80, dtype="bf16", keys="mixture",
             seed=63, hvaq=True),
    # the fp16 correction with eight children and D = 128 (two bf16 value planes)
    Workload("f16_c8_d128", B=2, T=257, S=2000, H=2, D=128, M0=160, C=8, P=20, dtype="f16", keys="aniso", seed=64),
]


def _forward(w: Workload, q, st, cb, tc: bool):
    os.environ["AVQ_DISABLE_TCGEN05"] = "0" if tc else "1"
    try:
        out, diag = ops.forward(heads_view(q, w.H), cb, st, min(w.P, w.M0), w.passes, w.pass_decay,
                                1 if w.hvaq else 0, w.D ** -0.5, 1.0, diagnostics=True)
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
    assert normrel(out_tc.cpu().numpy(), out_mma.cpu().numpy()) < 1e-5
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


QCASES = [
    Workload("q_tail_bf16", B=2, T=8, S=300, H=2, D=128, M0=200, C=3, P=8, dtype="bf16", keys="mixture", seed=51),
    Workload("q_d64_f16", B=1, T=8, S=1000, H=3, D=64, M0=136, C=8, P=8, dtype="f16", keys="aniso", seed=52),
    Workload("q_big_bf16", B=1, T=8, S=2048, H=2, D=128, M0=1024, C=4, P=8, dtype="bf16", keys="student_t", seed=53),
    # the child stage's other lane splits: 16 lanes per child row (C <= 2, D = 128), 8 (C = 1, D = 64)
    Workload("q_c2_bf16", B=1, T=8, S=900, H=2, D=128, M0=96, C=2, P=8, dtype="bf16", keys="mixture", seed=57),
    Workload("q_c1_f16", B=2, T=8, S=500, H=1, D=64, M0=64, C=1, P=8, dtype="f16", keys="aniso", seed=58),
]


def _quantize(w: Workload, k, v, cb, tc: bool):
    os.environ["AVQ_DISABLE_TCGEN05"] = "0" if tc else "1"
    try:
        st = ops.quantize(heads_view(k, w.H), heads_view(v, w.H), cb, keep_sums=True)
        torch.cuda.synchronize()
    finally:
        os.environ.pop("AVQ_DISABLE_TCGEN05", None)
    code = ctypes.c_int(-1)
    _lib.check(_lib.load().avq_device_fault(ctypes.byref(code), None), "avq_device_fault")
    assert code.value == 0
    return st


def _assert_same_quant(a, b, tag: str) -> None:
    for name in ("passign", "cassign", "pcnt", "ccnt", "nvalid", "gmin", "pacc", "cacc"):
        assert torch.equal(getattr(a, name), getattr(b, name)), f"{tag}: {name}"
    for name in ("pagg", "cagg"):
        assert torch.equal(getattr(a, name).view(torch.int16), getattr(b, name).view(torch.int16)), f"{tag}: {name}"


@pytest.mark.parametrize("w", QCASES, ids=lambda w: w.name)
def test_tcgen05_assignment_matches_mma_and_oracle(w: Workload) -> None:
    dt = w.dtype
    _, k, v = make_inputs(w)
    kn, vn = (O.rnd(x.numpy(), dt) for x in (k, v))
    kh0 = torch.from_numpy(kn).view(w.B, w.S, w.H, w.D).transpose(1, 2)[0]
    cbk = codebook_from_keys(kh0, w.M0, w.C, w.seed)
    cb = ops.prepare_codebook(cbk.parents, cbk.children, TORCH_DTYPE[dt], torch.device("cuda"))
    kd, vd = to_dev(kn, dt), to_dev(vn, dt)
    a = _quantize(w, kd, vd, cb, True)
    b = _quantize(w, kd, vd, cb, False)
    _assert_same_quant(a, b, w.name)
    pd, cd = O.cast_codebook(cbk.parents.numpy(), cbk.children.numpy(), dt)
    want = O.quantize(O.split_heads(kn, w.H), O.split_heads(vn, w.H), pd, cd, dt)
    check_quantization(quant_arrays(a, w.B, w.H), O.split_heads(kn, w.H), O.split_heads(vn, w.H), pd, cd, dt, want,
                       tag=w.name)


def test_tcgen05_assignment_non_finite_inputs() -> None:
    """A NaN distance wins the parent argmin (torch.argmin): a NaN key and a
    parent with an infinite element take the kernel's scalar path."""
    w = Workload("q_nonfinite", B=1, T=8, S=256, H=1, D=128, M0=128, C=4, P=8, dtype="bf16", keys="mixture", seed=54)
    _, k, v = make_inputs(w)
    kn, vn = (O.rnd(x.numpy(), "bf16") for x in (k, v))
    kn[0, 5, 3] = np.nan
    kh0 = torch.from_numpy(np.nan_to_num(kn)).view(w.B, w.S, w.H, w.D).transpose(1, 2)[0]
    cbk = codebook_from_keys(kh0, w.M0, w.C, w.seed)
    parents = cbk.parents.clone()
    parents[0, 17, 9] = float("inf")
    cb = ops.prepare_codebook(parents, cbk.children, torch.bfloat16, torch.device("cuda"))
    kd, vd = to_dev(kn, "bf16"), to_dev(vn, "bf16")
    a = _quantize(w, kd, vd, cb, True)
    b = _quantize(w, kd, vd, cb, False)
    assert torch.equal(a.passign, b.passign) and torch.equal(a.cassign, b.cassign)
    assert int(a.passign[0, 5]) == 0  # every distance of the NaN key is NaN: the first parent
    pd, cd = O.cast_codebook(parents.numpy(), cbk.children.numpy(), "bf16")
    want = O.quantize(O.split_heads(kn, w.H), O.split_heads(vn, w.H), pd, cd, "bf16")
    np.testing.assert_array_equal(a.passign.cpu().numpy(), want.parent_assignments)


@pytest.mark.parametrize("dt,D,C", [("bf16", 128, 4), ("f16", 64, 8), ("bf16", 128, 2)])
def test_tcgen05_assignment_integer_ties(dt: str, D: int, C: int) -> None:
    """Small-integer keys and codebooks: the child cross terms are integers
    whose dtype rounding often sits exactly on a tie, where the fp32 error
    bound cannot decide and the row is summed again in fp64; distance ties
    exercise the first-minimum rule."""
    B, S, H, M0 = 1, 1536, 2, 64
    g = torch.Generator().manual_seed(55 + D + C)
    kn = torch.randint(-6, 7, (B, S, H * D), generator=g).float().numpy()
    vn = O.rnd(torch.randn(B, S, H * D, generator=g).numpy(), dt)
    parents = torch.randint(-6, 7, (H, M0, D), generator=g).float()
    children = parents[:, :, None, :] + torch.randint(-2, 3, (H, M0, C, D), generator=g).float()
    cb = ops.prepare_codebook(parents, children, TORCH_DTYPE[dt], torch.device("cuda"))
    w = Workload("q_int", B=B, T=8, S=S, H=H, D=D, M0=M0, C=C, P=8, dtype=dt, keys="mixture", seed=55)
    kd, vd = to_dev(kn, dt), to_dev(vn, dt)
    a = _quantize(w, kd, vd, cb, True)
    b = _quantize(w, kd, vd, cb, False)
    _assert_same_quant(a, b, f"int_{dt}_{D}_{C}")
    pd, cd = O.cast_codebook(parents.numpy(), children.numpy(), dt)
    want = O.quantize(O.split_heads(kn, H), O.split_heads(vn, H), pd, cd, dt)
    np.testing.assert_array_equal(a.passign.cpu().numpy().reshape(want.parent_assignments.shape),
                                  want.parent_assignments)
    np.testing.assert_array_equal(a.cassign.cpu().numpy().reshape(want.child_assignments.shape),
                                  want.child_assignments)


def test_tcgen05_assignment_large_f16_takes_the_guarded_scan() -> None:
    """f16 keys large enough that k_sq + max p_sq exceeds a quarter of the
    f16 range: the parent scan keeps its NaN tracking and separate doubling."""
    w = Workload("q_large_f16", B=1, T=8, S=700, H=2, D=64, M0=96, C=4, P=8, dtype="f16", keys="mixture", seed=56)
    _, k, v = make_inputs(w)
    kn, vn = O.rnd(12.0 * k.numpy(), "f16"), O.rnd(v.numpy(), "f16")
    kh0 = torch.from_numpy(kn).view(w.B, w.S, w.H, w.D).transpose(1, 2)[0]
    cbk = codebook_from_keys(kh0, w.M0, w.C, w.seed)
    pd, cd = O.cast_codebook(cbk.parents.numpy(), cbk.children.numpy(), "f16")
    assert float(O.sq_norms(kn.reshape(-1, w.D), "f16").max() + O.sq_norms(pd.reshape(-1, w.D), "f16").max()) > 16376
    cb = ops.prepare_codebook(cbk.parents, cbk.children, torch.float16, torch.device("cuda"))
    kd, vd = to_dev(kn, "f16"), to_dev(vn, "f16")
    a = _quantize(w, kd, vd, cb, True)
    b = _quantize(w, kd, vd, cb, False)
    _assert_same_quant(a, b, w.name)
    want = O.quantize(O.split_heads(kn, w.H), O.split_heads(vn, w.H), pd, cd, "f16")
    check_quantization(quant_arrays(a, w.B, w.H), O.split_heads(kn, w.H), O.split_heads(vn, w.H), pd, cd, "f16", want,
                       tag=w.name)
