"""CUDA path vs the oracle on seeded synthetic inputs (sizes the oracle
finishes in seconds), including ragged sizes (M0, C, D, T not multiples of
the tile sizes), exact ties, empty codewords and budgets above the number
of valid parents."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from avqa_b200.codebook import codebook_from_keys
from avqa_b200.workloads import Workload, make_inputs
from oracle import avq_oracle as O
from parity import (OUT_TOL, check_quantization, check_routing, cuda_forward_heads, heads_view, normrel,
                    oracle_config, quant_arrays, to_dev)

pytestmark = pytest.mark.gpu

CASES = [
    Workload("mix_bf16_mid", B=2, T=512, S=1024, H=4, D=128, M0=128, C=4, P=16, dtype="bf16", keys="mixture", seed=21),
    Workload("mix_f16_mid", B=2, T=384, S=768, H=3, D=64, M0=96, C=4, P=12, dtype="f16", keys="mixture", seed=22),
    Workload("mix_f32_mid", B=1, T=256, S=512, H=4, D=64, M0=64, C=4, P=8, dtype="f32", keys="mixture", seed=23),
    Workload("aniso_bf16_c8", B=2, T=64, S=1024, H=2, D=128, M0=256, C=8, P=32, dtype="bf16", keys="aniso", seed=24),
    Workload("mp_hvaq_f16", B=2, T=512, S=512, H=2, D=64, M0=64, C=4, P=24, dtype="f16", keys="student_t", seed=25,
             passes=3, pass_decay=0.5, hvaq=True),
    Workload("ragged_bf16", B=3, T=37, S=301, H=2, D=72, M0=45, C=3, P=7, dtype="bf16", keys="mixture", seed=26),
    Workload("ragged_f32", B=1, T=33, S=100, H=3, D=40, M0=19, C=5, P=6, dtype="f32", keys="mixture", seed=27,
             passes=2, pass_decay=0.6),
    Workload("budget_gt_valid_bf16", B=1, T=16, S=6, H=2, D=32, M0=16, C=2, P=12, dtype="bf16", keys="mixture",
             seed=28),
    Workload("rope_bf16", B=1, T=96, S=2048, H=2, D=128, M0=256, C=8, P=32, dtype="bf16", keys="mixture_rope",
             seed=29),
    Workload("hvaq_lin_bf16", B=1, T=200, S=400, H=2, D=64, M0=40, C=4, P=10, dtype="bf16", keys="mixture", seed=30,
             hvaq=True),
    Workload("quirk_f32", B=1, T=12, S=64, H=2, D=16, M0=6, C=2, P=6, dtype="f32", keys="mixture", seed=31, passes=2,
             pass_decay=1.0),
    # routing orders of more than 256 parents: the bitonic sort instead of the radix select
    Workload("wide_budget_bf16", B=1, T=128, S=4096, H=2, D=128, M0=512, C=4, P=300, dtype="bf16", keys="mixture",
             seed=32),
    Workload("wide_budget_mp_f16", B=1, T=96, S=3072, H=2, D=64, M0=384, C=4, P=200, dtype="f16", keys="mixture",
             seed=33, passes=2, pass_decay=0.5),
]


def run_case(w: Workload, adaptive: str = "entropy", alpha: float = 1.0, ties: bool = False):
    from avqa_b200 import ops
    q, k, v = make_inputs(w)
    if ties:
        k = k[:, :4].repeat(1, w.S // 4, 1)
    dt = w.dtype
    TDT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dt]
    qn, kn, vn = (O.rnd(x.numpy(), dt) for x in (q, k, v))
    kh0 = torch.from_numpy(kn).view(w.B, w.S, w.H, w.D).transpose(1, 2)[0]
    cbk = codebook_from_keys(kh0, w.M0, w.C, w.seed)
    P32, C32 = cbk.parents.numpy(), cbk.children.numpy()
    if ties:
        C32 = C32.copy()
        C32[:, 1] = C32[:, 0]
        P32 = C32.mean(2)
    cb = ops.prepare_codebook(torch.from_numpy(P32), torch.from_numpy(C32), TDT, torch.device("cuda"))
    pd, cd = O.cast_codebook(P32, C32, dt)
    wd = dict(w.__dict__)
    cfg = oracle_config(wd, adaptive, alpha)
    res = O.forward(qn, kn, vn, pd, cd, cfg)
    st = ops.quantize(heads_view(to_dev(kn, dt), w.H), heads_view(to_dev(vn, dt), w.H), cb)
    quant = check_quantization(quant_arrays(st, w.B, w.H), O.split_heads(kn, w.H), O.split_heads(vn, w.H), pd, cd,
                               dt, res["quant"], tag=w.name)
    if quant is not res["quant"]:
        res = O.forward(qn, kn, vn, pd, cd, cfg, quant=quant)
    out, diag = cuda_forward_heads(heads_view(to_dev(qn, dt), w.H), st, cb, cfg)
    check_routing(diag, res, dt, tag=w.name)
    out_bte = out.transpose(0, 2, 1, 3).reshape(w.B, w.T, w.E)
    err = normrel(out_bte, res["out_bte"])
    assert err <= OUT_TOL[dt], f"{w.name}: output normrel {err}"
    return err


@pytest.mark.parametrize("w", CASES, ids=[c.name for c in CASES])
def test_random_case(w: Workload) -> None:
    adaptive = "linear" if w.name.startswith("hvaq_lin") else "entropy"
    run_case(w, adaptive=adaptive, alpha=0.7 if adaptive == "linear" else 1.0)


def test_exact_ties_bf16() -> None:
    w = Workload("ties", B=1, T=8, S=64, H=2, D=16, M0=8, C=2, P=8, dtype="bf16", keys="mixture", seed=32)
    run_case(w, ties=True)
