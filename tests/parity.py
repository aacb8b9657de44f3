"""Parity helpers: drive the CUDA path and the oracle on the same inputs and
compare them stage by stage.

Rules (the reference's parity contract):
* assignments, routed indices: bit-exact;
* counts: exact; aggregates: bit-exact (same fp32 key-order sums);
* outputs: normwise relative error <= 2e-5 (fp32) / 1e-2 (bf16, fp16),
  against the oracle and the recorded reference outputs.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import avq_oracle as O

TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
OUT_TOL = {"f32": 2e-5, "bf16": 1e-2, "f16": 1e-2}


def normrel(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))


def finite_normrel(got: np.ndarray, want: np.ndarray, tag: str = "") -> tuple[float, int]:
    """Normwise error over the finite entries, after checking that both sides
    have their non-finite entries (the reference's own NaN/inf outputs, e.g.
    fp16 overflow) in the same places; returns (error, non-finite rows)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    bad_g, bad_w = ~np.isfinite(got), ~np.isfinite(want)
    assert np.array_equal(bad_g, bad_w), (f"{tag}: non-finite outputs differ: {int(bad_g.sum())} on the GPU, "
                                          f"{int(bad_w.sum())} in the oracle")
    keep = ~bad_g
    return normrel(got[keep], want[keep]), int(bad_g.reshape(-1, got.shape[-1]).any(-1).sum())


def to_dev(x: np.ndarray, dt: str, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device=device, dtype=TD[dt])


def oracle_config(w: dict, adaptive: str = "entropy", alpha: float = 1.0, beta_init: float = 0.0) -> O.ForwardConfig:
    return O.ForwardConfig(num_heads=w["H"], num_codewords=w["M0"], children_per_codeword=w["C"],
                           refinement_budget=w["P"], dtype=w["dtype"], passes=w["passes"],
                           pass_decay=w["pass_decay"], hvaq=w["hvaq"], hvaq_adaptive=adaptive,
                           hvaq_beta_init=beta_init, hvaq_alpha=alpha)


def cuda_forward_heads(qg_bhtd: torch.Tensor, state, cb, cfg: O.ForwardConfig, present=None):
    """Run ops.forward with diagnostics; returns (out [B,H,T,D] numpy, diag)."""
    from avqa_b200 import ops
    D = qg_bhtd.shape[-1]
    hv = 0 if not cfg.hvaq or cfg.hvaq_adaptive == "none" else {"entropy": 1, "linear": 2}[cfg.hvaq_adaptive]
    beta0 = cfg.hvaq_beta_init if cfg.hvaq_beta_init > 0 else 1.0 / np.sqrt(D)
    out, diag = ops.forward(qg_bhtd, cb, state, min(cfg.refinement_budget, cfg.num_codewords), cfg.passes,
                            cfg.pass_decay, hv, float(beta0), cfg.hvaq_alpha, diagnostics=True, present=present)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), diag


def heads_view(x_bte: torch.Tensor, H: int) -> torch.Tensor:
    B, T, E = x_bte.shape
    return x_bte.view(B, T, H, E // H).transpose(1, 2)


def quant_arrays(state, B: int, H: int) -> dict:
    pc, cc = state.counts_in_dtype()
    G = B * H
    return {
        "passign": state.passign.long().cpu().numpy() if state.passign is not None else None,
        "cassign": state.cassign.long().cpu().numpy() if state.cassign is not None else None,
        "pagg": state.pagg.float().cpu().numpy(), "cagg": state.cagg.float().cpu().numpy(),
        "pcnt": pc.float().cpu().numpy().reshape(G, -1), "ccnt": cc.float().cpu().numpy().reshape(G, *cc.shape[1:]),
    }


def ulp(x: np.ndarray, dt: str) -> np.ndarray:
    """Spacing of dtype values at |x| (normal range)."""
    mant = {"f32": 23, "bf16": 7, "f16": 10}[dt]
    ax = np.maximum(np.abs(np.asarray(x, np.float64)), 1e-30)
    return np.exp2(np.floor(np.log2(ax)) - mant)


def possible_parent_distances(k: np.ndarray, p: np.ndarray, ksq: float, psq: float, dt: str) -> tuple[float, float]:
    """Range of the reference-rounded distance when the fp32 accumulation of
    k.p may err by up to 2^-20 |k||p| (any summation order, any tensor-core
    accumulation), i.e. the cross term may round to a neighbouring value."""
    x = float(np.dot(k.astype(np.float64), p.astype(np.float64)))
    delta = 2.0 ** -20 * float(np.linalg.norm(k) * np.linalg.norm(p)) + 1e-30
    t1 = O.rnd(np.float64(ksq) + np.float64(psq), dt)
    vals = []
    for xc in (x - delta, x, x + delta):
        cross = O.rnd(xc, dt)
        vals.append(float(O.rnd(np.float64(t1) - O.rnd(2.0 * np.float64(cross), dt), dt)))
    return min(vals), max(vals)


def certify_assignment_flips(keys: np.ndarray, parents: np.ndarray, H: int, got: np.ndarray, want: np.ndarray,
                             dt: str, tag: str = "") -> int:
    """Every key whose parent differs from the oracle's must be a near-tie
    that an fp32 accumulation difference explains; returns the count."""
    bad = np.argwhere(got != want)
    for g, s in bad:
        k = keys[g, s]
        pg = parents[g % H]
        ksq = O.sq_norms(k[None], dt)[0]
        pc, po = int(got[g, s]), int(want[g, s])
        lo_c, _ = possible_parent_distances(k, pg[pc], ksq, O.sq_norms(pg[pc][None], dt)[0], dt)
        _, hi_o = possible_parent_distances(k, pg[po], ksq, O.sq_norms(pg[po][None], dt)[0], dt)
        assert lo_c < hi_o or (lo_c == hi_o and pc < po), f"{tag}: key ({g},{s}) parent {pc} vs {po} is no near-tie"
    n = len(bad)
    assert n <= max(2, got.size // 1000), f"{tag}: {n} assignment flips of {got.size}"
    return n


def quant_from_arrays(got: dict, values: np.ndarray, M0: int, C: int, dt: str) -> O.Quantization:
    """The oracle's aggregation run on the CUDA assignments (checks the
    aggregation kernels independently of the distance kernel)."""
    pa, ca = got["passign"], got["cassign"]
    G = pa.shape[0]
    pagg = O.sequential_bucket_sums(values, pa, M0, dt)
    cagg = O.sequential_bucket_sums(values, pa * C + ca, M0 * C, dt).reshape(G, M0, C, -1)
    pce = np.stack([np.bincount(pa[g], minlength=M0) for g in range(G)])
    cce = np.stack([np.bincount(pa[g] * C + ca[g], minlength=M0 * C) for g in range(G)]).reshape(G, M0, C)
    sat = O.count_saturation(dt)
    return O.Quantization(pa, ca, pagg, cagg, np.minimum(pce, sat).astype(np.float32),
                          np.minimum(cce, sat).astype(np.float32), pce, cce)


def check_quantization(got: dict, keys_g: np.ndarray, values_g: np.ndarray, parents: np.ndarray,
                       children: np.ndarray, dt: str, want: O.Quantization, tag: str = "") -> O.Quantization:
    """Assignments equal the oracle's up to certified near-ties; children,
    counts and aggregates are then exact given the CUDA parent assignments.
    Returns the quantization the rest of the comparison should use."""
    H, M0, C, _ = children.shape

    def children_of(g: int, p: int) -> np.ndarray:
        return children[g % H, p]

    certify_assignment_flips(keys_g, parents, H, got["passign"], want.parent_assignments, dt, tag)
    same = got["passign"] == want.parent_assignments
    np.testing.assert_array_equal(got["cassign"][same], want.child_assignments[same], err_msg=f"{tag} children")
    if same.all():
        exact = want
    else:
        exact = quant_from_arrays(got, values_g, M0, C, dt)
        for g, s in np.argwhere(~same):  # child choice inside the CUDA-chosen parent, exactly
            ch = children_of(g, got["passign"][g, s])
            dc = O.child_distances(keys_g[g:g + 1, s:s + 1], ch[None, None], dt)
            assert int(O.first_argmin(dc)[0, 0]) == int(got["cassign"][g, s]), f"{tag} child of flipped key"
    np.testing.assert_array_equal(got["pcnt"], exact.parent_counts, err_msg=f"{tag} parent counts")
    np.testing.assert_array_equal(got["ccnt"], exact.child_counts, err_msg=f"{tag} child counts")
    np.testing.assert_array_equal(got["pagg"], exact.parent_aggregates, err_msg=f"{tag} parent aggregates")
    np.testing.assert_array_equal(got["cagg"], exact.child_aggregates, err_msg=f"{tag} child aggregates")
    return exact


def assert_quant_equal(got: dict, want: O.Quantization, tag: str = "") -> None:
    if got["passign"] is not None:
        np.testing.assert_array_equal(got["passign"], want.parent_assignments, err_msg=f"{tag} parent assignments")
        np.testing.assert_array_equal(got["cassign"], want.child_assignments, err_msg=f"{tag} child assignments")
    np.testing.assert_array_equal(got["pcnt"], want.parent_counts, err_msg=f"{tag} parent counts")
    np.testing.assert_array_equal(got["ccnt"], want.child_counts, err_msg=f"{tag} child counts")
    np.testing.assert_array_equal(got["pagg"], want.parent_aggregates, err_msg=f"{tag} parent aggregates")
    np.testing.assert_array_equal(got["cagg"], want.child_aggregates, err_msg=f"{tag} child aggregates")


def check_routing(diag, res: dict, dt: str, tag: str = "") -> None:
    """Importance equals the oracle's up to rare one-ulp differences (fp32
    accumulation inside the parent-logit MMA); the routed indices are the
    exact stable top-k of the CUDA importance, and equal the oracle's unless
    an importance difference explains the change."""
    imp = diag.importance.cpu().numpy()
    want = res["importance0"]
    diff = imp != want
    n = int(diff.sum())
    assert n <= max(2, imp.size // 500), f"{tag}: {n} importance differences"
    if n:
        assert np.all(np.abs(imp[diff] - want[diff]) <= 1.01 * ulp(want[diff], dt)), f"{tag}: importance off by > 1 ulp"
    sels = [s.long().cpu().numpy() for s in diag.selections()]
    assert len(sels) == len(res["selected"]), f"{tag}: pass count"
    np.testing.assert_array_equal(sels[0], O.stable_topk_desc(imp, sels[0].shape[-1]), err_msg=f"{tag} routing")
    for k, (a, b) in enumerate(zip(sels, res["selected"])):
        if n == 0:
            np.testing.assert_array_equal(a, b, err_msg=f"{tag} pass {k} selected indices")
        else:
            rows = np.unique(np.argwhere(diff)[:, 0])
            keep = np.setdiff1d(np.arange(a.shape[0]), rows)
            np.testing.assert_array_equal(a[keep], b[keep], err_msg=f"{tag} pass {k} selected indices")


def logit_near_ties(q: np.ndarray, parents: np.ndarray, dt: str) -> np.ndarray:
    """Per parent, whether the dtype rounding of the fp32-accumulated logit
    q.p could differ from the exactly rounded one: the exact value lies
    within 2^-20 |q||p| (any summation order, any tensor-core accumulation)
    of a dtype rounding boundary.  ``q`` [D], ``parents`` [M0, D]."""
    q64, p64 = np.asarray(q, np.float64), np.asarray(parents, np.float64)
    raw = p64 @ q64
    delta = 2.0 ** -20 * np.linalg.norm(q64) * np.linalg.norm(p64, axis=-1) + 1e-30
    return O.rnd(raw - delta, dt) != O.rnd(raw + delta, dt)


def check_routing_single_query(diag, res: dict, qg: np.ndarray, parents: np.ndarray, H: int, dt: str,
                               tag: str = "") -> int:
    """Routing of one query per (b,h) (decode).  The importance n * p then is
    a single query's probability, so one logit that the fp32 GEMM rounds to
    the neighbouring dtype value moves it by more than an ulp.  Every row
    whose importance differs from the oracle's must hold such a certified
    near-tie logit (``logit_near_ties``); the other rows must match exactly,
    and every row's selection must be the exact stable top-k of the GPU
    importance.  Returns the number of differing rows."""
    imp = diag.importance.cpu().numpy()
    want = res["importance0"]
    rows = np.unique(np.argwhere(imp != want)[:, 0])
    for g in rows:
        assert logit_near_ties(qg[g, 0], parents[g % H], dt).any(), f"{tag}: row {g} differs without a near-tie"
    assert len(rows) <= max(2, imp.shape[0] // 10), f"{tag}: {len(rows)} of {imp.shape[0]} rows differ"
    sels = [s.long().cpu().numpy() for s in diag.selections()]
    np.testing.assert_array_equal(sels[0], O.stable_topk_desc(imp, sels[0].shape[-1]), err_msg=f"{tag} routing")
    keep = np.setdiff1d(np.arange(imp.shape[0]), rows)
    for k, (a, b) in enumerate(zip(sels, res["selected"])):
        np.testing.assert_array_equal(a[keep], b[keep], err_msg=f"{tag} pass {k} selected indices")
    return len(rows)


def assert_routing_equal(diag, res: dict, tag: str = "") -> None:
    sels = [s.long().cpu().numpy() for s in diag.selections()]
    want = res["selected"]
    assert len(sels) == len(want), f"{tag}: {len(sels)} passes vs {len(want)}"
    for k, (a, b) in enumerate(zip(sels, want)):
        np.testing.assert_array_equal(a, b, err_msg=f"{tag} pass {k} selected indices")
    imp = diag.importance.cpu().numpy()
    np.testing.assert_array_equal(imp, res["importance0"], err_msg=f"{tag} importance")
