"""Parity at the benchmark configurations' real sizes.

The CUDA path runs a whole configuration (batch 1 where the benchmark's
batch only repeats independent (b,h) slices); sampled (b,h) slices are then
checked stage by stage against the oracle on the same inputs and codebook:

* assignments equal the oracle's up to certified near-ties (the count is
  printed and bounded), counts and aggregates exactly (given those
  assignments);
* importance equal up to rare one-ulp differences (counted, bounded), routed
  indices the exact stable top-k, equal to the oracle's where no importance
  difference explains a change;
* the output within 1e-2 normwise (bf16 / fp16).

The budget floor is the GPU's global one (min over every (b,h) of the
call); the oracle slice runs with it, as a head-sharded reference would.
Run with ``-s`` to see the per-case flip and importance-difference counts.
"""
from __future__ import annotations

import json
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from avqa_b200 import ops
from avqa_b200.codebook import codebook_from_keys
from avqa_b200.workloads import TORCH_DTYPE, WORKLOADS, Workload, make_decode_tokens, make_inputs
from oracle import avq_oracle as O
from parity import (OUT_TOL, certify_assignment_flips, check_quantization, check_routing,
                    check_routing_single_query, finite_normrel, quant_from_arrays)

pytestmark = pytest.mark.gpu


def _heads(x: torch.Tensor, H: int) -> torch.Tensor:
    B, T, E = x.shape
    return x.view(B, T, H, E // H).transpose(1, 2)


def _setup(w: Workload, B: int = 1):
    """Inputs generated on the GPU and rounded to the dtype; the key-based
    codebook from batch 0 (fp32 master on the GPU)."""
    dt = TORCH_DTYPE[w.dtype]
    q, k, v = make_inputs(w, device="cuda", B=B)
    q, k, v = q.to(dt), k.to(dt), v.to(dt)
    cb32 = codebook_from_keys(_heads(k, w.H)[0].float(), w.M0, w.C, w.seed)
    cb = ops.prepare_codebook(cb32.parents, cb32.children, dt, torch.device("cuda"))
    return q, k, v, cb32, cb


def _np(x: torch.Tensor) -> np.ndarray:
    return x.float().cpu().numpy()


def _slice_quant(st: ops.QuantState, g: int, dt: str) -> dict:
    pc, cc = st.counts_in_dtype()
    return {"passign": st.passign[g:g + 1].long().cpu().numpy() if st.passign is not None else None,
            "cassign": st.cassign[g:g + 1].long().cpu().numpy() if st.cassign is not None else None,
            "pagg": _np(st.pagg[g:g + 1]), "cagg": _np(st.cagg[g:g + 1]),
            "pcnt": _np(pc[g:g + 1]), "ccnt": _np(cc[g:g + 1])}


def _slice_diag(diag, g: int):
    sels = diag.selections()
    return SimpleNamespace(importance=diag.importance[g:g + 1], selections=lambda: [s[g:g + 1] for s in sels])


def _cfg(w: Workload) -> O.ForwardConfig:
    return O.ForwardConfig(1, w.M0, w.C, w.P, w.dtype, w.passes, w.pass_decay, w.hvaq)


def _report(tag: str, **kw) -> None:
    print(json.dumps({"case": tag, **kw}))


def _check_slice(tag, w, qg, kg, vg, cb32, hh, st, g, diag, out_g, floor, want_quant=None, srow=None):
    """Oracle comparison of query group g (head hh) whose key state is row
    ``srow`` of ``st`` (default g); ``*_g`` are numpy [1, n, D]."""
    dt = w.dtype
    pd, cd = O.cast_codebook(cb32.parents[hh:hh + 1].cpu().numpy(), cb32.children[hh:hh + 1].cpu().numpy(), dt)
    got = _slice_quant(st, g if srow is None else srow, dt)
    if want_quant is None:
        want_quant = O.quantize(kg, vg, pd, cd, dt)
    exact = check_quantization(got, kg, vg, pd, cd, dt, want_quant, tag=tag)
    flips = int((got["passign"] != want_quant.parent_assignments).sum())
    res = O.forward_heads(qg, kg, vg, pd, cd, _cfg(w), quant=exact, budget_floor=floor)
    sd = _slice_diag(diag, g)
    imp_diff = int((sd.importance.cpu().numpy() != res["importance0"]).sum())
    check_routing(sd, res, dt, tag=tag)
    err, nonfinite = finite_normrel(out_g, res["out"], tag)
    _report(tag, assignment_flips=flips, keys=int(kg.shape[1]), importance_diffs=imp_diff, parents=w.M0,
            output_normwise=err, nonfinite_rows=nonfinite, budget_floor=floor)
    assert err <= OUT_TOL[dt], f"{tag}: output normrel {err}"
    assert flips <= max(2, kg.shape[1] // 2000), f"{tag}: {flips} assignment flips"
    assert imp_diff <= max(2, w.M0 // 100), f"{tag}: {imp_diff} importance differences"


def test_c2_prefill_full_size() -> None:
    """c2: T=S=8192, 32 heads x 128, M0=512, C=4, P=32, bf16 (batch 1 of 4)."""
    w = WORKLOADS["c2"]
    q, k, v, cb32, cb = _setup(w)
    st = ops.quantize(_heads(k, w.H), _heads(v, w.H), cb)
    out, diag = ops.forward(_heads(q, w.H), cb, st, w.P, diagnostics=True)
    torch.cuda.synchronize()
    floor = int(st.gmin.item())
    D = w.D
    for hh in (0, 17):
        sl = lambda x: _np(x[:, :, hh * D:(hh + 1) * D])
        _check_slice(f"c2 h={hh}", w, sl(q), sl(k), sl(v), cb32, hh, st, hh, diag, _np(out[:, hh]), floor)


def test_c4_multipass_hvaq_full_size() -> None:
    """c4: T=S=16384, 16 heads x 64, M0=256, C=4, budgets 48/24/12, HVAQ
    entropy, fp16 (batch 1 of 8)."""
    w = WORKLOADS["c4"]
    q, k, v, cb32, cb = _setup(w)
    st = ops.quantize(_heads(k, w.H), _heads(v, w.H), cb)
    beta0 = 1.0 / np.sqrt(w.D)
    out, diag = ops.forward(_heads(q, w.H), cb, st, w.P, w.passes, w.pass_decay, 1, float(beta0), 1.0,
                            diagnostics=True)
    torch.cuda.synchronize()
    floor = int(st.gmin.item())
    hh = 5
    sl = lambda x: _np(x[:, :, hh * w.D:(hh + 1) * w.D])
    _check_slice(f"c4 h={hh}", w, sl(q), sl(k), sl(v), cb32, hh, st, hh, diag, _np(out[:, hh]), floor)


def test_c5_long_context_chunks_full_size() -> None:
    """c5: S=131072 keys quantized once, 2048 queries as eight 256-query
    chunks in one call (a batch-1 key state shared by the chunk batch),
    64 heads x 128, M0=4096, C=8, P=128, bf16.  Head 9, chunks 0 and 7."""
    w = WORKLOADS["c5"]
    q, k, v, cb32, cb = _setup(w)
    st = ops.quantize(_heads(k, w.H), _heads(v, w.H), cb)
    qh = _heads(q, w.H)  # [1, H, 2048, D]
    n, tc = w.T // w.q_chunk, w.q_chunk
    qc = qh.as_strided((n, w.H, tc, w.D), (qh.stride(2) * tc, qh.stride(1), qh.stride(2), qh.stride(3)))
    out, diag = ops.forward(qc, cb, st, w.P, diagnostics=True)  # out [n, H, tc, D]
    torch.cuda.synchronize()
    floor = int(st.gmin.item())
    hh, D = 9, w.D
    kg, vg = _np(k[:, :, hh * D:(hh + 1) * D]), _np(v[:, :, hh * D:(hh + 1) * D])
    pd, cd = O.cast_codebook(cb32.parents[hh:hh + 1].cpu().numpy(), cb32.children[hh:hh + 1].cpu().numpy(), w.dtype)
    want = O.quantize(kg, vg, pd, cd, w.dtype)  # once for both chunks
    wc = Workload(**{**w.__dict__, "T": tc})
    for c in (0, n - 1):
        qg = _np(q[:, c * tc:(c + 1) * tc, hh * D:(hh + 1) * D])
        g = c * w.H + hh
        # the key state is batch 1: query group g reads state row g % H = hh
        _check_slice(f"c5 h={hh} chunk={c}", wc, qg, kg, vg, cb32, hh, st, g, diag, _np(out[c:c + 1, hh]), floor,
                     want_quant=want, srow=hh)


def test_c3_decode_full_size() -> None:
    """c3: a 32768-token prior at M0=1024, C=8, P=64 (32 heads x 128, bf16,
    batch 1 of 64), then four decode steps through the incremental append;
    after each step the state equals the oracle's re-quantization of all
    keys and the T=1 forward matches the oracle."""
    w = WORKLOADS["c3"]
    dt = TORCH_DTYPE[w.dtype]
    q0, k, v, cb32, cb = _setup(w)
    st = ops.quantize(_heads(k, w.H), _heads(v, w.H), cb, keep_sums=True)
    hh, D = 3, w.D
    kg, vg = _np(k[:, :, hh * D:(hh + 1) * D]), _np(v[:, :, hh * D:(hh + 1) * D])
    pd, cd = O.cast_codebook(cb32.parents[hh:hh + 1].cpu().numpy(), cb32.children[hh:hh + 1].cpu().numpy(), w.dtype)
    want = O.quantize(kg, vg, pd, cd, w.dtype)
    got = _slice_quant(st, hh, w.dtype)
    exact = check_quantization(got, kg, vg, pd, cd, w.dtype, want, tag="c3 prior")
    flips = int((got["passign"] != want.parent_assignments).sum())
    pa, ca = exact.parent_assignments, exact.child_assignments
    for step, (qt, kt, vt) in enumerate(make_decode_tokens(w, 4, B=1)):
        qt, kt, vt = (x.to("cuda", dt) for x in (qt, kt, vt))
        pc0, cc0 = st.pcnt[hh].clone(), st.ccnt[hh].clone()
        ops.append(st, _heads(kt, w.H), _heads(vt, w.H), cb)
        out, diag = ops.forward(_heads(qt, w.H), cb, st, w.P, diagnostics=True)
        torch.cuda.synchronize()
        floor = int(st.gmin.item())
        kn, vn, qn = (_np(x[:, :, hh * D:(hh + 1) * D]) for x in (kt, vt, qt))
        kg, vg = np.concatenate([kg, kn], 1), np.concatenate([vg, vn], 1)
        # the new key's buckets on the GPU (the counts that grew) against the
        # oracle's assignment; a different parent must be a certified near-tie
        p_gpu = int(torch.nonzero(st.pcnt[hh] - pc0)[0, 0])
        c_gpu = int(torch.nonzero(st.ccnt[hh, p_gpu] - cc0[p_gpu])[0, 0])
        one = O.quantize(kn, vn, pd, cd, w.dtype)
        certify_assignment_flips(kn, pd, 1, np.array([[p_gpu]]), one.parent_assignments, w.dtype, f"c3 step {step}")
        if p_gpu == int(one.parent_assignments[0, 0]):
            assert c_gpu == int(one.child_assignments[0, 0]), f"c3 step {step}: child"
        pa = np.concatenate([pa, np.array([[p_gpu]])], 1)
        ca = np.concatenate([ca, np.array([[c_gpu]])], 1)
        exact = quant_from_arrays({"passign": pa, "cassign": ca}, vg, w.M0, w.C, w.dtype)
        sq = _slice_quant(st, hh, w.dtype)
        for key, ref in (("pagg", exact.parent_aggregates), ("cagg", exact.child_aggregates),
                         ("pcnt", exact.parent_counts), ("ccnt", exact.child_counts)):
            np.testing.assert_array_equal(sq[key], ref, err_msg=f"c3 step {step} {key}")
        res = O.forward_heads(qn, kg, vg, pd, cd, _cfg(w), quant=exact, budget_floor=floor)
        check_routing_single_query(_slice_diag(diag, hh), res, qn, pd, 1, w.dtype, tag=f"c3 step {step}")
        err, _ = finite_normrel(_np(out[:, hh]), res["out"], f"c3 step {step}")
        _report(f"c3 h={hh} step={step}", prior_assignment_flips=flips, keys=int(kg.shape[1]),
                output_normwise=err, budget_floor=floor)
        assert err <= OUT_TOL[w.dtype], f"c3 step {step}: output normrel {err}"
