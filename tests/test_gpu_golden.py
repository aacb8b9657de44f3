"""CUDA path vs the reference's recorded outputs (tests/golden) and the oracle.

Every golden case is replayed through the C ABI (quantize, forward, append):
assignments, counts, aggregates and routed indices must equal the reference
bit for bit; outputs must be within 2e-5 (fp32) / 1e-2 (bf16, fp16)
normwise of the reference, and match the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import golden_io as G
from oracle import avq_oracle as O
from parity import (OUT_TOL, assert_quant_equal, check_quantization, check_routing, cuda_forward_heads,
                    finite_normrel, heads_view, normrel, oracle_config, quant_arrays, to_dev)

pytestmark = pytest.mark.gpu


def _golden_quant(g: G.Golden, i: int, shape_g: tuple) -> dict:
    return {
        "passign": g.get(f"quant{i}_passign").reshape(shape_g[0], -1).astype(np.int64),
        "cassign": g.get(f"quant{i}_cassign").reshape(shape_g[0], -1).astype(np.int64),
        "pagg": g.f(f"quant{i}_pagg").reshape(shape_g[0], -1, shape_g[2]),
        "cagg": g.f(f"quant{i}_cagg").reshape(shape_g[0], -1, shape_g[1], shape_g[2]),
        "pcnt": g.get(f"quant{i}_pcnt").reshape(shape_g[0], -1),
        "ccnt": g.get(f"quant{i}_ccnt").reshape(shape_g[0], -1, shape_g[1]),
    }


def _cfg(g: G.Golden) -> O.ForwardConfig:
    hc = g.meta["config"]["hopfield"]
    return oracle_config(g.w, hc["adaptive"], hc["alpha"], hc["beta_init"])


@pytest.mark.parametrize("name", G.case_names())
def test_golden_case(name: str) -> None:
    from avqa_b200 import ops
    g = G.load(name)
    if g.meta.get("bcar_decay"):
        pytest.skip("BCAR adapts the codebook between quantization and attention: tests/test_gpu_bcar.py")
    if g.meta.get("dense"):
        pytest.skip("the dense path has no quantization: tests/test_gpu_dense.py")
    w, dt = g.w, g.dt
    cfg = _cfg(g)
    B, H, D, M0, C = w["B"], w["H"], w["D"], w["M0"], w["C"]
    q, k, v = g.inputs()
    P32, C32 = g.get("parents32"), g.get("children32")
    cb = ops.prepare_codebook(torch.from_numpy(P32), torch.from_numpy(C32), G.TD[dt], torch.device("cuda"))
    pd, cd = O.cast_codebook(P32, C32, dt)
    # the cast codebook equals the oracle's
    np.testing.assert_array_equal(cb.parents.float().cpu().numpy(), pd)
    np.testing.assert_array_equal(cb.children.float().cpu().numpy(), cd)
    qd, kd, vd = to_dev(q, dt), to_dev(k, dt), to_dev(v, dt)
    tol = OUT_TOL[dt]
    if w["decode_steps"]:
        from avqa_b200.workloads import Workload, make_decode_tokens
        st = ops.quantize(heads_view(kd, H), heads_view(vd, H), cb, keep_sums=True)
        toks = [tuple(O.rnd(x.numpy(), dt) for x in tok) for tok in make_decode_tokens(Workload(**w), w["decode_steps"])]

        def calls():
            kk, vv = k, v
            for (qt, kt, vt) in toks:
                ops.append(st, heads_view(to_dev(kt, dt), H), heads_view(to_dev(vt, dt), H), cb)
                kk, vv = np.concatenate([kk, kt], 1), np.concatenate([vv, vt], 1)
                yield to_dev(qt, dt), kk, vv, st, qt
    elif w["q_chunk"]:
        st = ops.quantize(heads_view(kd, H), heads_view(vd, H), cb)

        def calls():
            for c0 in range(0, w["T"], w["q_chunk"]):
                yield qd[:, c0:c0 + w["q_chunk"]], k, v, st, q[:, c0:c0 + w["q_chunk"]]
    else:
        st = ops.quantize(heads_view(kd, H), heads_view(vd, H), cb)

        def calls():
            yield qd, k, v, st, q
    sel_i = 0
    for ci, (qdev, kfull, vfull, st, qnp) in enumerate(calls()):
        mask = g.mask_for(qnp.shape[1], kfull.shape[1])
        res = O.forward(qnp, kfull, vfull, pd, cd, cfg, mask=mask)
        got_q = quant_arrays(st, B, H)
        if got_q["passign"] is not None:
            quant = check_quantization(got_q, O.split_heads(kfull, H), O.split_heads(vfull, H), pd, cd, dt,
                                       res["quant"], tag=f"{name} call{ci} vs oracle")
            if quant is not res["quant"]:
                res = O.forward(qnp, kfull, vfull, pd, cd, cfg, quant=quant, mask=mask)
        else:
            assert_quant_equal(got_q, res["quant"], tag=f"{name} call{ci} vs oracle")
        want = _golden_quant(g, ci, (B * H, C, D))
        if got_q["passign"] is not None:
            np.testing.assert_array_equal(got_q["passign"], want["passign"])
            np.testing.assert_array_equal(got_q["cassign"], want["cassign"])
        for key in ("pagg", "cagg", "pcnt", "ccnt"):
            np.testing.assert_array_equal(got_q[key], want[key], err_msg=f"{name} call{ci} {key} vs reference")
        if res.get("naive"):
            continue
        present = None
        if mask is not None:  # the codeword visibility bits, compared with the oracle's
            present = ops.codeword_presence(st, qnp.shape[1], torch.from_numpy(np.ascontiguousarray(mask)))
            bits = present.cpu().numpy().view(np.uint32)
            got_p = ((bits[..., :, None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(*bits.shape[:2], -1)
            np.testing.assert_array_equal(got_p[..., :M0].astype(bool), res["present"], err_msg=f"{name} present")
        out, diag = cuda_forward_heads(heads_view(qdev, H), st, cb, cfg, present)
        check_routing(diag, res, dt, tag=f"{name} call{ci}")
        for s in diag.selections():
            gs = g.get(f"sel{sel_i}").reshape(B * H, -1)
            np.testing.assert_array_equal(s.long().cpu().numpy(), gs, err_msg=f"{name} sel{sel_i} vs reference")
            sel_i += 1
        out_bte = out.transpose(0, 2, 1, 3).reshape(B, -1, H * D)
        ref_out = g.get(f"out{ci}").reshape(out_bte.shape)
        err_ref, _ = finite_normrel(out_bte, ref_out, f"{name} call{ci} vs reference")
        err_orc, _ = finite_normrel(out_bte, res["out_bte"], f"{name} call{ci} vs oracle")
        assert err_ref <= tol and err_orc <= tol, f"{name} call{ci}: {err_ref} vs reference, {err_orc} vs oracle"
