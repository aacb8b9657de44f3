"""The oracle (numpy restatement) against the reference's recorded outputs.

Pins the oracle: every case in tests/golden was produced by the reference
``AVQAttention`` itself (tests/golden/make_golden.py).  Indices, counts and
aggregates must match bit for bit; outputs within 2e-5 normwise (fp32) and
1e-2 (bf16/fp16) -- in practice they agree to ~1e-6.
"""
from __future__ import annotations

import numpy as np
import pytest

import golden_io as G
from avqa_b200.workloads import Workload, make_decode_tokens
from oracle import avq_oracle as O
from parity import OUT_TOL, finite_normrel, normrel, oracle_config


def _calls(g: G.Golden):
    w, dt = g.w, g.dt
    hc = g.meta["config"]["hopfield"]
    cfg = oracle_config(w, hc["adaptive"], hc["alpha"], hc["beta_init"])
    pd, cd = O.cast_codebook(g.get("parents32"), g.get("children32"), dt)
    q, k, v = g.inputs()
    if w["decode_steps"]:
        kk, vv = k, v
        for (qt, kt, vt) in make_decode_tokens(Workload(**w), w["decode_steps"]):
            qt, kt, vt = (O.rnd(x.numpy(), dt) for x in (qt, kt, vt))
            kk, vv = np.concatenate([kk, kt], 1), np.concatenate([vv, vt], 1)
            yield O.forward(qt, kk, vv, pd, cd, cfg)
    elif g.meta.get("bcar_decay"):
        # each call quantizes with the current codebook, adapts it (BCAR) and
        # attends with the adapted codebook over the unadapted quantization
        H, D = w["H"], w["D"]
        kg, vg = O.split_heads(k, H), O.split_heads(v, H)
        n_calls = g.meta["n_calls"]
        for _ in range(n_calls):
            quant = O.quantize(kg, vg, pd, cd, dt)
            pd, cd = O.bcar_update(kg, quant.parent_assignments, quant.child_assignments, pd, cd, w["B"],
                                   g.meta["bcar_decay"], dt)
            res = O.forward(q, k, v, pd, cd, cfg, quant=quant)
            res["codebook"] = (pd, cd)
            yield res
    elif w["q_chunk"]:
        for c0 in range(0, w["T"], w["q_chunk"]):
            qc = q[:, c0:c0 + w["q_chunk"]]
            yield O.forward(qc, k, v, pd, cd, cfg, mask=g.mask_for(qc.shape[1], k.shape[1]))
    else:
        yield O.forward(q, k, v, pd, cd, cfg, mask=g.mask_for(q.shape[1], k.shape[1]))


def _dense_out(g: G.Golden) -> np.ndarray:
    """The dense path (backend.py:190-203) on the fixture's inputs, [B, T, E]."""
    w, dt = g.w, g.dt
    H = w["H"]
    q, k, v = g.inputs()
    mask = g.mask_for(q.shape[1], k.shape[1])
    mg = None if mask is None else O.expand_mask(mask, w["B"], H)
    out = O.naive_attention(O.split_heads(q, H), O.split_heads(k, H), O.split_heads(v, H), dt, mg)
    return O.merge_heads(out, w["B"], H)


@pytest.mark.parametrize("name", G.case_names())
def test_oracle_matches_reference(name: str) -> None:
    g = G.load(name)
    w, dt = g.w, g.dt
    if g.meta.get("dense"):
        got, want = _dense_out(g), g.get("out0").reshape(w["B"], w["T"], -1)
        err, nonfinite = finite_normrel(got, want, name)
        assert err <= OUT_TOL[dt] and err <= 5e-3 * (dt != "f32") + 1e-6, err
        return
    G_ = w["B"] * w["H"]
    sel_i = imp_i = 0
    for ci, res in enumerate(_calls(g)):
        qn = res["quant"]
        np.testing.assert_array_equal(qn.parent_assignments, g.get(f"quant{ci}_passign").reshape(G_, -1))
        np.testing.assert_array_equal(qn.child_assignments, g.get(f"quant{ci}_cassign").reshape(G_, -1))
        np.testing.assert_array_equal(qn.parent_counts, g.get(f"quant{ci}_pcnt").reshape(G_, -1))
        np.testing.assert_array_equal(qn.child_counts, g.get(f"quant{ci}_ccnt").reshape(qn.child_counts.shape))
        np.testing.assert_array_equal(qn.parent_aggregates, g.f(f"quant{ci}_pagg").reshape(qn.parent_aggregates.shape))
        np.testing.assert_array_equal(qn.child_aggregates, g.f(f"quant{ci}_cagg").reshape(qn.child_aggregates.shape))
        if res.get("naive"):
            np.testing.assert_array_equal(res["out_bte"], g.get(f"out{ci}").reshape(res["out_bte"].shape))
            continue
        w_imp = g.f(f"imp{imp_i}").reshape(G_, -1)
        if dt == "f32":
            assert normrel(res["importance0"], w_imp) < 1e-6
        else:
            np.testing.assert_array_equal(res["importance0"], w_imp)
        imp_i += 1 + (len(res["selected"]) - 1 if w["passes"] > 1 else 0)
        for s in res["selected"]:
            np.testing.assert_array_equal(s, g.get(f"sel{sel_i}").reshape(G_, -1), err_msg=f"sel{sel_i}")
            sel_i += 1
        if "beta" in res:
            np.testing.assert_array_equal(res["beta"], g.f("beta0").reshape(res["beta"].shape))
        # the reference's own non-finite outputs (fp16) must sit in the same places
        err, _ = finite_normrel(res["out_bte"], g.get(f"out{ci}").reshape(res["out_bte"].shape), name)
        assert err <= OUT_TOL[dt], err
        if "codebook" in res:
            # the adapted codebook: bit for bit in bf16 / fp16, where the
            # reference's one-hot einsum sums the keys exactly in fp32; in fp32
            # that einsum rounds in its own order, so within a few ulp
            for got, key in zip(res["codebook"], ("parents", "children")):
                want = g.f(f"cb{ci}_{key}").reshape(got.shape)
                if dt == "f32":
                    np.testing.assert_allclose(got, want, rtol=4 * 2.0 ** -23, atol=1e-7, err_msg=f"{name} {key}")
                else:
                    np.testing.assert_array_equal(got, want, err_msg=f"{name} {key}")
        assert err <= 1e-5, f"oracle drifted from the reference: {err}"


def test_fixtures_cover_every_config_family() -> None:
    names = set(G.case_names())
    for must in ("c1_readme_f32", "mix_bf16", "mp_hvaq_f16", "decode_bf16", "rope_bf16", "empty_keys_bf16",
                 "ties_bf16", "mp_quirk_f32", "causal_bf16", "mask2_f32", "mask4_bf16", "bcar_bf16", "bcar_b2_f32",
                 "dense_ref_bf16", "dense_norefine_f32"):
        assert must in names
