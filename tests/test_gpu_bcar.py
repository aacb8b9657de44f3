"""BCAR online codebook adaptation through AVQAttention against the
reference's recorded calls (tests/golden/bcar_*.npz, online_adaptation.py:37-127).

Each fixture calls the reference module twice on the same inputs: the
codebook adapts after each quantization, the attention uses the adapted
codebook, and the second call quantizes against it.  The adapted codebook
must equal the reference's bit for bit in bf16 / fp16 (within a few ulp in
fp32, whose one-hot einsum rounds in its own order), the assignments and
routed indices of both calls exactly, the outputs within 1e-2 / 2e-5.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import golden_io as G
from avqa_b200 import AVQAttention, AVQConfig
from avqa_b200.config import AttentionShapeConfig, CodebookConfig, RefinementConfig, RoutingConfig
from parity import OUT_TOL, finite_normrel

pytestmark = pytest.mark.gpu

CASES = [n for n in G.case_names() if n.startswith("bcar")]


@pytest.mark.parametrize("name", CASES)
def test_bcar_matches_reference(name: str) -> None:
    g = G.load(name)
    w, dt = g.w, g.dt
    cfg = AVQConfig(attention=AttentionShapeConfig(embed_dim=w["H"] * w["D"], num_heads=w["H"]),
                    codebook=CodebookConfig(num_codewords=w["M0"], children_per_codeword=w["C"], bcar_enabled=True,
                                            bcar_decay=g.meta["bcar_decay"]),
                    routing=RoutingConfig(strategy="topp", refinement_budget=w["P"]),
                    refinement=RefinementConfig(passes=w["passes"], pass_decay=w["pass_decay"]))
    m = AVQAttention(cfg, in_proj=False, out_proj=False)
    m.codebook.parents = torch.from_numpy(g.get("parents32")).clone()
    m.codebook.children = torch.from_numpy(g.get("children32")).clone()
    q, k, v = (G.to_torch(x if x.dtype == np.uint16 else x, dt).cuda() for x in (g.get("q"), g.get("k"), g.get("v")))
    for ci in range(g.meta["n_calls"]):
        out = m(q, k, v).cpu().numpy()
        np.testing.assert_array_equal(m.last_parent_assignments.cpu().numpy().reshape(-1),
                                      g.get(f"quant{ci}_passign").reshape(-1), err_msg=f"{name} call {ci} assignments")
        for key, got in (("parents", m.codebook.parents), ("children", m.codebook.children)):
            got = got.float().cpu().numpy()
            want = g.f(f"cb{ci}_{key}").reshape(got.shape)
            if dt == "f32":
                np.testing.assert_allclose(got, want, rtol=4 * 2.0 ** -23, atol=1e-7, err_msg=f"{name} {key}")
            else:
                np.testing.assert_array_equal(got, want, err_msg=f"{name} call {ci} {key}")
        err, _ = finite_normrel(out, g.get(f"out{ci}").reshape(out.shape), f"{name} call {ci}")
        assert err <= OUT_TOL[dt], f"{name} call {ci}: {err}"
