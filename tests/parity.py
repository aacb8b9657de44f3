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


def to_dev(x: np.ndarray, dt: str, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device=device, dtype=TD[dt])


def oracle_config(w: dict, adaptive: str = "entropy", alpha: float = 1.0, beta_init: float = 0.0) -> O.ForwardConfig:
    return O.ForwardConfig(num_heads=w["H"], num_codewords=w["M0"], children_per_codeword=w["C"],
                           refinement_budget=w["P"], dtype=w["dtype"], passes=w["passes"],
                           pass_decay=w["pass_decay"], hvaq=w["hvaq"], hvaq_adaptive=adaptive,
                           hvaq_beta_init=beta_init, hvaq_alpha=alpha)


def cuda_forward_heads(qg_bhtd: torch.Tensor, state, cb, cfg: O.ForwardConfig):
    """Run ops.forward with diagnostics; returns (out [B,H,T,D] numpy, diag)."""
    from avqa_b200 import ops
    D = qg_bhtd.shape[-1]
    hv = 0 if not cfg.hvaq or cfg.hvaq_adaptive == "none" else {"entropy": 1, "linear": 2}[cfg.hvaq_adaptive]
    beta0 = cfg.hvaq_beta_init if cfg.hvaq_beta_init > 0 else 1.0 / np.sqrt(D)
    out, diag = ops.forward(qg_bhtd, cb, state, min(cfg.refinement_budget, cfg.num_codewords), cfg.passes,
                            cfg.pass_decay, hv, float(beta0), cfg.hvaq_alpha, diagnostics=True)
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


def assert_quant_equal(got: dict, want: O.Quantization, tag: str = "") -> None:
    if got["passign"] is not None:
        np.testing.assert_array_equal(got["passign"], want.parent_assignments, err_msg=f"{tag} parent assignments")
        np.testing.assert_array_equal(got["cassign"], want.child_assignments, err_msg=f"{tag} child assignments")
    np.testing.assert_array_equal(got["pcnt"], want.parent_counts, err_msg=f"{tag} parent counts")
    np.testing.assert_array_equal(got["ccnt"], want.child_counts, err_msg=f"{tag} child counts")
    np.testing.assert_array_equal(got["pagg"], want.parent_aggregates, err_msg=f"{tag} parent aggregates")
    np.testing.assert_array_equal(got["cagg"], want.child_aggregates, err_msg=f"{tag} child aggregates")


def assert_routing_equal(diag, res: dict, tag: str = "") -> None:
    sels = [s.long().cpu().numpy() for s in diag.selections()]
    want = res["selected"]
    assert len(sels) == len(want), f"{tag}: {len(sels)} passes vs {len(want)}"
    for k, (a, b) in enumerate(zip(sels, want)):
        np.testing.assert_array_equal(a, b, err_msg=f"{tag} pass {k} selected indices")
    imp = diag.importance.cpu().numpy()
    np.testing.assert_array_equal(imp, res["importance0"], err_msg=f"{tag} importance")
