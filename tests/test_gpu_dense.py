"""The dense softmax-attention path (reference backend.py:190-203,
:105-156; pipeline.py:261-273, 310-312) against the reference's recorded
outputs and the oracle.

Covers the module in execution.mode = "reference" and with refinement
disabled (tests/golden/dense_*.npz, causal and user masks), and the kernels
directly: the tcgen05 kernel (unmasked bf16 / fp16, D = 64 and 128, key
counts a multiple of 8 up to 8192), the mma.sync kernel (masked calls and the
other key counts) and the fp32 / other-D kernel, with key and query counts that are not multiples of the 64
tiles, rank-4 masks, fully masked queries (NaN, as torch.softmax gives) and a
KV cache.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import golden_io as G
from avqa_b200 import AVQAttention, AVQConfig, InMemoryKVCache, ops
from avqa_b200.backend import online_softmax_attention
from avqa_b200.config import AttentionShapeConfig, CodebookConfig, ExecutionConfig, RefinementConfig, RoutingConfig
from oracle import avq_oracle as O
from parity import OUT_TOL, finite_normrel

pytestmark = pytest.mark.gpu

TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


@pytest.mark.parametrize("name", [n for n in G.case_names() if n.startswith("dense")])
def test_dense_module_matches_reference(name: str) -> None:
    g = G.load(name)
    w, dt = g.w, g.dt
    c = g.meta["config"]
    cfg = AVQConfig(causal=c["causal"], attention=AttentionShapeConfig(embed_dim=w["H"] * w["D"], num_heads=w["H"]),
                    codebook=CodebookConfig(num_codewords=w["M0"], children_per_codeword=w["C"]),
                    routing=RoutingConfig(refinement_budget=w["P"]),
                    refinement=RefinementConfig(enabled=c["refinement"]["enabled"]),
                    execution=ExecutionConfig(mode=c["execution"]["mode"]))
    m = AVQAttention(cfg, in_proj=False, out_proj=False)
    q, k, v = (G.to_torch(g.get(x), dt).cuda() for x in ("q", "k", "v"))
    mask = g.mask_for(q.shape[1], k.shape[1]) if g.meta.get("mask") != "causal" else None
    out = m(q, k, v, mask=None if mask is None else torch.from_numpy(mask).cuda())
    assert out.dtype == TD[dt]  # the dense path keeps the input dtype, as the reference's does
    err, _ = finite_normrel(out.float().cpu().numpy(), g.get("out0").reshape(out.shape), name)
    assert err <= OUT_TOL[dt], f"{name}: {err}"


CASES = [
    # dtype, B, H, T, N, D, mask
    ("bf16", 2, 3, 100, 200, 64, None),
    ("f16", 1, 2, 64, 129, 128, "rank4"),
    ("bf16", 1, 2, 70, 64, 128, "rank2"),
    ("f32", 2, 2, 33, 90, 40, "rank4"),
    ("bf16", 1, 1, 20, 300, 72, None),  # D = 72: the fp32-accumulating kernel
    # unmasked bf16 / fp16 with D = 64 or 128 and N % 8 == 0: the tcgen05 kernel
    ("f16", 2, 2, 130, 256, 128, None),   # a partial second query tile
    ("bf16", 1, 2, 257, 1024, 128, None),  # sixteen key chunks
    ("f16", 1, 1, 5, 8, 64, None),        # one key row block, mostly padding
    ("bf16", 1, 1, 4, 8200, 64, None),    # above the tcgen05 kernel's key limit: mma.sync
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}_T{c[3]}_N{c[4]}_D{c[5]}_{c[6]}")
def test_dense_kernels_match_oracle(case) -> None:
    dt, B, H, T, N, D, kind = case
    g = torch.Generator().manual_seed(91 + D + T)
    q, k, v = (O.rnd(torch.randn(B, H, n, D, generator=g).numpy(), dt) for n in (T, N, N))
    mask = None
    if kind == "rank2":
        mask = (torch.rand(T, N, generator=g) < 0.3).numpy()
        mask[5] = False  # a query that sees nothing -> NaN
    elif kind == "rank4":
        mask = (torch.rand(B, H, T, N, generator=g) < 0.3).numpy()
    dev = [torch.from_numpy(x).to("cuda", TD[dt]) for x in (q, k, v)]
    mt = None if mask is None else torch.from_numpy(mask).cuda()
    out = ops.dense_attention(*dev, mt).float().cpu().numpy()
    mg = None if mask is None else O.expand_mask(mask, B, H)
    want = O.naive_attention(q.reshape(B * H, T, D), k.reshape(B * H, N, D), v.reshape(B * H, N, D), dt, mg)
    err, nonfinite = finite_normrel(out.reshape(B * H, T, D), want, f"{case}")
    assert err <= OUT_TOL[dt], f"{case}: {err}"
    if kind == "rank2":
        assert nonfinite == B * H  # the fully masked query, in every (b,h)
    again = online_softmax_attention(*dev, mask=mt).float().cpu().numpy()
    np.testing.assert_array_equal(again, out)


def test_dense_module_with_cache_matches_oracle() -> None:
    """Reference mode over a KV cache: the cached keys plus the new ones."""
    torch.manual_seed(7)
    B, H, D, S0 = 2, 2, 64, 50
    cfg = AVQConfig(attention=AttentionShapeConfig(embed_dim=H * D, num_heads=H),
                    execution=ExecutionConfig(mode="reference"))
    m = AVQAttention(cfg, in_proj=False, out_proj=False)
    cache = InMemoryKVCache(num_heads=H, head_dim_k=D, head_dim_v=D, device="cuda", dtype=torch.bfloat16)
    k0, v0 = (torch.randn(B, H, S0, D).to("cuda", torch.bfloat16) for _ in range(2))
    cache.append(k0, v0)
    q1, k1, v1 = (torch.randn(B, 3, H * D).to("cuda", torch.bfloat16) for _ in range(3))
    out = m(q1, k1, v1, kv_cache=cache).float().cpu().numpy()
    hv = lambda x: x.view(B, 3, H, D).transpose(1, 2)
    kf = torch.cat([k0, hv(k1)], 2).float().cpu().numpy().reshape(B * H, -1, D)
    vf = torch.cat([v0, hv(v1)], 2).float().cpu().numpy().reshape(B * H, -1, D)
    want = O.naive_attention(hv(q1).float().cpu().numpy().reshape(B * H, 3, D), kf, vf, "bf16")
    want = want.reshape(B, H, 3, D).transpose(0, 2, 1, 3).reshape(B, 3, H * D)
    assert finite_normrel(out, want, "cache")[0] <= 1e-2
    assert cache.size == S0 + 3
