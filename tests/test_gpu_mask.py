"""User and causal masks through the public API (reference pipeline.py:82-106,
attention_module.py:210-223, 369-390) against the oracle.

A parent is masked for a query when none of its keys is visible; the child
logits ignore the mask, as in the reference.  The cases reach every kernel
family that applies the mask bits: the tcgen05 parent attention and
correction (bf16, and fp16 with the HVAQ rescaling pass and three routing
passes), the mma.sync kernels (tcgen05 switched off; indices must equal the
tcgen05 run's), the fp32 / odd-C kernels, decode (one query sees every key),
and query chunks (each chunk a separate causal call).  Parent counts that
are not a multiple of 64 leave partial mask words.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from avqa_b200 import AVQAttention, AVQConfig, InMemoryKVCache, ops
from avqa_b200.codebook import codebook_from_keys
from avqa_b200.config import (AttentionShapeConfig, BackendConfig, CodebookConfig, HopfieldConfig, RefinementConfig,
                              RoutingConfig)
from oracle import avq_oracle as O
from parity import OUT_TOL, finite_normrel

pytestmark = pytest.mark.gpu

TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _module(E, H, M0, C, P, causal, passes=1, hvaq=False):
    cfg = AVQConfig(causal=causal, attention=AttentionShapeConfig(embed_dim=E, num_heads=H),
                    codebook=CodebookConfig(num_codewords=M0, children_per_codeword=C),
                    routing=RoutingConfig(strategy="budget", refinement_budget=P),
                    refinement=RefinementConfig(passes=passes, pass_decay=0.5),
                    backend=BackendConfig(hopfield=hvaq),
                    hopfield=HopfieldConfig(enabled=hvaq, adaptive="entropy" if hvaq else "none"))
    return AVQAttention(cfg, in_proj=False, out_proj=False)


def _run(dt, B, T, S, H, D, M0, C, P, kind, seed, passes=1, hvaq=False, tc=True):
    g = torch.Generator().manual_seed(seed)
    E = H * D
    q, k, v = (torch.randn(B, n, E, generator=g) for n in (T, S, S))
    if kind == "causal":
        mask = None
        mask_np = O.causal_mask(T, S)
    elif kind == "rank2":
        mask_np = (torch.rand(T, S, generator=g) < 0.2).numpy()
        mask_np[3] = False  # a query that sees nothing
        mask = torch.from_numpy(mask_np)
    else:
        mask_np = (torch.rand(B, H, T, S, generator=g) < 0.25).numpy()
        mask = torch.from_numpy(mask_np)
    qn, kn, vn = (O.rnd(x.numpy(), dt) for x in (q, k, v))
    kh0 = torch.from_numpy(kn).view(B, S, H, D).transpose(1, 2)[0]
    cb = codebook_from_keys(kh0, M0, C, seed)
    m = _module(E, H, M0, C, P, kind == "causal", passes, hvaq)
    m.codebook.parents, m.codebook.children = cb.parents.clone(), cb.children.clone()
    dev = [torch.from_numpy(x).to("cuda", TD[dt]) for x in (qn, kn, vn)]
    os.environ["AVQ_DISABLE_TCGEN05"] = "0" if tc else "1"
    try:
        out = m(*dev, mask=None if mask is None else mask.cuda()).cpu().numpy()
    finally:
        os.environ.pop("AVQ_DISABLE_TCGEN05", None)
    pd, cd = O.cast_codebook(cb.parents.numpy(), cb.children.numpy(), dt)
    res = O.forward(qn, kn, vn, pd, cd, O.ForwardConfig(H, M0, C, P, dt, passes, 0.5, hvaq), mask=mask_np)
    return out, res


CASES = [
    # dtype, B, T, S, H, D, M0, C, P, mask, seed, passes, hvaq
    ("bf16", 2, 300, 300, 2, 128, 200, 4, 16, "causal", 81, 1, False),
    ("f16", 1, 260, 260, 2, 64, 96, 4, 12, "causal", 82, 3, True),
    ("bf16", 2, 140, 400, 2, 64, 72, 4, 8, "rank4", 83, 1, False),
    ("bf16", 1, 64, 200, 2, 64, 40, 3, 6, "rank2", 84, 2, False),  # odd C: the exact kernels
    ("f32", 1, 96, 96, 2, 32, 24, 2, 6, "causal", 85, 1, False),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}_{c[9]}_p{c[11]}{'_hvaq' if c[12] else ''}")
def test_mask_matches_oracle(case) -> None:
    dt, B, T, S, H, D, M0, C, P, kind, seed, passes, hvaq = case
    out, res = _run(dt, B, T, S, H, D, M0, C, P, kind, seed, passes, hvaq)
    err, _ = finite_normrel(out, res["out_bte"], f"{dt} {kind}")
    assert err <= OUT_TOL[dt], f"{dt} {kind}: output normrel {err}"


def test_mask_mma_kernels_match_tcgen05() -> None:
    """Causal bf16 with tcgen05 off (mma.sync parent attention and correction)."""
    out_tc, res = _run("bf16", 2, 300, 300, 2, 128, 200, 4, 16, "causal", 81)
    out_mma, _ = _run("bf16", 2, 300, 300, 2, 128, 200, 4, 16, "causal", 81, tc=False)
    assert finite_normrel(out_mma, res["out_bte"], "mma")[0] <= 1e-2
    assert finite_normrel(out_tc, out_mma, "tc vs mma")[0] <= 1e-5


@pytest.mark.parametrize("M0", [80, 64, 512])
def test_causal_presence_bits_match_oracle(M0: int) -> None:
    """The causal bits alone, including the cached-prefix offset, for word
    counts of 3, 2 and 16 per query row."""
    g = torch.Generator().manual_seed(86)
    B, H, S, D, C, T = 2, 3, 500, 64, 4, 120
    k = torch.randn(B, S, H * D, generator=g).to(torch.bfloat16)
    kh = k.view(B, S, H, D).transpose(1, 2)
    cb32 = codebook_from_keys(kh[0].float(), M0, C, 1)
    cb = ops.prepare_codebook(cb32.parents, cb32.children, torch.bfloat16, torch.device("cuda"))
    st = ops.quantize(kh.cuda(), kh.cuda(), cb)
    bits = ops.codeword_presence(st, T).cpu().numpy().view(np.uint32)
    got = ((bits[..., :, None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(B * H, T, -1)[..., :M0].astype(bool)
    want = O.codeword_present(np.broadcast_to(O.causal_mask(T, S), (B * H, T, S)), st.passign.long().cpu().numpy(),
                              M0)
    np.testing.assert_array_equal(got, want)


def test_chunked_causal_equals_separate_calls() -> None:
    """Each 64-query chunk is its own causal call over all keys (offset S - 64)."""
    dt, T, S, H, D, M0, C, P = "bf16", 256, 512, 2, 64, 64, 4, 8
    g = torch.Generator().manual_seed(87)
    q, k, v = (torch.randn(1, n, H * D, generator=g) for n in (T, S, S))
    qn, kn, vn = (O.rnd(x.numpy(), dt) for x in (q, k, v))
    cb = codebook_from_keys(torch.from_numpy(kn).view(1, S, H, D).transpose(1, 2)[0], M0, C, 3)
    m = _module(H * D, H, M0, C, P, True)
    m.codebook.parents, m.codebook.children = cb.parents.clone(), cb.children.clone()
    qd, kd, vd = (torch.from_numpy(x).to("cuda", torch.bfloat16) for x in (qn, kn, vn))
    out = m.forward_chunked(qd, kd, vd, 64).cpu().numpy()
    pd, cd = O.cast_codebook(cb.parents.numpy(), cb.children.numpy(), dt)
    for t0 in range(0, T, 64):
        sep = m(qd[:, t0:t0 + 64], kd, vd).cpu().numpy()
        np.testing.assert_array_equal(out[:, t0:t0 + 64], sep)
        res = O.forward(qn[:, t0:t0 + 64], kn, vn, pd, cd, O.ForwardConfig(H, M0, C, P, dt),
                        mask=O.causal_mask(64, S))
        assert finite_normrel(out[:, t0:t0 + 64], res["out_bte"], f"chunk {t0}")[0] <= 1e-2


def test_causal_decode_sees_every_key() -> None:
    """One new query per step: the causal mask hides nothing (the cached
    prefix and the new key are all visible), so the output equals the
    unmasked decode."""
    torch.manual_seed(88)
    B, S0, H, D, M0, C, P = 2, 90, 2, 64, 16, 4, 5
    E = H * D
    k0, v0 = torch.randn(B, S0, E), torch.randn(B, S0, E)
    kh = lambda x: x.view(B, -1, H, D).transpose(1, 2).to("cuda", torch.bfloat16)
    cb = codebook_from_keys(k0.to(torch.bfloat16).view(B, S0, H, D).transpose(1, 2)[0].float(), M0, C, 2)
    outs = []
    for causal in (True, False):
        m = _module(E, H, M0, C, P, causal)
        m.codebook.parents, m.codebook.children = cb.parents.clone(), cb.children.clone()
        cache = InMemoryKVCache(num_heads=H, head_dim_k=D, head_dim_v=D, device="cuda", dtype=torch.bfloat16)
        cache.append(kh(k0), kh(v0))
        g = torch.Generator().manual_seed(5)
        steps = []
        for _ in range(3):
            qt, kt, vt = (torch.randn(B, 1, E, generator=g).to("cuda", torch.bfloat16) for _ in range(3))
            steps.append(m(qt, kt, vt, kv_cache=cache).cpu())
        outs.append(torch.stack(steps))
    assert torch.equal(outs[0], outs[1])
