"""AVQAttention / functional.attention / KV-cache decode through the public API."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from avqa_b200 import AVQAttention, AVQConfig, InMemoryKVCache, PagedKVCache
from avqa_b200.codebook import codebook_from_keys
from avqa_b200.config import AttentionShapeConfig, CodebookConfig, RoutingConfig
from avqa_b200.functional import attention
from oracle import avq_oracle as O
from parity import normrel

pytestmark = pytest.mark.gpu

TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _cfg(E=128, H=2, M0=16, C=4, P=4):
    return AVQConfig(attention=AttentionShapeConfig(embed_dim=E, num_heads=H),
                     codebook=CodebookConfig(num_codewords=M0, children_per_codeword=C),
                     routing=RoutingConfig(strategy="budget", refinement_budget=P))


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
def test_module_matches_oracle(dt: str) -> None:
    torch.manual_seed(0)
    B, T, S, E, H = 2, 48, 96, 128, 2
    cfg = _cfg(E, H)
    q, k, v = (torch.randn(B, n, E) for n in (T, S, S))
    qn, kn, vn = (O.rnd(x.numpy(), dt) for x in (q, k, v))
    kh0 = torch.from_numpy(kn).view(B, S, H, E // H).transpose(1, 2)[0]
    cb = codebook_from_keys(kh0, 16, 4, seed=3)
    m = AVQAttention(cfg, in_proj=False, out_proj=False)
    m.codebook.parents, m.codebook.children = cb.parents.clone(), cb.children.clone()
    dev = [torch.from_numpy(x).to("cuda", TD[dt]) for x in (qn, kn, vn)]
    out = m(*dev)
    assert out.dtype == torch.float32 and out.shape == (B, T, E)
    pd, cd = O.cast_codebook(cb.parents.numpy(), cb.children.numpy(), dt)
    res = O.forward(qn, kn, vn, pd, cd, O.ForwardConfig(H, 16, 4, 4, dt))
    assert normrel(out.cpu().numpy(), res["out_bte"]) <= (2e-5 if dt == "f32" else 1e-2)
    # the module's codebook now lives on the device in the input dtype, as in the reference
    assert m.codebook.parents.dtype == TD[dt] and m.codebook.parents.is_cuda


def test_functional_default_codebook_matches_oracle() -> None:
    torch.manual_seed(1)
    cfg = _cfg(64, 2, 8, 2, 3)
    q, k, v = (torch.randn(1, n, 64, device="cuda") for n in (5, 9, 9))
    torch.manual_seed(7)
    out = attention(q, k, v, cfg)
    torch.manual_seed(7)
    ref_mod = AVQAttention(cfg, in_proj=False, out_proj=False)  # same RNG draws as the functional call
    pd, cd = O.cast_codebook(ref_mod.codebook.parents.numpy(), ref_mod.codebook.children.numpy(), "f32")
    res = O.forward(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), pd, cd, O.ForwardConfig(2, 8, 2, 3, "f32"))
    assert normrel(out.cpu().numpy(), res["out_bte"]) <= 2e-5


@pytest.mark.parametrize("paged", [False, True])
def test_decode_with_cache_matches_oracle(paged: bool) -> None:
    torch.manual_seed(2)
    dt, B, S0, E, H, D = "bf16", 3, 70, 128, 2, 64
    cfg = _cfg(E, H, 16, 4, 5)
    k0, v0 = torch.randn(B, S0, E), torch.randn(B, S0, E)
    k0n, v0n = O.rnd(k0.numpy(), dt), O.rnd(v0.numpy(), dt)
    kh0 = torch.from_numpy(k0n).view(B, S0, H, D).transpose(1, 2)[0]
    cb = codebook_from_keys(kh0, 16, 4, seed=5)
    m = AVQAttention(cfg, in_proj=False, out_proj=False)
    m.codebook.parents, m.codebook.children = cb.parents.clone(), cb.children.clone()
    if paged:
        cache = PagedKVCache(page_size=32, num_heads=H, head_dim_k=D, head_dim_v=D, device="cuda",
                             dtype=torch.bfloat16)
    else:
        cache = InMemoryKVCache(num_heads=H, head_dim_k=D, head_dim_v=D, device="cuda", dtype=torch.bfloat16)
    to_h = lambda x: torch.from_numpy(x).view(B, -1, H, D).transpose(1, 2).to("cuda", torch.bfloat16)
    cache.append(to_h(k0n), to_h(v0n))
    pd, cd = O.cast_codebook(cb.parents.numpy(), cb.children.numpy(), dt)
    kk, vv = k0n, v0n
    for step in range(40):  # crosses page boundaries
        qt, kt, vt = (O.rnd(torch.randn(B, 1, E).numpy(), dt) for _ in range(3))
        out = m(*[torch.from_numpy(x).to("cuda", torch.bfloat16) for x in (qt, kt, vt)], kv_cache=cache)
        kk, vv = np.concatenate([kk, kt], 1), np.concatenate([vv, vt], 1)
        res = O.forward(qt, kk, vv, pd, cd, O.ForwardConfig(H, 16, 4, 5, dt))
        assert normrel(out.cpu().numpy(), res["out_bte"]) <= 1e-2, step
    assert cache.size == S0 + 40
    ck, cv = cache.lookup()
    np.testing.assert_array_equal(ck.float().cpu().numpy(), torch.from_numpy(kk).view(B, -1, H, D).transpose(1, 2))


@pytest.mark.parametrize("B", [1, 2])
def test_forward_chunked_equals_separate_calls(B: int) -> None:
    """Query chunks over keys quantized once (the long-context path): batch 1
    runs all whole chunks in one call against a shared key state, batch 2
    chunk by chunk; either way each chunk equals its own reference call."""
    torch.manual_seed(4)
    dt, T, S, E, H, chunk = "bf16", 3 * 64 + 37, 512, 128, 2, 64
    cfg = _cfg(E, H, 32, 4, 6)
    q, k, v = (torch.randn(B, n, E) for n in (T, S, S))
    qn, kn, vn = (O.rnd(x.numpy(), dt) for x in (q, k, v))
    kh0 = torch.from_numpy(kn).view(B, S, H, E // H).transpose(1, 2)[0]
    cb = codebook_from_keys(kh0, 32, 4, seed=9)
    m = AVQAttention(cfg, in_proj=False, out_proj=False)
    m.codebook.parents, m.codebook.children = cb.parents.clone(), cb.children.clone()
    qd, kd, vd = (torch.from_numpy(x).to("cuda", torch.bfloat16) for x in (qn, kn, vn))
    out = m.forward_chunked(qd, kd, vd, chunk).cpu().numpy()
    pd, cd = O.cast_codebook(cb.parents.numpy(), cb.children.numpy(), dt)
    for t0 in range(0, T, chunk):
        sep = m(qd[:, t0:t0 + chunk], kd, vd).cpu().numpy()
        np.testing.assert_array_equal(out[:, t0:t0 + chunk], sep)
        res = O.forward(qn[:, t0:t0 + chunk], kn, vn, pd, cd, O.ForwardConfig(H, 32, 4, 6, dt))
        assert normrel(out[:, t0:t0 + chunk], res["out_bte"]) <= 1e-2, t0
