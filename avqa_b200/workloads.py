"""Seeded synthetic workloads for the AVQ-attention hot path.

No public dataset is involved: every input is synthetic, generated with
``torch.Generator`` in fp32 and then cast to the working dtype.  Each recipe
returns module-layout tensors ``[B, T, E]`` (``E = H * D``), the layout that
``AVQAttention.forward`` accepts (reference ``attention_module.py:255-290``).

Recipes (keys are the interesting part; queries and values are N(0, 1)):

* ``readme``    -- iid N(0,1) q/k/v under ``torch.manual_seed(0)``, in README
                   order (reference ``README.md:84-96``).
* ``mixture``   -- keys from a per-head Gaussian mixture: centres ~ N(0,1),
                   uniform cluster weights, isotropic noise ``sigma``.
* ``aniso``     -- like ``mixture`` but with a per-centre, per-dimension noise
                   scale ~ U[0.1, 1] (anisotropic clusters).
* ``student_t`` -- keys ``0.5 * z / sqrt(chi2_3 / 3)`` (Student-t, nu = 3).
* ``mixture_rope`` -- mixture keys rotated by absolute position with RoPE
                   (half-split pairing: dims ``i`` and ``i + D/2`` rotate
                   together, ``theta_i = base^(-2i/D)``, base 10000).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

TORCH_DTYPE = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
DTYPE_NAME = {v: k for k, v in TORCH_DTYPE.items()}


@dataclass(frozen=True)
class Workload:
    """One benchmark / parity configuration."""

    name: str
    B: int
    T: int
    S: int
    H: int
    D: int
    M0: int
    C: int
    P: int
    dtype: str
    keys: str
    seed: int
    passes: int = 1
    pass_decay: float = 1.0
    hvaq: bool = False
    sigma: float = 0.3
    n_centres: int = 0  # 0 -> M0
    q_chunk: int = 0  # >0: queries processed in sequential chunks of this size
    decode_steps: int = 0  # >0: S prior tokens then this many T=1 steps
    page_size: int = 256

    @property
    def E(self) -> int:
        return self.H * self.D


WORKLOADS = {
    # README example, fp32 (reference README.md:84-96).
    "c1": Workload("c1", B=2, T=64, S=128, H=8, D=64, M0=64, C=4, P=8, dtype="f32", keys="readme", seed=0),
    # Prefill, bf16, Gaussian-mixture keys.
    "c2": Workload("c2", B=4, T=8192, S=8192, H=32, D=128, M0=512, C=4, P=32, dtype="bf16", keys="mixture", seed=1),
    # Decode with a paged KV cache, bf16.
    "c3": Workload("c3", B=64, T=1, S=32768, H=32, D=128, M0=1024, C=8, P=64, dtype="bf16", keys="aniso", seed=2,
                   decode_steps=128, page_size=256),
    # Multi-pass refinement + HVAQ entropy temperature, fp16.
    "c4": Workload("c4", B=8, T=16384, S=16384, H=16, D=64, M0=256, C=4, P=48, dtype="f16", keys="student_t", seed=3,
                   passes=3, pass_decay=0.5, hvaq=True),
    # Long context, head-sharded, bf16, 256-query chunks.
    "c5": Workload("c5", B=1, T=2048, S=131072, H=64, D=128, M0=4096, C=8, P=128, dtype="bf16", keys="mixture_rope",
                   seed=4, q_chunk=256),
}


def rope_rotate(x: torch.Tensor, positions: torch.Tensor, base: float = 10000.0) -> torch.Tensor:
    """Rotate ``x [..., S, D]`` by absolute ``positions [S]`` (half-split pairing)."""
    D = x.shape[-1]
    half = D // 2
    inv = base ** (-torch.arange(0, half, dtype=torch.float64, device=x.device) * 2.0 / D)
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    cos = torch.cos(ang).to(x.dtype)
    sin = torch.sin(ang).to(x.dtype)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)


def make_keys(w: Workload, B: int, S: int, gen: torch.Generator, device="cpu", pos0: int = 0,
              sample_gen: torch.Generator | None = None) -> torch.Tensor:
    """Keys ``[B, S, E]`` in fp32 following ``w.keys``.  The mixture's centres
    come from ``gen``; the samples from ``sample_gen`` (default ``gen``)."""
    H, D = w.H, w.D
    sgen = gen if sample_gen is None else sample_gen
    if w.keys == "readme":
        raise ValueError("readme keys are generated together with q/v")
    if w.keys in ("mixture", "aniso", "mixture_rope"):
        nc = w.n_centres or w.M0
        centres = torch.randn(H, nc, D, generator=gen, device=device)
        scale = None
        if w.keys == "aniso":
            scale = torch.rand(H, nc, D, generator=gen, device=device) * 0.9 + 0.1
        idx = torch.randint(0, nc, (B, H, S), generator=sgen, device=device)
        hix = torch.arange(H, device=device)[None, :, None].expand(B, H, S)
        noise = torch.randn(B, H, S, D, generator=sgen, device=device)
        if scale is None:
            k = centres[hix, idx] + w.sigma * noise
        else:
            k = centres[hix, idx] + scale[hix, idx] * noise
        if w.keys == "mixture_rope":
            k = rope_rotate(k, torch.arange(pos0, pos0 + S, device=device))
        return k.transpose(1, 2).reshape(B, S, H * D).contiguous()
    if w.keys == "student_t":
        z = torch.randn(B, S, H * D, generator=sgen, device=device)
        chi = (torch.randn(3, B, S, H * D, generator=sgen, device=device) ** 2).sum(0)
        return 0.5 * z / torch.sqrt(chi / 3.0)
    raise ValueError(f"unknown key recipe {w.keys!r}")


def make_inputs(w: Workload, device="cpu", B: int | None = None, T: int | None = None, S: int | None = None,
                part: int = 0):
    """Return fp32 ``(q [B,T,E], k [B,S,E], v [B,S,E])`` for workload ``w``.

    ``B``/``T``/``S`` override the sizes (parity tests use reduced sizes with
    the same distributions).  ``part`` > 0 draws another batch of the same
    distribution: the same mixture centres, independent samples (the batch
    shards of one global batch across ranks).
    """
    B = w.B if B is None else B
    T = w.T if T is None else T
    S = w.S if S is None else S
    E = w.E
    if w.keys == "readme":
        torch.manual_seed(w.seed)
        q = torch.randn(B, T, E)
        k = torch.randn(B, S, E)
        v = torch.randn(B, S, E)
        return q.to(device), k.to(device), v.to(device)
    gen = torch.Generator(device=device).manual_seed(w.seed)
    sgen = None if part == 0 else torch.Generator(device=device).manual_seed(w.seed + 7919 * part)
    k = make_keys(w, B, S, gen, device, sample_gen=sgen)
    g2 = gen if sgen is None else sgen
    q = torch.randn(B, T, E, generator=g2, device=device)
    v = torch.randn(B, S, E, generator=g2, device=device)
    return q, k, v


def make_decode_tokens(w: Workload, steps: int, B: int | None = None, device="cpu"):
    """Per-step decode tokens: ``steps`` triples of ``[B, 1, E]`` N(0,1) q/k/v."""
    B = w.B if B is None else B
    gen = torch.Generator(device=device).manual_seed(w.seed + 1000)
    out = []
    for _ in range(steps):
        q = torch.randn(B, 1, w.E, generator=gen, device=device)
        k = torch.randn(B, 1, w.E, generator=gen, device=device)
        v = torch.randn(B, 1, w.E, generator=gen, device=device)
        out.append((q, k, v))
    return out


__all__ = ["DTYPE_NAME", "TORCH_DTYPE", "WORKLOADS", "Workload", "make_decode_tokens", "make_inputs", "make_keys",
           "rope_rotate"]
