"""Hierarchical parent/child codebook storage.

``parents [H, M0, D]`` and ``children [H, M0, C, D]`` held as an fp32 master
copy, with the reference's initialisers and mean constraint
(``src/avqa/codebook.py:66-217``) and its ``state_dict`` schema
(``codebook.py:307-322``).  The forward pass casts the master copy to the
input dtype once per call, as the reference does
(``attention_module.py:344-348``).

:func:`codebook_from_keys` is the fixed key-based initialisation recipe used
by every benchmark and parity workload (the reference ships no key-based
initialiser):

1. ``parents0[h] = K[b=0, h, floor(linspace(0, S-1, M0))]`` (fp32 of the
   dtype-rounded keys);
2. children = parents0 + ``perturbation_scale`` x zero-mean Gaussian noise
   drawn from ``torch.Generator().manual_seed(seed)``; parents re-projected
   to the children's mean (``codebook.py:137-180``);
3. one Lloyd step in fp32 with the hierarchical quantizer, keys as values:
   children with a non-zero count move to the mean of their keys, then the
   parents are re-projected.
"""
from __future__ import annotations

import torch

from avqa_b200.exceptions import CodebookError


def _require_positive(value: int, name: str) -> None:
    if value <= 0:
        raise CodebookError(f"{name} must be > 0, got {value}", {name: value})


class HierarchicalCodebook:
    """Parent/child codebook of one attention layer (all heads)."""

    def __init__(self, num_heads: int = 1, num_parents: int = 64, children_per_parent: int = 4,
                 head_dim: int = 64, perturbation_scale: float = 0.1, device: str | torch.device = "cpu",
                 dtype: torch.dtype = torch.float32) -> None:
        _require_positive(num_heads, "num_heads")
        _require_positive(num_parents, "num_parents")
        _require_positive(children_per_parent, "children_per_parent")
        _require_positive(head_dim, "head_dim")
        if perturbation_scale <= 0:
            raise CodebookError(f"perturbation_scale must be > 0, got {perturbation_scale}")
        self.num_heads = num_heads
        self.num_parents = num_parents
        self.children_per_parent = children_per_parent
        self.head_dim = head_dim
        self.perturbation_scale = perturbation_scale
        self.parents = torch.zeros(num_heads, num_parents, head_dim, device=device, dtype=dtype)
        self.children = torch.zeros(num_heads, num_parents, children_per_parent, head_dim, device=device, dtype=dtype)

    def initialize_children_around_parents(self, perturbation: torch.Tensor | None = None,
                                           generator: torch.Generator | None = None) -> None:
        shape = (self.num_heads, self.num_parents, self.children_per_parent, self.head_dim)
        if perturbation is None:
            perturbation = torch.randn(*shape, device=self.children.device, dtype=self.children.dtype,
                                       generator=generator)
        elif tuple(perturbation.shape) != shape:
            raise CodebookError(f"perturbation shape {tuple(perturbation.shape)} != expected {shape}")
        perturbation = perturbation - perturbation.mean(dim=2, keepdim=True)
        self.children = self.parents.unsqueeze(2) + self.perturbation_scale * perturbation
        self.reproject_parents()

    def initialize_parents_random(self, generator: torch.Generator | None = None, scale: float = 1.0) -> None:
        self.parents = torch.randn(self.num_heads, self.num_parents, self.head_dim, device=self.parents.device,
                                   dtype=self.parents.dtype, generator=generator) * scale
        self.children = torch.zeros_like(self.children)
        self.initialize_children_around_parents(generator=generator)

    def reproject_parents(self) -> None:
        self.parents = self.children.mean(dim=2)

    def validate_mean_constraint(self, atol: float = 1e-5) -> None:
        diff = (self.parents - self.children.mean(dim=2)).abs().max().item()
        if diff > atol:
            raise CodebookError(f"mean constraint violated: max |parent - mean(child)| = {diff}", {"max_diff": diff})

    def state_dict(self) -> dict[str, torch.Tensor]:
        return {"parents": self.parents.detach().clone(), "children": self.children.detach().clone(),
                "schema_version": torch.tensor(1, dtype=torch.int32)}

    def load_state_dict(self, state: dict[str, torch.Tensor]) -> None:
        if "parents" not in state or "children" not in state:
            raise CodebookError("state_dict must contain 'parents' and 'children'")
        self.parents = state["parents"].to(self.parents.device, self.parents.dtype)
        self.children = state["children"].to(self.children.device, self.children.dtype)
        self.validate_mean_constraint()

    def __repr__(self) -> str:
        return (f"HierarchicalCodebook(H={self.num_heads}, M0={self.num_parents}, C={self.children_per_parent}, "
                f"D={self.head_dim}, device={self.parents.device}, dtype={self.parents.dtype})")


def _lloyd_children(keys: torch.Tensor, parents: torch.Tensor, children: torch.Tensor) -> torch.Tensor:
    """One fp32 hierarchical assignment of ``keys [H,S,D]``; returns child means.

    Same arithmetic as the reference quantizer in fp32 (``quantizer.py:196-269``).
    Heads are independent, so they run in groups that keep the ``[h, S, M0]``
    distance tensor near 2^28 elements (the long-context codebook would
    otherwise need 137 GB); every bucket sums its keys in the same order.
    """
    H, S, D = keys.shape
    M0 = children.shape[1]
    step = max(1, (1 << 28) // max(1, S * M0))
    if step < H:
        return torch.cat([_lloyd_children(keys[h:h + step], parents[h:h + step], children[h:h + step])
                          for h in range(0, H, step)])
    M0, C = children.shape[1], children.shape[2]
    k_sq = (keys * keys).sum(-1, keepdim=True)
    p_sq = (parents * parents).sum(-1).unsqueeze(1)
    dist = k_sq + p_sq - 2.0 * torch.matmul(keys, parents.transpose(-1, -2))
    pa = dist.argmin(-1)  # [H,S]
    g = torch.gather(children, 1, pa[..., None, None].expand(H, S, C, D))
    c_sq = (g * g).sum(-1)
    cross = (keys.unsqueeze(-2) * g).sum(-1)
    ca = (k_sq + c_sq - 2.0 * cross).argmin(-1)
    flat = (pa * C + ca + torch.arange(H, device=keys.device)[:, None] * (M0 * C)).reshape(-1)
    agg = torch.zeros(H * M0 * C, D, dtype=keys.dtype, device=keys.device)
    agg.index_add_(0, flat, keys.reshape(-1, D))
    cnt = torch.zeros(H * M0 * C, dtype=keys.dtype, device=keys.device)
    cnt.index_add_(0, flat, torch.ones(H * S, dtype=keys.dtype, device=keys.device))
    agg = agg.view(H, M0, C, D)
    cnt = cnt.view(H, M0, C)
    return torch.where((cnt > 0)[..., None], agg / cnt.clamp_min(1.0)[..., None], children)


def codebook_from_keys(keys_b0: torch.Tensor, num_parents: int, children_per_parent: int, seed: int,
                       perturbation_scale: float = 0.1) -> HierarchicalCodebook:
    """Key-based codebook initialisation (the recipe in the module docstring).

    ``keys_b0`` is ``[H, S, D]``: batch 0's keys, already rounded to the
    working dtype; the recipe runs in fp32 on ``keys_b0``'s device.
    """
    H, S, D = keys_b0.shape
    k32 = keys_b0.to(torch.float32)
    cb = HierarchicalCodebook(H, num_parents, children_per_parent, D, perturbation_scale=perturbation_scale,
                              device=k32.device)
    pos = torch.floor(torch.linspace(0, S - 1, num_parents, dtype=torch.float64)).long().to(k32.device)
    cb.parents = k32[:, pos].clone()
    gen = torch.Generator(device=k32.device).manual_seed(seed)
    cb.initialize_children_around_parents(generator=gen)
    cb.children = _lloyd_children(k32, cb.parents, cb.children)
    cb.reproject_parents()
    return cb


__all__ = ["HierarchicalCodebook", "codebook_from_keys"]
