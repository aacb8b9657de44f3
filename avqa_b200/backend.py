"""The Backend seam and the B200 ``CUDABackend``.

Same contract as the reference (``src/avqa/backend.py:48-102``): a backend
implements ``quantize(keys, values, codebook_parents, codebook_children)``
returning a :class:`QuantizationResult` and ``naive_attention(q, k, v,
mask)``.  ``Backend.create("cuda")`` returns :class:`CUDABackend`; the
pure-PyTorch ``"torch"`` backend is the reference package's own and is not
re-implemented here.

Beyond the two abstract methods, :class:`CUDABackend` exposes ``forward``:
stages 6-11 of the reference pipeline (``pipeline.py:322-393``) as one call
into the CUDA library, which ``AVQAttention`` uses.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass

import torch

from avqa_b200 import ops
from avqa_b200.exceptions import BackendError, ShapeError


@dataclass
class QuantizationResult:
    """Quantizer outputs (reference ``quantizer.py:32-49``).

    Assignments are int64 ``[B, H, N]``; aggregates and counts are in the
    value dtype, counts saturating exactly as the reference's ``index_add_``
    of ones does (256 in bf16, 2048 in fp16).
    """

    parent_assignments: torch.Tensor
    child_assignments: torch.Tensor
    parent_aggregates: torch.Tensor
    child_aggregates: torch.Tensor
    parent_counts: torch.Tensor
    child_counts: torch.Tensor

    def validate_shapes(self, num_heads: int, num_parents: int, children_per_parent: int, head_dim: int) -> None:
        B, H, N = self.parent_assignments.shape
        checks = {
            "child_assignments": (self.child_assignments, (B, H, N)),
            "parent_aggregates": (self.parent_aggregates, (B, H, num_parents, head_dim)),
            "child_aggregates": (self.child_aggregates, (B, H, num_parents, children_per_parent, head_dim)),
            "parent_counts": (self.parent_counts, (B, H, num_parents)),
            "child_counts": (self.child_counts, (B, H, num_parents, children_per_parent)),
        }
        for name, (t, shape) in checks.items():
            if tuple(t.shape) != shape:
                raise ShapeError(f"{name} shape mismatch", expected=shape, actual=tuple(t.shape))


class Backend(ABC):
    """Execution backend: ``quantize`` and ``naive_attention``."""

    name: str = "abstract"

    @classmethod
    def create(cls, name: str = "cuda") -> Backend:
        if name == "cuda":
            return CUDABackend()
        if name == "torch":
            raise BackendError("backend 'torch' is the reference package's pure-PyTorch backend; "
                               "this package provides 'cuda'", {"name": name})
        raise BackendError(f"backend '{name}' is not a known backend", {"name": name})

    @abstractmethod
    def quantize(self, keys: torch.Tensor, values: torch.Tensor, codebook_parents: torch.Tensor,
                 codebook_children: torch.Tensor) -> QuantizationResult:
        """Hierarchical VQ precompute."""

    @abstractmethod
    def naive_attention(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                        mask: torch.Tensor | None = None) -> torch.Tensor:
        """O(N^2) reference attention."""


class CUDABackend(Backend):
    """B200 kernels behind the reference's Backend interface."""

    name = "cuda"

    def __init__(self) -> None:
        self._cb_cache: dict = {}

    # -- codebook ------------------------------------------------------------

    def prepared_codebook(self, parents: torch.Tensor, children: torch.Tensor, dtype: torch.dtype,
                          device: torch.device) -> ops.PreparedCodebook:
        """The codebook cast to ``dtype`` on ``device`` (cached until either
        tensor is replaced or modified in place)."""
        key = (parents.data_ptr(), parents._version, children.data_ptr(), children._version, dtype, str(device),
               tuple(children.shape))
        hit = self._cb_cache.get("key")
        if hit != key:
            self._cb_cache = {"key": key, "cb": ops.prepare_codebook(parents, children, dtype, device)}
        return self._cb_cache["cb"]

    # -- Backend API ---------------------------------------------------------

    def quantize(self, keys: torch.Tensor, values: torch.Tensor, codebook_parents: torch.Tensor,
                 codebook_children: torch.Tensor) -> QuantizationResult:
        if keys.shape != values.shape:
            raise ShapeError("keys and values must have identical shapes", expected=tuple(keys.shape),
                             actual=tuple(values.shape))
        if keys.ndim != 4:
            raise ShapeError("keys must have rank 4 [B, H, N, D]", expected="[B, H, N, D]", actual=tuple(keys.shape))
        if codebook_parents.shape[-1] != keys.shape[-1]:
            raise ShapeError("key head_dim mismatch", expected=codebook_parents.shape[-1], actual=keys.shape[-1])
        cb = self.prepared_codebook(codebook_parents, codebook_children, keys.dtype, keys.device)
        st = ops.quantize(keys, values, cb)
        B, H, N, _ = keys.shape
        M0, C = cb.dims[1], cb.dims[2]
        pc, cc = st.counts_in_dtype()
        return QuantizationResult(
            parent_assignments=st.passign.view(B, H, N).long(),
            child_assignments=st.cassign.view(B, H, N).long(),
            parent_aggregates=st.pagg.view(B, H, M0, -1),
            child_aggregates=st.cagg.view(B, H, M0, C, -1),
            parent_counts=pc.view(B, H, M0),
            child_counts=cc.view(B, H, M0, C),
        )

    def naive_attention(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                        mask: torch.Tensor | None = None) -> torch.Tensor:
        """Dense softmax attention (backend.py:190-203) on the GPU, in the input dtype."""
        if key.shape[-2] == 0:
            # softmax over zero keys times zero values: the reference yields zeros
            return torch.zeros(*query.shape[:-1], value.shape[-1], dtype=query.dtype, device=query.device)
        if value.shape[-1] != query.shape[-1]:
            raise ShapeError("value head_dim must equal the query's", expected=query.shape[-1],
                             actual=value.shape[-1])
        return ops.dense_attention(query, key, value, mask)

    def online_softmax_attention(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                 block_size: int = 64, mask: torch.Tensor | None = None) -> torch.Tensor:
        """The tiled online-softmax form (backend.py:105-156); the kernel tiles
        by 64 keys whatever ``block_size`` says (the result is the same)."""
        return online_softmax_attention(query, key, value, block_size, mask)

    # -- fused forward -------------------------------------------------------

    def forward(self, q: torch.Tensor, cb: ops.PreparedCodebook, state: ops.QuantState, budget: int,
                passes: int = 1, pass_decay: float = 1.0, hvaq: int = 0, beta0: float = 0.0, alpha: float = 1.0,
                out: torch.Tensor | None = None, min_valid: torch.Tensor | None = None, diagnostics: bool = False,
                min_valid_ready: torch.cuda.Event | None = None, present: torch.Tensor | None = None):
        return ops.forward(q, cb, state, budget, passes, pass_decay, hvaq, beta0, alpha, out, min_valid, diagnostics,
                           min_valid_ready, present)


def online_softmax_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, block_size: int = 64,
                             mask: torch.Tensor | None = None) -> torch.Tensor:
    """Tiled online-softmax attention (backend.py:105-156) on the GPU."""
    if key.shape[-2] == 0:
        return torch.zeros(*query.shape[:-1], value.shape[-1], dtype=query.dtype, device=query.device)
    return ops.dense_attention(query, key, value, mask)


__all__ = ["Backend", "CUDABackend", "QuantizationResult", "online_softmax_attention"]
