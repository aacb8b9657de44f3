"""Causal incremental VQ on the GPU (reference ``streaming_vq.py:34-292``).

:class:`StreamingVQBuffer` keeps the same state as the reference's buffer --
running parent / child assignments, int64 counts and dtype aggregates -- and
``extend`` runs one library call (``avq_stream_extend``): parent and child
assignment of the new keys against the per-head codebook, the append to the
assignment record, and the ``index_add_`` of the keys into the aggregates,
with the reference's rounding and its head pairing for batches of more than
one key (row ``i`` of the flat ``[B*H]`` order adds key ``i // H`` to head
``i // B``).  The assignment record grows in place (capacity doubling), so
an extend costs O(B·H·M0·D) codebook work and no re-copy of the record.

All state lives on one CUDA device; there is no CPU path.
"""
from __future__ import annotations

import torch

from avqa_b200 import _lib
from avqa_b200.backend import QuantizationResult
from avqa_b200.exceptions import DeviceError, DtypeError, ShapeError


class StreamingVQBuffer:
    """Causal incremental VQ state (``streaming_vq.py:34-107``)."""

    def __init__(self, num_heads: int, num_parents: int, children_per_parent: int, head_dim: int, *,
                 device: str | torch.device = "cuda", dtype: torch.dtype = torch.float32) -> None:
        if num_heads <= 0 or num_parents <= 0 or children_per_parent <= 0:
            msg = f"invalid shape: H={num_heads}, M_0={num_parents}, C={children_per_parent}"
            raise ShapeError(msg, expected="H, M_0, C all > 0",
                             actual=(num_heads, num_parents, children_per_parent))
        device = torch.device(device)
        if device.type != "cuda":
            raise DeviceError("StreamingVQBuffer state lives on a CUDA device", expected="cuda", actual=str(device))
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if dtype not in _lib.DTYPE_CODE:
            raise DtypeError("unsupported dtype", expected="float32 | bfloat16 | float16", actual=str(dtype))
        self.num_heads = num_heads
        self.num_parents = num_parents
        self.children_per_parent = children_per_parent
        self.head_dim = head_dim
        self.device = device
        self.dtype = dtype
        H, M0, C, D = num_heads, num_parents, children_per_parent, head_dim
        self.parent_counts = torch.zeros(1, H, M0, dtype=torch.long, device=device)
        self.child_counts = torch.zeros(1, H, M0, C, dtype=torch.long, device=device)
        self.parent_aggregates = torch.zeros(1, H, M0, D, dtype=dtype, device=device)
        self.child_aggregates = torch.zeros(1, H, M0, C, D, dtype=dtype, device=device)
        self._prec = torch.zeros(1, H, 0, dtype=torch.long, device=device)
        self._crec = torch.zeros(1, H, 0, dtype=torch.long, device=device)
        self.size = 0
        self._started = False  # an extend (even of zero keys) has run since the last reset
        self._ws = None  # (stream handle, scratch): reused by later extends on the same stream

    def __len__(self) -> int:
        return self.size

    # The reference keeps the records as [1, H, N] tensors rebuilt by
    # torch.cat on every extend, and as an empty 1-D tensor before the first.
    @property
    def parent_assignments(self) -> torch.Tensor:
        return self._record(self._prec)

    @property
    def child_assignments(self) -> torch.Tensor:
        return self._record(self._crec)

    def _record(self, rec: torch.Tensor) -> torch.Tensor:
        if not self._started:
            return torch.empty(0, device=self.device)
        return rec[:, :, :self.size]

    def reset(self) -> None:
        """Drop all cached state (``streaming_vq.py:99-107``)."""
        self._prec = self._prec[:, :, :0]
        self._crec = self._crec[:, :, :0]
        self.parent_counts.zero_()
        self.child_counts.zero_()
        self.parent_aggregates.zero_()
        self.child_aggregates.zero_()
        self.size = 0
        self._started = False

    def _reserve(self, n: int) -> None:
        cap = self._prec.shape[-1]
        if self.size + n <= cap and self._prec.is_contiguous():
            return
        new_cap = max(self.size + n, 2 * cap, 64)
        H = self.num_heads
        grown = []
        for rec in (self._prec, self._crec):
            g = torch.zeros(1, H, new_cap, dtype=torch.long, device=self.device)
            g[:, :, :self.size] = rec[:, :, :self.size]
            grown.append(g)
        self._prec, self._crec = grown

    def extend(self, keys: torch.Tensor, parents: torch.Tensor,
               children: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Add one ``[B, D]`` batch of new keys; return the ``[B, H]`` int64
        (parent, child) assignments (``streaming_vq.py:109-229``)."""
        if keys.dim() != 2 or keys.shape[1] != self.head_dim:
            raise ShapeError("keys must be [B, D]", expected=f"[B, {self.head_dim}]", actual=tuple(keys.shape))
        if parents.shape != (self.num_heads, self.num_parents, self.head_dim):
            raise ShapeError("parents shape mismatch", expected=(self.num_heads, self.num_parents, self.head_dim),
                             actual=tuple(parents.shape))
        want_c = (self.num_heads, self.num_parents, self.children_per_parent, self.head_dim)
        if children.shape != want_c:
            raise ShapeError("children shape mismatch", expected=want_c, actual=tuple(children.shape))
        for name, t in (("keys", keys), ("parents", parents), ("children", children)):
            if t.device != self.device:
                raise DeviceError(f"{name} must be on the buffer's device", expected=str(self.device),
                                  actual=str(t.device))
            if t.dtype != self.dtype:
                # the reference's matmul / index_add_ reject mixed dtypes
                raise DtypeError(f"{name} dtype must match the buffer's", expected=str(self.dtype),
                                 actual=str(t.dtype))
        H, M0, D = parents.shape
        C = self.children_per_parent
        B = keys.shape[0]
        lib = _lib.load()
        if keys.stride(1) != 1 or (B > 1 and keys.stride(0) < D):
            keys = keys.contiguous()
        parents, children = parents.contiguous(), children.contiguous()
        pout = torch.empty(B, H, dtype=torch.long, device=self.device)
        cout = torch.empty(B, H, dtype=torch.long, device=self.device)
        self._reserve(B)
        ws_bytes = lib.avq_stream_workspace_size(B, H, M0, C)
        stream = _lib.stream_of(self.device)
        if self._ws is None or self._ws[0] != stream or self._ws[1].numel() < ws_bytes:
            self._ws = (stream, torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=self.device))
        ws = self._ws[1]
        rc = lib.avq_stream_extend(_lib.dtype_code(self.dtype), keys.data_ptr(), keys.stride(0) if B > 1 else D, B, H,
                                   M0, C, D, parents.data_ptr(), children.data_ptr(), pout.data_ptr(),
                                   cout.data_ptr(), self._prec.data_ptr(), self._crec.data_ptr(),
                                   self._prec.shape[-1], self.size, self.parent_counts.data_ptr(),
                                   self.child_counts.data_ptr(), self.parent_aggregates.data_ptr(),
                                   self.child_aggregates.data_ptr(), ws.data_ptr(), ws_bytes, stream)
        _lib.check(rc, "avq_stream_extend")
        self.size += B
        self._started = True
        return pout, cout

    def realize(self) -> QuantizationResult:
        """Snapshot the buffers into a :class:`QuantizationResult`
        (``streaming_vq.py:231-255``): the records as ``[1, H, N]`` copies,
        the aggregates as the live buffers, the counts cast to the dtype."""
        if self.size == 0:
            return empty_realisation(self.num_heads, self.num_parents, self.children_per_parent, self.head_dim,
                                     device=self.device, dtype=self.dtype)
        return QuantizationResult(
            parent_assignments=self.parent_assignments.contiguous(),
            child_assignments=self.child_assignments.contiguous(),
            parent_aggregates=self.parent_aggregates,
            child_aggregates=self.child_aggregates,
            parent_counts=self.parent_counts.to(dtype=self.dtype),
            child_counts=self.child_counts.to(dtype=self.dtype),
        )


def empty_realisation(num_heads: int, num_parents: int, children_per_parent: int, head_dim: int, *,
                      device: str | torch.device, dtype: torch.dtype) -> QuantizationResult:
    """Zero-tensor QuantizationResult for an empty buffer (``streaming_vq.py:258-292``)."""
    H, M0, C, D = num_heads, num_parents, children_per_parent, head_dim
    return QuantizationResult(
        parent_assignments=torch.zeros(1, H, 0, dtype=torch.int64, device=device),
        child_assignments=torch.zeros(1, H, 0, dtype=torch.int64, device=device),
        parent_aggregates=torch.zeros(1, H, M0, D, dtype=dtype, device=device),
        child_aggregates=torch.zeros(1, H, M0, C, D, dtype=dtype, device=device),
        parent_counts=torch.zeros(1, H, M0, dtype=dtype, device=device),
        child_counts=torch.zeros(1, H, M0, C, dtype=dtype, device=device),
    )


__all__ = ["StreamingVQBuffer", "empty_realisation"]
