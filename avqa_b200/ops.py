"""Tensor-level wrappers of the C ABI: device state objects and the calls
that fill them.  Every tensor passed here must live on one CUDA device.

``PreparedCodebook``  the codebook in the input dtype plus squared norms.
``QuantState``        the quantized key set of one (batch, heads) block:
                      assignments, dtype aggregates, fp32 bucket sums, exact
                      int32 counts, per-(b,h) valid-parent counts and their
                      minimum (the routing budget's floor).
"""
from __future__ import annotations

from dataclasses import dataclass

import ctypes

import torch

from avqa_b200 import _lib
from avqa_b200.exceptions import BackendError, DeviceError


def _cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise DeviceError(f"{name} must be a CUDA tensor", expected="cuda", actual=str(t.device))


@dataclass
class PreparedCodebook:
    parents: torch.Tensor  # [H, M0, D] dtype
    children: torch.Tensor  # [H, M0, C, D] dtype
    p_sq: torch.Tensor  # [H, M0] fp32
    c_sq: torch.Tensor  # [H, M0, C] fp32

    @property
    def dims(self) -> tuple[int, int, int, int]:
        H, M0, C, D = self.children.shape
        return H, M0, C, D


def prepare_codebook(parents: torch.Tensor, children: torch.Tensor, dtype: torch.dtype,
                     device: torch.device) -> PreparedCodebook:
    """Cast the codebook to ``dtype`` on ``device`` and compute its norms."""
    lib = _lib.load()
    p32 = parents.detach().to(device=device, dtype=torch.float32).contiguous()
    c32 = children.detach().to(device=device, dtype=torch.float32).contiguous()
    H, M0, C, D = c32.shape
    if tuple(p32.shape) != (H, M0, D):
        raise BackendError("codebook parents/children shapes disagree",
                           {"parents": tuple(p32.shape), "children": tuple(c32.shape)})
    out = PreparedCodebook(torch.empty(H, M0, D, dtype=dtype, device=device),
                           torch.empty(H, M0, C, D, dtype=dtype, device=device),
                           torch.empty(H, M0, dtype=torch.float32, device=device),
                           torch.empty(H, M0, C, dtype=torch.float32, device=device))
    rc = lib.avq_prepare_codebook(_lib.dtype_code(dtype), p32.data_ptr(), c32.data_ptr(), H, M0, C, D,
                                  out.parents.data_ptr(), out.children.data_ptr(), out.p_sq.data_ptr(),
                                  out.c_sq.data_ptr(), _lib.stream_of(device))
    _lib.check(rc, "avq_prepare_codebook")
    return out


@dataclass
class QuantState:
    B: int
    H: int
    S: int
    dtype: torch.dtype
    passign: torch.Tensor | None  # [G, S] int32 (None in append-only decode states)
    cassign: torch.Tensor | None
    pagg: torch.Tensor  # [G, M0, D] dtype
    cagg: torch.Tensor  # [G, M0, C, D] dtype
    pacc: torch.Tensor | None  # [G, M0, D] fp32 bucket sums (decode)
    cacc: torch.Tensor | None
    pcnt: torch.Tensor  # [G, M0] int32
    ccnt: torch.Tensor  # [G, M0, C] int32
    nvalid: torch.Tensor  # [G] int32
    gmin: torch.Tensor  # [1] int32: min over (b,h) of nvalid

    def counts_in_dtype(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Counts as the reference reports them: saturating at 2^(mantissa+1)."""
        sat = {torch.bfloat16: 256, torch.float16: 2048, torch.float32: 1 << 24}[self.dtype]
        return self.pcnt.clamp(max=sat).to(self.dtype), self.ccnt.clamp(max=sat).to(self.dtype)


def quantize(keys: torch.Tensor, values: torch.Tensor, cb: PreparedCodebook, keep_sums: bool = False) -> QuantState:
    """Quantize ``keys``/``values`` ``[B, H, S, D]`` views (any b/h/s strides)."""
    lib = _lib.load()
    _cuda(keys, "keys")
    dev = keys.device
    B, H, S, D = keys.shape
    Hc, M0, C, Dc = cb.dims
    if Hc != H or Dc != D:
        raise BackendError("codebook does not match the keys", {"heads": (Hc, H), "head_dim": (Dc, D)})
    if values.shape != keys.shape:
        raise BackendError("keys and values must have identical shapes",
                           {"keys": tuple(keys.shape), "values": tuple(values.shape)})
    dt = keys.dtype
    G = B * H
    i32 = dict(dtype=torch.int32, device=dev)
    st = QuantState(
        B, H, S, dt,
        torch.empty(G, S, **i32),
        torch.empty(G, S, **i32),
        torch.empty(G, M0, D, dtype=dt, device=dev),
        torch.empty(G, M0, C, D, dtype=dt, device=dev),
        torch.empty(G, M0, D, dtype=torch.float32, device=dev) if keep_sums else None,
        torch.empty(G, M0, C, D, dtype=torch.float32, device=dev) if keep_sums else None,
        torch.empty(G, M0, **i32), torch.empty(G, M0, C, **i32), torch.empty(G, **i32),
        torch.full((1,), 2 ** 31 - 1, **i32))
    ws_bytes = lib.avq_quantize_workspace_size(B, H, S, M0)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    rc = lib.avq_quantize(_lib.dtype_code(dt), keys.data_ptr(), _lib.strides3(keys), values.data_ptr(),
                          _lib.strides3(values), B, H, S, D, M0, C, cb.parents.data_ptr(), cb.p_sq.data_ptr(),
                          cb.children.data_ptr(), cb.c_sq.data_ptr(), _lib.ptr(st.passign), _lib.ptr(st.cassign),
                          st.pagg.data_ptr(), st.cagg.data_ptr(), _lib.ptr(st.pacc), _lib.ptr(st.cacc),
                          st.pcnt.data_ptr(), st.ccnt.data_ptr(), st.nvalid.data_ptr(), st.gmin.data_ptr(),
                          ws.data_ptr(), ws_bytes, _lib.stream_of(dev))
    _lib.check(rc, "avq_quantize")
    if G == 0:
        st.gmin.zero_()
    return st


def append(state: QuantState, k: torch.Tensor, v: torch.Tensor, cb: PreparedCodebook,
           kpage: torch.Tensor | None = None, vpage: torch.Tensor | None = None, slot0: int = 0) -> None:
    """Append ``k``/``v`` ``[B, H, Tn, D]`` to ``state`` in key order (and
    optionally write them into page slots ``slot0..`` of ``kpage``/``vpage``
    ``[B, H, page_size, D]``); refreshes ``state.gmin``."""
    lib = _lib.load()
    if state.pacc is None:
        raise BackendError("this quantization state keeps no fp32 bucket sums; quantize with keep_sums=True")
    B, H, Tn, D = k.shape
    _, M0, C, _ = cb.dims
    dev = k.device
    ws_bytes = lib.avq_append_workspace_size(B, H, Tn)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    rc = lib.avq_append(_lib.dtype_code(k.dtype), k.data_ptr(), _lib.strides3(k), v.data_ptr(), _lib.strides3(v),
                        B, H, Tn, D, M0, C, cb.parents.data_ptr(), cb.p_sq.data_ptr(), cb.children.data_ptr(),
                        cb.c_sq.data_ptr(), state.pacc.data_ptr(), state.cacc.data_ptr(), state.pagg.data_ptr(),
                        state.cagg.data_ptr(), state.pcnt.data_ptr(), state.ccnt.data_ptr(), state.nvalid.data_ptr(),
                        _lib.ptr(kpage), _lib.ptr(vpage), _lib.strides3(kpage) if kpage is not None else None,
                        slot0, ws.data_ptr(), ws_bytes, _lib.stream_of(dev))
    _lib.check(rc, "avq_append")
    state.S += Tn
    state.passign = None  # per-key assignments are not tracked across appends
    state.cassign = None
    rc = lib.avq_reduce_min(state.nvalid.data_ptr(), state.nvalid.numel(), state.gmin.data_ptr(),
                            _lib.stream_of(dev))
    _lib.check(rc, "avq_reduce_min")


def codeword_presence(state: QuantState, T: int, mask: torch.Tensor | None = None, causal_offset: int | None = None,
                      query_batch: int | None = None) -> torch.Tensor:
    """Codeword visibility bits ``[Bq*H, T, ceil(M0/32)]`` int32 for ``T``
    queries per (b,h) (pipeline.py:82-106): a parent is visible to a query
    when one of its keys is allowed by the mask.

    ``mask``: bool/uint8 ``[T, S]`` or ``[B, H, T, S]`` (True = attend; size-1
    leading dims broadcast); without it the causal mask, query t seeing keys
    ``0 .. t + causal_offset`` (the reference uses ``S - T``).  ``query_batch``
    is the query batch when the state (batch 1) serves several."""
    from avqa_b200.exceptions import NotInitializedError
    lib = _lib.load()
    if state.passign is None:
        raise NotInitializedError("the codeword mask needs the key assignments of this state (not kept after a "
                                  "decode append)")
    dev = state.pcnt.device
    Bq = state.B if query_batch is None else query_batch
    H, S, M0 = state.H, state.S, state.pcnt.shape[-1]
    W = lib.avq_presence_words(M0)
    out = torch.empty(Bq * H, T, W, dtype=torch.int32, device=dev)
    m, strides = _mask_operand(mask, Bq, H, T, S, dev)  # m stays referenced until the kernel is enqueued
    offset = (S - T) if causal_offset is None else causal_offset
    ws_bytes = lib.avq_presence_workspace_size(H, M0, state.B) if m is None else 0
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    rc = lib.avq_codeword_presence(_lib.ptr(state.passign), Bq, H, S, M0, T, state.B, _lib.ptr(m), strides, offset,
                                   out.data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_of(dev))
    _lib.check(rc, "avq_codeword_presence")
    return out


def _mask_operand(mask: torch.Tensor | None, B: int, H: int, T: int, S: int, dev):
    """(uint8 mask tensor or None, ctypes strides {b, h, t} or None) of a
    rank-2 [T, S] or rank-4 [B|1, H|1, T, S] mask (True = attend)."""
    from avqa_b200.exceptions import ConfigurationError, ShapeError
    if mask is None:
        return None, None
    if mask.ndim not in (2, 4):
        raise ConfigurationError("mask must be rank 2 [T_q, T_k] or rank 4 [B, H, T_q, T_k]", {"got_rank": mask.ndim})
    if tuple(mask.shape[-2:]) != (T, S):
        raise ShapeError("mask shape does not match the queries and keys", expected=(T, S),
                         actual=tuple(mask.shape[-2:]))
    m = mask.to(device=dev, dtype=torch.uint8)
    if m.stride(-1) != 1:
        m = m.contiguous()
    if m.ndim == 2:
        st = (0, 0, m.stride(0))
    else:
        if m.shape[0] not in (1, B) or m.shape[1] not in (1, H):
            raise ShapeError("rank-4 mask does not broadcast to [B, H, T, S]", expected=(B, H, T, S),
                             actual=tuple(m.shape))
        st = (m.stride(0) if m.shape[0] > 1 else 0, m.stride(1) if m.shape[1] > 1 else 0, m.stride(2))
    return m, (ctypes.c_longlong * 3)(*st)


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    mask: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(mask(q k^T / sqrt(D))) v for ``[B, H, T|N, D]`` views, in the
    input dtype (backend.py:190-203); returns a ``[B, H, T, D]`` view."""
    lib = _lib.load()
    _cuda(q, "query")
    B, H, T, D = q.shape
    N = k.shape[2]
    dev = q.device
    out = torch.empty(B, T, H, D, dtype=q.dtype, device=dev).permute(0, 2, 1, 3)
    m, mst = _mask_operand(mask, B, H, T, N, dev)
    rc = lib.avq_dense_attention(_lib.dtype_code(q.dtype), q.data_ptr(), _lib.strides3(q), k.data_ptr(),
                                 _lib.strides3(k), v.data_ptr(), _lib.strides3(v), B, H, T, N, D, _lib.ptr(m), mst,
                                 out.data_ptr(), _lib.strides3(out), _lib.stream_of(dev))
    _lib.check(rc, "avq_dense_attention")
    return out


def bcar_update(keys: torch.Tensor, state: QuantState, parents: torch.Tensor, children: torch.Tensor,
                decay: float) -> None:
    """BCAR (online_adaptation.py:37-127): adapt ``children`` [H, M0, C, D]
    toward the means of the keys ``[B, H, S, D]`` that ``state`` assigned to
    each child cell and re-derive ``parents`` [H, M0, D] as their children's
    means, in place, in the codebook dtype (= the keys' dtype)."""
    from avqa_b200.exceptions import NotInitializedError
    lib = _lib.load()
    if state.passign is None:
        raise NotInitializedError("BCAR needs the key assignments of this state (not kept after a decode append)")
    B, H, S, D = keys.shape
    _, M0, C, _ = children.shape
    dev = keys.device
    new_c = torch.empty_like(children)
    new_p = torch.empty_like(parents)
    ws_bytes = lib.avq_bcar_workspace_size(B, H, M0, C, D)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    rc = lib.avq_bcar_update(_lib.dtype_code(keys.dtype), keys.data_ptr(), _lib.strides3(keys),
                             _lib.ptr(state.passign), _lib.ptr(state.cassign), B, H, S, D, M0, C, float(decay),
                             children.data_ptr(), new_c.data_ptr(), new_p.data_ptr(), ws.data_ptr(), ws_bytes,
                             _lib.stream_of(dev))
    _lib.check(rc, "avq_bcar_update")
    children.copy_(new_c)
    parents.copy_(new_p)


@dataclass
class ForwardDiagnostics:
    importance: torch.Tensor  # [G, M0] fp32 (pre-HVAQ importance, dtype values)
    selected: torch.Tensor  # [G, stride] int32, -1 padded, pass after pass
    pass_counts: torch.Tensor  # [passes] int32
    stride: int
    caps: list[int]

    def selections(self) -> list[torch.Tensor]:
        """Per pass, the ``[G, n_k]`` selected parent indices."""
        out, off = [], 0
        counts = self.pass_counts.tolist()
        for cap, n in zip(self.caps, counts):
            if n > 0:
                out.append(self.selected[:, off:off + n])
            off += cap
        return out


def pass_caps(P: int, passes: int, decay: float) -> list[int]:
    return [max(1, round(P * (decay ** i))) if i else P for i in range(passes)]


def forward(q: torch.Tensor, cb: PreparedCodebook, st: QuantState, P: int, passes: int = 1, pass_decay: float = 1.0,
            hvaq: int = 0, beta0: float = 0.0, alpha: float = 1.0, out: torch.Tensor | None = None,
            min_valid: torch.Tensor | None = None, diagnostics: bool = False,
            min_valid_ready: torch.cuda.Event | None = None, present: torch.Tensor | None = None):
    """AVQ attention of ``q`` ``[B, H, T, D]`` over ``st``.

    ``st`` holds either B batches of keys, or one batch that every query
    batch attends to (query chunks of one sequence over keys quantized once;
    each batch entry is routed on its own, exactly as separate calls over the
    same keys).  ``min_valid_ready``: an event recorded after ``min_valid``
    was produced on another stream; the library waits on it only right
    before routing.  ``present``: codeword visibility bits of a mask
    (:func:`codeword_presence`) for these queries.

    Returns ``out`` as a ``[B, H, T, D]`` fp32 view (module layout when
    ``out`` is given as a ``[B, T, H, D]``-strided tensor) and optional
    diagnostics.
    """
    lib = _lib.load()
    _cuda(q, "query")
    B, H, T, D = q.shape
    _, M0, C, _ = cb.dims
    dev = q.device
    if st.B != B and st.B != 1:
        raise BackendError("quantized state batch must equal the query batch or be 1",
                           {"state_batch": st.B, "query_batch": B})
    if out is None:
        out = torch.empty(B, T, H, D, dtype=torch.float32, device=dev).permute(0, 2, 1, 3)
    ws_bytes = lib.avq_forward_workspace_size(_lib.dtype_code(q.dtype), B, H, T, D, M0, C, P, passes, pass_decay, hvaq)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    diag = None
    imp = sel = pc = None
    if diagnostics:
        stride = lib.avq_selection_stride(P, passes, pass_decay)
        imp = torch.empty(B * H, M0, dtype=torch.float32, device=dev)
        sel = torch.full((B * H, stride), -1, dtype=torch.int32, device=dev)
        pc = torch.zeros(passes, dtype=torch.int32, device=dev)
        diag = ForwardDiagnostics(imp, sel, pc, stride, pass_caps(P, passes, pass_decay))
    mv = st.gmin if min_valid is None else min_valid
    rc = lib.avq_forward(_lib.dtype_code(q.dtype), q.data_ptr(), _lib.strides3(q), B, H, T, D, M0, C,
                         cb.parents.data_ptr(), cb.children.data_ptr(), st.pagg.data_ptr(), st.cagg.data_ptr(),
                         st.pcnt.data_ptr(), st.ccnt.data_ptr(), st.B, mv.data_ptr(),
                         None if min_valid_ready is None else min_valid_ready.cuda_event, _lib.ptr(present), P,
                         passes, pass_decay,
                         hvaq, beta0, alpha, out.data_ptr(), _lib.strides3(out), _lib.ptr(imp), _lib.ptr(sel),
                         _lib.ptr(pc), ws.data_ptr(), ws_bytes, _lib.stream_of(dev))
    _lib.check(rc, "avq_forward")
    return out, diag


__all__ = ["ForwardDiagnostics", "PreparedCodebook", "QuantState", "append", "bcar_update", "codeword_presence",
           "dense_attention", "forward", "pass_caps", "prepare_codebook", "quantize"]
