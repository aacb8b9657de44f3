"""CPU restatement (numpy) of the sachncs/avqa AVQ-attention forward.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA path: it is
imported by ``tests/``, by ``__graft_entry__.smoke()`` and by the CPU-baseline
leg of ``bench.py``.  The product path (``avqa_b200``) never imports it.

What it models
--------------
The reference runs every stage in the input dtype on the CPU (torch ops).  Each
torch op computes in fp32 ("opmath") and rounds its result once to the tensor
dtype.  This restatement reproduces those rounding points exactly:

* every elementwise op, matmul and reduction is evaluated in float64 (exact
  for the products and sums that occur here), rounded to fp32 and then to the
  dtype, both with round-to-nearest-even -- torch's fp32 "opmath" followed by
  the narrowing store;
* ``index_add_`` aggregation of values is a sequential fp32 sum per bucket in
  key order, rounded once to the dtype (``quantizer.py:242-244,258-260``),
  reproduced bit-for-bit;
* counts are ``index_add_`` of ones in the value dtype, so they saturate at
  256 (bf16), 2048 (fp16) and 2**24 (fp32);
* the refinement correction is promoted to fp32 (``refinement.py:314-358``,
  ``attention.py:138-163``) and the output is fp32 for every input dtype.

The one thing it cannot reproduce is the reference's own fp32 accumulation
order inside BLAS/oneDNN GEMMs and vectorised sums.  Those differ from the
exactly-rounded value in ~6e-5 of bf16 GEMM entries; an index that flips
because of that is a certified near-tie (see ``tests/parity.py``).

Layout: tensors are ``[G, ...]`` with ``G = B*H`` and head ``h = g % H``
(the reference's ``split_heads``, ``attention_module.py:198-202``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

DTYPES = ("f32", "bf16", "f16")

# ---------------------------------------------------------------------------
# Rounding
# ---------------------------------------------------------------------------


def _bf16_from_f32(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bf16 (RNE), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    nan = np.isnan(x)
    r = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    with np.errstate(over="ignore"):
        out = ((u + r) & np.uint32(0xFFFF0000)).view(np.float32)  # +inf rounds to +inf; wraps only for NaN
    if nan.any():
        out = np.where(nan, x, out)
    return out


def rnd(x, dt: str) -> np.ndarray:
    """Round values to ``dt`` the way a torch CPU op does; returns float32.

    torch computes every op in fp32 ("opmath") and then narrows, so the
    value is first rounded to fp32 and then to the dtype (RNE both times).
    The intermediate fp32 rounding matters when an operand is an fp32
    scalar (``x / sqrt(D)``, ``alpha * h``): ``0.7 * bf16(1.7578125)``
    rounds to the fp32 tie ``1.23046875`` and then to even, 1.234375.
    """
    x = np.asarray(x)
    with np.errstate(over="ignore", invalid="ignore"):
        f = x.astype(np.float32)
        if dt == "f32":
            return f
        if dt == "f16":
            return f.astype(np.float16).astype(np.float32)
        if dt == "bf16":
            return _bf16_from_f32(f)
    raise ValueError(f"unknown dtype {dt!r}")


def scalar_in_dt(v: float, dt: str) -> float:
    """A Python scalar cast to the tensor dtype (``clamp_min``'s bound)."""
    return float(rnd(np.array([v], np.float64), dt)[0])


def opmath_scalar(v: float) -> np.float64:
    """A Python scalar as the fp32 opmath operand of a tensor-scalar op."""
    return np.float64(np.float32(v))


def count_saturation(dt: str) -> int:
    """Largest count reachable by repeated ``+1`` in ``dt`` (index_add_ of ones)."""
    return {"f32": 1 << 24, "f16": 2048, "bf16": 256}[dt]


EPS = 1e-12  # pipeline.py:37, attention_module.py:534


def _f64(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float64)


# ---------------------------------------------------------------------------
# Quantizer: quantizer.py:166-278
# ---------------------------------------------------------------------------


@dataclass
class Quantization:
    parent_assignments: np.ndarray  # [G,S] int64
    child_assignments: np.ndarray  # [G,S] int64
    parent_aggregates: np.ndarray  # [G,M0,D] f32 (dt values)
    child_aggregates: np.ndarray  # [G,M0,C,D]
    parent_counts: np.ndarray  # [G,M0] f32 (dt values, saturating)
    child_counts: np.ndarray  # [G,M0,C]
    parent_counts_exact: np.ndarray = field(default=None)  # [G,M0] int64
    child_counts_exact: np.ndarray = field(default=None)


def sq_norms(x: np.ndarray, dt: str) -> np.ndarray:
    """``(x*x).sum(-1)`` with the product rounded to dt (quantizer.py:207-208,224)."""
    return rnd(rnd(_f64(x) * x, dt).astype(np.float64).sum(-1), dt)


def parent_distances(keys, parents_g, dt: str) -> np.ndarray:
    """``k_sq + p_sq - 2*(k @ p^T)``, each op rounded (quantizer.py:207-210)."""
    k_sq = sq_norms(keys, dt)[..., None]  # [G,S,1]
    p_sq = sq_norms(parents_g, dt)[:, None, :]  # [G,1,M0]
    cross = rnd(np.matmul(_f64(keys), _f64(parents_g).transpose(0, 2, 1)), dt)
    two_cross = rnd(2.0 * _f64(cross), dt)
    return rnd(_f64(rnd(_f64(k_sq) + p_sq, dt)) - two_cross, dt)


def first_argmin(d: np.ndarray) -> np.ndarray:
    """``torch.argmin``: first index of the minimum; a NaN wins (propagates)."""
    nan = np.isnan(d)
    idx = np.argmin(np.where(nan, np.inf, d), axis=-1)
    if nan.any():
        has = nan.any(-1)
        idx = np.where(has, np.argmax(nan, axis=-1), idx)
    return idx.astype(np.int64)


def child_distances(keys, children_sel, dt: str) -> np.ndarray:
    """``k_sq + c_sq - 2*sum(k*c)`` over the assigned parent's children.

    The cross term is an elementwise product rounded to dt, then summed
    (quantizer.py:223-226) -- not a matmul.
    """
    k_sq = sq_norms(keys, dt)[..., None]  # [G,S,1]
    c_sq = sq_norms(children_sel, dt)  # [G,S,C]
    prod = rnd(_f64(keys)[:, :, None, :] * children_sel, dt)
    cross = rnd(prod.astype(np.float64).sum(-1), dt)
    two_cross = rnd(2.0 * _f64(cross), dt)
    return rnd(_f64(rnd(_f64(k_sq) + c_sq, dt)) - two_cross, dt)


def sequential_bucket_sums(values: np.ndarray, bucket: np.ndarray, nb: int, dt: str) -> np.ndarray:
    """Per-bucket sums in key order, as the reference's 2-D ``index_add_`` does.

    The row-wise ``index_add_`` accumulates each bucket sequentially in fp32
    (key order) and rounds once to the dtype at the end; pinned bit-exact
    against the reference for fp32, bf16 and fp16 (tests/golden).
    values ``[G,S,D]``, bucket ``[G,S]`` in ``[0,nb)``; returns ``[G,nb,D]``.
    """
    G, S, D = values.shape
    flat = (np.arange(G)[:, None] * nb + bucket).ravel()
    order = np.argsort(flat, kind="stable")
    fb = flat[order]
    counts = np.bincount(flat, minlength=G * nb)
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int64)
    rank = np.arange(G * S) - starts[fb]
    vals = values.reshape(G * S, D)[order]
    acc = np.zeros((G * nb, D), np.float32)
    top = int(counts.max()) if counts.size else 0
    for r in range(top):
        sel = rank == r
        ids = fb[sel]
        acc[ids] = (acc[ids] + vals[sel]).astype(np.float32)
    return rnd(acc, dt).reshape(G, nb, D)


def quantize(keys, values, parents, children, dt: str) -> Quantization:
    """EuclideanHierarchicalQuantizer.precompute (quantizer.py:166-278).

    keys/values ``[G,S,D]``; parents ``[H,M0,D]``; children ``[H,M0,C,D]``
    (all holding dt-representable values).
    """
    G, S, D = keys.shape
    H, M0, C, _ = children.shape
    hidx = np.arange(G) % H
    pg = parents[hidx]  # [G,M0,D]
    if S == 0:
        z = np.zeros((G, 0), np.int64)
        return Quantization(z, z.copy(), np.zeros((G, M0, D), np.float32),
                            np.zeros((G, M0, C, D), np.float32), np.zeros((G, M0), np.float32),
                            np.zeros((G, M0, C), np.float32), np.zeros((G, M0), np.int64),
                            np.zeros((G, M0, C), np.int64))
    # quantizer.py:211 and :217-227, in blocks of keys so that the [G, block, M0]
    # distances stay small (every key's argmin depends on that key alone)
    blk = max(1, (1 << 24) // max(1, G * M0))
    passign = np.empty((G, S), np.int64)
    cassign = np.empty((G, S), np.int64)
    for s0 in range(0, S, blk):
        kb = keys[:, s0:s0 + blk]
        pa = first_argmin(parent_distances(kb, pg, dt))
        csel = children[hidx[:, None], pa]  # [G,blk,C,D]
        passign[:, s0:s0 + blk] = pa
        cassign[:, s0:s0 + blk] = first_argmin(child_distances(kb, csel, dt))
    pagg = sequential_bucket_sums(values, passign, M0, dt)  # quantizer.py:242-244
    flat_child = passign * C + cassign  # quantizer.py:256
    cagg = sequential_bucket_sums(values, flat_child, M0 * C, dt).reshape(G, M0, C, D)
    pcnt_exact = np.stack([np.bincount(passign[g], minlength=M0) for g in range(G)])
    ccnt_exact = np.stack([np.bincount(flat_child[g], minlength=M0 * C) for g in range(G)]).reshape(G, M0, C)
    sat = count_saturation(dt)
    return Quantization(passign, cassign, pagg, cagg,
                        np.minimum(pcnt_exact, sat).astype(np.float32),
                        np.minimum(ccnt_exact, sat).astype(np.float32),
                        pcnt_exact, ccnt_exact)


# ---------------------------------------------------------------------------
# Streaming VQ: streaming_vq.py:34-255 (StreamingVQBuffer)
# ---------------------------------------------------------------------------


@dataclass
class StreamState:
    """StreamingVQBuffer's buffers: counts exact, aggregates in the dtype."""

    pcnt: np.ndarray  # [H, M0] int64
    ccnt: np.ndarray  # [H, M0, C] int64
    pagg: np.ndarray  # [H, M0, D] f32 (dt values)
    cagg: np.ndarray  # [H, M0, C, D]
    passign: list = field(default_factory=list)  # per extend: [H, B] (the reference's reshape(1, H, B))
    cassign: list = field(default_factory=list)


def stream_init(H: int, M0: int, C: int, D: int) -> StreamState:
    return StreamState(np.zeros((H, M0), np.int64), np.zeros((H, M0, C), np.int64),
                       np.zeros((H, M0, D), np.float32), np.zeros((H, M0, C, D), np.float32))


def stream_extend(st: StreamState, keys: np.ndarray, parents: np.ndarray, children: np.ndarray,
                  dt: str) -> tuple[np.ndarray, np.ndarray]:
    """StreamingVQBuffer.extend (streaming_vq.py:109-229) for ``keys`` [B, D]
    (the same keys for every head); returns ``(parent, child)`` [B, H].

    * distance ``DT(DT(k_sq - DT(2 DT(k.p))) + p_sq)`` (:172-177, that order);
    * child ``DT(sum DT(DT(k - c)^2))`` over the assigned parent's children (:185-187);
    * the aggregates gain the keys by ``index_add_`` with row i of the flat
      ``[B*H]`` order: destination head ``i // B`` (``repeat_interleave``),
      parent ``assign.reshape(-1)[i]`` and key ``i // H`` (:191-209); each
      destination row adds its keys to the stored dtype value in fp32, in row
      order, and narrows once per call;
    * the record appends ``assign.reshape(1, H, B)`` (:212-223).
    """
    H, M0, D = parents.shape
    C = children.shape[2]
    B = keys.shape[0]
    f64 = np.float64
    k_sq = sq_norms(keys, dt)  # [B]
    p_sq = sq_norms(parents, dt)  # [H, M0]
    cross = rnd(np.einsum("bd,hmd->bhm", _f64(keys), _f64(parents)), dt)
    with np.errstate(invalid="ignore", over="ignore"):
        dist = rnd(_f64(rnd(_f64(k_sq)[:, None, None] - _f64(rnd(2.0 * _f64(cross), dt)), dt)) + p_sq[None], dt)
    pa = first_argmin(dist)  # [B, H]
    chosen = children[np.arange(H)[None, :], pa]  # [B, H, C, D]
    diff = rnd(_f64(keys)[:, None, None, :] - chosen, dt)
    cd = rnd(rnd(_f64(diff) * diff, dt).astype(f64).sum(-1), dt)
    ca = first_argmin(cd)  # [B, H]
    rows = np.arange(B * H)
    head = rows // B
    fp, fc = pa.reshape(-1), (pa * C + ca).reshape(-1)
    kf = keys[rows // H]
    for flat_dst, agg, cnt, width in ((head * M0 + fp, st.pagg.reshape(-1, D), st.pcnt.reshape(-1), M0),
                                      (head * M0 * C + fc, st.cagg.reshape(-1, D), st.ccnt.reshape(-1), M0 * C)):
        acc = {}
        for i in range(B * H):
            d = int(flat_dst[i])
            if d not in acc:
                acc[d] = agg[d].astype(np.float32).copy()
            acc[d] = (acc[d] + kf[i].astype(np.float32)).astype(np.float32)
            cnt[d] += 1
        for d, a in acc.items():
            agg[d] = rnd(a, dt)
    st.passign.append(pa.reshape(H, B))
    st.cassign.append(ca.reshape(H, B))
    return pa, ca


# ---------------------------------------------------------------------------
# Dense attention: backend.py:190-203 (TorchBackend.naive_attention)
# ---------------------------------------------------------------------------


def naive_attention(qg, kg, vg, dt: str, mask_g: np.ndarray | None = None) -> np.ndarray:
    """``softmax(mask(DT(DT(q k^T) * D^-1/2))) v`` in the dtype: the logits
    and the probabilities rounded to the dtype, the product rounded once.
    ``[G, T|N, D]`` inputs, ``mask_g`` [G, T, N] (True = attend); a fully
    masked query is NaN (softmax over -inf)."""
    D = qg.shape[-1]
    scale = opmath_scalar(float(D ** -0.5))
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        s = rnd(rnd(np.matmul(_f64(qg), _f64(kg).swapaxes(-1, -2)), dt).astype(np.float64) * scale, dt)
        if mask_g is not None:
            s = np.where(mask_g, s, np.float32(-np.inf))
        mx = s.max(-1, keepdims=True)
        e = np.exp(_f64(s) - mx)
        probs = rnd(e / e.sum(-1, keepdims=True), dt)
        return rnd(np.matmul(_f64(probs), _f64(vg)), dt)


# ---------------------------------------------------------------------------
# BCAR online codebook adaptation: online_adaptation.py:37-127
# ---------------------------------------------------------------------------


def bcar_update(keys_g: np.ndarray, passign: np.ndarray, cassign: np.ndarray, parents: np.ndarray,
                children: np.ndarray, B: int, decay: float, dt: str) -> tuple[np.ndarray, np.ndarray]:
    """One EMA step of the child codebook, parents re-derived as the mean of
    their children; returns the new ``(parents, children)`` in ``dt``.

    ``keys_g`` [G, S, D], assignments [G, S] (G = B*H, g = b*H + h),
    ``parents`` [H, M0, D], ``children`` [H, M0, C, D] holding dt values.
    Follows the reference op by op in the codebook dtype:

    * per group and cell: the key sum (an einsum with a one-hot matrix:
      the exact sum rounded through fp32), the count (a sum, rounded), its
      reciprocal, the mean ``DT(sum * DT(1 / count))`` (online_adaptation.py:99-108);
    * ``new = DT(c + DT(w * DT(mean - c)))`` with ``w = DT(fp32(1 - decay))``
      where the cell received keys, else 0 (:113-115);
    * the tiled codebook is ``children.repeat_interleave(B, dim=0)`` while
      the groups are ordered b-major, so group ``i = b*H + h`` updates the
      children of head ``i // B`` and the results are averaged over ``b``
      as ``view(B, H, ...)`` reads them (:95, :116) -- for B > 1 the head
      pairing is the reference's own;
    * cells that received no key in any b keep their children (:117-123);
      then ``parents = DT(mean over c)`` (:126).
    """
    G, S, D = keys_g.shape
    H, M0, C, _ = children.shape
    MC = M0 * C
    f64 = np.float64
    sums = np.zeros((G, MC, D), f64)
    cnts = np.zeros((G, MC), np.int64)
    cell = passign.astype(np.int64) * C + cassign.astype(np.int64)
    for g in range(G):
        np.add.at(sums[g], cell[g], keys_g[g].astype(f64))
        cnts[g] = np.bincount(cell[g], minlength=MC)
    sum_dt = rnd(sums, dt)
    cnt_dt = rnd(cnts.astype(f64), dt)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.where(cnt_dt > 0, rnd(1.0 / np.where(cnt_dt > 0, cnt_dt, 1.0).astype(f64), dt), np.float32(0))
    mean = rnd(sum_dt.astype(f64) * inv[..., None].astype(f64), dt)
    has = cnts > 0
    w = np.where(has, np.float32(rnd(np.array([np.float32(1.0 - decay)], f64), dt)[0]), np.float32(0))
    src = children.reshape(H, MC, D)[np.arange(G) // B]  # repeat_interleave(B, dim=0)
    with np.errstate(invalid="ignore", over="ignore"):
        diff = rnd(mean.astype(f64) - src, dt)
        upd = rnd(w[..., None].astype(f64) * diff, dt)
        new_bh = rnd(src.astype(f64) + upd, dt)
        per_h = rnd(new_bh.reshape(B, H, MC, D).astype(f64).sum(0).astype(np.float32).astype(f64) / B, dt)
    any_b = has.reshape(B, H, MC).any(0)
    new_children = np.where(any_b[..., None], per_h, children.reshape(H, MC, D)).reshape(H, M0, C, D)
    new_parents = rnd(new_children.astype(f64).sum(2).astype(np.float32).astype(f64) / C, dt)
    return new_parents.astype(np.float32), new_children.astype(np.float32)


# ---------------------------------------------------------------------------
# Parent attention: pipeline.py:46-151
# ---------------------------------------------------------------------------


def scaled_logits(q, keys_g, D: int, dt: str) -> np.ndarray:
    """``rnd(rnd(q @ k^T) / sqrt(D))`` (pipeline.py:81, :184)."""
    raw = rnd(np.matmul(_f64(q), _f64(keys_g).swapaxes(-1, -2)), dt)
    return rnd(_f64(raw) / opmath_scalar(math.sqrt(D)), dt)


def causal_mask(t_q: int, t_k: int) -> np.ndarray:
    """attention_module.py:210-223: ``[T_q, T_k]``, query i sees keys
    ``0 .. i + (t_k - t_q)`` (the cached prefix is visible to every query)."""
    i = np.arange(t_q)[:, None]
    j = np.arange(t_k)[None, :]
    return j <= i + (t_k - t_q)


def codeword_present(mask_g: np.ndarray, passign: np.ndarray, M0: int) -> np.ndarray:
    """pipeline.py:98-105: parent p is visible to query t when at least one
    key assigned to p is allowed by the mask.  ``mask_g`` [G, T, S] bool,
    ``passign`` [G, S]; returns [G, T, M0] bool."""
    G, T, S = mask_g.shape
    out = np.zeros((G, T, M0), bool)
    for g in range(G):
        onehot = np.zeros((S, M0), np.float32)
        onehot[np.arange(S), passign[g]] = 1.0
        out[g] = (mask_g[g].astype(np.float32) @ onehot) > 0
    return out


def expand_mask(mask: np.ndarray, B: int, H: int) -> np.ndarray:
    """A rank-2 ``[T, S]`` or rank-4 ``[B, H, T, S]`` mask as ``[G, T, S]``
    (pipeline.py:93-97)."""
    mask = np.asarray(mask, bool)
    if mask.ndim == 2:
        return np.broadcast_to(mask, (B * H,) + mask.shape)
    if mask.ndim == 4:
        return np.broadcast_to(mask, (B, H) + mask.shape[2:]).reshape((B * H,) + mask.shape[2:])
    raise ValueError("mask must be rank 2 [T_q, T_k] or rank 4 [B, H, T_q, T_k]")


def parent_logits(q, parents, pcnt, H: int, dt: str, present: np.ndarray | None = None) -> np.ndarray:
    """pipeline.py:46-108: logits, -inf where the codeword has no key visible
    to the query (``present``, from a user or causal mask) and where
    count == 0."""
    G = q.shape[0]
    D = q.shape[-1]
    s = scaled_logits(q, parents[np.arange(G) % H], D, dt)
    if present is not None:
        s = np.where(present, s, np.float32(-np.inf))
    return np.where((pcnt > 0)[:, None, :], s, np.float32(-np.inf)).astype(np.float32)


@dataclass
class SoftmaxState:
    m: np.ndarray  # [G,T] f32
    l: np.ndarray  # [G,T] f32
    a: np.ndarray  # [G,T,D] f32
    probs: np.ndarray  # [G,T,M0] f32 (dt values)
    tile_exp: np.ndarray  # [G,T,M0]
    z: np.ndarray  # [G,T]  rounded row sum of tile_exp (before clamp)


def online_softmax(s, pagg, pcnt, dt: str) -> SoftmaxState:
    """pipeline.py:111-151 with OnlineSoftmaxState.merge into an empty fp32 state."""
    with np.errstate(invalid="ignore", over="ignore"):
        tmax = s.max(-1, keepdims=True) if s.shape[-1] else np.full(s.shape[:-1] + (1,), -np.inf, np.float32)
        safe = np.where(np.isneginf(tmax), np.float32(0), tmax).astype(np.float32)  # :137-141
        diff = rnd(_f64(s) - safe, dt)
        e = rnd(np.exp(_f64(diff)), dt)  # :142
        e = np.where(np.isnan(e), np.float32(0), e).astype(np.float32)  # :143-145
        l = rnd(rnd(_f64(e) * pcnt[:, None, :], dt).astype(np.float64).sum(-1), dt)  # :146
        a = rnd(np.matmul(_f64(e), _f64(pagg)), dt)  # :147 einsum
        z = rnd(_f64(e).sum(-1), dt)  # :150
        zc = np.maximum(z, np.float32(scalar_in_dt(EPS, dt)))
        probs = rnd(_f64(e) / zc[..., None], dt)
    # merge into the empty state (attention.py:86-98, numerics.py:17-65):
    # m = max(-inf, safe) = safe; alpha = 0, beta = 1 -> l, a promoted to fp32.
    return SoftmaxState(safe[..., 0], l.astype(np.float32), a.astype(np.float32), probs, e, z)


def importance(probs, pcnt, dt: str) -> np.ndarray:
    """routing.py:61-63: ``counts * probs.sum(dim=-2)``."""
    total = rnd(_f64(probs).sum(-2), dt)
    return rnd(_f64(pcnt) * total, dt)


def stable_topk_desc(w: np.ndarray, k: int) -> np.ndarray:
    """``torch.sort(descending=True, stable=True)[..., :k]`` (routing.py:164-170).

    NaN sorts first (torch treats NaN as the largest value); ties keep
    ascending index order.
    """
    G, M = w.shape
    key = np.where(np.isnan(w), -np.inf, -w.astype(np.float64))
    nanfirst = ~np.isnan(w)  # False (0) sorts before True (1)
    idx = np.lexsort((np.broadcast_to(np.arange(M), (G, M)), key, nanfirst), axis=-1)
    return idx[:, :k].astype(np.int64)


# ---------------------------------------------------------------------------
# HVAQ: pipeline.py:192-258, hopfield.py:55-144
# ---------------------------------------------------------------------------


def hvaq_logits(s, probs, sel, D: int, dt: str, beta_init: float, adaptive: str, alpha: float = 1.0):
    """Return (scaled logits, beta_q) for the HVAQ temperature schedule."""
    if beta_init <= 0.0:
        beta_init = 1.0 / math.sqrt(D)  # hopfield.py:38-43
    G, T, M0 = probs.shape
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        gathered = np.take_along_axis(probs, np.broadcast_to(sel[:, None, :], (G, T, sel.shape[-1])), -1)
        gs = rnd(_f64(gathered).sum(-1), dt)
        gs = np.maximum(gs, np.float32(scalar_in_dt(EPS, dt)))
        top = rnd(_f64(gathered) / gs[..., None], dt)  # pipeline.py:238
        if adaptive == "none":
            beta = np.full((G, T), np.float32(rnd(np.array([beta_init]), dt)[0]), np.float32)
        else:
            logp = np.where(top > 0, rnd(np.log(np.where(top > 0, _f64(top), 1.0)), dt), np.float32(0))
            h = -rnd(rnd(_f64(top) * logp, dt).astype(np.float64).sum(-1), dt)  # hopfield.py:100
            if adaptive == "entropy":
                one_p = rnd(1.0 + _f64(h), dt)
                sched = rnd(1.0 + _f64(rnd(1.0 / _f64(one_p), dt)), dt)
            elif adaptive == "linear":
                sched = rnd(1.0 + _f64(rnd(opmath_scalar(alpha) * h, dt)), dt)
            else:
                raise ValueError(adaptive)
            beta = rnd(opmath_scalar(beta_init) * sched, dt)  # hopfield.py:102
        raw = rnd(_f64(s) * opmath_scalar(math.sqrt(D)), dt)  # pipeline.py:256
        scaled = rnd(_f64(beta)[..., None] * raw, dt)  # hopfield.py:144 (parent_beta = 1.0)
    return scaled.astype(np.float32), beta


# ---------------------------------------------------------------------------
# Child logits + correction: pipeline.py:154-189, refinement.py:82-304
# ---------------------------------------------------------------------------


def child_logits_sel(q, children, sel, ccnt, H: int, dt: str) -> np.ndarray:
    """pipeline.py:154-189: ``[G,T,P,C]`` logits of the selected parents' children."""
    G, T, D = q.shape
    C = children.shape[2]
    hidx = np.arange(G) % H
    ch = children[hidx[:, None], sel]  # [G,P,C,D]
    P = sel.shape[-1]
    u = scaled_logits(q, ch.reshape(G, P * C, D), D, dt).reshape(G, T, P, C)
    cnt = np.take_along_axis(ccnt, sel[..., None].repeat(C, -1), 1)  # [G,P,C]
    return np.where((cnt > 0)[:, None], u, np.float32(-np.inf)).astype(np.float32)


def correction(m, l, a, probs, pagg, pcnt, cagg, ccnt, sel, u):
    """vectorized_correction + OnlineSoftmaxState.replace (fp32 promoted).

    ``u`` is ``[G,T,P,C]`` child logits aligned with ``sel`` slots.
    Returns the new (l, a) in fp32.
    """
    G, T = m.shape
    P = sel.shape[-1]
    C = ccnt.shape[-1]
    f32 = np.float32
    with np.errstate(over="ignore", invalid="ignore"):
        x = np.take_along_axis(probs, np.broadcast_to(sel[:, None, :], (G, T, P)), -1)  # refinement.py:233
        nsel = np.take_along_axis(pcnt, sel, -1)  # :249
        vsel = np.take_along_axis(pagg, sel[..., None], 1)  # [G,P,D] :241-246
        csel = np.take_along_axis(cagg, sel[..., None, None], 1)  # [G,P,C,D] :229-230
        ncsel = np.take_along_axis(ccnt, sel[..., None], 1)  # [G,P,C]
        mm = m[..., None].astype(f32)
        # fp32 weights (exp is the correctly rounded fp32 value); the weighted
        # value sums are evaluated exactly in float64 and rounded once to fp32
        # (refinement.py:335-348 sums fp32 products in fp32).
        pe = (exp32((x - mm).astype(f32)) * nsel[:, None, :]).astype(f32)  # :335
        r_l = pe.sum(-1, dtype=np.float64)
        r_a = np.einsum("gtp,gpd->gtd", pe.astype(np.float64), vsel.astype(np.float64))  # :337
        ce = (exp32((u - mm[..., None]).astype(f32)) * ncsel[:, None]).astype(f32)  # :341
        a_l = ce.sum((-1, -2), dtype=np.float64)
        a_a = np.einsum("gtk,gkd->gtd", ce.reshape(G, T, P * C).astype(np.float64),
                        csel.reshape(G, P * C, -1).astype(np.float64))  # :346
        l_new = ((l.astype(f32) - r_l.astype(f32)).astype(f32) + a_l.astype(f32)).astype(f32)  # attention.py:149-153
        a_new = ((a.astype(f32) - r_a.astype(f32)).astype(f32) + a_a.astype(f32)).astype(f32)
    return l_new, a_new


def exp32(x: np.ndarray) -> np.ndarray:
    """Correctly rounded fp32 ``exp`` of fp32 values."""
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        return np.exp(x.astype(np.float64)).astype(np.float32)


def compute_pass_budgets(base: int, passes: int, decay: float) -> list[int]:
    """multipass.py:40-67 (Python ``round`` is half-to-even)."""
    return [max(1, round(base * (decay ** i))) for i in range(passes)]


# ---------------------------------------------------------------------------
# Whole forward: pipeline.py:276-399 + attention_module.py:471-544
# ---------------------------------------------------------------------------


@dataclass
class ForwardConfig:
    num_heads: int
    num_codewords: int
    children_per_codeword: int
    refinement_budget: int
    dtype: str = "f32"
    passes: int = 1
    pass_decay: float = 1.0
    hvaq: bool = False
    hvaq_adaptive: str = "entropy"
    hvaq_beta_init: float = 0.0
    hvaq_alpha: float = 1.0


def split_heads(x: np.ndarray, H: int) -> np.ndarray:
    """``[B,T,E] -> [B*H,T,D]`` (attention_module.py:198-202)."""
    B, T, E = x.shape
    D = E // H
    return x.reshape(B, T, H, D).transpose(0, 2, 1, 3).reshape(B * H, T, D)


def merge_heads(x: np.ndarray, B: int, H: int) -> np.ndarray:
    """``[B*H,T,D] -> [B,T,E]`` (attention_module.py:205-208)."""
    G, T, D = x.shape
    return x.reshape(B, H, T, D).transpose(0, 2, 1, 3).reshape(B, T, H * D)


def forward_heads(qg, kg, vg, parents, children, cfg: ForwardConfig, quant: Quantization | None = None,
                  budget_floor: int | None = None, mask_g: np.ndarray | None = None) -> dict:
    """Run the AVQ forward on head-split tensors ``[G,T,D]`` / ``[G,S,D]``.

    ``parents``/``children`` must already be cast to ``cfg.dtype``
    (attention_module.py:344-348).  ``quant`` reuses a precomputed
    quantization (result-identical to recomputing it).  ``budget_floor``
    replaces the local ``min_valid`` with a global one (head sharding).
    Returns a dict with every intermediate and ``out`` ``[G,T,D]`` fp32.
    """
    dt = cfg.dtype
    H = cfg.num_heads
    G, T, D = qg.shape
    res: dict = {}
    if quant is None:
        quant = quantize(kg, vg, parents, children, dt)
    res["quant"] = quant
    pc = quant.parent_counts
    present = None
    if mask_g is not None:  # pipeline.py:82-106; the child logits ignore the mask
        present = codeword_present(mask_g, quant.parent_assignments, parents.shape[1])
        res["present"] = present
    s = parent_logits(qg, parents, pc, H, dt, present)
    st = online_softmax(s, quant.parent_aggregates, pc, dt)
    res["logits"], res["state0"] = s, st
    w = importance(st.probs, pc, dt)
    res["importance0"] = w
    min_valid = int((pc > 0).sum(-1).min()) if G else 0
    if budget_floor is not None:
        min_valid = budget_floor
    budget = min(cfg.refinement_budget, min_valid)  # pipeline.py:340-343
    res["budget"] = budget
    if budget <= 0:  # pipeline.py:344-345 -> naive attention over zero keys
        res["out"] = np.zeros((G, T, D), np.float32)
        res["naive"] = True
        return res
    sel0 = stable_topk_desc(w, budget)
    res["selected"] = [sel0]
    if cfg.hvaq and cfg.hvaq_adaptive != "none":
        s2, beta = hvaq_logits(s, st.probs, sel0, D, dt, cfg.hvaq_beta_init, cfg.hvaq_adaptive, cfg.hvaq_alpha)
        st = online_softmax(s2, quant.parent_aggregates, pc, dt)
        res["beta"], res["state1"] = beta, st
    l, a = st.l, st.a
    if cfg.passes <= 1:
        u = child_logits_sel(qg, children, sel0, quant.child_counts, H, dt)
        l, a = correction(st.m, l, a, st.probs, quant.parent_aggregates, pc,
                          quant.child_aggregates, quant.child_counts, sel0, u)
    else:
        M0 = cfg.num_codewords
        C = cfg.children_per_codeword
        budgets = compute_pass_budgets(budget, cfg.passes, cfg.pass_decay)
        res["pass_budgets"] = budgets
        refined = np.zeros((G, M0), bool)
        wpost = None
        sels = []
        for pb in budgets:
            if pb <= 0:
                break
            if refined.any():  # multipass.py:213-222
                if wpost is None:
                    wpost = importance(st.probs, pc, dt)
                wm = np.where(refined, np.float32(-np.inf), wpost).astype(np.float32)
                remaining = int((~refined).sum(-1).min())
                cur = min(pb, remaining)
                if cur <= 0:
                    break
                sel = stable_topk_desc(wm, cur)
            else:
                sel = sel0
                cur = sel0.shape[-1]
            if cur == M0:
                # refinement.py:256-260: logits already [.., M0, C] are used
                # without the gather, i.e. slot j carries parent j's logits.
                ident = np.broadcast_to(np.arange(M0), (G, M0))
                u = child_logits_sel(qg, children, ident, quant.child_counts, H, dt)
            else:
                u = child_logits_sel(qg, children, sel, quant.child_counts, H, dt)
            l, a = correction(st.m, l, a, st.probs, quant.parent_aggregates, pc,
                              quant.child_aggregates, quant.child_counts, sel, u)
            np.put_along_axis(refined, sel, True, -1)
            sels.append(sel)
        res["selected"] = sels
        res["importance_post"] = wpost
    with np.errstate(divide="ignore", invalid="ignore"):
        out = (a / np.maximum(l, np.float32(EPS))[..., None]).astype(np.float32)  # attention_module.py:532-535
    res["l_final"], res["a_final"] = l, a
    res["out"] = out
    return res


def forward(q, k, v, parents, children, cfg: ForwardConfig, mask: np.ndarray | None = None, **kw) -> dict:
    """Module-layout forward: ``[B,T,E]`` inputs, ``[B,T,E]`` fp32 output;
    ``mask`` rank 2 ``[T, S]`` or rank 4 ``[B, H, T, S]`` (True = attend)."""
    B = q.shape[0]
    H = cfg.num_heads
    if mask is not None:
        kw["mask_g"] = expand_mask(mask, B, H)
    res = forward_heads(split_heads(q, H), split_heads(k, H), split_heads(v, H), parents, children, cfg, **kw)
    res["out_bte"] = merge_heads(res["out"], B, H)
    return res


def cast_codebook(parents32: np.ndarray, children32: np.ndarray, dt: str):
    """attention_module.py:344-348: the fp32 master codebook cast to the input dtype."""
    return rnd(parents32, dt), rnd(children32, dt)


__all__ = [
    "DTYPES", "EPS", "ForwardConfig", "Quantization", "SoftmaxState", "bcar_update", "cast_codebook",
    "naive_attention", "stream_extend", "stream_init", "StreamState",
    "causal_mask",
    "codeword_present", "expand_mask",
    "child_logits_sel", "compute_pass_budgets", "correction", "count_saturation", "first_argmin",
    "forward", "forward_heads", "hvaq_logits", "importance", "merge_heads", "online_softmax",
    "parent_distances", "parent_logits", "quantize", "rnd", "sequential_bucket_sums",
    "split_heads", "stable_topk_desc",
]
