"""``AVQAttention``: the AVQ-attention nn.Module on B200 kernels.

Constructor, attribute names and forward signature follow the reference
(``src/avqa/attention_module.py:70-316``); parameters are created in the same
order, so under the same RNG seed the projections and the default codebook
equal the reference's.  The forward pass runs the reference pipeline
(``pipeline.py:276-399``) with every stage from VQ precompute to the final
reduction executed by the CUDA library:

    validate -> project -> split heads -> codebook cast -> KV cache ->
    quantize (or incremental append) -> parent attention -> routing ->
    [HVAQ] -> child correction (1..passes) -> merge heads -> out_proj

The output is fp32 for every input dtype, as in the reference (its online
softmax state is fp32, ``attention.py:37-68``).  User and causal masks
follow ``pipeline.py:82-106`` and ``attention_module.py:369-390``: a parent
is masked for a query when none of its keys is visible.  Features the
reference offers but no benchmark configuration uses -- BCAR codebook
adaptation, the threshold router, the adaptive budget scheduler, learnable
HVAQ parameters and the dense "reference" execution mode -- raise
:class:`BackendError` instead of silently running elsewhere.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from avqa_b200 import ops
from avqa_b200.backend import Backend, CUDABackend
from avqa_b200.cache import KVCache, PagedKVCache
from avqa_b200.codebook import HierarchicalCodebook
from avqa_b200.config import AVQConfig
from avqa_b200.exceptions import BackendError, DeviceError, DtypeError, RoutingError, ShapeError

SUPPORTED_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


class AVQAttention(nn.Module):
    """AVQ attention (hierarchical VQ keys, parent attention, routed child correction)."""

    def __init__(self, config: AVQConfig, *, in_proj: bool = True, out_proj: bool = True) -> None:
        super().__init__()
        self.config = config
        self.backend = Backend.create(config.backend.name)
        E = config.attention.embed_dim
        if in_proj:
            self.q_proj = nn.Linear(E, E, bias=False)
            self.k_proj = nn.Linear(E, E, bias=False)
            self.v_proj = nn.Linear(E, E, bias=False)
        else:
            self.q_proj = nn.Identity()
            self.k_proj = nn.Identity()
            self.v_proj = nn.Identity()
        self.out_proj = nn.Linear(E, E, bias=False) if out_proj else nn.Identity()
        self.codebook = HierarchicalCodebook(
            num_heads=config.attention.num_heads, num_parents=config.codebook.num_codewords,
            children_per_parent=config.codebook.children_per_codeword, head_dim=E // config.attention.num_heads,
            perturbation_scale=config.codebook.perturbation_scale, device="cpu", dtype=torch.float32)
        self.codebook.initialize_children_around_parents()
        self.dropout = nn.Dropout(config.dropout) if config.dropout > 0 else nn.Identity()
        self.last_keys: torch.Tensor | None = None
        self.last_parent_assignments: torch.Tensor | None = None
        self.process_group = None  # set by avqa_b200.parallel for head sharding
        self._check_supported()

    # -- configuration -----------------------------------------------------------

    def _check_supported(self) -> None:
        c = self.config
        unsupported = []
        if c.routing.strategy == "threshold":
            unsupported.append("routing.strategy='threshold'")
        if c.refinement.adaptive_budget:
            unsupported.append("refinement.adaptive_budget")
        if c.hopfield.learnable_parent_beta or c.hopfield.learnable_alpha:
            unsupported.append("hopfield.learnable_*")
        if c.execution.compile_enabled:
            unsupported.append("execution.compile_enabled")
        if unsupported:
            raise BackendError("not supported by the cuda backend: " + ", ".join(unsupported))
        if c.refinement.passes <= 0:
            raise RoutingError(f"passes must be positive, got {c.refinement.passes}")
        if c.refinement.passes > 1 and not 0.0 < c.refinement.pass_decay <= 1.0:
            raise RoutingError(f"decay must be in (0, 1], got {c.refinement.pass_decay}")
        if c.refinement.passes > 8:
            raise BackendError("at most 8 refinement passes are supported", {"passes": c.refinement.passes})

    # -- helpers -----------------------------------------------------------------

    @staticmethod
    def split_heads(tensor: torch.Tensor, num_heads: int) -> torch.Tensor:
        """``[B, T, E]`` -> ``[B, H, T, D]`` (a view)."""
        B, T, E = tensor.shape
        return tensor.view(B, T, num_heads, E // num_heads).transpose(1, 2)

    @staticmethod
    def merge_heads(tensor: torch.Tensor) -> torch.Tensor:
        B, H, T, D = tensor.shape
        return tensor.transpose(1, 2).contiguous().view(B, T, H * D)

    def maybe_project(self, query, key, value):
        return self.q_proj(query), self.k_proj(key), self.v_proj(value)

    def validate_inputs(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> None:
        """Same checks as the reference (attention_module.py:321-342)."""
        if self.config.backend.skip_validation:
            return
        E = self.config.attention.embed_dim
        for name, t in (("query", query), ("key", key), ("value", value)):
            if t.ndim != 3:
                raise ShapeError(f"{name} must have rank 3", expected=3, actual=t.ndim)
            if t.dtype not in SUPPORTED_DTYPES:
                raise DtypeError(f"{name} has unsupported dtype", expected=[str(d) for d in SUPPORTED_DTYPES],
                                 actual=str(t.dtype))
            if t.shape[-1] != E:
                raise ShapeError(f"{name} embed dim mismatch", expected=E, actual=t.shape[-1])
        devs = {t.device for t in (query, key, value)}
        if len(devs) > 1:
            raise DeviceError("query/key/value are on different devices", actual=[str(d) for d in devs])
        if key.shape != value.shape:
            raise ShapeError("value shape mismatch", expected=tuple(key.shape), actual=tuple(value.shape))

    def sync_codebook_device(self, q: torch.Tensor) -> None:
        """Cast the codebook to the input's device and dtype (attention_module.py:344-348)."""
        if self.codebook.parents.device != q.device or self.codebook.parents.dtype != q.dtype:
            self.codebook.parents = self.codebook.parents.to(device=q.device, dtype=q.dtype)
            self.codebook.children = self.codebook.children.to(device=q.device, dtype=q.dtype)

    # -- forward -----------------------------------------------------------------

    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, mask: torch.Tensor | None = None,
                kv_cache: KVCache | None = None) -> torch.Tensor:
        c = self.config
        if c.precision.autocast:
            with torch.autocast(device_type=query.device.type, dtype=getattr(torch, c.precision.dtype)):
                return self.forward_impl(query, key, value, mask, kv_cache)
        return self.forward_impl(query, key, value, mask, kv_cache)

    def forward_impl(self, query, key, value, mask=None, kv_cache=None) -> torch.Tensor:
        return cuda_run_pipeline(self, query, key, value, mask, kv_cache)

    def forward_chunked(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                        chunk_size: int) -> torch.Tensor:
        """``forward`` of ``query`` in sequential chunks of ``chunk_size``
        queries over the same ``key``/``value``.

        The result equals one ``forward(query[:, chunk], key, value)`` call per
        chunk, concatenated: each chunk gets its own routing (importance summed
        over its own queries), and every chunk sees the same budget because the
        keys are the same.  The reference re-quantizes the keys on every such
        call (``attention_module.py:392-440``); quantization is deterministic,
        so here it runs once and every chunk attends to the cached state.  With
        batch 1 all chunks run in one launch sequence.
        """
        if chunk_size <= 0:
            raise ShapeError("chunk_size must be positive", expected="> 0", actual=chunk_size)
        return cuda_run_pipeline(self, query, key, value, None, None, chunk_size=chunk_size)


def hvaq_mode(config: AVQConfig) -> int:
    """0 off, 1 entropy, 2 linear (the gate of pipeline.py:353)."""
    if not (config.backend.hopfield and config.hopfield.adaptive != "none"):
        return 0
    return {"entropy": 1, "linear": 2}[config.hopfield.adaptive]


def cuda_run_pipeline(m, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                      mask: torch.Tensor | None = None, kv_cache=None, chunk_size: int = 0) -> torch.Tensor:
    """The reference pipeline (pipeline.py:276-399) on the CUDA library.

    ``m`` is any module with the reference ``AVQAttention`` attributes
    (``config``, ``codebook``, ``q_proj``/``k_proj``/``v_proj``/``out_proj``,
    ``dropout``, ``validate_inputs``, ``sync_codebook_device``) whose
    ``backend`` is a :class:`CUDABackend` -- this package's module or the
    reference's own one, once its ``run_pipeline`` is routed here.
    """
    c = m.config
    if mask is not None and chunk_size > 0:
        raise BackendError("a user mask with query chunks is not supported; pass each chunk's mask to forward")
    m.validate_inputs(query, key, value)
    if not query.is_cuda:
        raise DeviceError("the cuda backend needs CUDA tensors", expected="cuda", actual=str(query.device))
    qp, kp, vp = m.q_proj(query), m.k_proj(key), m.v_proj(value)
    H = c.attention.num_heads
    q = AVQAttention.split_heads(qp, H)
    k = AVQAttention.split_heads(kp, H)
    v = AVQAttention.split_heads(vp, H)
    m.sync_codebook_device(q)
    backend: CUDABackend = m.backend  # type: ignore[assignment]
    if not c.refinement.enabled or c.execution.mode == "reference":
        # pipeline.py:310-312: no scheduler, or the reference mode: dense
        # attention over the (cached) keys with the resolved mask
        return dense_path(m, q, k, v, mask, kv_cache, chunk_size)
    cb = backend.prepared_codebook(m.codebook.parents, m.codebook.children, q.dtype, q.device)
    state = resolve_quantization(m, k, v, cb, kv_cache)
    if c.codebook.bcar_enabled and state.S > 0:
        # run_vq_precompute (attention_module.py:420-428): the codebook adapts
        # to this call's keys after their quantization; the attention below
        # uses the adapted codebook over the unadapted quantization
        if state.passign is None:
            raise BackendError("BCAR over a KV cache after a decode step is not supported by the cuda backend: "
                               "its decode state keeps no per-key assignments")
        kf = k if kv_cache is None else _full_keys(kv_cache, k)
        ops.bcar_update(kf, state, m.codebook.parents, m.codebook.children, c.codebook.bcar_decay)
        cb = backend.prepared_codebook(m.codebook.parents, m.codebook.children, q.dtype, q.device)
    B, _, T, D = q.shape
    if state.S == 0:
        # pipeline.py:344-345: budget 0 -> naive attention over zero keys
        attn = backend.naive_attention(q, k, v)
        return m.dropout(m.out_proj(AVQAttention.merge_heads(attn)))
    min_valid, ready = global_min_valid(state, getattr(m, "process_group", None))
    out = torch.empty(B, T, H * D, dtype=torch.float32, device=q.device)
    beta0 = c.hopfield.beta_init if c.hopfield.beta_init > 0 else 1.0 / math.sqrt(D)
    args = (min(c.routing.refinement_budget, cb.dims[1]), c.refinement.passes, c.refinement.pass_decay, hvaq_mode(c),
            beta0, c.hopfield.alpha)
    for q_part, out_part in query_chunks(q, out, H, chunk_size):
        Bq, _, Tq, _ = q_part.shape
        present = codeword_mask(c, state, Tq, mask, Bq if Bq != state.B else None)
        backend.forward(q_part, cb, state, *args, out=out_part, min_valid=min_valid, min_valid_ready=ready,
                        present=present)
        ready = None  # later chunks are ordered after the first one's wait
    return m.dropout(m.out_proj(out))


def dense_path(m, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None, kv_cache,
               chunk_size: int = 0) -> torch.Tensor:
    """naive_fallback (pipeline.py:261-273) after resolve_kv_cache and
    resolve_mask (attention_module.py:350-390): dense attention, merge heads,
    output projection, dropout; the output keeps the input dtype.  Query
    chunks are separate calls (each with its own causal offset)."""
    if kv_cache is not None:
        ck, cv = kv_cache.lookup()
        new_k, new_v = k, v
        if ck.shape[-2] > 0:
            k = torch.cat([ck.to(device=k.device, dtype=k.dtype), k], dim=-2)
            v = torch.cat([cv.to(device=v.device, dtype=v.dtype), v], dim=-2)
        kv_cache.append(new_k, new_v)
        _cache_states(kv_cache).clear()  # quantized states no longer cover the cache
    B, H, T, D = q.shape
    S = k.shape[-2]
    out = torch.empty(B, H, T, D, dtype=q.dtype, device=q.device)
    step = chunk_size if chunk_size > 0 else max(T, 1)
    for t0 in range(0, T, step):
        qc = q[:, :, t0:t0 + step]
        Tq = qc.shape[2]
        mk = mask
        if mk is None and m.config.causal:
            mk = torch.arange(S, device=q.device)[None, :] <= torch.arange(Tq, device=q.device)[:, None] + (S - Tq)
        out[:, :, t0:t0 + Tq] = m.backend.naive_attention(qc, k, v, mk)
    return m.dropout(m.out_proj(AVQAttention.merge_heads(out)))


def codeword_mask(config: AVQConfig, state: ops.QuantState, T: int, mask: torch.Tensor | None,
                  query_batch: int | None = None) -> torch.Tensor | None:
    """The codeword visibility bits of one call (pipeline.py:82-106), or None.

    A user mask is used as given; otherwise, with ``config.causal``, the
    causal mask of ``resolve_mask`` (attention_module.py:369-390): query t
    sees keys ``0 .. t + S - T``, so a single query (decode) sees every key
    and needs no mask."""
    if mask is None and not config.causal:
        return None
    if mask is None and T == 1:
        return None
    if state.passign is None:
        raise BackendError("a mask over a KV cache with more than one new query is not supported by the cuda "
                           "backend: its decode state keeps no per-key assignments")
    return ops.codeword_presence(state, T, mask, None, query_batch)


def query_chunks(q: torch.Tensor, out: torch.Tensor, H: int, chunk: int):
    """``(queries [b, H, t, D], output [b, H, t, D] view)`` pairs covering
    ``q [B, H, T, D]`` in chunks of ``chunk`` queries (all of T when 0).

    With batch 1 the whole chunks form one query batch (chunk c = batch entry
    c, a strided view) that attends to the batch-1 key state in one call; the
    ragged tail and batches > 1 go chunk by chunk."""
    B, _, T, D = q.shape
    out4 = out.view(B, T, H, D)
    if chunk <= 0 or chunk >= T:
        yield q, out4.transpose(1, 2)
        return
    full = T // chunk
    if B == 1 and full > 1:
        qs = q.as_strided((full, H, chunk, D), (q.stride(2) * chunk, q.stride(1), q.stride(2), q.stride(3)))
        os_ = out4.as_strided((full, H, chunk, D), (out4.stride(1) * chunk, out4.stride(2), out4.stride(1), 1))
        yield qs, os_
        start = full * chunk
    else:
        start = 0
    for t0 in range(start, T, chunk):
        t1 = min(t0 + chunk, T)
        yield q[:, :, t0:t1], out4[:, t0:t1].transpose(1, 2)


_SIDE_STREAMS: dict = {}


def global_min_valid(state: ops.QuantState, group=None) -> tuple[torch.Tensor, torch.cuda.Event | None]:
    """The budget floor: min over every (b,h) of the call -- and of every
    rank of ``group`` when batches or heads are sharded.

    With a group the all-reduce(MIN) runs on a side stream after the
    quantization; the returned event marks its completion, and the forward
    waits on it only before routing, so parent attention overlaps it."""
    if group is None:
        return state.gmin, None
    import torch.distributed as dist
    dev = state.gmin.device
    main = torch.cuda.current_stream(dev)
    side = _SIDE_STREAMS.get(dev)
    if side is None:
        side = _SIDE_STREAMS[dev] = torch.cuda.Stream(dev)
    g = state.gmin.clone()
    side.wait_stream(main)
    with torch.cuda.stream(side):
        dist.all_reduce(g, op=dist.ReduceOp.MIN, group=group)
        ready = torch.cuda.Event()
        ready.record(side)
    g.record_stream(side)
    return g, ready


def _full_keys(kv_cache, k: torch.Tensor) -> torch.Tensor:
    """The cached keys followed by none: after the first call with a cache,
    the cache holds every key the state quantized (resolve_kv_cache)."""
    ck, _ = kv_cache.lookup()
    return ck.to(device=k.device, dtype=k.dtype)


def _cache_states(kv_cache) -> dict:
    states = getattr(kv_cache, "quant_states", None)
    if states is None:  # a reference KVCache: attach the device state to it
        states = {}
        kv_cache.quant_states = states
    return states


def resolve_quantization(m, k: torch.Tensor, v: torch.Tensor, cb: ops.PreparedCodebook,
                         kv_cache=None) -> ops.QuantState:
    """Quantize ``k``/``v`` -- or, with a cache, extend the cache's device state
    (resolve_kv_cache, attention_module.py:350-367, then the quantizer)."""
    if kv_cache is None:
        st = ops.quantize(k, v, cb)
        m.last_keys = k.detach()
        m.last_parent_assignments = st.passign.view(k.shape[:3]).long()
        return st
    states = _cache_states(kv_cache)
    skey = (id(m), id(cb), k.dtype)
    st = states.get(skey)
    if st is not None and (st.B != k.shape[0] or st.H != k.shape[1]):
        st = None
    if st is None:
        ck, cv = kv_cache.lookup()
        if ck.shape[-2] > 0:
            ck = ck.to(device=k.device, dtype=k.dtype)
            cv = cv.to(device=v.device, dtype=v.dtype)
            kf, vf = torch.cat([ck, k], dim=-2), torch.cat([cv, v], dim=-2)
        else:
            kf, vf = k, v
        st = ops.quantize(kf, vf, cb, keep_sums=True)
        kv_cache.append(k, v)
        states.clear()
        states[skey] = st
        return st
    if isinstance(kv_cache, PagedKVCache) and str(kv_cache.device) == str(k.device) and kv_cache.dtype == k.dtype:
        cursor = 0
        for page, slot0, take in kv_cache.reserve(k.shape[0], k.shape[2]):
            ops.append(st, k[:, :, cursor:cursor + take], v[:, :, cursor:cursor + take], cb,
                       kv_cache.key_pages[page], kv_cache.value_pages[page], slot0)
            cursor += take
    else:
        ops.append(st, k, v, cb)
        kv_cache.append(k, v)
    return st


__all__ = ["AVQAttention", "codeword_mask", "cuda_run_pipeline", "global_min_valid", "hvaq_mode", "query_chunks",
           "resolve_quantization"]
