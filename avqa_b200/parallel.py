"""Head-sharded AVQ attention across the ranks of a process group.

Every (b,h) of the AVQ forward is independent except for the routing budget,
``min(P, min over all (b,h) of non-empty parents)`` (reference
``pipeline.py:340-343``).  A head shard therefore needs exactly one
collective per forward -- an all-reduce(MIN) of one int32 -- plus the
all-gather of the fp32 output head-slices.  Rank r owns the contiguous heads
``head_range(H, world, r)`` and the matching codebook slice.

The per-rank compute is pluggable (``ShardCompute``): ``CudaShardCompute``
runs the CUDA library; tests plug in a CPU implementation to exercise the
sharding logic on gloo ranks.
"""
from __future__ import annotations

from typing import Protocol

import torch
import torch.distributed as dist

from avqa_b200.config import AVQConfig
from avqa_b200.exceptions import ConfigurationError


def head_range(num_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous head slice [h0, h1) of ``rank``; the first ``H % world`` ranks get one more."""
    if world <= 0 or not 0 <= rank < world:
        raise ConfigurationError("bad rank/world", {"rank": rank, "world": world})
    base, extra = divmod(num_heads, world)
    h0 = rank * base + min(rank, extra)
    return h0, h0 + base + (1 if rank < extra else 0)


class ShardCompute(Protocol):
    def quantize(self, k: torch.Tensor, v: torch.Tensor):
        """Quantize ``[B,h,S,D]`` keys/values; returns (state, local min-valid int32 tensor [1])."""

    def forward(self, q: torch.Tensor, state, min_valid: torch.Tensor, chunk_size: int = 0,
                ready: torch.cuda.Event | None = None) -> torch.Tensor:
        """AVQ forward of ``[B,h,T,D]`` queries (in chunks of ``chunk_size``
        queries when > 0, each routed on its own); returns ``[B,h,T,D]`` fp32.
        ``ready``: event after which ``min_valid`` holds the global floor."""


class CudaShardCompute:
    """The CUDA library on this rank's device."""

    def __init__(self, config: AVQConfig, parents: torch.Tensor, children: torch.Tensor, dtype: torch.dtype,
                 device: torch.device):
        from avqa_b200 import ops
        self.ops = ops
        self.config = config
        self.cb = ops.prepare_codebook(parents, children, dtype, device)

    def quantize(self, k, v, kv_cache=None):
        """Quantize the keys -- or, with a KV cache of this rank's heads,
        extend the cache's quantized state by the new tokens (decode)."""
        if kv_cache is None:
            st = self.ops.quantize(k, v, self.cb)
        else:
            from avqa_b200.attention_module import resolve_quantization
            st = resolve_quantization(self, k, v, self.cb, kv_cache)
        return st, st.gmin

    def forward(self, q, state, min_valid, chunk_size=0, ready=None):
        import math
        from avqa_b200.attention_module import hvaq_mode, query_chunks
        c = self.config
        B, h, T, D = q.shape
        hv = hvaq_mode(c)
        beta0 = c.hopfield.beta_init if c.hopfield.beta_init > 0 else 1.0 / math.sqrt(D)
        out = torch.empty(B, T, h * D, dtype=torch.float32, device=q.device)
        args = (min(c.routing.refinement_budget, self.cb.dims[1]), c.refinement.passes, c.refinement.pass_decay, hv,
                beta0, c.hopfield.alpha)
        for q_part, o_part in query_chunks(q, out, h, chunk_size):
            self.ops.forward(q_part, self.cb, state, *args, out=o_part, min_valid=min_valid, min_valid_ready=ready)
            ready = None
        return out.view(B, T, h, D).transpose(1, 2)


_SIDE: dict = {}


def reduce_min(mv: torch.Tensor, group=None) -> tuple[torch.Tensor, torch.cuda.Event | None]:
    """All-reduce(MIN) of the budget floor over ``group``.  For a CUDA tensor
    it runs on a side stream and returns an event marking its completion (the
    forward waits on it only before routing); on the CPU it is synchronous."""
    g = mv.clone()
    if not g.is_cuda:
        dist.all_reduce(g, op=dist.ReduceOp.MIN, group=group)
        return g, None
    main = torch.cuda.current_stream(g.device)
    side = _SIDE.get(g.device)
    if side is None:
        side = _SIDE[g.device] = torch.cuda.Stream(g.device)
    side.wait_stream(main)
    with torch.cuda.stream(side):
        dist.all_reduce(g, op=dist.ReduceOp.MIN, group=group)
        ready = torch.cuda.Event()
        ready.record(side)
    g.record_stream(side)
    return g, ready


class ShardedAVQAttention:
    """AVQ attention over the heads of a process group (no projections).

    ``forward(query, key, value, chunk_size=0)`` takes the full ``[B, T, E]``
    tensors on every rank and returns the full ``[B, T, E]`` fp32 output on
    every rank.  Rank r quantizes the keys of its heads once, attends to them
    (chunk by chunk when ``chunk_size`` > 0) and the output head-slices meet
    in one all-gather.
    """

    def __init__(self, config: AVQConfig, parents32: torch.Tensor, children32: torch.Tensor,
                 group=None, compute_factory=None, device: torch.device | None = None,
                 dtype: torch.dtype = torch.bfloat16):
        self.config = config
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        H = config.attention.num_heads
        self.h0, self.h1 = head_range(H, self.world, self.rank)
        self.D = config.attention.embed_dim // H
        p_loc = parents32[self.h0:self.h1]
        c_loc = children32[self.h0:self.h1]
        if compute_factory is None:
            self.compute = CudaShardCompute(config, p_loc, c_loc, dtype, device or torch.device("cuda"))
        else:
            self.compute = compute_factory(p_loc, c_loc)

    def _local(self, x: torch.Tensor) -> torch.Tensor:
        B, T, _ = x.shape
        return x[:, :, self.h0 * self.D:self.h1 * self.D].reshape(B, T, self.h1 - self.h0, self.D).transpose(1, 2)

    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                chunk_size: int = 0, kv_cache=None) -> torch.Tensor:
        """``kv_cache``: a cache of this rank's heads (``num_heads`` = its
        head count); the new tokens are appended and attention covers the
        cached ones too, as in ``AVQAttention.forward``."""
        if kv_cache is None:
            st, mv = self.compute.quantize(self._local(key), self._local(value))
        else:
            st, mv = self.compute.quantize(self._local(key), self._local(value), kv_cache)
        ready = None
        if self.world > 1:
            mv, ready = reduce_min(mv, self.group)
        out = self.compute.forward(self._local(query), st, mv, chunk_size, ready)  # [B, h, T, D]
        B, h, T, D = out.shape
        local = out.transpose(1, 2).reshape(B, T, h * D).contiguous()
        if self.world == 1:
            return local
        H = self.config.attention.num_heads
        sizes = [head_range(H, self.world, r) for r in range(self.world)]
        hmax = max(b - a for a, b in sizes)
        if all(b - a == hmax for a, b in sizes):
            parts = [torch.empty_like(local) for _ in sizes]
            dist.all_gather(parts, local, group=self.group)
            return torch.cat(parts, dim=-1)
        padded = torch.zeros(B, T, hmax * D, dtype=local.dtype, device=local.device)
        padded[:, :, :h * D] = local
        parts = [torch.empty_like(padded) for _ in sizes]
        dist.all_gather(parts, padded, group=self.group)
        return torch.cat([p[:, :, :(b - a) * D] for p, (a, b) in zip(parts, sizes)], dim=-1)

    __call__ = forward


__all__ = ["CudaShardCompute", "ShardCompute", "ShardedAVQAttention", "head_range", "reduce_min"]
