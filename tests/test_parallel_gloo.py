"""Head sharding over two gloo ranks on the CPU.

The sharding logic (head ranges, codebook slices, the all-reduce(MIN) of the
budget floor and the output all-gather) runs with the oracle as the per-rank
compute; the result must equal one unsharded oracle forward over all heads.
The data make one head's valid-parent count the global minimum, so a rank
that used its local minimum would route differently.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from avqa_b200.config import AttentionShapeConfig, AVQConfig, CodebookConfig, RoutingConfig
from avqa_b200.parallel import ShardedAVQAttention, head_range
from oracle import avq_oracle as O

H, D, M0, C, P, B, T, S = 4, 16, 12, 2, 8, 2, 10, 40


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(B, n, H * D, generator=g) for n in (T, S, S))
    parents = torch.randn(H, M0, D, generator=g)
    children = parents[:, :, None] + 0.1 * torch.randn(H, M0, C, D, generator=g)
    parents = children.mean(2)
    # head 3: all keys sit on two parents -> min valid over (b,h) is 2 < P
    kk = k.view(B, S, H, D)
    kk[:, :, 3] = parents[3, torch.arange(S) % 2] + 1e-3 * torch.randn(B, S, D, generator=g)
    return q, k, v, parents, children


class OracleShard:
    """Per-rank compute backed by the oracle (head-split numpy)."""

    def __init__(self, parents, children):
        self.p = parents.numpy()
        self.c = children.numpy()

    def quantize(self, k, v):
        Bq, h, Sq, Dq = k.shape
        kg = k.reshape(Bq * h, Sq, Dq).numpy()
        vg = v.reshape(Bq * h, Sq, Dq).numpy()
        st = O.quantize(kg, vg, self.p, self.c, "f32")
        mv = int((st.parent_counts > 0).sum(-1).min())
        return (st, h), torch.tensor([mv], dtype=torch.int32)

    def forward(self, q, state, min_valid, chunk_size=0, ready=None):
        st, h = state
        Bq, _, Tq, Dq = q.shape
        cfg = O.ForwardConfig(h, M0, C, P, "f32")
        step = chunk_size if chunk_size > 0 else Tq
        outs = []
        for t0 in range(0, Tq, step):  # each chunk a separate call over the same quantized keys
            qc = q[:, :, t0:t0 + step]
            res = O.forward_heads(qc.reshape(Bq * h, qc.shape[2], Dq).numpy(), None, None, self.p, self.c, cfg,
                                  quant=st, budget_floor=int(min_valid.item()))
            outs.append(torch.from_numpy(res["out"]).view(Bq, h, qc.shape[2], Dq))
        return torch.cat(outs, dim=2)


def _worker(rank: int, world: int, port: int, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, parents, children = _data()
        cfg = AVQConfig(attention=AttentionShapeConfig(embed_dim=H * D, num_heads=H),
                        codebook=CodebookConfig(num_codewords=M0, children_per_codeword=C),
                        routing=RoutingConfig(refinement_budget=P))
        mod = ShardedAVQAttention(cfg, parents, children, compute_factory=OracleShard)
        out = mod(q, k, v)
        out_c = mod(q, k, v, chunk_size=4)  # chunks of 4, 4 and 2 queries
        out_q.put((rank, (out.numpy(), out_c.numpy())))
    finally:
        dist.destroy_process_group()


def test_head_range_partitions() -> None:
    for Hh in (1, 4, 7, 64):
        for world in (1, 2, 3, 8):
            rngs = [head_range(Hh, world, r) for r in range(world)]
            assert rngs[0][0] == 0 and rngs[-1][1] == Hh
            assert all(a[1] == b[0] for a, b in zip(rngs, rngs[1:]))


@pytest.mark.timeout(120)
def test_two_gloo_ranks_match_unsharded_oracle() -> None:
    q, k, v, parents, children = _data()
    full = O.forward(q.numpy(), k.numpy(), v.numpy(), parents.numpy(), children.numpy(),
                     O.ForwardConfig(H, M0, C, P, "f32"))
    assert full["budget"] == 2  # the global floor comes from head 3 only
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict(out_q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    chunked = [O.forward(q[:, t0:t0 + 4].numpy(), k.numpy(), v.numpy(), parents.numpy(), children.numpy(),
                         O.ForwardConfig(H, M0, C, P, "f32"))["out_bte"] for t0 in range(0, T, 4)]
    chunked = np.concatenate(chunked, axis=1)
    for r in range(2):
        np.testing.assert_allclose(outs[r][0], full["out_bte"], rtol=0, atol=1e-6)
        np.testing.assert_allclose(outs[r][1], chunked, rtol=0, atol=1e-6)
