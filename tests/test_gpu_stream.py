"""StreamingVQBuffer on the GPU (reference streaming_vq.py:34-292).

* every fixture recorded from the reference buffer, replayed call by call:
  returned assignments, record, int64 counts, dtype aggregates and realize()
  bit for bit (NaN positions included);
* seeded larger streams against the oracle: one key per call (the token
  stream), batches with several heads (the reference's head pairing) and a
  batch far larger than the codebook (many keys of one call on one codeword);
* the reference's own unit-test properties: counts add up to the keys seen,
  reset clears, the empty buffer realizes zero tensors, shape errors.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from avqa_b200 import StreamingVQBuffer
from avqa_b200.exceptions import DtypeError, ShapeError
from golden_io import from_bits
from oracle import avq_oracle as O
from test_stream_oracle import load_stream, stream_cases

pytestmark = pytest.mark.gpu

TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def dev(a: np.ndarray, dt: str) -> torch.Tensor:
    return torch.from_numpy(from_bits(a, dt).copy()).to("cuda", TD[dt])


def host(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


@pytest.mark.parametrize("name", stream_cases())
def test_stream_replays_reference(name: str) -> None:
    meta, arrs = load_stream(name)
    dt, H, M0, C, D = meta["dtype"], meta["H"], meta["M0"], meta["C"], meta["D"]
    parents, children = dev(arrs["parents"], dt), dev(arrs["children"], dt)
    buf = StreamingVQBuffer(H, M0, C, D, dtype=TD[dt])
    for i, _ in enumerate(meta["batches"]):
        keys = dev(arrs[f"keys{i}"], dt).reshape(-1, D)
        p, c = buf.extend(keys, parents, children)
        assert p.dtype == torch.int64 and tuple(p.shape) == (keys.shape[0], H)
        np.testing.assert_array_equal(p.cpu().numpy(), arrs[f"passign{i}"], err_msg=f"call {i} parents")
        np.testing.assert_array_equal(c.cpu().numpy(), arrs[f"cassign{i}"], err_msg=f"call {i} children")
    assert len(buf) == meta["size"]
    np.testing.assert_array_equal(buf.parent_counts.cpu().numpy(), arrs["pcnt"])
    np.testing.assert_array_equal(buf.child_counts.cpu().numpy(), arrs["ccnt"])
    np.testing.assert_array_equal(host(buf.parent_aggregates), from_bits(arrs["pagg"], dt))
    np.testing.assert_array_equal(host(buf.child_aggregates), from_bits(arrs["cagg"], dt))
    r = buf.realize()
    np.testing.assert_array_equal(r.parent_assignments.cpu().numpy(), arrs["rec_passign"])
    np.testing.assert_array_equal(r.child_assignments.cpu().numpy(), arrs["rec_cassign"])
    np.testing.assert_array_equal(host(r.parent_counts), from_bits(arrs["real_pcnt"], dt))
    np.testing.assert_array_equal(host(r.child_counts), from_bits(arrs["real_ccnt"], dt))


def _codebook(H, M0, C, D, dt, g):
    parents = torch.randn(H, M0, D, generator=g)
    children = parents[:, :, None] + 0.3 * torch.randn(H, M0, C, D, generator=g)
    return O.rnd(parents.numpy(), dt), O.rnd(children.numpy(), dt)


STREAMS = [
    # dtype, H, M0, C, D, batch sizes, seed
    ("bf16", 8, 256, 8, 128, [1] * 40, 31),          # token stream
    ("f16", 4, 96, 4, 64, [7, 1, 33, 0, 12], 32),     # head pairing, odd batches
    ("f32", 3, 40, 2, 32, [5, 9], 33),
    ("bf16", 2, 8, 4, 64, [700, 300], 34),            # many keys per codeword in one call
    ("bf16", 16, 512, 4, 256, [64], 35),              # several key tiles and parent tiles
    ("bf16", 3, 24, 3, 20, [1, 5, 1], 37),            # D not a multiple of 8: scalar parent loads; odd C
    ("f16", 2, 16, 6, 40, [1, 7, 1], 38),             # C > 4: two batches of child rows
    ("f32", 4, 300, 2, 512, [1, 3], 39),              # the widest head dimension, a partial parent tile
]


@pytest.mark.parametrize("case", STREAMS, ids=lambda c: f"{c[0]}_h{c[1]}_m{c[2]}_d{c[4]}_n{sum(c[5])}")
def test_stream_matches_oracle(case) -> None:
    dt, H, M0, C, D, batches, seed = case
    g = torch.Generator().manual_seed(seed)
    pn, cn = _codebook(H, M0, C, D, dt, g)
    parents, children = (torch.from_numpy(x).to("cuda", TD[dt]) for x in (pn, cn))
    buf = StreamingVQBuffer(H, M0, C, D, dtype=TD[dt])
    st = O.stream_init(H, M0, C, D)
    for i, B in enumerate(batches):
        kn = O.rnd(torch.randn(B, D, generator=g).numpy(), dt)
        p, c = buf.extend(torch.from_numpy(kn).to("cuda", TD[dt]), parents, children)
        po, co = O.stream_extend(st, kn, pn, cn, dt)
        np.testing.assert_array_equal(p.cpu().numpy(), po, err_msg=f"call {i} parents")
        np.testing.assert_array_equal(c.cpu().numpy(), co, err_msg=f"call {i} children")
    np.testing.assert_array_equal(buf.parent_counts[0].cpu().numpy(), st.pcnt)
    np.testing.assert_array_equal(buf.child_counts[0].cpu().numpy(), st.ccnt)
    np.testing.assert_array_equal(host(buf.parent_aggregates[0]), st.pagg)
    np.testing.assert_array_equal(host(buf.child_aggregates[0]), st.cagg)
    np.testing.assert_array_equal(buf.parent_assignments[0].cpu().numpy(), np.concatenate(st.passign, -1))
    np.testing.assert_array_equal(buf.child_assignments[0].cpu().numpy(), np.concatenate(st.cassign, -1))
    # every (key, head) row lands once in the parent and once in the child counts
    assert int(buf.parent_counts.sum()) == int(buf.child_counts.sum()) == sum(batches) * H


def test_strided_keys_equal_contiguous() -> None:
    """Keys as a strided row view of a wider matrix give the same state."""
    g = torch.Generator().manual_seed(36)
    H, M0, C, D = 4, 64, 4, 64
    pn, cn = _codebook(H, M0, C, D, "bf16", g)
    parents, children = (torch.from_numpy(x).to("cuda", torch.bfloat16) for x in (pn, cn))
    wide = torch.randn(10, 3 * D, generator=g).to("cuda", torch.bfloat16)
    a, b = StreamingVQBuffer(H, M0, C, D, dtype=torch.bfloat16), StreamingVQBuffer(H, M0, C, D, dtype=torch.bfloat16)
    pa, ca = a.extend(wide[:, D:2 * D], parents, children)
    pb, cb = b.extend(wide[:, D:2 * D].contiguous(), parents, children)
    assert torch.equal(pa, pb) and torch.equal(ca, cb)
    assert torch.equal(a.child_aggregates, b.child_aggregates) and torch.equal(a.parent_counts, b.parent_counts)


def test_reference_unit_properties() -> None:
    """The reference's unit tests (tests/unit/test_streaming_vq.py) on the GPU buffer."""
    torch.manual_seed(0)
    H, M0, C, D = 1, 4, 2, 8
    parents = torch.randn(H, M0, D, device="cuda")
    children = parents[:, :, None] + 0.1 * torch.randn(H, M0, C, D, device="cuda")
    buf = StreamingVQBuffer(num_heads=H, num_parents=M0, children_per_parent=C, head_dim=D)
    empty = buf.realize()
    assert tuple(empty.parent_assignments.shape) == (1, 1, 0)
    assert tuple(empty.parent_aggregates.shape) == (1, 1, 4, 8) and tuple(empty.parent_counts.shape) == (1, 1, 4)
    assert buf.parent_assignments.numel() == 0
    p, c = buf.extend(torch.randn(8, D, device="cuda"), parents, children)
    assert tuple(p.shape) == (8, 1) and tuple(c.shape) == (8, 1) and len(buf) == 8
    r = buf.realize()
    assert tuple(r.parent_assignments.shape) == (1, 1, 8) and tuple(r.child_aggregates.shape) == (1, 1, 4, 2, 8)
    assert tuple(r.child_counts.shape) == (1, 1, 4, 2) and r.parent_counts.dtype == torch.float32
    for _ in range(2):
        buf.extend(torch.randn(8, D, device="cuda"), parents, children)
    assert int(buf.parent_counts.sum()) == 24 and (buf.parent_aggregates != 0).any()
    buf.reset()
    assert int(buf.parent_counts.sum()) == 0 and len(buf) == 0 and buf.parent_assignments.numel() == 0
    with pytest.raises(ShapeError):
        buf.extend(torch.randn(2, 2, 8, device="cuda"), parents, children)
    with pytest.raises(ShapeError):
        buf.extend(torch.randn(2, 8, device="cuda"), torch.zeros(1, 4, 7, device="cuda"), children)
    with pytest.raises(DtypeError):
        buf.extend(torch.randn(2, 8, device="cuda", dtype=torch.bfloat16), parents, children)
    with pytest.raises(ShapeError):
        StreamingVQBuffer(num_heads=0, num_parents=4, children_per_parent=2, head_dim=8)
