"""Serialization formats of the caches and the codebook (reference
cache.py:163-198, 305-323 and codebook.py:307-322), on the CPU.

The state dicts have the reference's keys and meaning, so checkpoints move
between the two packages: where the reference source is present, a state dict
written by one package is loaded by the other and gives the same contents.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

from avqa_b200 import HierarchicalCodebook, InMemoryKVCache, PagedKVCache
from avqa_b200.exceptions import CodebookError, ShapeError

REF_SRC = Path(os.environ.get("AVQ_REFERENCE_SRC", "/root/reference/src"))
HAVE_REF = (REF_SRC / "avqa" / "__init__.py").exists()


def _filled_cache(cls_kwargs=None) -> InMemoryKVCache:
    g = torch.Generator().manual_seed(3)
    c = InMemoryKVCache(num_heads=2, head_dim_k=8, head_dim_v=8, **(cls_kwargs or {}))
    for n in (5, 3):
        c.append(torch.randn(1, 2, n, 8, generator=g), torch.randn(1, 2, n, 8, generator=g))
    return c


def test_in_memory_cache_round_trip() -> None:
    c = _filled_cache()
    st = c.state_dict()
    assert set(st) == {"schema_version", "num_heads", "head_dim_k", "head_dim_v", "size", "cache_key", "cache_value"}
    assert int(st["size"]) == 8 and int(st["schema_version"]) == 1
    d = InMemoryKVCache(num_heads=2, head_dim_k=8, head_dim_v=8)
    d.load_state_dict(st)
    for a, b in zip(c.lookup(), d.lookup()):
        assert torch.equal(a, b)
    assert d.size == 8
    # the snapshot is a copy: later appends do not change it
    c.append(torch.zeros(1, 2, 1, 8), torch.zeros(1, 2, 1, 8))
    assert st["cache_key"].shape[-2] == 8
    # an empty snapshot resets
    d.load_state_dict(InMemoryKVCache(num_heads=2, head_dim_k=8, head_dim_v=8).state_dict())
    assert d.size == 0


@pytest.mark.parametrize("field", ["num_heads", "head_dim_k", "head_dim_v"])
def test_in_memory_cache_rejects_mismatch(field: str) -> None:
    st = _filled_cache().state_dict()
    st[field] = torch.tensor(int(st[field]) + 1, dtype=torch.int32)
    with pytest.raises(ShapeError):
        InMemoryKVCache(num_heads=2, head_dim_k=8, head_dim_v=8).load_state_dict(st)


def test_paged_cache_metadata() -> None:
    c = PagedKVCache(page_size=4, num_heads=2, head_dim_k=8, head_dim_v=8)
    c.append(torch.randn(1, 2, 6, 8), torch.randn(1, 2, 6, 8))
    st = c.state_dict()
    assert {k: int(v) for k, v in st.items()} == {"schema_version": 1, "page_size": 4, "num_pages": 2, "size": 6}
    # the page table is metadata only (the data lives on the device): loading resets
    c.load_state_dict(st)
    assert c.size == 0 and c.num_pages == 0
    with pytest.raises(ShapeError):
        PagedKVCache(page_size=8).load_state_dict(st)


def test_codebook_round_trip() -> None:
    cb = HierarchicalCodebook(num_heads=2, num_parents=4, children_per_parent=3, head_dim=8)
    cb.initialize_parents_random(generator=torch.Generator().manual_seed(1))
    st = cb.state_dict()
    assert set(st) == {"parents", "children", "schema_version"}
    other = HierarchicalCodebook(num_heads=2, num_parents=4, children_per_parent=3, head_dim=8)
    other.load_state_dict(st)
    assert torch.equal(other.parents, cb.parents) and torch.equal(other.children, cb.children)
    with pytest.raises(CodebookError):
        other.load_state_dict({"parents": st["parents"]})
    bad = {"parents": st["parents"] + 1.0, "children": st["children"]}  # breaks parent = mean(children)
    with pytest.raises(CodebookError):
        other.load_state_dict(bad)


@pytest.fixture(scope="module")
def ref():
    if not HAVE_REF:
        pytest.skip("reference source not present")
    sys.path.insert(0, str(REF_SRC))
    try:
        import avqa.cache
        import avqa.codebook
        yield avqa
    finally:
        sys.path.remove(str(REF_SRC))


def test_state_dicts_move_between_packages(ref) -> None:
    ours = _filled_cache()
    theirs = ref.cache.InMemoryKVCache(num_heads=2, head_dim_k=8, head_dim_v=8)
    theirs.load_state_dict(ours.state_dict())
    for a, b in zip(ours.lookup(), theirs.lookup()):
        assert torch.equal(a, b)
    back = InMemoryKVCache(num_heads=2, head_dim_k=8, head_dim_v=8)
    back.load_state_dict(theirs.state_dict())
    for a, b in zip(ours.lookup(), back.lookup()):
        assert torch.equal(a, b)
    rcb = ref.codebook.HierarchicalCodebook(num_heads=2, num_parents=4, children_per_parent=3, head_dim=8)
    rcb.initialize_parents_random(generator=torch.Generator().manual_seed(2))
    cb = HierarchicalCodebook(num_heads=2, num_parents=4, children_per_parent=3, head_dim=8)
    cb.load_state_dict(rcb.state_dict())
    assert torch.equal(cb.parents, rcb.parents) and torch.equal(cb.children, rcb.children)
    rcb2 = ref.codebook.HierarchicalCodebook(num_heads=2, num_parents=4, children_per_parent=3, head_dim=8)
    rcb2.load_state_dict(cb.state_dict())
    assert torch.equal(rcb2.children, cb.children)
    pst = PagedKVCache(page_size=4).state_dict()
    ref.cache.PagedKVCache(page_size=4).load_state_dict(pst)
