"""CPU model of the routing kernels' top-k selection (avq_select.cuh).

``select_smallest`` picks the k smallest of n unique 64-bit routing keys by a
radix select on the high word (four 8-bit rounds), takes the keys below the
boundary value and the smallest indices among the keys equal to it, and
places them by rank.  This model repeats those steps in numpy and checks them
against a full sort on random, tie-heavy, all-equal and bf16-valued keys.
"""
from __future__ import annotations

import numpy as np
import pytest


def select_model(keys: np.ndarray, k: int) -> np.ndarray:
    hw = keys >> np.uint64(32)
    prefix, pmask, remaining = 0, 0, k
    for shift in (24, 16, 8, 0):
        cand = (hw & np.uint64(pmask)) == np.uint64(prefix)
        digit = ((hw >> np.uint64(shift)) & np.uint64(255)).astype(np.int64)
        hist = np.bincount(digit[cand], minlength=256)
        before = np.cumsum(hist) - hist
        hit = [j for j in range(256) if before[j] < remaining <= before[j] + hist[j]]
        assert len(hit) == 1
        d = hit[0]
        remaining -= int(before[d])
        prefix |= d << shift
        pmask |= 255 << shift
    less = keys[hw < np.uint64(prefix)]
    ties = np.nonzero(hw == np.uint64(prefix))[0]  # ascending index = ascending low word
    chosen = np.concatenate([less, keys[ties[:remaining]]])
    assert len(chosen) == k
    rank = np.array([(chosen < c).sum() for c in chosen])
    out = np.empty(k, np.uint64)
    out[rank] = chosen
    return out


@pytest.mark.parametrize("kind", ["random", "ties", "equal", "bf16", "nan_first"])
def test_select_matches_sort(kind: str) -> None:
    rng = np.random.default_rng(hash(kind) % 2**32)
    for _ in range(300):
        n = int(rng.integers(1, 4097))
        k = int(rng.integers(1, min(n, 256) + 1))
        if kind == "random":
            hw = rng.integers(0, 2**32, n, dtype=np.uint64)
        elif kind == "ties":
            hw = rng.integers(0, 4, n, dtype=np.uint64) << np.uint64(20)
        elif kind == "equal":
            hw = np.full(n, 0xFFFFFFFF, np.uint64)
        elif kind == "bf16":  # ~float_order_key of bf16 importance values: low 16 bits all ones
            hw = (rng.integers(0x3F00, 0x3F80, n, dtype=np.uint64) << np.uint64(16)) | np.uint64(0xFFFF)
        else:  # NaN importance sorts first (high word 0)
            hw = rng.integers(1, 2**32, n, dtype=np.uint64)
            hw[rng.random(n) < 0.1] = 0
        keys = (hw << np.uint64(32)) | np.arange(n, dtype=np.uint64)
        np.testing.assert_array_equal(select_model(keys, k), np.sort(keys)[:k])
