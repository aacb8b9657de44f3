"""The argmin keys of the tcgen05 parent pass (avqa_b200/csrc/avq_assign_tc.cu),
modelled on the CPU with numpy.

A distance pair is a dtype x2 word.  The kernel's key for parent j is
(order16(d_j) << 16) | j as a signed 32-bit integer, and the minimum key is
torch.argmin's choice: the smallest distance, the first index on ties.  (A
distance is one fma, s - 2x; an exact cancellation rounds to +0 in
round-to-nearest, so -0 does not occur.)  order16 flips the magnitude bits
of negative values.  While no distance of a quarter has its sign bit set, the
kernel skips order16 and uses the raw bits.  This test checks that:
- raw and transformed keys then pick the same parent;
- the sign-bit gather flags every quarter where they could differ;
- the transformed keys always reproduce numpy's first-minimum argmin.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import avq_oracle as O


def bits16(x: np.ndarray, dt: str) -> np.ndarray:
    """The dtype bits of float32 values already rounded to the dtype."""
    if dt == "bf16":
        return (x.astype(np.float32).view(np.uint32) >> 16).astype(np.uint32)
    return x.astype(np.float16).view(np.uint16).astype(np.uint32)


def order16(b: np.ndarray) -> np.ndarray:
    neg = (b & 0x8000) != 0
    return np.where(neg, b ^ 0x7FFF, b)


def keys(b: np.ndarray, ordered: bool) -> np.ndarray:
    hi = order16(b) if ordered else b
    k = ((hi << 16) | np.arange(b.shape[-1], dtype=np.uint32)).astype(np.uint32)
    return k.view(np.int32)


def argmin_first(d: np.ndarray) -> np.ndarray:
    """torch.argmin on finite values: the first minimum."""
    return np.argmin(d, axis=-1)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_raw_keys_match_while_no_sign_bit(dt: str) -> None:
    rng = np.random.default_rng(5)
    n = 32  # one quarter
    for case in range(400):
        scale = 10.0 ** rng.integers(-3, 3)
        d = O.rnd(np.abs(rng.standard_normal((64, n))) * scale, dt)
        if case % 4 == 0:  # ties
            d[:, rng.integers(0, n, 8)] = d[:, :1]
        if case % 4 == 1:  # exact zeros, as for a key equal to a parent
            d[:, rng.integers(0, n, 3)] = 0.0
        b = bits16(d, dt)
        assert not (b & 0x8000).any()
        raw = keys(b, ordered=False).min(axis=-1) & 0xFFFF
        ordk = keys(b, ordered=True).min(axis=-1) & 0xFFFF
        np.testing.assert_array_equal(raw, ordk)
        np.testing.assert_array_equal(ordk, argmin_first(d))


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_sign_bits_flag_every_quarter_that_needs_the_transform(dt: str) -> None:
    rng = np.random.default_rng(6)
    n = 32
    for case in range(400):
        d = O.rnd(rng.standard_normal((64, n)) * 0.01, dt)  # near-zero distances, both signs
        if case % 3 == 0:  # exact zeros and ties among the negatives
            d[:, rng.integers(0, n, 4)] = 0.0
            d[:, rng.integers(0, n, 4)] = d[:, :1]
        b = bits16(d, dt)
        flagged = (b & 0x8000).any(axis=-1)
        raw = keys(b, ordered=False).min(axis=-1) & 0xFFFF
        ordk = keys(b, ordered=True).min(axis=-1) & 0xFFFF
        # a row whose raw choice differs is always flagged (the kernel redoes it)
        assert not ((raw != ordk) & ~flagged).any()
        # the transformed keys are torch.argmin's first minimum
        np.testing.assert_array_equal(ordk, argmin_first(d))
