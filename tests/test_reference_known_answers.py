"""Known-answer tests of the reference's own test suite, replayed on the oracle.

Sources (sachncs/avqa): tests/reference/test_hand_computed.py:30-171,
tests/unit/test_spec_fixes.py:93-154, tests/unit/test_routing.py:87-105,184-196,
tests/unit/test_multipass.py:16-46,134-142, tests/unit/test_quantizer.py:117-126.
"""
from __future__ import annotations

import numpy as np

from oracle import avq_oracle as O


def _quant(keys, values, parents, children, dt="f32"):
    k = np.asarray(keys, np.float32)[None]
    v = np.asarray(values, np.float32)[None]
    return O.quantize(k, v, np.asarray(parents, np.float32)[None], np.asarray(children, np.float32)[None], dt)


def test_known_assignment() -> None:
    r = _quant([[0.05, 0.05], [-0.05, -0.05], [10.05, 10.05], [9.95, 9.95]],
               [[1, 2], [3, 4], [5, 6], [7, 8]], [[0, 0], [10, 10]],
               [[[0.1, 0.1], [-0.1, -0.1]], [[10.1, 10.1], [9.9, 9.9]]])
    assert r.parent_assignments.tolist() == [[0, 0, 1, 1]]
    np.testing.assert_allclose(r.parent_aggregates[0], [[4, 6], [12, 14]], atol=1e-5)
    assert r.parent_counts.tolist() == [[2.0, 2.0]]


def test_single_key_exact_match() -> None:
    parents = np.eye(3, 4, dtype=np.float32)
    children = np.stack([np.stack([p * 1.1, p * 0.9]) for p in parents])
    r = _quant([[0, 1, 0, 0]], [[10, 20, 30, 40]], parents, children)
    assert r.parent_assignments.item() == 1
    np.testing.assert_allclose(r.parent_aggregates[0, 1], [10, 20, 30, 40], atol=1e-5)


def test_conservation() -> None:
    r = _quant([[0, 0], [5, 5]], [[1, 2], [3, 4]], [[0, 0], [5, 5]],
               [[[0.1, 0.1], [-0.1, -0.1]], [[5.1, 5.1], [4.9, 4.9]]])
    np.testing.assert_allclose(r.parent_aggregates[0].sum(0), [4, 6], atol=1e-5)


def test_n_a_weighting() -> None:
    parents = [[1, 0, 0, 0], [0, 1, 0, 0]]
    children = [[[1.1, 0, 0, 0], [0.9, 0, 0, 0]], [[0, 1.1, 0, 0], [0, 0.9, 0, 0]]]
    keys = [[1, 0, 0, 0], [1, 0, 0, 0], [1, 0, 0, 0], [0, 1, 0, 0]]
    vals = [[1, 0, 0, 0], [2, 0, 0, 0], [3, 0, 0, 0], [0, 10, 0, 0]]
    r = _quant(keys, vals, parents, children)
    assert r.parent_counts[0].tolist() == [3.0, 1.0]
    np.testing.assert_allclose(r.parent_aggregates[0], [[6, 0, 0, 0], [0, 10, 0, 0]])


def test_router_selection_and_ties() -> None:
    assert O.stable_topk_desc(np.array([[0.4, 0.9, 0.1, 0.7]], np.float32), 2).tolist() == [[1, 3]]
    assert O.stable_topk_desc(np.array([[0.5, 0.5, 0.5]], np.float32), 2).tolist() == [[0, 1]]
    assert O.stable_topk_desc(np.array([[0.1, 0.2, 0.3]], np.float32), 3).tolist() == [[2, 1, 0]]
    assert O.stable_topk_desc(np.array([[0.1, 0.7, 0.3, 0.5]], np.float32), 2).tolist() == [[1, 3]]
    assert O.stable_topk_desc(np.array([[0.5, 0.5, 0.5, 0.5]], np.float32), 2).tolist() == [[0, 1]]
    # torch.sort(descending) puts NaN first
    assert O.stable_topk_desc(np.array([[0.2, np.nan, 0.9]], np.float32), 2).tolist() == [[1, 2]]


def test_pass_budgets() -> None:
    assert O.compute_pass_budgets(8, 4, 0.5) == [8, 4, 2, 1]
    assert O.compute_pass_budgets(8, 4, 1.0) == [8, 8, 8, 8]
    assert O.compute_pass_budgets(8, 5, 0.3) == [8, 2, 1, 1, 1]
    assert O.compute_pass_budgets(1, 4, 0.1) == [1, 1, 1, 1]
    assert O.compute_pass_budgets(48, 3, 0.5) == [48, 24, 12]


def test_entropy_beta_one_hot_doubles() -> None:
    probs = np.array([[[1.0, 0.0, 0.0, 0.0]]], np.float32)
    s = np.zeros_like(probs)
    sel = np.array([[0, 1, 2, 3]])
    _, beta = O.hvaq_logits(s, probs, sel, 64, "f32", 1.0, "entropy")
    assert beta.item() == 2.0
    _, beta = O.hvaq_logits(s, probs, sel, 64, "f32", 1.5, "linear", 0.7)
    assert beta.item() == 1.5


def test_importance_formula() -> None:
    probs = np.full((1, 8, 4), 0.25, np.float32)
    n = np.array([[1.0, 2.0, 3.0, 4.0]], np.float32)
    np.testing.assert_allclose(O.importance(probs, n, "f32"), 2.0 * n)


def test_bf16_scalar_rounding_goes_through_fp32() -> None:
    # torch: 0.7 * bf16(1.7578125) -> fp32 tie 1.23046875 -> bf16 1.234375
    assert O.rnd(np.float64(np.float32(0.7)) * 1.7578125, "bf16").item() == 1.234375


def test_count_saturation() -> None:
    assert O.count_saturation("bf16") == 256 and O.count_saturation("f16") == 2048
    k = np.zeros((1, 5000, 2), np.float32)
    r = O.quantize(k, k, np.zeros((1, 1, 2), np.float32), np.zeros((1, 1, 1, 2), np.float32), "bf16")
    assert r.parent_counts.item() == 256.0 and r.parent_counts_exact.item() == 5000
