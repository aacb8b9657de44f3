"""The oracle's streaming-VQ restatement against the reference's recorded
``StreamingVQBuffer`` runs (tests/golden/stream, made by
tests/golden/make_stream_golden.py): every returned assignment, the
assignment record, the int64 counts and the dtype aggregates bit for bit
(NaN positions included)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from golden_io import from_bits
from oracle import avq_oracle as O

STREAM = Path(__file__).resolve().parent / "golden" / "stream"


def stream_cases() -> list[str]:
    return sorted(p.stem for p in STREAM.glob("*.npz"))


def load_stream(name: str) -> tuple[dict, dict]:
    z = np.load(STREAM / f"{name}.npz")
    arrs = {k: z[k] for k in z.files}
    return json.loads(arrs.pop("meta_json").tobytes().decode()), arrs


def oracle_run(meta: dict, arrs: dict) -> tuple[O.StreamState, list]:
    dt, H, M0, C, D = meta["dtype"], meta["H"], meta["M0"], meta["C"], meta["D"]
    parents, children = from_bits(arrs["parents"], dt), from_bits(arrs["children"], dt)
    st = O.stream_init(H, M0, C, D)
    outs = []
    for i, _ in enumerate(meta["batches"]):
        keys = from_bits(arrs[f"keys{i}"], dt).reshape(-1, D)
        outs.append(O.stream_extend(st, keys, parents, children, dt))
    return st, outs


def test_cases_present() -> None:
    assert len(stream_cases()) >= 8


@pytest.mark.parametrize("name", stream_cases())
def test_oracle_stream_matches_reference(name: str) -> None:
    meta, arrs = load_stream(name)
    dt = meta["dtype"]
    st, outs = oracle_run(meta, arrs)
    for i, (p, c) in enumerate(outs):
        np.testing.assert_array_equal(p, arrs[f"passign{i}"], err_msg=f"call {i} parents")
        np.testing.assert_array_equal(c, arrs[f"cassign{i}"], err_msg=f"call {i} children")
    np.testing.assert_array_equal(st.pcnt, arrs["pcnt"].reshape(st.pcnt.shape))
    np.testing.assert_array_equal(st.ccnt, arrs["ccnt"].reshape(st.ccnt.shape))
    np.testing.assert_array_equal(st.pagg, from_bits(arrs["pagg"], dt).reshape(st.pagg.shape))
    np.testing.assert_array_equal(st.cagg, from_bits(arrs["cagg"], dt).reshape(st.cagg.shape))
    rec_p = np.concatenate(st.passign, -1)[None]
    rec_c = np.concatenate(st.cassign, -1)[None]
    np.testing.assert_array_equal(rec_p, arrs["rec_passign"])
    np.testing.assert_array_equal(rec_c, arrs["rec_cassign"])
    assert rec_p.shape[-1] == meta["size"]


def test_collide_case_exercises_narrow_once() -> None:
    """The bf16 collision case must differ from per-row rounding, or it does
    not test the fp32-accumulate-once rule."""
    meta, arrs = load_stream("h3_collide_bf16")
    dt, H, M0, C, D = meta["dtype"], meta["H"], meta["M0"], meta["C"], meta["D"]
    parents, children = from_bits(arrs["parents"], dt), from_bits(arrs["children"], dt)
    agg = np.zeros((H, M0, D), np.float32)
    for i, B in enumerate(meta["batches"]):
        keys = from_bits(arrs[f"keys{i}"], dt).reshape(-1, D)
        pa = arrs[f"passign{i}"].reshape(-1)
        for r in range(B * H):  # per-row rounding, the rule the reference does not follow
            h, p = r // B, pa[r]
            agg[h, p] = O.rnd(agg[h, p] + keys[r // H], dt)
    assert not np.array_equal(agg, from_bits(arrs["pagg"], dt).reshape(agg.shape))
