"""Every kernel the library times (AVQ_TIMED labels in avqa_b200/csrc) has an
algorithmic-work entry in bench.py, so that each kernel in a bench line's
kernel table carries an achieved rate and a roofline fraction; and the
prefill and decode work tables keep their bound kinds."""
from __future__ import annotations

import re
from pathlib import Path
from types import SimpleNamespace

ROOT = Path(__file__).resolve().parent.parent


def timed_labels() -> set[str]:
    labels = set()
    for f in (ROOT / "avqa_b200" / "csrc").glob("*.cu"):
        labels |= set(re.findall(r'AVQ_TIMED\("([a-z_0-9]+)"', f.read_text()))
    return labels


def test_every_timed_kernel_has_a_work_entry() -> None:
    text = (ROOT / "bench.py").read_text()
    keys = set(re.findall(r'"([a-z_0-9]+)": \("(?:hbm|tensor)"', text))
    missing = sorted(timed_labels() - keys)
    assert not missing, f"kernels without an algorithmic-work entry in bench.py: {missing}"


def test_work_tables_cover_the_forward() -> None:
    import bench
    w = SimpleNamespace(T=8192, H=32, S=8192, D=128, M0=512, C=4, P=32, dtype="bf16")
    prefill = bench.algorithmic_work(w, 4)
    for k in ("assign_tc", "child", "aggregate", "bucket_sort", "parent_attn_tc", "correct_tc", "route"):
        assert k in prefill, k
    assert prefill["assign_tc"][0] == "tensor" and prefill["child"][0] == "hbm"
    # the parent pass counts only the parent distances: 2 G S M0 D
    assert prefill["assign_tc"][1] == 2.0 * 4 * 32 * 8192 * 512 * 128
    decode = bench.algorithmic_work(w, 4, T=1, decode=True)
    for k in ("decode_value", "decode_route", "decode_logits", "append", "append_assign"):
        assert k in decode, k
    assert decode["decode_value"][0] == "hbm"
