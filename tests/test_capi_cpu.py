"""The C-ABI library loads and exports every declared symbol; host-side
argument checks work without a GPU (no kernel is launched)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from avqa_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "avqa_b200.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(avq_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_binding() -> None:
    assert set(declared()) == set(_lib.exported_symbols())


def test_library_exports_every_declared_symbol() -> None:
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.avq_version().startswith(b"avqa_b200")


def test_selection_stride_matches_pass_caps() -> None:
    from avqa_b200.ops import pass_caps
    lib = _lib.load()
    assert lib.avq_selection_stride(48, 3, 0.5) == 48 + 24 + 12 == sum(pass_caps(48, 3, 0.5))
    assert lib.avq_selection_stride(8, 1, 1.0) == 8
    assert lib.avq_selection_stride(5, 3, 0.3) == sum(pass_caps(5, 3, 0.3))


@pytest.mark.parametrize("call", ["bad_dtype", "bad_budget", "null", "state_batch"])
def test_forward_rejects_bad_arguments(call: str) -> None:
    lib = _lib.load()
    s = (ctypes.c_longlong * 3)(1, 1, 1)
    args = dict(dtype=1, P=4, M0=8, q=None)
    if call == "bad_dtype":
        args["dtype"] = 7
    if call == "bad_budget":
        args["P"] = 9
    sb = 3 if call == "state_batch" else 1
    rc = lib.avq_forward(args["dtype"], args["q"], s, 1, 1, 1, 8, args["M0"], 2, None, None, None, None, None, None,
                         sb, None, None, None, args["P"], 1, 1.0, 0, 0.0, 1.0, None, s, None, None, None, None, 0, None)
    assert rc == 1
    msg = _lib.last_error()
    assert msg.startswith("avq_forward")
    if call == "bad_budget":
        assert "exceeds number of parents" in msg
    if call == "state_batch":
        assert "state_batch" in msg


def test_group_count_overflow_is_rejected() -> None:
    """B*H beyond INT_MAX is refused before any size is derived from it."""
    lib = _lib.load()
    s = (ctypes.c_longlong * 3)(1, 1, 1)
    assert lib.avq_quantize_workspace_size(1 << 16, 1 << 16, 8, 8) == 0
    rc = lib.avq_quantize_noalloc(1, None, s, None, s, 1 << 16, 1 << 16, 8, 8, 8, 2, None, None, None, None, None,
                                  None, None, None, None, None, None, None, None, None, None)
    assert rc == 1 and "exceeds INT_MAX" in _lib.last_error()


def test_workspace_queries() -> None:
    lib = _lib.load()
    assert lib.avq_quantize_workspace_size(4, 32, 8192, 512) > 4 * 32 * 8192 * 4
    assert lib.avq_forward_workspace_size(1, 1, 1, 1, 8, 4, 2, 2, 1, 1.0, 0) > 0
    # the tensor-core path keeps no fp32 logits when they fit in shared memory
    mma = lib.avq_forward_workspace_size(1, 4, 32, 8192, 128, 512, 4, 32, 1, 1.0, 0)
    exact = lib.avq_forward_workspace_size(0, 4, 32, 8192, 128, 512, 4, 32, 1, 1.0, 0)
    assert 0 < mma < exact


@pytest.mark.parametrize("case", ["bad_dtype", "bad_sizes", "head_dim", "null", "record", "workspace"])
def test_stream_extend_rejects_bad_arguments(case: str) -> None:
    """avq_stream_extend validates before touching device memory."""
    lib = _lib.load()
    dummy = 16  # any non-null address: every case fails before a dereference
    a = dict(dtype=1, B=2, H=2, M0=4, C=2, D=8, ptr=dummy, rec=dummy, stride=8, size=0, ws=1 << 20)
    if case == "bad_dtype":
        a["dtype"] = 9
    elif case == "bad_sizes":
        a["M0"] = 0
    elif case == "head_dim":
        a["D"] = 1024
    elif case == "null":
        a["ptr"] = None
    elif case == "record":
        a["stride"] = 1  # record row narrower than size + B
    elif case == "workspace":
        a["ws"] = 8
    p, r = a["ptr"], a["rec"]
    rc = lib.avq_stream_extend(a["dtype"], dummy, a["D"], a["B"], a["H"], a["M0"], a["C"], a["D"], p, p, p, p, r, r,
                               a["stride"], a["size"], p, p, p, p, dummy, a["ws"], None)
    assert rc == {"head_dim": 3, "workspace": 4}.get(case, 1), _lib.last_error()
    assert _lib.last_error().startswith("avq_stream_extend")


def test_stream_workspace_query() -> None:
    lib = _lib.load()
    assert lib.avq_stream_workspace_size(1, 8, 256, 8) >= 8 * 8 + 8 * 256 * 4 + 8 * 256 * 8 * 4
    assert lib.avq_stream_workspace_size(1 << 16, 1 << 16, 8, 8) == 0
    # zero keys: a no-op that needs no pointers
    assert lib.avq_stream_extend(1, None, 8, 0, 2, 4, 2, 8, None, None, None, None, None, None, 0, 0, None, None,
                                 None, None, None, 0, None) == 0
