"""Model check, on the CPU, of the lane arithmetic of the child assignment kernel
(child_bucket_kernel in avqa_b200/csrc/avq_assign_tc.cu).

A warp takes four keys at a time.  Lane (rsub, vg) of a G-lane row holds, for
each of the four keys, the partial sum of child row ps*R + rsub over its
chunks vg + G*t.  A reduce-scatter (lanes G/2 and G/4 apart) and a butterfly
over the remaining bits leave each lane with the whole-row sum of one key kq.
An xor-min over the row bits then combines the rows, and key kk is read from
the lane at (kk >> 1) * G/2 + (kk & 1) * G/4.

The sums are modelled as sets of (vg, key) contributions.  For every
(D, C) -> (NV, NP) choice of the launcher, the test checks that:
- every lane ends with exactly the G contributions of its key kq;
- the lane read for key kk finishes key kk;
- the passes' child rows cover 0 .. C-1 once.
"""
from __future__ import annotations

import pytest

KP = 4


def dispatch(D: int, C: int) -> tuple[int, int]:
    """(NV, NP) as launch_child_bucket picks them."""
    if D == 128:
        return (1, 1) if C <= 2 else (2, 1) if C <= 4 else (2, 2)
    return (1, 1) if C <= 4 else (2, 1)


def shfl_xor(vals: list, o: int) -> list:
    return [vals[lane ^ o] for lane in range(32)]


def lane_sums(G: int) -> tuple[list, list]:
    """Each lane's final sum (a frozenset of (vg, key)) and its key kq."""
    vg = [lane % G for lane in range(32)]
    hb1 = [(v & (G // 2)) != 0 for v in vg]
    hb2 = [(v & (G // 4)) != 0 for v in vg]
    kq = [(2 if a else 0) + (1 if b else 0) for a, b in zip(hb1, hb2)]
    sx = [[frozenset({(vg[lane], kk)}) for kk in range(KP)] for lane in range(32)]
    s0 = [sx[i][0] if hb1[i] else sx[i][2] for i in range(32)]
    s1 = [sx[i][1] if hb1[i] else sx[i][3] for i in range(32)]
    r0, r1 = shfl_xor(s0, G // 2), shfl_xor(s1, G // 2)
    w0 = [(sx[i][2] if hb1[i] else sx[i][0]) | r0[i] for i in range(32)]
    w1 = [(sx[i][3] if hb1[i] else sx[i][1]) | r1[i] for i in range(32)]
    r = shfl_xor([w0[i] if hb2[i] else w1[i] for i in range(32)], G // 4)
    sv = [(w1[i] if hb2[i] else w0[i]) | r[i] for i in range(32)]
    o = 1
    while o < G // 4:
        other = shfl_xor(sv, o)
        assert all(not (sv[i] & other[i]) for i in range(32)), "a contribution added twice"
        sv = [sv[i] | other[i] for i in range(32)]
        o <<= 1
    return sv, kq


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("C", list(range(1, 9)))
def test_child_lane_map(D: int, C: int) -> None:
    nv, npass = dispatch(D, C)
    cpr = D // 8
    G = cpr // nv
    R = 32 // G
    assert G >= KP and G % KP == 0 and 32 % G == 0
    assert R * npass >= C
    sv, kq = lane_sums(G)
    for lane in range(32):
        assert sv[lane] == frozenset((v, kq[lane]) for v in range(G)), f"lane {lane}"
    for kk in range(KP):
        src = (kk >> 1) * (G // 2) + (kk & 1) * (G // 4)
        assert src < G and kq[src] == kk  # row 0 holds the key after the xor-min over rows
    # each lane's chunks vg + G*t (t < NV) tile the row's CPR chunks once
    chunks = sorted(v + G * t for v in range(G) for t in range(nv))
    assert chunks == list(range(cpr))
    rows = sorted(ps * R + rsub for ps in range(npass) for rsub in range(R) if ps * R + rsub < C)
    assert rows == list(range(C))
