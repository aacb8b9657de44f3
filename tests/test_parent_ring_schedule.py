"""Model check of the tile and logit-slot schedule of the tcgen05 parent
attention kernel (avqa_b200/csrc/avq_parent_tc.cu), on CPU.

The kernel streams, after the query tile, one sequence of ring tiles through
four shared-memory buffers: the parent tiles P_0..P_{n-1} of pass 1, then
P_0, V_0, P_1, V_1, ... of pass 2.  Pass 1 has four TMEM logit slots (chunk v
in slot v % 4), pass 2 two (chunk v in slot v % 2).  The MMA thread issues a
chunk's logits when the previous user of its slot has been consumed by the
row threads; the producer refills a buffer once its last tile was consumed.
This restates those rules and checks, for every parent-chunk count the kernel
admits (M0 <= 2048), that each chunk is issued once, into a free slot, that
every buffer's tiles are consumed in fill order (so the mbarrier phases
match), that pass 1's slots in O's columns are read before the first e @ V
MMA, and that producer, MMA thread and row threads never wait on each other
in a cycle.
"""
from __future__ import annotations

import pytest

NRING = 4


def _schedule(nch: int):
    nv = 2 * nch

    def s_tile(w: int) -> int:
        return w if w < nch else nch + 2 * (w - nch)

    def v_tile(u: int) -> int:
        return nch + 2 * u + 1

    def slot(v: int) -> int:
        return v & 3 if v < nch else v & 1

    def next_user(v: int) -> int:
        if v >= nch:
            return v + 2 if v + 2 < nv else -1
        if v + 4 < nch:
            return v + 4
        k = v & 3
        w = nch + ((k - nch) & 1)
        return w if k < 2 and w < nv else -1

    # the MMA thread's operations, in issue order
    ops = [("S", w) for w in range(min(4, nch))]
    if nch == 1:
        ops.append(("S", 1))
    for v in range(nv):
        ops.append(("E", v))  # wait: the row threads consumed chunk v's slot
        if v >= nch:
            ops.append(("V", v - nch))  # e @ V of second-pass chunk v - nch
        w = next_user(v)
        if w >= 0:
            ops.append(("S", w))
    return nv, ops, s_tile, v_tile, slot


@pytest.mark.parametrize("nch", range(1, 33))
def test_ring_schedule(nch: int) -> None:
    nv, ops, s_tile, v_tile, slot = _schedule(nch)
    ntl = nch + nv
    issued = [w for o, w in ops if o == "S"]
    assert sorted(issued) == list(range(nv))
    pos = {o: i for i, o in enumerate(ops)}
    for w in range(nv):
        prev = [v for v in range(w) if slot(v) == slot(w)]
        if prev:  # the slot's previous user was consumed before the issue
            assert pos[("E", prev[-1])] < pos[("S", w)]
    assert max(pos[("E", v)] for v in range(nch)) < pos[("V", 0)]
    consumed = [s_tile(x) if o == "S" else v_tile(x) for o, x in ops if o in ("S", "V")]
    assert sorted(consumed) == list(range(ntl))
    for k in range(NRING):
        seq = [t for t in consumed if t % NRING == k]
        assert seq == sorted(seq)
    # run producer, MMA thread and row threads until none can move
    loaded, done, mi, rows, avail = 0, set(), 0, 0, set()
    while True:
        moved = False
        if loaded < ntl and (loaded < NRING or loaded - NRING in done):
            loaded += 1
            moved = True
        if mi < len(ops):
            o, x = ops[mi]
            t = s_tile(x) if o == "S" else v_tile(x) if o == "V" else None
            if (t is not None and t < loaded) or (o == "E" and rows > x):
                if t is not None:
                    done.add(t)
                if o == "S":
                    avail.add(x)
                mi += 1
                moved = True
        if rows < nv and rows in avail:
            rows += 1
            moved = True
        if not moved:
            break
    assert (loaded, mi, rows) == (ntl, len(ops), nv), "the schedule stalls"
