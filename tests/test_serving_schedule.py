"""The N-GPU serving loop's schedule (decode_opt_b200.tp.serving_schedule),
checked on the CPU: the happens-before relation of its three streams (H2D
copies, fused GEMMs, D2H copies; each in issue order, plus the declared
cross-stream waits) must order every reuse of an input slot and of a gathered
buffer set, including the cross-rank rule -- a peer's GEMM j stores into set
j % (2*group) once this rank finished GEMM j-1, so the set's previous D2H
copy must come before this rank's GEMM j-1 -- and only a group's first GEMM
may wait on another stream (the others keep their PDL edge).  Mutated
schedules show that the checker catches a missing wait."""

import pytest

from decode_opt_b200 import tp

STREAM = {"h2d": 0, "gemm": 1, "d2h": 2}


def happens_before(ops):
    """{(kind, j): bitmask of ops that happen before it}, ops in issue order."""
    index = {(kind, j): i for i, (kind, j, _) in enumerate(ops)}
    assert len(index) == len(ops), "an operation is issued twice"
    reach = []
    last_on_stream = {}
    for i, (kind, j, waits) in enumerate(ops):
        preds = []
        if kind in last_on_stream:
            preds.append(last_on_stream[kind])
        for w in waits:
            assert w in index, f"{kind} {j} waits on {w}, which is not in the schedule"
            assert index[w] < i, f"{kind} {j} waits on {w}, issued after it"
            preds.append(index[w])
        mask = 0
        for p in preds:
            mask |= reach[p] | (1 << p)
        reach.append(mask)
        last_on_stream[kind] = i
    return index, reach


def check(ops, base, count, group, ring):
    nset = 2 * group
    index, reach = happens_before(ops)

    def hb(a, b):
        return bool(reach[index[b]] >> index[a] & 1)

    js = range(base, base + count)
    for kind in STREAM:
        assert [j for k, j, _ in ops if k == kind] == list(js), f"{kind} ops out of order"
    for j in js:
        assert hb(("h2d", j), ("gemm", j)), f"GEMM {j} may read its input before the copy lands"
        assert hb(("gemm", j), ("d2h", j)), f"D2H {j} may read before GEMM {j}"
        if j - nset >= base:
            assert hb(("gemm", j - nset), ("h2d", j)), f"H2D {j} may overwrite the slot GEMM {j - nset} reads"
            assert hb(("d2h", j - nset), ("gemm", j - 1)), \
                f"a peer's GEMM {j} may store into set {j % nset} before D2H {j - nset} read it"
    # PDL: only a group's first GEMM waits on another stream
    for kind, j, waits in ops:
        if kind == "gemm" and (j - base) % group != 0:
            assert not waits, f"GEMM {j} (not first in its group) waits on {waits}"
    # event ring: a waited op's slot was not re-recorded before the wait
    issued = {k: [] for k in STREAM}
    for kind, j, waits in ops:
        for wk, wj in waits:
            later = [x for x in issued[wk] if x > wj]
            assert len(later) < ring, f"event of {wk} {wj} reused before {kind} {j} waits on it"
        issued[kind].append(j)


@pytest.mark.parametrize("group", [1, 2, 3, 4, 8, 16])
@pytest.mark.parametrize("base,count", [(0, 1), (0, 7), (0, 64), (496, 37), (10, 96)])
def test_schedule_orders_every_reuse(group, base, count):
    ops = tp.serving_schedule(base, count, group)
    check(ops, base, count, group, ring=2 * (2 * group) + 2)


def test_only_group_heads_wait_and_waits_stay_in_chunk():
    ops = tp.serving_schedule(100, 40, 8)
    heads = [j for k, j, w in ops if k == "gemm" and w]
    assert heads == list(range(100, 140, 8))
    for kind, j, waits in ops:
        assert all(wj >= 100 for _, wj in waits)


@pytest.mark.parametrize("mutation", ["drop_d2h_wait", "drop_h2d_slot_wait", "late_h2d_wait", "wait_every_gemm"])
def test_checker_catches_planted_mistakes(mutation):
    group, base, count = 4, 0, 48
    ops = [list(op) for op in tp.serving_schedule(base, count, group)]
    if mutation == "drop_d2h_wait":
        for op in ops:
            if op[0] == "gemm":
                op[2] = [w for w in op[2] if w[0] != "d2h"]
    elif mutation == "drop_h2d_slot_wait":
        for op in ops:
            if op[0] == "h2d":
                op[2] = []
    elif mutation == "late_h2d_wait":
        # the group head waits on its own H2D only, not on the group's last
        for op in ops:
            if op[0] == "gemm" and op[2]:
                op[2] = [("h2d", op[1]) if w[0] == "h2d" else w for w in op[2]]
    elif mutation == "wait_every_gemm":
        for op in ops:
            if op[0] == "gemm" and not op[2]:
                op[2] = [("h2d", op[1])]
    with pytest.raises(AssertionError):
        check([tuple(op) for op in ops], base, count, group, ring=2 * (2 * group) + 2)


def test_rejects_bad_arguments():
    with pytest.raises(ValueError):
        tp.serving_schedule(0, 4, 0)
    with pytest.raises(ValueError):
        tp.serving_schedule(0, -1, 2)
    assert tp.serving_schedule(0, 0, 4) == []
