"""The oracle's group lanes (slot-keeping restatement of the reference's
kv_touch / grp_trim / own_release / kv_live_owned / kv_handoff_owned,
src/runtime/wla_multigpu.cuh:1867-2015, cap_mode 1 capacities of
src/workloads/missstream.cuh:91-94) against a direct deque/set/dict
restatement of the same functions: hit/miss of every touch, LRU contents,
owner masks and owned counts identical over a seeded scenario with members
finishing and being stolen; the slot rules keep the occupied slots [0, size)."""
import numpy as np
import pytest

from tests.group_scenario import RefMirror, events

GROUPS, MEMBERS, LAYERS, IDS, HOT = 3, 4, 2, 64, 10
LANES, CAPMAX = GROUPS * LAYERS, HOT * MEMBERS


def _pages(o, lane):
    ps, order, size = o.state(lane)
    inv = {int(s): p for p, s in enumerate(ps) if s >= 0}
    assert sorted(int(x) for x in order) == list(range(size))   # occupied slots are [0, size)
    assert len(inv) == size
    return [inv[int(s)] for s in order]


def _masks(o, lane):
    ps, _, _ = o.state(lane)
    m, cap = o.owned_state(lane)
    return {p: int(m[s]) for p, s in enumerate(ps) if s >= 0 and m[s]}, cap


@pytest.mark.parametrize("dup,seed", [(False, 5), (True, 11), (False, 23)])
def test_oracle_group_lanes_match_reference_restatement(dup, seed):
    import oracle

    orc = [oracle.LruLanes(LANES, CAPMAX, IDS) for _ in range(2)]
    ref = [RefMirror(LANES, CAPMAX) for _ in range(2)]
    for o in orc:
        o.group_enable()
    n_touch = n_hit = n_trim_moves = 0
    for ev in events(groups=GROUPS, members=MEMBERS, layers=LAYERS, ids=IDS, hot=HOT, seed=seed, dup=dup):
        kind = ev[0]
        if kind == "touch":
            _, g, r, lanes, sel, bit = ev
            is_miss, *_ = orc[g].step_owned(lanes, sel, np.full(len(lanes), bit, np.uint32))
            for i, l in enumerate(lanes):
                hits = ref[g].touch(int(l), sel[i], bit)
                assert (is_miss[i] == 0).tolist() == hits
                n_touch += len(hits)
                n_hit += sum(hits)
        elif kind == "cap":
            _, g, lanes, caps = ev
            before = {int(l): _pages(orc[g], int(l)) for l in lanes}
            orc[g].set_capacity(lanes, caps)
            for l, c in zip(lanes, caps):
                ref[g].set_cap(int(l), int(c))
                n_trim_moves += len(before[int(l)]) - len(ref[g].dq[int(l)])
        elif kind == "release":
            _, g, lanes, bit = ev
            orc[g].release(lanes, bit)
            for l in lanes:
                ref[g].release(int(l), bit)
        elif kind == "count":
            _, g, lanes, bit = ev
            got = orc[g].count_owned(lanes, bit)
            assert got.tolist() == [ref[g].count_owned(int(l), bit) for l in lanes]
        elif kind == "handoff":
            _, v, c, lanes, bit = ev
            orc[c].handoff(orc[v], lanes, lanes, 2, bit)
            for l in lanes:
                ref[c].handoff_owned(ref[v], int(l), int(l), bit)
        for g in range(2):
            for l in (ev[2] if kind in ("cap", "release", "count") else ev[3]):
                l = int(l)
                assert _pages(orc[g], l) == list(ref[g].dq[l])
                m, cap = _masks(orc[g], l)
                assert m == {b: v for b, v in ref[g].own[l].items() if v}
                assert cap == ref[g].cap[l]
    assert n_touch > 1000 and 0 < n_hit < n_touch and n_trim_moves > 0


def test_oracle_handoff_drop_and_carry():
    import oracle

    a, b = oracle.LruLanes(2, 8, 32), oracle.LruLanes(2, 8, 32)
    a.group_enable()
    b.group_enable()
    a.step_owned([0, 1], np.array([[1, 2, 3, 4], [5, 6, 7, 8]], np.int32), np.array([1, 2], np.uint32))
    b.step_owned([0], np.array([[9, 10]], np.int32), np.array([4], np.uint32))
    b.handoff(a, [1], [0], 1)                   # carry: b's lane 0 becomes a's lane 1
    assert _pages(b, 0) == [5, 6, 7, 8] and _masks(b, 0)[0] == {5: 2, 6: 2, 7: 2, 8: 2}
    b.handoff(a, None, [0], 0)                  # drop: empty
    assert _pages(b, 0) == [] and _masks(b, 0)[0] == {}
    b.set_capacity([1], [2])
    with pytest.raises(ValueError):
        b.handoff(a, [0], [1], 1)               # 4 pages do not fit a lane of capacity 2
