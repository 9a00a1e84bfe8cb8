"""Device group lanes (ferry_lru_group_enable / touch_owned / set_capacity /
release / count_owned / handoff, csrc/group.cu) against the oracle's group
lanes over the seeded scenario of tests/group_scenario.py: every touch's
miss flags, slots and miss lists, every lane's page table, LRU order, owner
masks and capacity, and every owned count identical -- the reference's
prefix-group-shared LRU with cap_mode 1 and per-request ownership carry
(src/runtime/wla_multigpu.cuh:1867-2015). Both GPUs' mirrors on one device,
and, with two GPUs, the victim's lanes read over NVLink by the consumer."""
import ctypes as C

import numpy as np
import pytest

from tests.group_scenario import events

pytestmark = pytest.mark.gpu

GROUPS, MEMBERS, LAYERS = 3, 4, 2
LANES = GROUPS * LAYERS
IDS, HOT, K = 64, 10, 12           # warp-per-lane kernel (capacity <= 128)
BIG = dict(ids=512, hot=40, k=48)  # capacity 160: the CTA-per-lane kernel


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


class DevLanes:
    def __init__(self, t, device, ids=IDS, hot=HOT):
        from ferry_b200 import _abi

        self.t, self.a, self.dev = t, _abi, t.device("cuda", device)
        self.ids, self.cap = ids, hot * MEMBERS
        self.h = C.c_void_p()
        _abi.call("ferry_lru_create", device, LANES, self.cap, ids, C.byref(self.h))
        _abi.call("ferry_lru_group_enable", self.h)

    def d(self, x):
        return self.t.from_numpy(np.ascontiguousarray(x)).to(self.dev)

    @staticmethod
    def p(x):
        return None if x is None else C.c_void_p(x.data_ptr())

    def stream(self):
        return C.c_void_p(self.t.cuda.current_stream(self.dev).cuda_stream)

    def touch(self, lanes, sel, bit, distinct):
        t = self.t
        n, k = sel.shape
        lanes_d, sel_d = self.d(lanes.astype(np.int32)), self.d(sel.astype(np.int32))
        ns_d = self.d(np.full(n, k, np.int32))
        bits_d = self.d(np.full(n, bit, np.uint32).view(np.int32))
        im = t.zeros((n, k), dtype=t.uint8, device=self.dev)
        isl, mp, ms = (t.full((n, k), -1, dtype=t.int32, device=self.dev) for _ in range(3))
        nm = t.zeros(n, dtype=t.int32, device=self.dev)
        self.a.call("ferry_lru_touch_owned", self.h, self.stream(), self.p(lanes_d), None, n, self.p(sel_d), k,
                    self.p(ns_d), self.a.LRU_DISTINCT if distinct else 0, self.p(bits_d), self.p(im), self.p(isl),
                    self.p(mp), self.p(ms), self.p(nm))
        t.cuda.synchronize(self.dev)
        return im.cpu().numpy(), isl.cpu().numpy(), mp.cpu().numpy(), ms.cpu().numpy(), nm.cpu().numpy()

    # device copies are held in locals until the launch is queued: a temporary
    # freed early hands its memory to the next copy, and two arguments alias
    def set_capacity(self, lanes, caps):
        l, c = self.d(lanes.astype(np.int32)), self.d(caps.astype(np.int32))
        self.a.call("ferry_lru_set_capacity", self.h, self.stream(), self.p(l), self.p(c), len(lanes))

    def release(self, lanes, bit):
        l = self.d(lanes.astype(np.int32))
        self.a.call("ferry_lru_release", self.h, self.stream(), self.p(l), len(lanes), bit)

    def count_owned(self, lanes, bit):
        out = self.t.zeros(len(lanes), dtype=self.t.int32, device=self.dev)
        l = self.d(lanes.astype(np.int32))
        self.a.call("ferry_lru_count_owned", self.h, self.stream(), self.p(l), len(lanes), bit, self.p(out))
        return out.cpu().numpy()

    def handoff(self, src, lanes, mode, bit):
        l = self.d(lanes.astype(np.int32))
        self.a.call("ferry_lru_handoff", self.h, self.stream(), src.h, self.p(l), self.p(l), len(lanes), mode, bit)
        self.t.cuda.synchronize(self.dev)

    def state(self, lane):
        ps = np.zeros(self.ids, np.int32)
        order = np.zeros(self.cap, np.int32)
        size = np.zeros(1, np.int32)
        self.a.call("ferry_lru_read", self.h, lane, ps.ctypes.data, order.ctypes.data, size.ctypes.data)
        masks = np.zeros(self.cap, np.uint32)
        cap = np.zeros(1, np.int32)
        self.a.call("ferry_lru_read_owned", self.h, lane, masks.ctypes.data, cap.ctypes.data)
        n = int(size[0])
        m = np.where(np.arange(self.cap) < n, masks, 0)  # slots past size hold no page
        return ps, order[:n].copy(), n, m, int(cap[0])

    def close(self):
        if self.h:
            self.a.call("ferry_lru_destroy", self.h)
            self.h = None


def _check_lane(dev, orc, lane):
    ps, order, n, m, cap = dev.state(lane)
    ops, oorder, on = orc.state(lane)
    om, ocap = orc.owned_state(lane)
    assert n == on and (order == oorder).all() and (ps == ops).all()
    assert (m == om).all() and cap == ocap


@pytest.mark.parametrize("devices,dup,seed,big", [((0, 0), False, 5, False), ((0, 0), True, 11, False),
                                                  ((0, 0), False, 7, True), ((0, 1), False, 23, False)])
def test_group_lanes_match_oracle(torch_cuda, devices, dup, seed, big):
    import oracle

    t = torch_cuda
    if max(devices) >= t.cuda.device_count():
        pytest.skip("needs two GPUs")
    sz = BIG if big else dict(ids=IDS, hot=HOT, k=K)
    dev = [DevLanes(t, d, sz["ids"], sz["hot"]) for d in devices]
    orc = [oracle.LruLanes(LANES, sz["hot"] * MEMBERS, sz["ids"]) for _ in range(2)]
    for o in orc:
        o.group_enable()
    try:
        touches = handoffs = 0
        for ev in events(groups=GROUPS, members=MEMBERS, layers=LAYERS, seed=seed, dup=dup, **sz):
            kind = ev[0]
            if kind == "touch":
                _, g, r, lanes, sel, bit = ev
                got = dev[g].touch(lanes, sel, bit, distinct=not dup)
                ref = orc[g].step_owned(lanes, sel, np.full(len(lanes), bit, np.uint32))
                im, isl, mp, ms, nm = got
                rim, risl, rmp, rms, rnm = ref
                assert (im == rim).all() and (isl == risl).all() and (nm == rnm).all()
                for i in range(len(lanes)):
                    assert (mp[i, : nm[i]] == rmp[i, : rnm[i]]).all() and (ms[i, : nm[i]] == rms[i, : rnm[i]]).all()
                touches += 1
                lanes_chk = lanes
            elif kind == "cap":
                _, g, lanes, caps = ev
                dev[g].set_capacity(lanes, caps)
                orc[g].set_capacity(lanes, caps)
                lanes_chk = lanes
            elif kind == "release":
                _, g, lanes, bit = ev
                dev[g].release(lanes, bit)
                orc[g].release(lanes, bit)
                lanes_chk = lanes
            elif kind == "count":
                _, g, lanes, bit = ev
                assert (dev[g].count_owned(lanes, bit) == orc[g].count_owned(lanes, bit)).all()
                lanes_chk = lanes
            else:
                _, v, c, lanes, bit = ev
                dev[c].handoff(dev[v], lanes, 2, bit)
                orc[c].handoff(orc[v], lanes, lanes, 2, bit)
                handoffs += 1
                g = c
                lanes_chk = lanes
            for gg in range(2):
                for l in lanes_chk:
                    _check_lane(dev[gg], orc[gg], int(l))
        assert touches > 100 and handoffs > 0
    finally:
        for d in dev:
            d.close()


def test_group_handoff_drop_carry_and_errors(torch_cuda):
    import oracle
    from ferry_b200 import _abi

    t = torch_cuda
    a, b = DevLanes(t, 0), DevLanes(t, 0)
    oa, ob = oracle.LruLanes(LANES, HOT * MEMBERS, IDS), oracle.LruLanes(LANES, HOT * MEMBERS, IDS)
    oa.group_enable()
    ob.group_enable()
    try:
        sel = np.array([[1, 2, 3, 4, 5], [6, 7, 8, 9, 10]], np.int32)
        lanes = np.array([0, 1], np.int32)
        a.touch(lanes, sel, 1, True)
        oa.step_owned(lanes, sel, np.full(2, 1, np.uint32))
        b.touch(lanes[:1], sel[:1] + 20, 2, True)
        ob.step_owned(lanes[:1], sel[:1] + 20, np.full(1, 2, np.uint32))
        b.handoff(a, lanes, _abi.HANDOFF_CARRY, 0)
        ob.handoff(oa, lanes, lanes, 1)
        for l in (0, 1):
            _check_lane(b, ob, l)
        b.handoff(a, lanes[:1], _abi.HANDOFF_DROP, 0)
        ob.handoff(oa, None, lanes[:1], 0)
        _check_lane(b, ob, 0)
        with pytest.raises(_abi.FerryError):
            _abi.call("ferry_lru_handoff", b.h, b.stream(), a.h, None, None, 1, _abi.HANDOFF_OWNED, 0)  # bit 0
        b.set_capacity(np.array([2], np.int32), np.array([3], np.int32))
        b.handoff(a, np.array([2], np.int32), _abi.HANDOFF_DROP, 0)
        # carry of a 5-page lane into a lane of capacity 3: a range error, the lane untouched
        l2 = b.d(np.array([0], np.int32))
        l3 = b.d(np.array([2], np.int32))
        _abi.call("ferry_lru_handoff", b.h, b.stream(), a.h, b.p(l2), b.p(l3), 1, _abi.HANDOFF_CARRY, 0)
        with pytest.raises(_abi.FerryError) as e:
            b.state(2)
        assert e.value.code == _abi.E_RANGE
        plain = C.c_void_p()
        _abi.call("ferry_lru_create", 0, 2, 4, 8, C.byref(plain))
        try:
            with pytest.raises(_abi.FerryError) as e:
                _abi.call("ferry_lru_release", plain, None, None, 0, 1)   # not enabled
            assert e.value.code == _abi.E_STATE
        finally:
            _abi.call("ferry_lru_destroy", plain)
    finally:
        a.close()
        b.close()


def test_group_lanes_replay_cap_mode_1(torch_cuda):
    """The reference's prefix-shared block stream (prefix group 4, 8 shared
    steps) on group lanes with cap_mode 1 capacities, hot x members
    (wla_group_cap, src/workloads/missstream.cuh:91-94; wla_recompute_stats,
    src/runtime/wla_multigpu.cuh:376-417): lanes allocated at twice that,
    capacities set per lane; the device misses equal the oracle's totals,
    and the larger group capacity hits more often than cap_mode 0."""
    import oracle
    from ferry_b200 import _abi

    t = torch_cuda
    pg = 4
    sp1 = oracle.miss_spec(prefix_group=pg, prefix_steps=8, cap_mode=1)
    sp0 = oracle.miss_spec(prefix_group=pg, prefix_steps=8, cap_mode=0)
    R, L_, S, G, hot = sp1.num_requests, sp1.num_layers, sp1.steps, sp1.sel_blocks, sp1.hot_blocks
    blocks, _, _ = oracle.replay_miss_stream(sp1)
    shared, tot1 = oracle.prefix_share_stats(sp1, blocks.copy())
    _, tot0 = oracle.prefix_share_stats(sp0, blocks.copy())
    B = shared.reshape(R, S, L_, G).astype(np.int32)
    ngrp, ids = R // pg, 64 + 8 * S
    dev = DevLanes.__new__(DevLanes)
    dev.t, dev.a, dev.dev, dev.ids, dev.cap = t, _abi, t.device("cuda", 0), ids, 2 * hot * pg
    dev.h = C.c_void_p()
    _abi.call("ferry_lru_create", 0, ngrp * L_, dev.cap, ids, C.byref(dev.h))
    try:
        _abi.call("ferry_lru_group_enable", dev.h)
        lanes = (np.arange(ngrp)[:, None] * L_ + np.arange(L_)[None]).ravel().astype(np.int32)
        dev.set_capacity(lanes, np.full(len(lanes), hot * pg, np.int32))
        misses = 0
        for m in range(pg):
            for s in range(S):
                sel = B[np.arange(ngrp) * pg + m, s].reshape(ngrp * L_, G)
                *_, nm = dev.touch(lanes, sel, 1 << m, distinct=False)
                misses += int(nm.sum())
        assert misses == int(tot1[1]) and misses < int(tot0[1])
        # every resident page was touched by some member
        for lane in lanes[:4]:
            ps, order, n, masks, cap = dev.state(int(lane))
            assert cap == hot * pg and n <= cap and (masks[:n] != 0).all()
    finally:
        dev.close()
