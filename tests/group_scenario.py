"""A seeded group-lane scenario shared by the oracle and GPU tests.

Prefix groups of P members touch their group's lane per layer on the GPU
they live on (the reference's kv_touch keyed by (GPU, group, layer),
src/runtime/wla_multigpu.cuh:1937-1962). Capacities follow cap_mode 1
(hot x resident members of the group on that GPU, wla_group_cap,
src/workloads/missstream.cuh:91-94). Members finish (own_release, then
grp_trim: :836-862) or are stolen to the other GPU (member counts move, the
consumer's lanes take the member's exclusively owned pages with
kv_handoff_owned, the victim releases the member's bit and trims:
:1200-1332). Lane of (gpu, group, layer) = (group * L + layer) in that GPU's
lane set.

``events(...)`` yields the operations in order; ``RefMirror`` is a direct
restatement of those reference functions on deques, sets and mask dicts (no
slots), the cross-check of the oracle's slot-keeping version.
"""
from __future__ import annotations

import collections

import numpy as np


def events(groups=3, members=4, layers=2, steps=24, k=12, ids=64, hot=10, gpus=2, seed=5, dup=False):
    """Operations (dup: a touch row may repeat a page):
    ("touch", gpu, member, lanes, sel[len(lanes), k], bit),
    ("cap", gpu, lanes, caps), ("release", gpu, lanes, bit),
    ("handoff", victim, consumer, lanes, bit), ("count", gpu, lanes, bit)."""
    rng = np.random.default_rng(seed)
    R = groups * members
    home = [r % gpus for r in range(R)]               # member r lives on GPU home[r]
    length = rng.integers(steps // 2, steps + 1, R)   # decode steps of each member
    alive = [True] * R
    n_on = collections.Counter((home[r], r // members) for r in range(R))
    cap = {}

    def lanes_of(q):
        return np.arange(q * layers, (q + 1) * layers, dtype=np.int32)

    out = []
    for g in range(gpus):  # initial capacities
        for q in range(groups):
            c = hot * max(1, n_on[(g, q)])
            cap[(g, q)] = c
            out.append(("cap", g, lanes_of(q), np.full(layers, c, np.int32)))
    # a group's members share a drifting hot set of ids (prefix sharing)
    base = rng.integers(0, ids, (groups, layers, 3 * k))
    for s in range(steps):
        for r in range(R):
            if not alive[r]:
                continue
            q, g = r // members, home[r]
            pool = base[q]
            sel = np.stack([rng.choice(np.unique(np.concatenate([pool[l], rng.integers(0, ids, k)])), k,
                                       replace=dup) for l in range(layers)]).astype(np.int32)
            out.append(("touch", g, r, lanes_of(q), sel, 1 << (r % members)))
            if s + 1 >= length[r]:  # the member finishes on this GPU
                alive[r] = False
                n_on[(g, q)] -= 1
                out.append(("release", g, lanes_of(q), 1 << (r % members)))
                c = hot * max(1, n_on[(g, q)])
                cap[(g, q)] = c
                out.append(("cap", g, lanes_of(q), np.full(layers, c, np.int32)))
        # every 5 steps the less loaded GPU steals one member
        if s % 5 == 4 and gpus > 1:
            load = [sum(1 for r in range(R) if alive[r] and home[r] == g) for g in range(gpus)]
            v, c = int(np.argmax(load)), int(np.argmin(load))
            cand = [r for r in range(R) if alive[r] and home[r] == v]
            if v != c and cand:
                r = cand[int(rng.integers(len(cand)))]
                q, bit = r // members, 1 << (r % members)
                n_on[(v, q)] -= 1
                n_on[(c, q)] += 1
                cc = hot * max(1, n_on[(c, q)])
                if cc != cap[(c, q)]:
                    cap[(c, q)] = cc
                    out.append(("cap", c, lanes_of(q), np.full(layers, cc, np.int32)))
                out.append(("count", v, lanes_of(q), bit))
                out.append(("handoff", v, c, lanes_of(q), bit))
                out.append(("release", v, lanes_of(q), bit))
                cv = hot * max(1, n_on[(v, q)])
                cap[(v, q)] = cv
                out.append(("cap", v, lanes_of(q), np.full(layers, cv, np.int32)))
                home[r] = c
        for g in range(gpus):
            for q in range(groups):
                out.append(("count", g, lanes_of(q), 1 << (q % members)))
    return out


class RefMirror:
    """kv_touch / grp_trim / own_release / kv_live_owned / kv_handoff_owned
    on one GPU's lanes, as the reference keeps them (deque, set, mask dict)."""

    def __init__(self, lanes: int, cap: int):
        self.dq = [collections.deque() for _ in range(lanes)]
        self.cap = [cap] * lanes
        self.own = [dict() for _ in range(lanes)]

    def touch(self, lane, blocks, bit):
        hits = []
        dq, own = self.dq[lane], self.own[lane]
        for b in blocks:
            b = int(b)
            hit = b in dq
            if hit:
                dq.remove(b)
                dq.append(b)
            else:
                while len(dq) >= self.cap[lane]:
                    own.pop(dq.popleft(), None)
                dq.append(b)
            own[b] = own.get(b, 0) | bit
            hits.append(hit)
        return hits

    def set_cap(self, lane, c):
        self.cap[lane] = c
        dq, own = self.dq[lane], self.own[lane]
        while len(dq) > c:
            own.pop(dq.popleft(), None)

    def release(self, lane, bit):
        own = self.own[lane]
        for b in list(own):
            own[b] &= ~bit
            if not own[b]:
                del own[b]

    def count_owned(self, lane, bit):
        return sum(1 for b in self.dq[lane] if self.own[lane].get(b, 0) == bit)

    def handoff_owned(self, src: "RefMirror", src_lane, lane, bit):
        dq, own = self.dq[lane], self.own[lane]
        for b in list(src.dq[src_lane]):
            if src.own[src_lane].get(b, 0) != bit:
                continue
            if b in dq:
                own[b] = own.get(b, 0) | bit
                continue
            while len(dq) >= self.cap[lane]:
                own.pop(dq.popleft(), None)
            dq.append(b)
            own[b] = own.get(b, 0) | bit
