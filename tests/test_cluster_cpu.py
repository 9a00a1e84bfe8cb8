"""Host-side logic of the multi-GPU runtime on CPU: rank assignment, the
ownership table, and the ownership exchange across two gloo ranks."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def test_assign_ranks_policies():
    from ferry_b200.cluster import assign_ranks

    rr = assign_ranks(10, 4, "rr")
    assert rr.tolist() == [0, 1, 2, 3, 0, 1, 2, 3, 0, 1]
    z = assign_ranks(4000, 8, "zipf", seed=42)
    assert (z == assign_ranks(4000, 8, "zipf", seed=42)).all()
    share = np.bincount(z, minlength=8) / len(z)
    assert share[:2].sum() > 0.7 and share[0] > share[1] > share[7]


def test_merge_ownership():
    from ferry_b200.cluster import merge_ownership, ownership_row

    rows = np.stack([ownership_row(3, 7, np.array([0, 5, 6]), 4),
                     ownership_row(1, 2, np.array([2]), 4)])
    owner, fin, adm = merge_ownership(rows, 8)
    assert owner.tolist() == [0, -1, 1, -1, -1, 0, 0, -1] and fin == 4 and adm == 9


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _exchange_worker(rank, world, port, out):
    import torch.distributed as dist

    from ferry_b200.cluster import exchange_ownership

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    owned = np.array([rank, rank + 2], np.int32)
    owner, fin, adm = exchange_ownership(finished=rank + 1, admitted=10 * (rank + 1), owned=owned,
                                         cap=4, total_requests=6)
    out.put((rank, owner.tolist(), fin, adm))
    dist.destroy_process_group()


def test_exchange_ownership_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    for rank, owner, fin, adm in res:
        assert owner == [0, 1, 0, 1, -1, -1] and fin == 3 and adm == 30


# --------------------------------------------------------------------------- steal policy E


def _filter(pol, remain, live, step_ms):
    import ctypes as C

    from ferry_b200 import _abi

    n = len(remain)
    r = np.ascontiguousarray(remain, np.int32)
    lb = np.ascontiguousarray(live, np.int64)
    v = np.zeros(n, np.float64)
    c = np.zeros(n, np.float64)
    acc = C.c_int()
    _abi.call("ferry_steal_filter", C.byref(pol), n, r.ctypes.data_as(C.c_void_p),
              lb.ctypes.data_as(C.c_void_p), C.c_double(step_ms), v.ctypes.data_as(C.c_void_p),
              c.ctypes.data_as(C.c_void_p), C.byref(acc))
    return acc.value, v, c


def test_steal_filter_prices_candidates_like_policy_e():
    """value = remaining steps x step time; cost = kappa x live bytes / link
    + fixed; the accepted candidates are the longest prefix with value >=
    margin x cost (cost_filter_ok, wla_multigpu.cuh:942-1061)."""
    from ferry_b200 import _abi

    pol = _abi.StealPolicy(cost_filter=1, margin=2.0, cost_scale=3.0, link_gbs=16.6, fixed_ms=0.06)
    remain = [40, 5, 2, 30]
    live = [24 << 20, 24 << 20, 24 << 20, 1 << 20]
    acc, v, c = _filter(pol, remain, live, 1.5)
    ms_per_b = 1e3 / (16.6e9)
    exp_c = [3.0 * b * ms_per_b + 0.06 for b in live]
    exp_v = [r * 1.5 for r in remain]
    np.testing.assert_allclose(c, exp_c, rtol=1e-12)
    np.testing.assert_allclose(v, exp_v, rtol=1e-12)
    ok = [vv >= 2.0 * cc for vv, cc in zip(exp_v, exp_c)]
    assert ok == [True, False, False, True]
    assert acc == 1  # the prefix stops at the first rejection
    # the NVLink link prices the same candidates as cheap
    pol.link_gbs = 700.0
    assert _filter(pol, remain, live, 1.5)[0] == 4
    # margin 0 takes everything; without the filter every candidate passes
    pol.link_gbs, pol.margin = 16.6, 0.0
    assert _filter(pol, remain, live, 1.5)[0] == 4
    pol.margin, pol.cost_filter = 2.0, 0
    assert _filter(pol, remain, live, 1.5)[0] == 4


def test_steal_filter_rejects_bad_policy():
    import ctypes as C

    from ferry_b200 import _abi

    pol = _abi.StealPolicy(cost_filter=1, margin=2.0, cost_scale=3.0, link_gbs=0.0, fixed_ms=0.06)
    acc = C.c_int()
    lib = _abi.lib()
    assert lib.ferry_steal_filter(C.byref(pol), 0, None, None, C.c_double(1.0), None, None,
                                  C.byref(acc)) == _abi.E_INVAL
    assert lib.ferry_exec_policy(None, C.byref(pol)) == _abi.E_INVAL


# --------------------------------------------------------------------------- failures on the host


def test_merge_rejects_corrupt_rows():
    from ferry_b200.cluster import merge_ownership, ownership_row

    rows = np.stack([ownership_row(0, 2, np.array([0, 1]), 4), ownership_row(1, 2, np.array([2, 3]), 4)])
    owner, fin, adm = merge_ownership(rows, 8)
    assert owner.tolist() == [0, 0, 1, 1, -1, -1, -1, -1] and (fin, adm) == (1, 4)
    bad = rows.copy()
    bad[1, 2] = 99  # a garbled count
    with pytest.raises(ValueError):
        merge_ownership(bad, 8)
    bad = rows.copy()
    bad[0, 1] = -5
    with pytest.raises(ValueError):
        merge_ownership(bad, 8)


def _leaving_rank(rank, port, out):
    import datetime

    import torch.distributed as dist

    from ferry_b200.cluster import exchange_ownership

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    if rank == 1:  # leaves between steps, before the exchange
        out.put((1, "left"))
        dist.destroy_process_group()
        return
    try:
        exchange_ownership(0, 4, np.arange(4), 8, 8)
        out.put((0, "no error"))
    except Exception as e:  # the collective ends with an error instead of waiting for good
        out.put((0, type(e).__name__))


def test_a_rank_that_leaves_ends_the_exchange_with_an_error():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_leaving_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    try:
        res = dict(q.get(timeout=90) for _ in ps)
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[1] == "left" and res[0] != "no error"


def test_llx_plan_matches_the_rebalancer_rule():
    """rebalance_llumnix (wla_multigpu.cuh:2084-2112): spread / mean > thr ->
    the least loaded pulls clamp((usage[src] - mean) // (mean // n_src + 1), 1, 4)."""
    from ferry_b200.cluster import llx_plan

    # usage 120 / 0 / 60, mean 60, spread 2.0 > 0.25; per = 60 // 4 + 1 = 16; k = 60 // 16 = 3
    assert llx_plan([120, 0, 60], [4, 0, 2]) == (0, 1, 3)
    # balanced within the threshold: nothing to do
    assert llx_plan([100, 90, 95], [5, 5, 5]) is None
    # the pull is capped at 4 and floored at 1
    assert llx_plan([1000, 0], [40, 0]) == (0, 1, 4)   # per = 500 // 40 + 1 = 13, 500 // 13 = 38
    assert llx_plan([1000, 0], [2, 0]) == (0, 1, 1)    # per = 251, 500 // 251 = 1
    assert llx_plan([10, 0], [10, 0]) == (0, 1, 4)     # per = 1, k = 5 -> 4
    assert llx_plan([3, 1], [1, 1]) == (0, 1, 1)       # over 1 < per 3: floored at 1
    # idle job, single GPU
    assert llx_plan([0, 0], [0, 0]) is None and llx_plan([50], [3]) is None
    # ties: the first maximum and the first minimum, as the reference's strict comparisons
    assert llx_plan([80, 80, 0, 0], [2, 2, 0, 0])[:2] == (0, 2)


def test_exchange_over_a_communicator_merges_its_int32_rows():
    """The runner's exchange through the C ABI's communicator: the rows come
    back as int32 (the NCCL all_gather's type) and merge exactly like the
    process group's int64 rows. A stand-in communicator plays the other rank."""
    from ferry_b200.cluster import exchange_ownership, llx_plan, ownership_row

    other = ownership_row(3, 9, np.array([1, 4, 6], np.int32), cap=8, usage=40)

    class TwoRanks:
        def all_gather(self, row):
            assert row.dtype == np.int64 and len(row) == len(other)
            return np.stack([np.asarray(row, np.int32), other.astype(np.int32)])

    (owner, fin, adm), rows = exchange_ownership(2, 5, np.array([0, 2, 5], np.int32), 8, 8,
                                                 usage=7, with_rows=True, comm=TwoRanks())
    assert rows.dtype == np.int64 and rows.shape == (2, 12)
    assert fin == 5 and adm == 14
    assert owner.tolist() == [0, 1, 0, -1, 1, 0, 1, -1]
    # loads 7 and 40, 3 requests each: mean 23.5, rank 0 pulls (40 - 23) // (23.5 // 3 + 1) = 2
    assert llx_plan(rows[:, 3], rows[:, 2], 0.25) == (1, 0, 2)


def test_job_schedule_scales_the_box_rate_and_config_generators():
    """The multi-GPU bench's job: homes round-robin, Poisson arrivals at N x the
    single-GPU rate (each GPU sees the configs[0] rate); the configs[3] ON/OFF
    generator puts its first requests in one ON period and then pauses; ragged
    contexts are whole pages inside the configured token range."""
    import numpy as np

    from ferry_b200.cluster import job_schedule
    from ferry_b200.workload import CFG1, onoff_arrival_ticks, pages_after, ragged_pages

    home, join = job_schedule(CFG1, 64, 4, "rr", rate=CFG1.arrival_rate * 4)
    assert (home == np.arange(64) % 4).all() and join.min() == 0
    _, join1 = job_schedule(CFG1, 16, 1, "rr")
    # four times the requests at four times the rate arrive over a similar span
    assert 0.5 < join.max() / max(1, join1.max()) < 2.0
    j = onoff_arrival_ticks(2000, 2000.0, 200.0, 800.0, seed=3)
    assert (np.diff(j) >= 0).all() and j[0] == 0
    gaps = np.diff(np.unique(j))
    assert gaps.max() >= 10  # an OFF period of >= 200 ms on a 20 ms tick
    per_tick = np.bincount(j)
    assert per_tick.max() >= 30  # ~40 arrivals per 20 ms tick while ON
    p = ragged_pages(1000, 8192, 32768, seed=1)
    assert p.min() >= 512 and p.max() <= 2048
    assert (pages_after(np.array([10, 2047]), 40, 1, 2048) == [12, 2048]).all()
