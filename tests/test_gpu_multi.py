"""Multi-GPU building blocks on the device: the work-stealing deque and request
migration (bit-exact state + cache transfer, then identical decoding on the
thief). Same-device variants run on one GPU; cross-device variants need two."""
import ctypes as C
import multiprocessing as mp

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _p(t):
    return C.c_void_p(t.data_ptr())


# --------------------------------------------------------------------------- deque


@pytest.mark.parametrize("cap,n,thieves,batch", [(1024, 1 << 16, 64, 16), (8, 20000, 31, 3),
                                                 (1 << 16, 1 << 17, 128, 32)])
def test_deque_exactly_once_under_contention(torch_cuda, cap, n, thieves, batch):
    from ferry_b200 import _abi

    taken = C.c_uint64()
    bad = C.c_int32()
    _abi.call("ferry_deque_stress", 0, cap, n, thieves, batch, C.byref(taken), C.byref(bad))
    assert taken.value == n and bad.value == 0


def test_deque_owner_and_thief_ends(torch_cuda):
    from ferry_b200 import _abi

    t = torch_cuda
    q = C.c_void_p()
    _abi.call("ferry_deque_create", 0, 16, C.byref(q))
    try:
        st = C.c_void_p(t.cuda.current_stream().cuda_stream)
        tasks = t.arange(10, dtype=t.int64, device="cuda")
        cnt = t.zeros(1, dtype=t.int32, device="cuda")
        out = t.full((16,), -1, dtype=t.int64, device="cuda")
        size = t.zeros(1, dtype=t.int64, device="cuda")
        _abi.call("ferry_deque_push", q, st, _p(tasks), 10, _p(cnt))
        assert cnt.item() == 10
        _abi.call("ferry_deque_steal", q, st, _p(out), 3, _p(cnt))
        assert cnt.item() == 3 and out[:3].tolist() == [0, 1, 2]
        _abi.call("ferry_deque_pop", q, st, _p(out), 2, _p(cnt))
        assert cnt.item() == 2 and out[:2].tolist() == [9, 8]
        _abi.call("ferry_deque_size", q, st, _p(size))
        assert size.item() == 5
        # overflow: capacity 16 holds 11 more at most
        more = t.arange(100, 120, dtype=t.int64, device="cuda")
        _abi.call("ferry_deque_push", q, st, _p(more), 20, _p(cnt))
        assert cnt.item() == 11
        _abi.call("ferry_deque_pop", q, st, _p(out), 16, _p(cnt))
        assert cnt.item() == 16 and out[:16].tolist() == list(range(110, 99, -1)) + [7, 6, 5, 4, 3]
        _abi.call("ferry_deque_steal", q, st, _p(out), 4, _p(cnt))
        assert cnt.item() == 0
    finally:
        _abi.call("ferry_deque_destroy", q)


def test_deque_peek_takes_nothing(torch_cuda):
    from ferry_b200 import _abi

    t = torch_cuda
    q = C.c_void_p()
    _abi.call("ferry_deque_create", 0, 8, C.byref(q))
    try:
        st = C.c_void_p(t.cuda.current_stream().cuda_stream)
        cnt = t.zeros(1, dtype=t.int32, device="cuda")
        out = t.full((8,), -1, dtype=t.int64, device="cuda")
        size = t.zeros(1, dtype=t.int64, device="cuda")
        _abi.call("ferry_deque_peek", q, st, _p(out), 4, _p(cnt))
        assert cnt.item() == 0
        # wrap the ring: push 6, steal 5, push 5 -> tasks 5..10 with top at 5
        _abi.call("ferry_deque_push", q, st, _p(t.arange(6, dtype=t.int64, device="cuda")), 6, _p(cnt))
        _abi.call("ferry_deque_steal", q, st, _p(out), 5, _p(cnt))
        _abi.call("ferry_deque_push", q, st, _p(t.arange(6, 11, dtype=t.int64, device="cuda")), 5, _p(cnt))
        _abi.call("ferry_deque_peek", q, st, _p(out), 4, _p(cnt))
        assert cnt.item() == 4 and out[:4].tolist() == [5, 6, 7, 8]
        _abi.call("ferry_deque_peek", q, st, _p(out), 8, _p(cnt))
        assert cnt.item() == 6 and out[:6].tolist() == [5, 6, 7, 8, 9, 10]
        _abi.call("ferry_deque_size", q, st, _p(size))
        assert size.item() == 6                       # nothing taken
        _abi.call("ferry_deque_steal", q, st, _p(out), 2, _p(cnt))
        assert out[:2].tolist() == [5, 6]             # the peeked ones are what a steal takes
    finally:
        _abi.call("ferry_deque_destroy", q)


def test_deque_steal_from_peer_device(torch_cuda):
    from ferry_b200 import _abi

    t = torch_cuda
    if t.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    q = C.c_void_p()
    v = C.c_void_p()
    _abi.call("ferry_deque_create", 0, 64, C.byref(q))
    _abi.call("ferry_deque_peer_view", 1, q, C.byref(v))
    try:
        with t.cuda.device(0):
            tasks = t.arange(40, dtype=t.int64, device="cuda:0")
            cnt0 = t.zeros(1, dtype=t.int32, device="cuda:0")
            _abi.call("ferry_deque_push", q, C.c_void_p(t.cuda.current_stream(0).cuda_stream), _p(tasks), 40, _p(cnt0))
            t.cuda.synchronize(0)
        with t.cuda.device(1):
            out = t.full((32,), -1, dtype=t.int64, device="cuda:1")
            cnt1 = t.zeros(1, dtype=t.int32, device="cuda:1")
            _abi.call("ferry_deque_steal", v, C.c_void_p(t.cuda.current_stream(1).cuda_stream), _p(out), 25, _p(cnt1))
            t.cuda.synchronize(1)
            assert cnt1.item() == 25 and out[:25].tolist() == list(range(25))
        with t.cuda.device(0):
            out0 = t.full((32,), -1, dtype=t.int64, device="cuda:0")
            _abi.call("ferry_deque_pop", q, C.c_void_p(t.cuda.current_stream(0).cuda_stream), _p(out0), 32, _p(cnt0))
            t.cuda.synchronize(0)
            assert cnt0.item() == 15 and sorted(out0[:15].tolist()) == list(range(25, 40))
    finally:
        _abi.call("ferry_deque_destroy", v)
        _abi.call("ferry_deque_destroy", q)


# --------------------------------------------------------------------------- migration


def _workload():
    from ferry_b200.workload import small

    return small(num_requests=4, num_layers=2, q_heads=8, kv_heads=4, ctx_tokens=1024, top_k=16,
                 cache_frac=0.5)


def _q(w, reqs, step):
    from ferry_b200.workload import q_stream

    return np.stack([q_stream(w, int(r), steps=step + 1)[step] for r in reqs])


def _lane_state(dec, w, req):
    LH, N, C_ = w.lanes_per_req, w.max_pages, w.cache_pages
    lanes = range(req * LH, (req + 1) * LH)
    out = []
    for l in lanes:
        size = int(dec.debug_read(3, np.int32, 1, offset_elems=l)[0])
        order = dec.debug_read(2, np.int32, C_, offset_elems=l * C_)[:size]
        ps = dec.debug_read(1, np.int32, N, offset_elems=l * N)
        cache = dec.debug_read(0, np.uint16, size * 4096, offset_elems=l * C_ * 4096) if size else np.zeros(0, np.uint16)
        out.append((size, order.copy(), ps.copy(), cache.copy()))
    return out


def _run_steps(t, dec, w, reqs, steps, dev):
    ids = t.from_numpy(np.asarray(reqs, np.int32)).to(dev)
    out = t.zeros((len(reqs), w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
    for s in steps:
        q = t.from_numpy(_q(w, reqs, s)).to(dev)
        dec.step(q, ids, out)
    t.cuda.synchronize(dev)
    dec.check()
    return out.cpu().numpy()


@pytest.mark.parametrize("devices,mode", [((0, 0), 1), ((0, 0), 0), ((0, 1), 1)])
def test_migrate_requests_bit_exact_then_same_decode(torch_cuda, devices, mode):
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder

    t = torch_cuda
    if max(devices) >= t.cuda.device_count():
        pytest.skip("needs two GPUs")
    w = _workload()
    src, dst = Decoder(w, devices[0]), Decoder(w, devices[1])
    try:
        d0, d1 = t.device("cuda", devices[0]), t.device("cuda", devices[1])
        for dec, d in ((src, d0), (dst, d1)):
            dec.register_pool()
            ids = t.arange(4, dtype=t.int32, device=d)
            dec.begin(ids, t.full((4,), w.max_pages, dtype=t.int32, device=d))
        _run_steps(t, src, w, [0, 1, 2, 3], range(3), d0)
        _run_steps(t, dst, w, [0, 1, 2, 3], [7], d1)  # the thief's slots hold other state
        before = {r: _lane_state(src, w, r) for r in (1, 3)}
        _abi.call("ferry_ctx_link", dst.ctx, 0, src.ctx)
        with t.cuda.device(d1):
            s_ids = t.tensor([1, 3], dtype=t.int32, device=d1)
            d_ids = t.tensor([0, 2], dtype=t.int32, device=d1)
            _abi.call("ferry_migrate_requests", dst.ctx, C.c_void_p(t.cuda.current_stream(d1).cuda_stream),
                      0, _p(s_ids), _p(d_ids), 2, mode)
            t.cuda.synchronize(d1)
        dst.check()
        for sr, dr in ((1, 0), (3, 2)):
            got = _lane_state(dst, w, dr)
            for (sz, order, ps, cache), (sz2, order2, ps2, cache2) in zip(before[sr], got):
                assert sz == sz2 and (order == order2).all() and (ps == ps2).all() and (cache == cache2).all()
        states = np.zeros(w.num_requests, np.int32)
        _abi.call("ferry_slot_states", src.ctx, states.ctypes.data_as(C.c_void_p), 1)
        assert states.tolist() == [0, 2, 0, 2]
        units, nbytes, mu, mb = dst.all_stats()[:4]
        resident = sum(s[0] for r in (1, 3) for s in before[r])
        assert mu == (resident if mode == 1 else 2 * w.lanes_per_req * w.cache_pages) and mb == mu * 8192
        # the thief decodes the migrated requests exactly as the victim would
        out_v = _run_steps(t, src, w, [1, 3], [3, 4], d0)
        out_t = _run_steps(t, dst, w, [0, 2], [], d1)  # no-op (keeps state)
        ids_t = t.tensor([0, 2], dtype=t.int32, device=d1)
        o = t.zeros((2, w.num_layers, w.q_heads, 128), dtype=t.float32, device=d1)
        for s in (3, 4):
            # queries of the original request ids
            q = t.from_numpy(_q(w, [1, 3], s)).to(d1)
            dst.step(q, ids_t, o)
        t.cuda.synchronize(d1)
        dst.check()
        assert (o.cpu().numpy().view(np.uint32) == out_v.view(np.uint32)).all()
        del out_t
    finally:
        dst.close()
        src.close()


@pytest.mark.parametrize("devices", [(0, 0), (0, 1)])
def test_migrate_drop_starts_cold(torch_cuda, devices):
    """FERRY_MIGRATE_DROP (the reference's kv-mode drop, wla_multigpu.cuh:1314):
    no page moves; the thief's lanes are empty, the request keeps its context
    length and pool home, and it decodes exactly as a cold restart of the
    same request would (every selected page refilled by a miss)."""
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder

    t = torch_cuda
    if max(devices) >= t.cuda.device_count():
        pytest.skip("needs two GPUs")
    w = _workload()
    src, dst, cold = Decoder(w, devices[0]), Decoder(w, devices[1]), Decoder(w, devices[1])
    try:
        d0, d1 = t.device("cuda", devices[0]), t.device("cuda", devices[1])
        for dec, d in ((src, d0), (dst, d1), (cold, d1)):
            dec.register_pool()
            ids = t.arange(4, dtype=t.int32, device=d)
            dec.begin(ids, t.full((4,), w.max_pages, dtype=t.int32, device=d))
        _run_steps(t, src, w, [0, 1, 2, 3], range(3), d0)
        _run_steps(t, dst, w, [0, 1, 2, 3], [7], d1)  # the thief's slots hold other state
        _abi.call("ferry_ctx_link", dst.ctx, 0, src.ctx)
        with t.cuda.device(d1):
            s_ids = t.tensor([1, 3], dtype=t.int32, device=d1)
            d_ids = t.tensor([0, 2], dtype=t.int32, device=d1)
            _abi.call("ferry_migrate_requests", dst.ctx, C.c_void_p(t.cuda.current_stream(d1).cuda_stream),
                      0, _p(s_ids), _p(d_ids), 2, _abi.MIGRATE_DROP)
            t.cuda.synchronize(d1)
        dst.check()
        for dr in (0, 2):
            for sz, _, ps, _ in _lane_state(dst, w, dr):
                assert sz == 0 and (ps == -1).all()
        states = np.zeros(w.num_requests, np.int32)
        _abi.call("ferry_slot_states", src.ctx, states.ctypes.data_as(C.c_void_p), 1)
        assert states.tolist() == [0, 2, 0, 2]
        assert dst.all_stats()[2] == 0  # no page migrated
        # slots 1 and 3 of `cold` start cold with requests 1 and 3's homes (default bases)
        ids_t = t.tensor([0, 2], dtype=t.int32, device=d1)
        ids_c = t.tensor([1, 3], dtype=t.int32, device=d1)
        cold.begin(ids_c, t.full((2,), w.max_pages, dtype=t.int32, device=d1))
        o = t.zeros((2, w.num_layers, w.q_heads, 128), dtype=t.float32, device=d1)
        oc = t.zeros_like(o)
        dst.all_stats(reset=True)
        cold.all_stats(reset=True)
        for s in (3, 4):
            q = t.from_numpy(_q(w, [1, 3], s)).to(d1)
            dst.step(q, ids_t, o)
            cold.step(q, ids_c, oc)
            t.cuda.synchronize(d1)
            assert (o.cpu().numpy().view(np.uint32) == oc.cpu().numpy().view(np.uint32)).all()
        assert dst.all_stats()[0] == cold.all_stats()[0] > 0
        dst.check()
    finally:
        cold.close()
        dst.close()
        src.close()


def _ipc_owner(conn, device):
    import torch

    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder

    w = _workload()
    dec = Decoder(w, device)
    dec.register_pool()
    d = torch.device("cuda", device)
    ids = torch.arange(4, dtype=torch.int32, device=d)
    dec.begin(ids, torch.full((4,), w.max_pages, dtype=torch.int32, device=d))
    _run_steps(torch, dec, w, [0, 1, 2, 3], range(3), d)
    handle = (C.c_uint8 * _abi.CTX_HANDLE_BYTES)()
    _abi.call("ferry_ctx_export", dec.ctx, handle)
    conn.send((bytes(handle), _lane_state(dec, w, 2)))
    conn.recv()  # wait until the importer is done
    states = np.zeros(4, np.int32)
    _abi.call("ferry_slot_states", dec.ctx, states.ctypes.data_as(C.c_void_p), 0)
    conn.send(states.tolist())
    dec.close()


def test_migrate_over_cuda_ipc(torch_cuda):
    """One process per GPU: the owner exports its ctx, a second process imports
    it and pulls a request (same device when only one GPU is present)."""
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder

    t = torch_cuda
    dev_owner = 1 if t.cuda.device_count() > 1 else 0
    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe()
    p = ctx.Process(target=_ipc_owner, args=(child, dev_owner))
    p.start()
    try:
        handle, expected = parent.recv()
        w = _workload()
        dec = Decoder(w, 0)
        try:
            dec.register_pool()
            buf = (C.c_uint8 * _abi.CTX_HANDLE_BYTES).from_buffer_copy(handle)
            _abi.call("ferry_ctx_import", dec.ctx, 3, buf)
            s_ids = t.tensor([2], dtype=t.int32, device="cuda:0")
            d_ids = t.tensor([1], dtype=t.int32, device="cuda:0")
            _abi.call("ferry_migrate_requests", dec.ctx, C.c_void_p(t.cuda.current_stream(0).cuda_stream), 3,
                      _p(s_ids), _p(d_ids), 1, 1)
            t.cuda.synchronize(0)
            dec.check()
            got = _lane_state(dec, w, 1)
            for (sz, order, ps, cache), (sz2, order2, ps2, cache2) in zip(expected, got):
                assert sz == sz2 and (order == order2).all() and (ps == ps2).all() and (cache == cache2).all()
        finally:
            dec.close()
        parent.send("done")
        assert parent.recv() == [0, 0, 2, 0]
    finally:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()


# --------------------------------------------------------------------------- executor


def _cluster_worker(rank, world, port, devices, out, policy=None, llx=None, nccl_exchange=False, log_dir=None):
    import os

    import torch
    import torch.distributed as dist

    from ferry_b200 import _abi
    from ferry_b200.cluster import RankRunner

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = _workload()
    w = type(w)(**{**w.__dict__, "steps": 6})
    total = 12
    home = np.zeros(total, np.int32)          # every request starts on rank 0
    join = np.zeros(total, np.int64)
    # FULL migration: every stolen request carries all of its lanes' cache
    # slots, so the unit count is deterministic (owners pop LIFO and thieves
    # take the oldest tasks, which may not have run yet: DELTA could move 0)
    pol = None if policy is None else _abi.StealPolicy(cost_filter=1, margin=policy, cost_scale=3.0,
                                                        link_gbs=700.0, fixed_ms=0.06)
    log = None if log_dir is None else os.path.join(log_dir, f"rank{rank}.log")
    runner = RankRunner(w, total, world, rank, devices[rank], slots=total + 4, max_batch=4,
                        steal_batch=4, migrate_mode=_abi.MIGRATE_FULL, policy=pol, log_path=log)
    try:
        stats = runner.run(home, join, epoch=2, max_ticks=400, llx=llx,
                           exchange_device=devices[rank] if nccl_exchange else None)
    finally:
        runner.close()
    out.put((rank, stats.tokens, stats.stolen_tasks, stats.migrated_units, stats.ticks, stats.rebalances,
             stats.migrated_bytes))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("policy", [None, 0.0, 1e12])
def test_executor_two_ranks_steal_and_migrate(torch_cuda, policy):
    """Rank 1 starts idle, steals from rank 0's deque and migrates the stolen
    requests over NVLink / IPC; every (request, step) decodes exactly once.
    policy: None = water-level steal; a margin = plus the value/cost filter
    (0 accepts every candidate, 1e12 rejects every one)."""
    import socket

    t = torch_cuda
    devices = [0, 1] if t.cuda.device_count() > 1 else [0, 0]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_cluster_worker, args=(r, 2, port, devices, q, policy)) for r in range(2)]
    for p in ps:
        p.start()
    try:
        res = sorted(q.get(timeout=300) for _ in ps)
    finally:
        for p in ps:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    (r0, tok0, st0, mig0, ticks0, _, _), (r1, tok1, st1, mig1, ticks1, _, _) = res
    assert tok0 + tok1 == 12 * 6
    if policy is not None and policy > 1e9:
        assert st0 == st1 == 0 and tok1 == 0 and mig1 == 0   # every candidate priced out
        return
    assert st1 > 0 and tok1 > 0
    w = _workload()
    per_req = w.lanes_per_req * w.cache_pages
    assert mig1 == st1 * per_req and mig0 == st0 * per_req
    assert ticks0 == ticks1


def test_executor_ownership_over_nccl_comm(torch_cuda):
    """The same two-rank job with the ownership exchange on the C ABI's NCCL
    communicator (ferry_exchange_ownership) instead of the process group:
    the job ends on both ranks together and every (request, step) decodes
    exactly once."""
    import socket

    t = torch_cuda
    if t.cuda.device_count() < 2:
        pytest.skip("needs two GPUs (one NCCL rank per GPU)")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_cluster_worker, args=(r, 2, port, [0, 1], q, None, None, True)) for r in range(2)]
    for p in ps:
        p.start()
    try:
        res = sorted(q.get(timeout=300) for _ in ps)
    finally:
        for p in ps:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    (_, tok0, st0, _, ticks0, _, _), (_, tok1, st1, _, ticks1, _, _) = res
    assert tok0 + tok1 == 12 * 6 and st1 > 0 and tok1 > 0
    assert ticks0 == ticks1


def test_executor_rebalance_orders_move_work(torch_cuda):
    """The cost filter rejects every water-level candidate; only the
    rebalancer's orders (usage exchanged with the ownership rows) move
    requests to the idle rank, bypassing the filter as the reference's does."""
    import socket

    t = torch_cuda
    devices = [0, 1] if t.cuda.device_count() > 1 else [0, 0]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_cluster_worker, args=(r, 2, port, devices, q, 1e12, 0.25)) for r in range(2)]
    for p in ps:
        p.start()
    try:
        res = sorted(q.get(timeout=300) for _ in ps)
    finally:
        for p in ps:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    (r0, tok0, st0, mig0, ticks0, rb0, _), (r1, tok1, st1, mig1, ticks1, rb1, _) = res
    assert tok0 + tok1 == 12 * 6
    assert rb1 > 0 and st1 > 0 and tok1 > 0 and rb0 == 0


def test_executor_decision_log(torch_cuda, tmp_path):
    """Both ranks log their steals (ferry_exec_log): the records add up to the
    runner's stolen tasks and migrated bytes, every stolen request appears
    with its step and slots, and ferry_b200.decisions prices each one under
    a0 / delta / full / drop (full = the mode the job ran: its priced bytes
    equal the measured ones)."""
    import socket

    from ferry_b200 import decisions

    t = torch_cuda
    devices = [0, 1] if t.cuda.device_count() > 1 else [0, 0]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_cluster_worker, args=(r, 2, port, devices, q, None, None, False, str(tmp_path)))
          for r in range(2)]
    for p in ps:
        p.start()
    try:
        res = sorted(q.get(timeout=300) for _ in ps)
    finally:
        for p in ps:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    w = _workload()
    for rank, _, stolen, _, _, _, mig_bytes in res:
        hdr, ds = decisions.read_log(str(tmp_path / f"rank{rank}.log"))
        assert hdr["rank"] == rank and hdr["world"] == 2 and hdr["migrate_mode"] == 0
        assert sum(d.taken for d in ds) == stolen
        assert sum(d.mig_bytes for d in ds) == mig_bytes
        for d in ds:
            assert d.victim == 1 - rank and 0 < d.taken <= d.planned and len(d.tasks) == d.taken
            for task in d.tasks:
                assert 0 <= task.request < 12 and 0 <= task.step < 6
                assert 0 <= task.resident_units <= w.lanes_per_req * w.cache_pages
            rows = decisions.price(hdr, d, 700.0, 50.0)
            full = sum(r[2] for r in rows if r[0] == "full")
            assert full == d.mig_bytes  # FULL moves every slot of every lane
    assert res[1][2] > 0  # the idle rank stole
    csv = decisions.counterfactuals([str(tmp_path / "rank1.log")], 700.0, 50.0)
    assert len(csv) == 1 + 4 * res[1][2]
