"""Page-owner stores (pages sharded by page id across GPUs) vs the host-pool
gather: misses served from the owning rank's store must put the same bytes in
the cache as the host path, decode outputs must be bit-identical, and the
per-source counters must account for every gathered unit. The ranks of one
job are several ctxs on one GPU here (plain device pointers); with two GPUs
the peer stores are read over NVLink."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _q(w, reqs, step):
    from ferry_b200.workload import q_stream

    return np.stack([q_stream(w, int(r), steps=step + 1)[step] for r in reqs])


def _job(t, world, devices, kv_dtype="f16", global_frac=1.0):
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    w = small(num_requests=4, num_layers=2, q_heads=8, kv_heads=2, ctx_tokens=2048, top_k=24,
              kv_dtype=kv_dtype)
    decs = [Decoder(w, devices[r]) for r in range(world)]
    gl = int(w.num_requests * w.lanes_per_req * global_frac)
    for r, d in enumerate(decs):
        d.register_pool()
        d.store_create(world, r, gl)
        d.store_fill()
    t.cuda.synchronize()
    for r, d in enumerate(decs):
        slot = 0
        for p, e in enumerate(decs):
            if p != r:
                _abi.call("ferry_ctx_link", d.ctx, slot, e.ctx)
                slot += 1
    return w, decs


def _run(t, dec, w, reqs, steps, dev):
    outs = []
    ids = t.from_numpy(np.asarray(reqs, np.int32)).to(dev)
    dec.begin(ids, t.full((len(reqs),), w.max_pages, dtype=t.int32, device=dev))
    for s in range(steps):
        out = t.zeros((len(reqs), w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
        dec.step(t.from_numpy(_q(w, reqs, s)).to(dev), ids, out)
        outs.append(out.cpu().numpy())
    t.cuda.synchronize(dev)
    dec.check()
    return outs


@pytest.mark.parametrize("world,kv_dtype", [(4, "f16"), (3, "e4m3"), (1, "f16")])
def test_owner_gather_matches_host_gather(torch_cuda, world, kv_dtype):
    from ferry_b200 import _abi

    t = torch_cuda
    dev = t.device("cuda", 0)
    w, decs = _job(t, world, [0] * world, kv_dtype)
    from ferry_b200.engine import Decoder

    host = Decoder(w, 0)
    try:
        host.register_pool()
        reqs = list(range(w.num_requests))
        decs[0].gather_source(_abi.SRC_OWNER)
        decs[0].all_stats(reset=True)
        a = _run(t, decs[0], w, reqs, 3, dev)
        b = _run(t, host, w, reqs, 3, dev)
        for x, y in zip(a, b):
            assert (x.view(np.uint32) == y.view(np.uint32)).all()
        ub = w.unit_bytes
        C_, LH = w.cache_pages, w.lanes_per_req
        ca = decs[0].debug_read(0, np.uint8, w.num_requests * LH * C_ * ub)
        cb = host.debug_read(0, np.uint8, w.num_requests * LH * C_ * ub)
        assert (ca == cb).all()
        st = decs[0].all_stats()
        units, peer_u, self_u = st[0], st[4], st[6]
        assert units > 0 and peer_u + self_u == units          # every miss from a store
        assert st[5] == peer_u * ub and st[7] == self_u * ub
        if world == 1:
            assert peer_u == 0
        else:
            # pages are spread over owners by page id: this rank holds ~1/world
            assert 0 < self_u < units and peer_u > 0
    finally:
        host.close()
        for d in decs:
            d.close()


def test_lanes_outside_the_store_come_from_host(torch_cuda):
    from ferry_b200 import _abi

    t = torch_cuda
    dev = t.device("cuda", 0)
    w, decs = _job(t, 2, [0, 0], global_frac=0.5)  # stores cover requests 0, 1 only
    try:
        decs[0].gather_source(_abi.SRC_OWNER)
        decs[0].all_stats(reset=True)
        _run(t, decs[0], w, [2, 3], 2, dev)
        st = decs[0].all_stats()
        assert st[0] > 0 and st[4] == 0 and st[6] == 0   # all from the host pool
        decs[0].all_stats(reset=True)
        _run(t, decs[0], w, [0, 1], 2, dev)
        st = decs[0].all_stats()
        assert st[0] > 0 and st[4] + st[6] == st[0]
    finally:
        for d in decs:
            d.close()


def test_store_arguments_rejected(torch_cuda):
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    w = small(num_requests=2)
    d = Decoder(w, 0)
    try:
        with pytest.raises(_abi.FerryError):
            d.gather_source(_abi.SRC_OWNER)             # no store yet
        with pytest.raises(_abi.FerryError):
            d.store_create(3, 3)                          # rank outside world
        with pytest.raises(_abi.FerryError):
            d.store_create(0, 0)
        d.store_create(2, 1)
        with pytest.raises(_abi.FerryError):
            d.store_create(2, 1)                          # one store per ctx
        with pytest.raises(_abi.FerryError):
            d.gather_source(7)
    finally:
        d.close()


def test_owner_gather_over_nvlink(torch_cuda):
    from ferry_b200 import _abi

    t = torch_cuda
    if t.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    w, decs = _job(t, 2, [0, 1])
    from ferry_b200.engine import Decoder

    host = Decoder(w, 0)
    try:
        host.register_pool()
        dev = t.device("cuda", 0)
        reqs = list(range(w.num_requests))
        decs[0].gather_source(_abi.SRC_OWNER)
        decs[0].all_stats(reset=True)
        a = _run(t, decs[0], w, reqs, 2, dev)
        b = _run(t, host, w, reqs, 2, dev)
        for x, y in zip(a, b):
            assert (x.view(np.uint32) == y.view(np.uint32)).all()
        st = decs[0].all_stats()
        assert st[4] > 0 and st[4] + st[6] == st[0]
    finally:
        host.close()
        for d in decs:
            d.close()


def _stores_only_job(t, world, kv_dtype, select_mode):
    """The same job with no host pool: every rank's store filled and linked,
    summaries from the stores."""
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    w = small(num_requests=4, num_layers=2, q_heads=8, kv_heads=2, ctx_tokens=2048, top_k=24,
              kv_dtype=kv_dtype)
    decs = [Decoder(w, 0, select_mode=select_mode) for _ in range(world)]
    for r, d in enumerate(decs):
        d.store_create(world, r)
        d.register_stores(w.pool_units)
        d.store_fill(pool_units=w.pool_units)
    t.cuda.synchronize()
    for r, d in enumerate(decs):
        slot = 0
        for p, e in enumerate(decs):
            if p != r:
                _abi.call("ferry_ctx_link", d.ctx, slot, e.ctx)
                slot += 1
    return w, decs


@pytest.mark.parametrize("world,kv_dtype,mode", [(1, "e4m3", 0), (3, "e4m3", 0), (2, "f16", 1), (4, "f16", 0)])
def test_stores_only_job_matches_host_pool(torch_cuda, world, kv_dtype, mode):
    """ferry_kv_register_stores + ferry_page_summary_from_stores: summaries
    (mean rows or Quest bounds), cache bytes and decode outputs bit-identical
    to the host-pool path on the same content."""
    from ferry_b200.engine import Decoder

    t = torch_cuda
    dev = t.device("cuda", 0)
    w, decs = _stores_only_job(t, world, kv_dtype, mode)
    host = Decoder(w, 0, select_mode=mode)
    try:
        host.register_pool()
        reqs = list(range(w.num_requests))
        ids = t.from_numpy(np.asarray(reqs, np.int32)).to(dev)
        d = decs[0]
        d.begin(ids, t.full((len(reqs),), w.max_pages, dtype=t.int32, device=dev))
        d.summaries_from_stores(ids)
        t.cuda.synchronize()
        d.check()
        row = 256 if mode == 1 else 128
        sa = d.debug_read(4, np.float32, w.pool_units * row)
        sb = host.debug_read(4, np.float32, w.pool_units * row)
        assert (sa.view(np.uint32) == sb.view(np.uint32)).all()
        d.all_stats(reset=True)
        outs = []
        for s in range(3):
            out = t.zeros((len(reqs), w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
            d.step(t.from_numpy(_q(w, reqs, s)).to(dev), ids, out)
            outs.append(out.cpu().numpy())
        t.cuda.synchronize()
        d.check()
        ref = _run(t, host, w, reqs, 3, dev)
        for x, y in zip(outs, ref):
            assert (x.view(np.uint32) == y.view(np.uint32)).all()
        n = w.num_requests * w.lanes_per_req * w.cache_pages * w.unit_bytes
        assert (d.debug_read(0, np.uint8, n) == host.debug_read(0, np.uint8, n)).all()
        st = d.all_stats()
        assert st[0] > 0 and st[4] + st[6] == st[0]  # every miss from a store
    finally:
        host.close()
        for x in decs:
            x.close()


def test_stores_only_rejects_host_paths_and_unmapped_owners(torch_cuda):
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    t = torch_cuda
    dev = t.device("cuda", 0)
    w = small(num_requests=2, ctx_tokens=1024, top_k=16)
    d = Decoder(w, 0)
    try:
        with pytest.raises(_abi.FerryError):
            d.register_stores(w.pool_units)               # no store yet
        d.store_create(2, 0)                               # rank 1 is never linked
        d.register_stores(w.pool_units)
        d.store_fill(pool_units=w.pool_units)
        with pytest.raises(_abi.FerryError):
            d.gather_source(_abi.SRC_HOST)                # there is no host pool
        with pytest.raises(_abi.FerryError):
            d.register_pool()                             # nor can one be added
        ids = t.tensor([0, 1], dtype=t.int32, device=dev)
        d.begin(ids, t.full((2,), w.max_pages, dtype=t.int32, device=dev))
        d.summaries_from_stores(ids)
        t.cuda.synchronize()
        with pytest.raises(_abi.FerryError) as e:         # the odd pages have no mapped owner
            d.check()
        assert e.value.code == _abi.E_RANGE
    finally:
        d.close()


@pytest.mark.parametrize("world,kv_dtype,chunks", [(2, "e4m3", 3), (3, "f16", 4), (1, "f16", 2)])
def test_pipelined_step_matches_plain_step(torch_cuda, world, kv_dtype, chunks):
    """ferry_step_chunks: each chunk's selection on the caller's stream
    overlaps the previous chunk's detect / gather / attention on the ctx's
    side stream; outputs, cache bytes and gather counts equal the plain
    step's."""
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder

    t = torch_cuda
    dev = t.device("cuda", 0)
    w, decs = _job(t, world, [0] * world, kv_dtype)
    plain = Decoder(w, 0)
    try:
        plain.register_pool()
        reqs = list(range(w.num_requests))
        decs[0].gather_source(_abi.SRC_OWNER)
        decs[0].step_chunks(chunks)
        decs[0].all_stats(reset=True)
        a = _run(t, decs[0], w, reqs, 4, dev)
        b = _run(t, plain, w, reqs, 4, dev)
        for x, y in zip(a, b):
            assert (x.view(np.uint32) == y.view(np.uint32)).all()
        n = w.num_requests * w.lanes_per_req * w.cache_pages * w.unit_bytes
        assert (decs[0].debug_read(0, np.uint8, n) == plain.debug_read(0, np.uint8, n)).all()
        assert decs[0].all_stats()[0] == plain.all_stats()[0] > 0
        with pytest.raises(_abi.FerryError):
            decs[0].step_chunks(17)
    finally:
        plain.close()
        for d in decs:
            d.close()
