"""Decode appends on the GPU (B200 only): every step adds its token to the
request's context; a page becomes selectable when its 16th token arrives and
its summary is computed then (ferry_requests_append / ferry_decode_appends).

Against the oracle, step after step: the context in whole pages, selections,
miss lists, slots and gathered bytes bit-exact, attention within 2e-3. The
fused step with appends equals the separate calls plus ferry_requests_append
bit for bit; a request migrated in the middle of a page keeps its partial
page; contexts stop at max_pages; the CPU pipeline with growing contexts gives
the GPU's outputs."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ATTN_RTOL = 2e-3


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _q(w, reqs, step):
    from ferry_b200.workload import q_stream

    return np.stack([q_stream(w, int(r), steps=step + 1)[step] for r in reqs])


def _rel_err(gpu, ref):
    g = gpu.reshape(-1, 128).astype(np.float64)
    r = ref.reshape(-1, 128).astype(np.float64)
    return float((np.abs(g - r).max(1) / np.maximum(np.abs(r).max(1), 1e-30)).max())


@pytest.mark.parametrize("kv_dtype,shape,quest", [
    ("f16", dict(q_heads=4, kv_heads=4), False),
    ("f16", dict(q_heads=8, kv_heads=2, cache_frac=0.5), False),
    ("e4m3", dict(q_heads=16, kv_heads=2), False),
    ("f16", dict(q_heads=8, kv_heads=2), True),
])
def test_appends_match_oracle(torch_cuda, kv_dtype, shape, quest):
    import oracle
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import pages_after, small

    t = torch_cuda
    # 5 tokens per step: a page fills every 3-4 steps; 12 steps add 3-4 pages
    w = small(kv_dtype=kv_dtype, ctx_tokens=1024, top_k=16, steps=12, append=5, **shape)
    assert w.max_pages == 64 + 4 and w.init_pages == 64
    dev = t.device("cuda", 0)
    LH, N, k, C_, U, UB, G = (w.lanes_per_req, w.max_pages, w.top_k, w.cache_pages, w.pool_units,
                              w.unit_bytes, w.group)
    dec = Decoder(w, 0, select_mode=_abi.SELECT_QUEST if quest else _abi.SELECT_MEAN)
    try:
        pool = dec.register_pool()
        f8 = kv_dtype == "e4m3"
        units = pool.numpy(np.uint8).reshape(U, UB)
        if quest:
            summ = oracle.page_minmax_e4m3(units) if f8 else oracle.page_minmax(units.view(np.uint16))
        else:
            summ = oracle.page_summary_e4m3(units) if f8 else oracle.page_summary(units.view(np.uint16))
        R = w.num_requests
        reqs = np.arange(R, dtype=np.int32)
        init = np.array([w.init_pages, w.init_pages - 3, k - 1, 2], np.int32)[:R]
        ids = t.from_numpy(reqs).to(dev)
        dec.begin(ids, t.from_numpy(init).to(dev))
        lru = oracle.LruLanes(R * LH, C_, N)
        gl = (reqs[:, None] * LH + np.arange(LH)[None]).ravel()
        nl = R * LH
        for step in range(w.steps):
            pages = pages_after(init, step, w.append, N)
            state = dec.debug_read(5, np.int32, 2 * R)
            assert (state[:R] == pages).all(), step
            # the partial page's tokens (a full context keeps none)
            assert (state[R:] == np.where(pages < N, (step * w.append) % 16, 0)).all(), step
            qn = _q(w, reqs, step)
            q = t.from_numpy(qn).to(dev)
            out = t.zeros((R, w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
            dec.select(q, ids)
            dec.detect(ids)
            dec.gather(ids)
            dec.attention(q, ids, out)
            dec.append(ids)
            t.cuda.synchronize()
            dec.check()
            if quest:
                grp = gl.reshape(R * w.num_layers, w.kv_heads)
                mm = summ[(grp[:, :, None] * N + np.arange(N)[None, None]) % U]
                sel_g, ns_g = oracle.select_quest(qn.reshape(R * w.num_layers, w.q_heads, 128), w.kv_heads, mm,
                                                  np.repeat(pages, w.num_layers), k)
                sel_ref, ns_ref = np.repeat(sel_g, w.kv_heads, 0), np.repeat(ns_g, w.kv_heads)
            else:
                sel_ref, ns_ref = oracle.select_topk(qn.reshape(nl, G, 128).view(np.uint16),
                                                     summ[(gl[:, None] * N + np.arange(N)[None]) % U],
                                                     np.repeat(pages, LH), k)
            assert (dec.n_sel[:nl].cpu().numpy() == ns_ref).all(), step
            assert (dec.sel[:nl].cpu().numpy() == sel_ref).all(), step
            im, islot, mp, ms, nm = lru.step(gl.astype(np.int32), sel_ref, n_sel=ns_ref)
            assert (dec.n_miss[:nl].cpu().numpy() == nm).all()
            assert (dec.item_slot[:nl].cpu().numpy() == islot).all()
            cache = dec.debug_read(0, np.uint8, nl * C_ * UB).reshape(-1, UB)
            js = np.arange(k)[None] < ns_ref[:, None]
            sel_units = cache[gl[:, None] * C_ + np.where(js, islot, 0)]
            want = units[(gl[:, None] * N + np.where(js, sel_ref, 0)) % U]
            assert (sel_units[js] == want[js]).all()
            if f8:
                pg = oracle.e4m3_dequant(sel_units.reshape(-1, UB)).reshape(nl, k, 4096)
                ref = oracle.sparse_decode_f32(qn.reshape(nl, G, 128), pg, ns_ref, 128 ** -0.5)
            else:
                ref = oracle.sparse_decode(qn.reshape(nl, G, 128).view(np.uint16), sel_units.view(np.uint16),
                                           ns_ref, 128 ** -0.5)
            assert _rel_err(out.cpu().numpy(), ref) <= ATTN_RTOL, step
        # every request grew: the last ones by whole pages since they started short
        final = dec.debug_read(5, np.int32, 2 * R)[:R]
        assert (final == pages_after(init, w.steps, w.append, N)).all() and (final > init).all()
    finally:
        dec.close()


def test_fused_step_appends_like_separate_calls(torch_cuda):
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    t = torch_cuda
    w = small(q_heads=8, kv_heads=2, steps=20, append=3)
    a, b = Decoder(w, 0), Decoder(w, 0)
    try:
        dev = t.device("cuda", 0)
        reqs = np.arange(w.num_requests, dtype=np.int32)
        ids = t.from_numpy(reqs).to(dev)
        for d in (a, b):
            d.register_pool()
            d.begin(ids, t.full((len(reqs),), w.init_pages - 2, dtype=t.int32, device=dev))
        for step in range(w.steps):
            q = t.from_numpy(_q(w, reqs, step)).to(dev)
            oa = t.zeros((len(reqs), w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
            ob = t.zeros_like(oa)
            a.select(q, ids)
            a.detect(ids)
            a.gather(ids)
            a.attention(q, ids, oa)
            a.append(ids)
            b.step(q, ids, ob)  # appends w.append tokens itself
            t.cuda.synchronize()
            assert (oa.cpu().numpy().view(np.uint32) == ob.cpu().numpy().view(np.uint32)).all(), step
        sa, sb = a.debug_read(5, np.int32, 2 * w.num_requests), b.debug_read(5, np.int32, 2 * w.num_requests)
        assert (sa == sb).all() and (sa[: w.num_requests] > w.init_pages - 2).all()
        a.check()
        b.check()
    finally:
        a.close()
        b.close()


def test_contexts_stop_at_max_pages(torch_cuda):
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    t = torch_cuda
    w = small(num_requests=2, steps=4, append=16)  # room for 4 more pages
    d = Decoder(w, 0)
    try:
        dev = t.device("cuda", 0)
        d.register_pool()
        ids = t.tensor([0, 1], dtype=t.int32, device=dev)
        d.begin(ids, t.tensor([w.max_pages - 2, 3], dtype=t.int32, device=dev))
        d.append(ids, 7)
        d.append(ids, 16 * 10)
        t.cuda.synchronize()
        d.check()
        st = d.debug_read(5, np.int32, 2 * w.num_requests)
        assert st[0] == w.max_pages and st[2] == 0            # full: no partial page kept
        assert st[1] == min(w.max_pages, 3 + (7 + 160) // 16) and st[3] == (7 + 160) % 16
    finally:
        d.close()


def test_migration_keeps_the_partial_page(torch_cuda):
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    t = torch_cuda
    w = small(num_requests=4, steps=12, append=5)
    src, dst = Decoder(w, 0), Decoder(w, 0)
    try:
        dev = t.device("cuda", 0)
        for d in (src, dst):
            d.register_pool()
            ids = t.arange(4, dtype=t.int32, device=dev)
            d.begin(ids, t.full((4,), w.init_pages, dtype=t.int32, device=dev))
        ids = t.arange(4, dtype=t.int32, device=dev)
        out = t.zeros((4, w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
        for s in range(3):  # 15 tokens: the partial page holds 15
            src.step(t.from_numpy(_q(w, range(4), s)).to(dev), ids, out)
        _abi.call("ferry_ctx_link", dst.ctx, 0, src.ctx)
        s_ids, d_ids = t.tensor([2], dtype=t.int32, device=dev), t.tensor([1], dtype=t.int32, device=dev)
        _abi.call("ferry_migrate_requests", dst.ctx, C.c_void_p(t.cuda.current_stream().cuda_stream), 0,
                  C.c_void_p(s_ids.data_ptr()), C.c_void_p(d_ids.data_ptr()), 1, _abi.MIGRATE_DELTA)
        t.cuda.synchronize()
        a, b = src.debug_read(5, np.int32, 8), dst.debug_read(5, np.int32, 8)
        assert b[1] == a[2] and b[4 + 1] == a[4 + 2] == 15
        # both sides decode request 2 onward identically (the next token completes the page)
        o1 = t.zeros((1, w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
        o2 = t.zeros_like(o1)
        for s in (3, 4):
            q = t.from_numpy(_q(w, [2], s)).to(dev)
            src.step(q, s_ids, o1)
            dst.step(q, d_ids, o2)
            t.cuda.synchronize()
            assert (o1.cpu().numpy().view(np.uint32) == o2.cpu().numpy().view(np.uint32)).all()
        src.check()
        dst.check()
    finally:
        dst.close()
        src.close()


def test_cpu_pipeline_with_growing_contexts_matches_gpu(torch_cuda):
    """The timed CPU baseline's pipeline (oracle) and the GPU's fused step over
    the same job ticks with appends: the bench's parity check, on a small job."""
    import importlib.util
    import os

    from ferry_b200.engine import Decoder
    from ferry_b200.workload import Schedule, q_stream, small

    t = torch_cuda
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    w = small(num_requests=4, num_layers=1, q_heads=8, kv_heads=4, steps=10, append=4, arrival_rate=100.0)
    sch = Schedule(w)
    _, _, _, per_tick = bench.cpu_baseline(w, threads=2, ticks=sch.length, keep=sch.length)
    dev = t.device("cuda", 0)
    dec = Decoder(w, 0)
    try:
        dec.register_pool()
        qs = [q_stream(w, r) for r in range(w.num_requests)]
        n_pages = t.full((w.num_requests,), w.init_pages, dtype=t.int32, device=dev)
        outs = []
        dec.stats(reset=True)
        for i in range(sch.length):
            active, steps, _ = sch.tick(i)
            if len(active) == 0:
                outs.append(None)
                continue
            new = active[steps == 0]
            if len(new):
                dec.begin(t.from_numpy(new).to(dev), n_pages[: len(new)])
            q = t.from_numpy(np.stack([qs[r][s] for r, s in zip(active, steps)])).to(dev)
            out = t.zeros((len(active), 1, w.q_heads, 128), dtype=t.float32, device=dev)
            dec.step(q, t.from_numpy(active).to(dev), out)
            outs.append(out.cpu().numpy())
        t.cuda.synchronize()
        dec.check()
        units = dec.stats()[0]
    finally:
        dec.close()
    p = bench.parity_vs_cpu(w, outs, units, per_tick)
    assert p["status"] == "ok", p
