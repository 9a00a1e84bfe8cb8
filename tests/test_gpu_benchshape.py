"""Parity at the shapes the bench times (B200 only).

* the exact configs[0] job (``WORKLOADS["cfg1"]``): its Schedule, its AR(1)
  queries and its 1 GiB procedural pool, tick after tick from the first
  arrival until all 16 requests decode together (512 lanes, N = 256, k = 64,
  C = 64);
* four requests of the configs[4] slice at its true per-lane shape (N = 8192,
  k = 512, C = 1229, GQA group 8, e4m3 KV with per-page scales) with misses
  gathered from the page-owner store (world 1);
* the LRU alone at that shape: 1229 slots, selections of 512 distinct pages out
  of 8192 with ~256 misses (and, once full, evictions) per lane per step.

Selections, miss lists, slot assignment, page tables and gathered bytes are
compared bit for bit with the CPU oracle; attention within 2e-3 relative error
per output row (fp32 accumulation), as in the small-shape parity tests.
"""
import ctypes as C
import dataclasses

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


def _rel_err(gpu, ref):
    g = gpu.reshape(-1, 128).astype(np.float64)
    r = ref.reshape(-1, 128).astype(np.float64)
    return float((np.abs(g - r).max(1) / np.maximum(np.abs(r).max(1), 1e-30)).max())


def _glanes(reqs, LH):
    reqs = np.asarray(reqs, np.int64)
    return (reqs[:, None] * LH + np.arange(LH)[None]).ravel()


def _check_tables(dec, lru, w, gl):
    """Page table, LRU order and size of every lane in gl vs the oracle."""
    N, C_ = w.max_pages, w.cache_pages
    lanes = w.num_requests * w.lanes_per_req
    ps = dec.debug_read(1, np.int32, lanes * N).reshape(lanes, N)
    order = dec.debug_read(2, np.int32, lanes * C_).reshape(lanes, C_)
    size = dec.debug_read(3, np.int32, lanes)
    for lane in gl:
        r_ps, r_order, r_size = lru.state(int(lane))
        assert size[lane] == r_size, lane
        assert (ps[lane] == r_ps).all(), lane
        assert (order[lane, :r_size] == r_order).all(), lane


def test_cfg1_job_ticks_match_oracle(torch_cuda):
    """The bench's own job, ticks 0..T: every intermediate bit-exact and the
    attention within tolerance, with a fused-step decoder alongside that must
    give bit-identical outputs, and a fused step pipelined over three request
    chunks (ferry_step_chunks, what the bench times) whose selections, miss
    lists and slots must be bit-identical and whose attention -- split over
    warps by each chunk's own size, so rounded differently -- must meet the
    same tolerance against the oracle."""
    import oracle
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import WORKLOADS, Schedule, q_stream

    t = torch_cuda
    w = WORKLOADS["cfg1"]
    dev = t.device("cuda", 0)
    LH, N, k, C_, U = w.lanes_per_req, w.max_pages, w.top_k, w.cache_pages, w.pool_units
    sep, fus, pipe = Decoder(w, 0), Decoder(w, 0), Decoder(w, 0)
    try:
        pool = sep.register_pool()
        fus.register_pool()
        pipe.register_pool()
        pipe.step_chunks(3)
        units = pool.numpy(np.uint16).reshape(U, 4096)
        summ = oracle.page_summary(units)
        gpu_summ = sep.debug_read(4, np.float32, U * 128).reshape(U, 128)
        assert (gpu_summ.view(np.uint32) == summ.view(np.uint32)).all()
        lru = oracle.LruLanes(w.num_requests * LH, C_, N)
        sch = Schedule(w)
        qs = [q_stream(w, r) for r in range(w.num_requests)]
        n_pages = t.full((w.num_requests,), N, dtype=t.int32, device=dev)
        full_batches = checked = total_miss = 0
        i = 0
        while full_batches < 3:
            active, steps, job = sch.tick(i)
            i += 1
            assert job == 0
            if len(active) == 0:
                continue
            new = active[steps == 0]
            if len(new):
                nid = t.from_numpy(new).to(dev)
                for d in (sep, fus, pipe):
                    d.begin(nid, n_pages[: len(new)])
                gln = _glanes(new, LH).astype(np.int32)
                lru.step(gln, np.zeros((len(gln), k), np.int32), n_sel=np.zeros(len(gln), np.int32),
                         reset=np.ones(len(gln), np.uint8))
            n = len(active)
            qn = np.stack([qs[r][s] for r, s in zip(active, steps)])
            q = t.from_numpy(qn).to(dev)
            ids = t.from_numpy(active).to(dev)
            out = t.zeros((n, 1, w.q_heads, 128), dtype=t.float32, device=dev)
            out_f = t.zeros_like(out)
            out_p = t.zeros_like(out)
            sep.select(q, ids)
            sep.detect(ids)
            sep.gather(ids)
            sep.attention(q, ids, out)
            fus.step(q, ids, out_f)
            pipe.step(q, ids, out_p)
            t.cuda.synchronize()
            sep.check()
            fus.check()
            pipe.check()
            assert (out.cpu().numpy().view(np.uint32) == out_f.cpu().numpy().view(np.uint32)).all()
            nl = n * LH
            gl = _glanes(active, LH)
            idx = (gl[:, None] * N + np.arange(N)[None]) % U
            sel_ref, ns_ref = oracle.select_topk(qn.reshape(nl, 1, 128).view(np.uint16), summ[idx],
                                                 np.full(nl, N, np.int32), k)
            assert (sep.n_sel[:nl].cpu().numpy() == ns_ref).all()
            assert (sep.sel[:nl].cpu().numpy() == sel_ref).all()
            # the pipelined step's workspace (selections, slots, miss lists and
            # counts of every lane) equals the plain fused step's
            ws_words = w.num_requests * LH * (4 * k + 2)
            assert (pipe.debug_read(6, np.int32, ws_words) == fus.debug_read(6, np.int32, ws_words)).all()
            im, islot, mp, ms, nm = lru.step(gl.astype(np.int32), sel_ref, n_sel=ns_ref)
            assert (sep.n_miss[:nl].cpu().numpy() == nm).all()
            assert (sep.is_miss[:nl].cpu().numpy() == im).all()
            assert (sep.item_slot[:nl].cpu().numpy() == islot).all()
            gmp, gms = sep.miss_page[:nl].cpu().numpy(), sep.miss_slot[:nl].cpu().numpy()
            mask = np.arange(k)[None] < nm[:, None]
            assert (gmp[mask] == mp[mask]).all() and (gms[mask] == ms[mask]).all()
            _check_tables(sep, lru, w, gl)
            # gathered bytes: every selected page's slot holds its pool unit
            cache = sep.debug_read(0, np.uint16, w.num_requests * LH * C_ * 4096).reshape(-1, 4096)
            pages = cache[gl[:, None] * C_ + islot]
            assert (pages == units[(gl[:, None] * N + sel_ref) % U]).all()
            ref = oracle.sparse_decode(qn.reshape(nl, 1, 128).view(np.uint16), pages, ns_ref, 128 ** -0.5)
            err = _rel_err(out.cpu().numpy(), ref)
            assert err <= ATTN_RTOL, (i, err)
            err_p = _rel_err(out_p.cpu().numpy(), ref)
            assert err_p <= ATTN_RTOL, (i, err_p)
            checked += 1
            total_miss += int(nm.sum())
            full_batches += int(n == w.num_requests)
        assert checked >= 3 and total_miss > 0
        nlanes = w.num_requests * LH
        for which, count in ((1, nlanes * N), (2, nlanes * C_), (3, nlanes)):
            assert (pipe.debug_read(which, np.int32, count) == fus.debug_read(which, np.int32, count)).all()
    finally:
        sep.close()
        fus.close()
        pipe.close()


def test_cfg5s_requests_at_true_lane_shape_match_oracle(torch_cuda):
    """Four requests of the configs[4] slice (64 lanes of N = 8192, k = 512,
    C = 1229, G = 8, e4m3), misses from this GPU's page-owner store, three
    steady decode steps."""
    import oracle
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import CFG5S, q_stream

    t = torch_cuda
    w = dataclasses.replace(CFG5S, num_requests=4)
    assert (w.max_pages, w.top_k, w.cache_pages, w.group) == (8192, 512, 1229, 8)
    dev = t.device("cuda", 0)
    LH, N, k, C_, U, UB = w.lanes_per_req, w.max_pages, w.top_k, w.cache_pages, w.pool_units, w.unit_bytes
    dec = Decoder(w, 0)
    try:
        pool = dec.register_pool()
        dec.store_create(1, 0)
        dec.store_fill()
        dec.gather_source(_abi.SRC_OWNER)
        units = pool.numpy(np.uint8).reshape(U, UB)
        summ = oracle.page_summary_e4m3(units)
        reqs = np.arange(w.num_requests, dtype=np.int32)
        ids = t.from_numpy(reqs).to(dev)
        dec.begin(ids, t.full((len(reqs),), N, dtype=t.int32, device=dev))
        nl = len(reqs) * LH
        gl = _glanes(reqs, LH)
        lru = oracle.LruLanes(nl, C_, N)
        qs = [q_stream(w, int(r), steps=3) for r in reqs]
        dec.all_stats(reset=True)
        for step in range(3):
            qn = np.stack([qs[r][step] for r in reqs])
            q = t.from_numpy(qn).to(dev)
            out = t.zeros((len(reqs), w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
            dec.select(q, ids)
            dec.detect(ids)
            dec.gather(ids)
            dec.attention(q, ids, out)
            t.cuda.synchronize()
            dec.check()
            sel_ref, ns_ref = oracle.select_topk(qn.reshape(nl, w.group, 128).view(np.uint16),
                                                 summ[(gl[:, None] * N + np.arange(N)[None]) % U],
                                                 np.full(nl, N, np.int32), k)
            assert (dec.sel[:nl].cpu().numpy() == sel_ref).all()
            im, islot, mp, ms, nm = lru.step(gl.astype(np.int32), sel_ref, n_sel=ns_ref)
            assert (dec.n_miss[:nl].cpu().numpy() == nm).all()
            assert (dec.item_slot[:nl].cpu().numpy() == islot).all()
            gmp, gms = dec.miss_page[:nl].cpu().numpy(), dec.miss_slot[:nl].cpu().numpy()
            mask = np.arange(k)[None] < nm[:, None]
            assert (gmp[mask] == mp[mask]).all() and (gms[mask] == ms[mask]).all()
            _check_tables(dec, lru, w, gl)
            cache = dec.debug_read(0, np.uint8, nl * C_ * UB).reshape(-1, UB)
            got = out.cpu().numpy().reshape(nl, w.group, 128)
            for a0 in range(0, nl, 16):  # dequantise 16 lanes at a time (bounded host memory)
                a1 = min(nl, a0 + 16)
                sel_units = cache[gl[a0:a1, None] * C_ + islot[a0:a1]]
                assert (sel_units == units[(gl[a0:a1, None] * N + sel_ref[a0:a1]) % U]).all()
                pages = oracle.e4m3_dequant(sel_units.reshape(-1, UB)).reshape(a1 - a0, k, 4096)
                ref = oracle.sparse_decode_f32(qn.reshape(nl, w.group, 128)[a0:a1], pages, ns_ref[a0:a1],
                                               128 ** -0.5)
                err = _rel_err(got[a0:a1], ref)
                assert err <= ATTN_RTOL, (step, a0, err)
        st = dec.all_stats()
        assert st[0] > 0 and st[6] == st[0] and st[4] == 0  # every miss from the own store
    finally:
        dec.close()


def test_lru_at_configs4_lane_shape(torch_cuda):
    """1229 slots, 512 distinct ascending pages of 8192 per step, half of them
    new each step: the warp-parallel eviction path at the benchmarked shape."""
    import oracle
    from ferry_b200 import _abi

    t = torch_cuda
    rng = np.random.default_rng(1229)
    lanes_n, cap, ids, k = 64, 1229, 8192, 512
    h = C.c_void_p()
    _abi.call("ferry_lru_create", 0, lanes_n, cap, ids, C.byref(h))
    mirror = oracle.LruLanes(lanes_n, cap, ids)
    prev = [rng.choice(ids, k, replace=False) for _ in range(lanes_n)]
    dev = t.device("cuda", 0)
    st = t.cuda.current_stream()
    p = lambda x: C.c_void_p(x.data_ptr())
    misses = 0
    try:
        for s in range(10):
            sel = np.empty((lanes_n, k), np.int32)
            for ln in range(lanes_n):
                keep = prev[ln][rng.random(k) < 0.5]
                fresh = rng.choice(np.setdiff1d(np.arange(ids), keep), k - len(keep), replace=False)
                prev[ln] = np.sort(np.concatenate([keep, fresh]))
                sel[ln] = prev[ln]
            lanes = t.arange(lanes_n, dtype=t.int32, device=dev)
            d_sel = t.from_numpy(sel).to(dev)
            d_ns = t.full((lanes_n,), k, dtype=t.int32, device=dev)
            im = t.zeros((lanes_n, k), dtype=t.uint8, device=dev)
            isl, mp, ms = (t.full((lanes_n, k), -1, dtype=t.int32, device=dev) for _ in range(3))
            nm = t.zeros(lanes_n, dtype=t.int32, device=dev)
            _abi.call("ferry_lru_touch", h, C.c_void_p(st.cuda_stream), p(lanes), None, lanes_n, p(d_sel), k,
                      p(d_ns), _abi.LRU_DISTINCT, p(im), p(isl), p(mp), p(ms), p(nm))
            t.cuda.synchronize()
            rim, risl, rmp, rms, rnm = mirror.step(np.arange(lanes_n, dtype=np.int32), sel)
            nm_h = nm.cpu().numpy()
            assert (nm_h == rnm).all()
            assert (im.cpu().numpy() == rim).all() and (isl.cpu().numpy() == risl).all()
            mask = np.arange(k)[None] < rnm[:, None]
            assert (mp.cpu().numpy()[mask] == rmp[mask]).all() and (ms.cpu().numpy()[mask] == rms[mask]).all()
            if s >= 3:
                misses += int(nm_h.sum())
        for lane in range(lanes_n):
            ps = np.zeros(ids, np.int32)
            order = np.zeros(cap, np.int32)
            size = np.zeros(1, np.int32)
            _abi.call("ferry_lru_read", h, lane, ps.ctypes.data_as(C.c_void_p),
                      order.ctypes.data_as(C.c_void_p), size.ctypes.data_as(C.c_void_p))
            r = mirror.state(lane)
            assert (ps == r[0]).all() and (order[: size[0]] == r[1]).all() and size[0] == r[2]
        # lanes fill (1229 slots) during the fourth step; from then on every
        # miss evicts, ~256 per lane and step
        assert misses / (7 * lanes_n) > 200
    finally:
        _abi.call("ferry_lru_destroy", h)
