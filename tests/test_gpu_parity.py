"""CUDA path vs the CPU oracle on the same seeded inputs (B200 only).

Selections, miss lists, page tables, slot assignment and gathered bytes must be
bit-exact; attention outputs within 2e-3 relative error, measured per output
row (lane, q head) as max|gpu - ref| / max|ref|.
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATTN_RTOL = 2e-3
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _rel_err(gpu, ref):
    g = gpu.reshape(-1, 128).astype(np.float64)
    r = ref.reshape(-1, 128).astype(np.float64)
    scale = np.maximum(np.abs(r).max(axis=1), 1e-30)
    return float((np.abs(g - r).max(axis=1) / scale).max())


class Harness:
    """A Decoder plus the oracle state that mirrors it."""

    def __init__(self, torch, w, n_pages=None, source=None):
        import oracle
        from ferry_b200.engine import Decoder

        self.t, self.w, self.o = torch, w, oracle
        self.dec = Decoder(w, 0)
        self.pool = self.dec.register_pool()
        if source is not None:
            self.dec.gather_source(source)
        U = w.pool_units
        self.units = self.pool.numpy(np.uint16).reshape(U, 4096)
        self.summ = oracle.page_summary(self.units)
        self.N, self.LH = w.max_pages, w.lanes_per_req
        self.lru = oracle.LruLanes(w.num_requests * self.LH, w.cache_pages, self.N)
        self.n_pages = np.full(w.num_requests, self.N, np.int32) if n_pages is None else np.asarray(n_pages, np.int32)
        self.dev = torch.device("cuda", 0)

    def begin(self, reqs):
        reqs = np.asarray(reqs, np.int32)
        t = self.t
        self.dec.begin(t.from_numpy(reqs).to(self.dev), t.from_numpy(self.n_pages[reqs]).to(self.dev))
        # mirror: empty the lanes in the oracle
        lanes = (reqs[:, None] * self.LH + np.arange(self.LH)[None]).ravel().astype(np.int32)
        k = self.w.top_k
        self.lru.step(lanes, np.zeros((len(lanes), k), np.int32), n_sel=np.zeros(len(lanes), np.int32),
                      reset=np.ones(len(lanes), np.uint8))

    def glanes(self, reqs):
        reqs = np.asarray(reqs, np.int32)
        return (reqs[:, None] * self.LH + np.arange(self.LH)[None]).ravel().astype(np.int32)

    def oracle_select(self, q, reqs):
        w = self.w
        gl = self.glanes(reqs)
        idx = (gl[:, None].astype(np.int64) * self.N + np.arange(self.N)[None]) % w.pool_units
        summ = self.summ[idx]
        npg = np.repeat(self.n_pages[np.asarray(reqs)], self.LH)
        qq = q.reshape(len(gl), w.group, 128).view(np.uint16)
        return self.o.select_topk(qq, summ, npg, w.top_k)

    def run_step(self, q_np, reqs, fused=False):
        t, w, dec = self.t, self.w, self.dec
        ids = t.from_numpy(np.asarray(reqs, np.int32)).to(self.dev)
        q = t.from_numpy(q_np).to(self.dev)
        out = t.zeros((len(reqs), w.num_layers, w.q_heads, 128), dtype=t.float32, device=self.dev)
        if fused:
            dec.step(q, ids, out)
        else:
            dec.select(q, ids)
            dec.detect(ids)
            dec.gather(ids)
            dec.attention(q, ids, out)
        t.cuda.synchronize()
        dec.check()
        return out.cpu().numpy()

    def check_step(self, q_np, reqs):
        """Separate-call step, every intermediate compared with the oracle."""
        w, dec = self.w, self.dec
        out = self.run_step(q_np, reqs)
        nl = len(reqs) * self.LH
        sel_ref, ns_ref = self.oracle_select(q_np, reqs)
        sel = dec.sel[:nl].cpu().numpy()
        ns = dec.n_sel[:nl].cpu().numpy()
        assert (ns == ns_ref).all()
        assert (sel == sel_ref).all()
        gl = self.glanes(reqs)
        im, islot, mp, ms, nm = self.lru.step(gl, sel_ref, n_sel=ns_ref)
        assert (dec.n_miss[:nl].cpu().numpy() == nm).all()
        assert (dec.is_miss[:nl].cpu().numpy() == im).all()
        assert (dec.item_slot[:nl].cpu().numpy() == islot).all()
        gmp, gms = dec.miss_page[:nl].cpu().numpy(), dec.miss_slot[:nl].cpu().numpy()
        for a in range(nl):
            assert (gmp[a, : nm[a]] == mp[a, : nm[a]]).all()
            assert (gms[a, : nm[a]] == ms[a, : nm[a]]).all()
        # gathered bytes: every selected page's slot holds that page's pool unit
        C_ = w.cache_pages
        pages = np.zeros((nl, w.top_k, 4096), np.uint16)
        for a in range(nl):
            for j in range(ns_ref[a]):
                unit = (int(gl[a]) * self.N + int(sel_ref[a, j])) % w.pool_units
                cached = dec.debug_read(0, np.uint16, 4096, offset_elems=(int(gl[a]) * C_ + int(islot[a, j])) * 4096)
                assert (cached == self.units[unit]).all()
                pages[a, j] = self.units[unit]
        ref = self.o.sparse_decode(q_np.reshape(nl, w.group, 128).view(np.uint16), pages, ns_ref, 128 ** -0.5)
        assert _rel_err(out.reshape(nl, w.group, 128), ref) <= ATTN_RTOL
        return out, int(nm.sum())

    def close(self):
        self.dec.close()


def _q(w, reqs, step, job=0):
    from ferry_b200.workload import q_stream

    return np.stack([q_stream(w, int(r), steps=step + 1, job=job)[step] for r in reqs])


def test_kvgen_and_summaries_bit_exact(torch_cuda):
    from ferry_b200.workload import small

    import oracle

    w = small(num_requests=2)
    h = Harness(torch_cuda, w)
    try:
        U = w.pool_units
        for u in [0, 1, 17, U // 2, U - 1]:
            assert (h.units[u] == oracle.kv_gen(w.seed, u, 1)[0]).all()
        gpu_summ = h.dec.debug_read(4, np.float32, U * 128).reshape(U, 128)
        assert (gpu_summ.view(np.uint32) == h.summ.view(np.uint32)).all()
    finally:
        h.close()


@pytest.mark.parametrize("shape", [
    dict(),                                            # G=1, C=k
    dict(q_heads=8, kv_heads=2, cache_frac=0.5),       # GQA group 4, C=2k
    dict(q_heads=8, kv_heads=1, ctx_tokens=2048, top_k=32, cache_frac=0.25),  # group 8
    # long lanes: selection scores them in several chunks (one CTA each)
    dict(num_layers=1, q_heads=8, kv_heads=1, ctx_tokens=65536, top_k=64),  # N 4096, G 8
    dict(num_layers=1, q_heads=4, kv_heads=2, ctx_tokens=40000, top_k=48),  # N 2500, G 2
    # the largest lanes of the 4-warp kernel (warp-level select over 1024 keys)
    # and the smallest of the 8-warp one (one chunk of 2048 pages)
    dict(num_layers=1, q_heads=4, kv_heads=4, ctx_tokens=16384, top_k=96),  # N 1024, G 1
    dict(num_layers=1, q_heads=4, kv_heads=4, ctx_tokens=32768, top_k=128),  # N 2048, G 1
])
def test_decode_steps_match_oracle(torch_cuda, shape):
    from ferry_b200.workload import small

    w = small(**shape)
    reqs = list(range(w.num_requests))
    n_pages = [w.max_pages, w.max_pages - 5, w.top_k // 2, w.top_k][: w.num_requests]
    h = Harness(torch_cuda, w, n_pages=n_pages)
    try:
        h.begin(reqs)
        misses = []
        for s in range(4):
            _, nm = h.check_step(_q(w, reqs, s), reqs)
            misses.append(nm)
        assert misses[0] > 0 and misses[1] < misses[0]    # warm cache after the first step
        # restart two requests mid-run: their lanes come back cold
        h.begin([1, 3])
        h.check_step(_q(w, reqs, 4, job=1), reqs)
        # a partial batch in a different order
        h.check_step(_q(w, [2, 0], 5), [2, 0])
    finally:
        h.close()


@pytest.mark.parametrize("shape", [dict(), dict(q_heads=8, kv_heads=2, cache_frac=0.5)])
def test_host_bulk_gather_matches_oracle(torch_cuda, shape):
    """FERRY_SRC_HOST_BULK: host-pool misses moved by TMA bulk copies land the
    same bytes in the same slots as the SM-load gather; every intermediate and
    the attention match the oracle, cold and warm steps, restarts and a
    partial batch."""
    from ferry_b200 import _abi
    from ferry_b200.workload import small

    w = small(**shape)
    reqs = list(range(w.num_requests))
    h = Harness(torch_cuda, w, n_pages=[w.max_pages, w.max_pages - 5, w.top_k // 2, w.top_k][: w.num_requests],
                source=_abi.SRC_HOST_BULK)
    try:
        h.begin(reqs)
        total = 0
        for s in range(3):
            total += h.check_step(_q(w, reqs, s), reqs)[1]
        h.begin([0, 2])
        total += h.check_step(_q(w, reqs, 3, job=1), reqs)[1]
        total += h.check_step(_q(w, [3, 1], 4), [3, 1])[1]
        assert total > 0 and h.dec.all_stats()[0] == total
    finally:
        h.close()


@pytest.mark.parametrize("shape", [dict(), dict(q_heads=8, kv_heads=2, cache_frac=0.5)])
def test_empty_and_single_page_contexts(torch_cuda, shape):
    """Requests with no page, one page and k - 1 pages beside a full one: the
    empty request's lanes select nothing, miss nothing and decode to exact
    zeros, and every other intermediate matches the oracle."""
    from ferry_b200.workload import small

    w = small(**shape)
    k, N = w.top_k, w.max_pages
    reqs = list(range(w.num_requests))
    h = Harness(torch_cuda, w, n_pages=[0, 1, k - 1, N][: w.num_requests])
    try:
        h.begin(reqs)
        for s in range(3):
            out, _ = h.check_step(_q(w, reqs, s), reqs)
            assert (out[0] == 0).all()
            assert (h.dec.n_sel[: h.LH].cpu().numpy() == 0).all()
    finally:
        h.close()


def test_longest_lane(torch_cuda):
    """Lanes of the maximum 16384 pages (16 selection chunks of 1024, the
    keys of a lane filling the shared-memory ring), GQA group 8."""
    from ferry_b200.workload import small

    w = small(num_requests=2, num_layers=1, q_heads=8, kv_heads=1, ctx_tokens=16384 * 16, top_k=64)
    assert w.max_pages == 16384
    reqs = [0, 1]
    h = Harness(torch_cuda, w, n_pages=[w.max_pages, w.max_pages - 3])
    try:
        h.begin(reqs)
        for s in range(2):
            h.check_step(_q(w, reqs, s), reqs)
    finally:
        h.close()


@pytest.mark.parametrize("ctx_tokens", [2048, 16384, 32768, 65536])
def test_select_ties_and_signed_zeros(torch_cuda, ctx_tokens):
    """All-zero queries score every page +-0 (ties everywhere, and -0 < +0 in
    key order); identical q heads tie the GQA maximum on every page. Lanes of
    128 and 1024 pages take the 4-warp kernel with the warp-level select,
    2048 pages the 8-warp kernel in one chunk, 4096 pages several chunks."""
    from ferry_b200.workload import small

    t = torch_cuda
    w = small(num_requests=3, num_layers=1, q_heads=8, kv_heads=2, ctx_tokens=ctx_tokens, top_k=40)
    h = Harness(t, w)
    try:
        reqs = [0, 1, 2]
        h.begin(reqs)
        q = _q(w, reqs, 0)
        q[0] = 0                                   # request 0: zero queries
        q[1, :, :, :] = q[1, :, :1, :]             # request 1: every head equal to head 0
        q[2, :, 1::2, :] = -q[2, :, 0::2, :]       # request 2: heads mirrored in each group
        ids = t.from_numpy(np.asarray(reqs, np.int32)).to(h.dev)
        h.dec.select(t.from_numpy(q).to(h.dev), ids)
        t.cuda.synchronize()
        h.dec.check()
        nl = len(reqs) * h.LH
        sel_ref, ns_ref = h.oracle_select(q, reqs)
        assert (h.dec.n_sel[:nl].cpu().numpy() == ns_ref).all()
        assert (h.dec.sel[:nl].cpu().numpy() == sel_ref).all()
    finally:
        h.close()


def test_fused_step_equals_separate_calls(torch_cuda):
    from ferry_b200.workload import small

    w = small()
    reqs = [0, 1, 2, 3]
    a, b = Harness(torch_cuda, w), Harness(torch_cuda, w)
    try:
        a.begin(reqs)
        b.begin(reqs)
        for s in range(3):
            q = _q(w, reqs, s)
            oa = a.run_step(q, reqs)
            ob = b.run_step(q, reqs, fused=True)
            assert (oa.view(np.uint32) == ob.view(np.uint32)).all()
        la = a.dec.debug_read(1, np.int32, w.num_requests * w.lanes_per_req * w.max_pages)
        lb = b.dec.debug_read(1, np.int32, w.num_requests * w.lanes_per_req * w.max_pages)
        assert (la == lb).all()
        ua, _ = a.dec.stats()
        ub, nb = b.dec.stats()
        assert ua == ub and nb == ub * 8192
    finally:
        a.close()
        b.close()


@pytest.mark.parametrize("shape,chunks", [(dict(), 2), (dict(), 4), (dict(q_heads=8, kv_heads=2, cache_frac=0.5), 3),
                                          (dict(kv_dtype="e4m3", q_heads=8, kv_heads=1, ctx_tokens=2048, top_k=40), 2)])
def test_pipelined_host_step_matches_oracle_checked_step(torch_cuda, shape, chunks):
    """ferry_step_chunks with host-pool gathers: chunk i's selection and miss
    detection on the caller's stream, chunk i-1's gather and chunk i-2's
    attention on the ctx's two streams. Outputs, page tables, cache bytes and
    gather counts equal those of a step whose every intermediate is checked
    against the oracle (fp16), or of the plain fused step (e4m3); full,
    partial and reordered batches, a restart in between."""
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    t = torch_cuda
    w = small(**shape)
    dev = t.device("cuda", 0)
    f16 = w.kv_dtype != "e4m3"
    a = Decoder(w, 0)
    b = Harness(t, w) if f16 else None
    pb = None if f16 else Decoder(w, 0)
    try:
        a.register_pool()
        a.step_chunks(chunks)
        if pb is not None:
            pb.register_pool()
        ref_dec = b.dec if f16 else pb

        def begin(reqs):
            ids = t.from_numpy(np.asarray(reqs, np.int32)).to(dev)
            a.begin(ids, t.full((len(reqs),), w.max_pages, dtype=t.int32, device=dev))
            if f16:
                b.begin(reqs)
            else:
                pb.begin(ids, t.full((len(reqs),), w.max_pages, dtype=t.int32, device=dev))

        def step(q, reqs):
            ids = t.from_numpy(np.asarray(reqs, np.int32)).to(dev)
            qd = t.from_numpy(q).to(dev)
            out = t.zeros((len(reqs), w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
            a.step(qd, ids, out)
            if f16:
                ref = b.check_step(q, reqs)[0]
            else:
                ro = t.zeros_like(out)
                pb.step(qd, ids, ro)
                ref = ro.cpu().numpy()
            t.cuda.synchronize()
            a.check()
            assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()

        reqs = list(range(w.num_requests))
        begin(reqs)
        for s in range(3):
            step(_q(w, reqs, s), reqs)
        begin([1, 2])
        step(_q(w, reqs, 3, job=1), reqs)
        step(_q(w, [3, 0, 2], 4), [3, 0, 2])
        nl = w.num_requests * w.lanes_per_req
        assert (a.debug_read(1, np.int32, nl * w.max_pages) == ref_dec.debug_read(1, np.int32, nl * w.max_pages)).all()
        n = nl * w.cache_pages * w.unit_bytes
        assert (a.debug_read(0, np.uint8, n) == ref_dec.debug_read(0, np.uint8, n)).all()
        assert a.stats()[0] == ref_dec.stats()[0] > 0
    finally:
        a.close()
        if b is not None:
            b.close()
        if pb is not None:
            pb.close()


def _lru_touch(torch, L, lanes, sel, n_sel=None, reset=None, distinct=False):
    from ferry_b200 import _abi

    dev = torch.device("cuda", 0)
    n, k = sel.shape
    d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    lanes_d, sel_d = d(lanes.astype(np.int32)), d(sel.astype(np.int32))
    ns_d = d(np.full(n, k, np.int32) if n_sel is None else n_sel.astype(np.int32))
    rs_d = None if reset is None else d(reset.astype(np.uint8))
    im = torch.zeros((n, k), dtype=torch.uint8, device=dev)
    isl, mp, ms = (torch.full((n, k), -1, dtype=torch.int32, device=dev) for _ in range(3))
    nm = torch.zeros(n, dtype=torch.int32, device=dev)
    p = lambda t: None if t is None else C.c_void_p(t.data_ptr())
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _abi.call("ferry_lru_touch", L, st, p(lanes_d), p(rs_d), n, p(sel_d), k, p(ns_d),
              _abi.LRU_DISTINCT if distinct else 0, p(im), p(isl), p(mp), p(ms), p(nm))
    torch.cuda.synchronize()
    return im.cpu().numpy(), isl.cpu().numpy(), mp.cpu().numpy(), ms.cpu().numpy(), nm.cpu().numpy()


def _lru_state(L, lane, ids, cap):
    from ferry_b200 import _abi

    ps = np.zeros(ids, np.int32)
    order = np.zeros(cap, np.int32)
    size = np.zeros(1, np.int32)
    _abi.call("ferry_lru_read", L, lane, ps.ctypes.data_as(C.c_void_p), order.ctypes.data_as(C.c_void_p),
              size.ctypes.data_as(C.c_void_p))
    return ps, order[: size[0]], int(size[0])


@pytest.mark.parametrize("which", ["fixture", "default"])
def test_lru_kernel_on_reference_block_stream(torch_cuda, which):
    """The device LRU replays the reference's own per-(request, layer) block
    stream (duplicates included) with the reference's exact hit/miss flags."""
    import oracle
    from ferry_b200 import _abi

    if which == "fixture":
        z = np.load(os.path.join(GOLDEN, "refstream_small.npz"))
        R, L_, S, G, hot = [int(x) for x in z["spec"][:5]]
        blocks, miss = z["blocks"], z["is_miss"]
    else:
        R, L_, S, G, hot = 48, 12, 16, 64, 128
        blocks, miss, tot = oracle.replay_miss_stream(oracle.miss_spec())
        assert int(tot[1]) == 79550
    ids = 64 + 8 * S
    B = blocks.reshape(R, S, L_, G).astype(np.int32)
    M = miss.reshape(R, S, L_, G)
    h = C.c_void_p()
    _abi.call("ferry_lru_create", 0, R * L_, hot, ids, C.byref(h))
    mirror = oracle.LruLanes(R * L_, hot, ids)
    try:
        lanes = np.arange(R * L_, dtype=np.int32)
        total_miss = 0
        for s in range(S):
            sel = B[:, s].reshape(R * L_, G)
            im, isl, mp, ms, nm = _lru_touch(torch_cuda, h, lanes, sel)
            assert (im == M[:, s].reshape(R * L_, G)).all()
            rim, risl, rmp, rms, rnm = mirror.step(lanes, sel)
            assert (isl == risl).all() and (nm == rnm).all()
            for a in range(0, R * L_, 7):
                assert (mp[a, : nm[a]] == rmp[a, : nm[a]]).all() and (ms[a, : nm[a]] == rms[a, : nm[a]]).all()
            total_miss += int(nm.sum())
        assert total_miss == int(M.sum())
        for lane in [0, 1, R * L_ // 2, R * L_ - 1]:
            g = _lru_state(h, lane, ids, hot)
            r = mirror.state(lane)
            assert (g[0] == r[0]).all() and (g[1] == r[1]).all() and g[2] == r[2]
    finally:
        _abi.call("ferry_lru_destroy", h)


def test_lru_kernel_over_capacity_and_resets(torch_cuda):
    """k > capacity (intra-step self eviction), resets and partial n_sel."""
    import oracle
    from ferry_b200 import _abi

    rng = np.random.default_rng(9)
    lanes_n, cap, ids, k = 16, 6, 40, 10
    h = C.c_void_p()
    _abi.call("ferry_lru_create", 0, lanes_n, cap, ids, C.byref(h))
    mirror = oracle.LruLanes(lanes_n, cap, ids)
    try:
        for s in range(12):
            lanes = rng.permutation(lanes_n)[:11].astype(np.int32)
            sel = rng.integers(0, ids, size=(11, k)).astype(np.int32)
            n_sel = rng.integers(0, k + 1, size=11).astype(np.int32)
            reset = (rng.random(11) < 0.2).astype(np.uint8)
            im, isl, mp, ms, nm = _lru_touch(torch_cuda, h, lanes, sel, n_sel, reset)
            rim, risl, rmp, rms, rnm = mirror.step(lanes, sel, n_sel=n_sel, reset=reset)
            for a in range(11):
                n = n_sel[a]
                assert (im[a, :n] == rim[a, :n]).all() and nm[a] == rnm[a]
                assert (mp[a, : nm[a]] == rmp[a, : nm[a]]).all()
        for lane in range(lanes_n):
            g, r = _lru_state(h, lane, ids, cap), mirror.state(lane)
            assert (g[0] == r[0]).all() and (g[1] == r[1]).all() and g[2] == r[2]
    finally:
        _abi.call("ferry_lru_destroy", h)


@pytest.mark.parametrize("cap,k,ids,reuse", [
    (48, 16, 200, 0.7),   # evictions reach only untouched pages: warp-parallel path
    (16, 16, 60, 0.5),    # cache = k: touched pages at the LRU front, serial replay
    (24, 16, 40, 0.9),    # mixed: some steps each way
    (300, 128, 2000, 0.5),  # decode-step shape: touched pages interleave the evicted front
    # lanes of more than 128 slots take the CTA-per-lane kernel: its parallel
    # path, its serial replay (cache = k) and a mix
    (400, 96, 3000, 0.7),
    (160, 160, 400, 0.5),
    (200, 128, 320, 0.9),
])
def test_lru_distinct_selections_both_paths(torch_cuda, cap, k, ids, reuse):
    """Distinct ascending selections (the decode step's case) against the
    sequential oracle, step after step, with partial selections and resets."""
    import oracle
    from ferry_b200 import _abi

    rng = np.random.default_rng(cap * 1000 + k)
    lanes_n = 24
    h = C.c_void_p()
    _abi.call("ferry_lru_create", 0, lanes_n, cap, ids, C.byref(h))
    mirror = oracle.LruLanes(lanes_n, cap, ids)
    prev = [rng.choice(ids, k, replace=False) for _ in range(lanes_n)]
    try:
        for s in range(20):
            lanes = rng.permutation(lanes_n)[:17].astype(np.int32)
            sel = np.full((17, k), -1, np.int32)
            for a, ln in enumerate(lanes):
                keep = prev[ln][rng.random(k) < reuse]
                fresh = rng.choice(np.setdiff1d(np.arange(ids), keep), k - len(keep), replace=False)
                pages = np.sort(np.concatenate([keep, fresh]))
                prev[ln] = pages
                sel[a] = pages
            n_sel = np.where(rng.random(17) < 0.8, k, rng.integers(0, k + 1, 17)).astype(np.int32)
            reset = (rng.random(17) < 0.05).astype(np.uint8)
            im, isl, mp, ms, nm = _lru_touch(torch_cuda, h, lanes, sel, n_sel, reset, distinct=True)
            rim, risl, rmp, rms, rnm = mirror.step(lanes, sel, n_sel=n_sel, reset=reset)
            for a in range(17):
                n = n_sel[a]
                assert nm[a] == rnm[a]
                assert (im[a, :n] == rim[a, :n]).all() and (isl[a, :n] == risl[a, :n]).all()
                assert (mp[a, : nm[a]] == rmp[a, : nm[a]]).all() and (ms[a, : nm[a]] == rms[a, : nm[a]]).all()
        for lane in range(lanes_n):
            g, r = _lru_state(h, lane, ids, cap), mirror.state(lane)
            assert (g[0] == r[0]).all() and (g[1] == r[1]).all() and g[2] == r[2]
    finally:
        _abi.call("ferry_lru_destroy", h)


def test_out_of_range_ids_are_reported_not_faulted(torch_cuda):
    from ferry_b200 import _abi

    h = C.c_void_p()
    _abi.call("ferry_lru_create", 0, 2, 4, 8, C.byref(h))
    try:
        sel = np.array([[1, 99, 2, -3]], np.int32)
        im, isl, mp, ms, nm = _lru_touch(torch_cuda, h, np.array([1], np.int32), sel)
        assert nm.tolist() == [2] and im.tolist() == [[1, 0, 1, 0]]
        ps = np.zeros(8, np.int32)
        order = np.zeros(4, np.int32)
        size = np.zeros(1, np.int32)
        rc = _abi.lib().ferry_lru_read(h, 1, ps.ctypes.data_as(C.c_void_p), order.ctypes.data_as(C.c_void_p),
                                       size.ctypes.data_as(C.c_void_p))
        assert rc == _abi.E_RANGE
        assert size[0] == 2 and ps[1] == 0 and ps[2] == 1
    finally:
        _abi.call("ferry_lru_destroy", h)


def test_empty_batch_and_bad_batch(torch_cuda):
    from ferry_b200 import FerryError
    from ferry_b200.workload import small

    w = small(num_requests=2)
    h = Harness(torch_cuda, w)
    try:
        t = torch_cuda
        ids = t.zeros(0, dtype=t.int32, device="cuda")
        q = t.zeros((0, w.num_layers, w.q_heads, 128), dtype=t.float16, device="cuda")
        out = t.zeros((0, w.num_layers, w.q_heads, 128), dtype=t.float32, device="cuda")
        h.dec.step(q, ids, out)
        with pytest.raises(FerryError):
            big = t.zeros(3, dtype=t.int32, device="cuda")
            h.dec.step(q, big, out)
        h.dec.check()
    finally:
        h.close()


def test_lru_kernel_replays_prefix_group_lanes(torch_cuda):
    """Prefix-group-shared LRU (the reference's kv_touch keyed by (GPU, prefix
    group, layer), wla_multigpu.cuh:1937-1962, and its statistics replay
    wla_recompute_stats, :376-417): every member of a group of 4 touches the
    group's lane, members in request order, the first 8 steps of each member
    being its group head's (wla_apply_prefix_sharing, :355-369). The device
    LRU on group lanes reproduces the oracle's totals and the reference's
    published hit rate 0.921 and 731.31 MB (results/wla_pathdep_20261018/
    base_s42.log:12,14)."""
    import oracle
    from ferry_b200 import _abi

    sp = oracle.miss_spec(prefix_group=4, prefix_steps=8)
    R, L_, S, G, hot, pg = sp.num_requests, sp.num_layers, sp.steps, sp.sel_blocks, sp.hot_blocks, 4
    blocks, _, _ = oracle.replay_miss_stream(sp)
    shared, tot = oracle.prefix_share_stats(sp, blocks)
    B = shared.reshape(R, S, L_, G).astype(np.int32)
    ngrp, ids = R // pg, 64 + 8 * S
    h = C.c_void_p()
    _abi.call("ferry_lru_create", 0, ngrp * L_, hot, ids, C.byref(h))
    try:
        lanes = (np.arange(ngrp)[:, None] * L_ + np.arange(L_)[None]).ravel().astype(np.int32)
        misses = 0
        for m in range(pg):  # members in request order; a member runs all its steps
            for s in range(S):
                sel = B[np.arange(ngrp) * pg + m, s].reshape(ngrp * L_, G)
                _, _, _, _, nm = _lru_touch(torch_cuda, h, lanes, sel)
                misses += int(nm.sum())
        assert misses == int(tot[1])
        selects = R * S * L_ * G
        c4 = 4 * 2 * sp.kv_heads * sp.head_dim * 2
        assert round(1.0 - misses / selects, 3) == 0.921
        assert round(misses * c4 / 1048576.0, 2) == 731.31
    finally:
        _abi.call("ferry_lru_destroy", h)
