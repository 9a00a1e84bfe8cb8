"""e4m3 KV path (per-page fp32 scales) on the GPU vs the CPU oracle:
quantised pool bytes and page summaries bit-exact, selections / miss lists /
slots / gathered bytes bit-exact, and the tcgen05 GQA attention within 2e-3
relative error per output row against fp64 attention over the dequantised
pages."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ATTN_RTOL = 2e-3
UB = 4112


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


def _q(w, reqs, step):
    from ferry_b200.workload import q_stream

    return np.stack([q_stream(w, int(r), steps=step + 1)[step] for r in reqs])


def test_e4m3_pool_and_summaries_bit_exact(torch_cuda):
    import oracle
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    w = small(num_requests=2, kv_dtype="e4m3")
    dec = Decoder(w, 0)
    try:
        pool = dec.register_pool()
        U = w.pool_units
        units = pool.numpy(np.uint8).reshape(U, UB)
        for u in [0, 3, U // 2, U - 1]:
            assert (units[u] == oracle.kv_gen_e4m3(w.seed, u, 1)[0]).all(), u
        summ = dec.debug_read(4, np.float32, U * 128).reshape(U, 128)
        ref = oracle.page_summary_e4m3(units)
        assert (summ.view(np.uint32) == ref.view(np.uint32)).all()
    finally:
        dec.close()


@pytest.mark.parametrize("shape", [
    dict(q_heads=32, kv_heads=4),                    # GQA group 8 (the long-context config)
    dict(q_heads=8, kv_heads=2, cache_frac=0.5),     # group 4
    dict(q_heads=4, kv_heads=2),                     # group 2: one head per softmax warpgroup
    dict(q_heads=4, kv_heads=4),                     # group 1
    dict(q_heads=32, kv_heads=4, n_pages="edge"),    # no page, one page, k - 1, full
])
def test_e4m3_decode_matches_oracle(torch_cuda, shape):
    import oracle
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    t = torch_cuda
    shape = dict(shape)
    edge = shape.pop("n_pages", None) == "edge"
    w = small(kv_dtype="e4m3", ctx_tokens=2048, top_k=40, **shape)
    dec = Decoder(w, 0)
    try:
        pool = dec.register_pool()
        U, N, LH, k = w.pool_units, w.max_pages, w.lanes_per_req, w.top_k
        units = pool.numpy(np.uint8).reshape(U, UB)
        summ = oracle.page_summary_e4m3(units)
        dq = oracle.e4m3_dequant(units)
        n_pages = np.array([0, 1, k - 1, N] if edge else [N, N - 7, k - 9, k], np.int32)[: w.num_requests]
        reqs = np.arange(w.num_requests, dtype=np.int32)
        dev = t.device("cuda", 0)
        dec.begin(t.from_numpy(reqs).to(dev), t.from_numpy(n_pages).to(dev))
        lru = oracle.LruLanes(w.num_requests * LH, w.cache_pages, N)
        for step in range(3):
            qn = _q(w, reqs, step)
            q = t.from_numpy(qn).to(dev)
            ids = t.from_numpy(reqs).to(dev)
            out = t.zeros((len(reqs), w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
            dec.select(q, ids)
            dec.detect(ids)
            dec.gather(ids)
            dec.attention(q, ids, out)
            t.cuda.synchronize()
            dec.check()
            nl = len(reqs) * LH
            gl = (reqs[:, None] * LH + np.arange(LH)[None]).ravel()
            idx = (gl[:, None].astype(np.int64) * N + np.arange(N)[None]) % U
            sel_ref, ns_ref = oracle.select_topk(qn.reshape(nl, w.group, 128).view(np.uint16), summ[idx],
                                                 np.repeat(n_pages, LH), k)
            assert (dec.sel[:nl].cpu().numpy() == sel_ref).all()
            im, islot, mp, ms, nm = lru.step(gl.astype(np.int32), sel_ref, n_sel=ns_ref)
            assert (dec.item_slot[:nl].cpu().numpy() == islot).all()
            assert (dec.n_miss[:nl].cpu().numpy() == nm).all()
            pages = np.zeros((nl, k, 4096), np.float32)
            for a in range(nl):
                for j in range(ns_ref[a]):
                    unit = (int(gl[a]) * N + int(sel_ref[a, j])) % U
                    cached = dec.debug_read(0, np.uint8, UB, offset_elems=(int(gl[a]) * w.cache_pages + int(islot[a, j])) * UB)
                    assert (cached == units[unit]).all()
                    pages[a, j] = dq[unit]
            ref = oracle.sparse_decode_f32(qn.reshape(nl, w.group, 128), pages, ns_ref, 128 ** -0.5)
            err = _rel_err(out.cpu().numpy().reshape(nl, w.group, 128), ref)
            assert err <= ATTN_RTOL, (step, err)
    finally:
        dec.close()


def test_e4m3_fused_step_equals_separate(torch_cuda):
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    t = torch_cuda
    w = small(kv_dtype="e4m3", q_heads=32, kv_heads=4, ctx_tokens=2048, top_k=40)
    a, b = Decoder(w, 0), Decoder(w, 0)
    try:
        dev = t.device("cuda", 0)
        reqs = np.arange(w.num_requests, dtype=np.int32)
        for d in (a, b):
            d.register_pool()
            d.begin(t.from_numpy(reqs).to(dev), t.full((len(reqs),), w.max_pages, dtype=t.int32, device=dev))
        for step in range(2):
            q = t.from_numpy(_q(w, reqs, step)).to(dev)
            ids = t.from_numpy(reqs).to(dev)
            oa = t.zeros((len(reqs), w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
            ob = t.zeros_like(oa)
            a.select(q, ids)
            a.detect(ids)
            a.gather(ids)
            a.attention(q, ids, oa)
            b.step(q, ids, ob)
            t.cuda.synchronize()
            assert (oa.cpu().numpy().view(np.uint32) == ob.cpu().numpy().view(np.uint32)).all()
        a.check()
        b.check()
    finally:
        a.close()
        b.close()
