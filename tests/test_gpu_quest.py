"""Quest selection on the GPU (FERRY_SELECT_QUEST) against the reference's own
selector and the oracle (B200 only).

* the fixture cases: page sets that the reference's Selector.on_layer
  (method "quest", tools/capture_miss_trace.py:128-159) chose for the same keys
  and queries -- one set per (request, layer), repeated in every kv-head lane;
* procedural shapes, fp16 and e4m3 (configs[4] lane shape): bit-exact with the
  oracle restatement (same fixed arithmetic, so near-ties agree too), and a
  whole decode step driven by the Quest selection matches the oracle.
"""
import dataclasses
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATTN_RTOL = 2e-3
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quest_selector.npz")


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.mark.parametrize("name", ["cfg1_shape", "gqa8", "ragged", "few_pages"])
def test_quest_kernel_matches_reference_selector(torch_cuda, name):
    import oracle
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import Workload

    t = torch_cuda
    z = np.load(GOLDEN)
    R, L, Hq, Hkv, N, T, k = [int(x) for x in z[f"{name}_shape"]]
    w = Workload(name=name, num_requests=R, num_layers=L, q_heads=Hq, kv_heads=Hkv, ctx_tokens=N * 16,
                 top_k=k, cache_frac=0.5, steps=1, arrival_rate=1.0, seed=int(z["kv_seed"]))
    dev = t.device("cuda", 0)
    dec = Decoder(w, 0, select_mode=_abi.SELECT_QUEST)
    try:
        pool = dec.register_pool()
        U = w.pool_units
        mm = dec.debug_read(4, np.float32, U * 256).reshape(U, 256)
        ref_mm = oracle.page_minmax(pool.numpy(np.uint16).reshape(U, 4096))
        assert (mm.view(np.uint32) == ref_mm.view(np.uint32)).all()
        reqs = np.arange(R, dtype=np.int32)
        ids = t.from_numpy(reqs).to(dev)
        dec.begin(ids, t.full((R,), T // 16, dtype=t.int32, device=dev))
        q = t.from_numpy(z[f"{name}_q"].view(np.float16)).to(dev)  # [R][L][Hq][128]
        dec.select(q, ids)
        t.cuda.synchronize()
        dec.check()
        nl = R * L * Hkv
        sel = dec.sel[:nl].cpu().numpy().reshape(R, L, Hkv, k)
        ns = dec.n_sel[:nl].cpu().numpy()
        ref = z[f"{name}_sel"]
        assert (ns == min(T // 16, k)).all()
        for h in range(Hkv):
            assert (sel[:, :, h] == ref).all(), h
    finally:
        dec.close()


@pytest.mark.parametrize("kv_dtype,shape", [
    ("f16", dict(num_requests=3, num_layers=2, q_heads=32, kv_heads=32, ctx_tokens=4096, top_k=64)),
    ("f16", dict(num_requests=2, num_layers=2, q_heads=16, kv_heads=2, ctx_tokens=2048, top_k=24)),
    ("e4m3", dict(num_requests=2, num_layers=2, q_heads=64, kv_heads=8, ctx_tokens=131072, top_k=512)),
])
def test_quest_decode_step_matches_oracle(torch_cuda, kv_dtype, shape):
    """Selection bit-exact with the oracle (ragged contexts included), then the
    rest of the step (miss detect, gather, attention) over those pages."""
    import oracle
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import q_stream, small

    t = torch_cuda
    w = small(kv_dtype=kv_dtype, cache_frac=0.15 if shape["top_k"] == 512 else 0.25, **shape)
    dev = t.device("cuda", 0)
    LH, N, k, C_, U, UB = w.lanes_per_req, w.max_pages, w.top_k, w.cache_pages, w.pool_units, w.unit_bytes
    R, L, Hkv, G = w.num_requests, w.num_layers, w.kv_heads, w.group
    dec = Decoder(w, 0, select_mode=_abi.SELECT_QUEST)
    try:
        pool = dec.register_pool()
        f8 = kv_dtype == "e4m3"
        units = pool.numpy(np.uint8).reshape(U, UB)
        mm = oracle.page_minmax_e4m3(units) if f8 else oracle.page_minmax(units.view(np.uint16))
        reqs = np.arange(R, dtype=np.int32)
        n_pages = np.array([N, N - 37, k - 5][:R], np.int32)
        ids = t.from_numpy(reqs).to(dev)
        dec.begin(ids, t.from_numpy(n_pages).to(dev))
        lru = oracle.LruLanes(R * LH, C_, N)
        gl = (reqs[:, None] * LH + np.arange(LH)[None]).ravel()
        for step in range(2):
            qn = np.stack([q_stream(w, int(r), steps=step + 1)[step] for r in reqs])
            q = t.from_numpy(qn).to(dev)
            out = t.zeros((R, L, w.q_heads, 128), dtype=t.float32, device=dev)
            dec.select(q, ids)
            dec.detect(ids)
            dec.gather(ids)
            dec.attention(q, ids, out)
            t.cuda.synchronize()
            dec.check()
            grp_units = (gl.reshape(R * L, Hkv)[:, :, None] * N + np.arange(N)[None, None]) % U
            sel_g, ns_g = oracle.select_quest(qn.reshape(R * L, Hkv * G, 128), Hkv, mm[grp_units],
                                              np.repeat(n_pages, L), k)
            sel_ref = np.repeat(sel_g, Hkv, axis=0)
            ns_ref = np.repeat(ns_g, Hkv)
            nl = R * LH
            assert (dec.n_sel[:nl].cpu().numpy() == ns_ref).all()
            assert (dec.sel[:nl].cpu().numpy() == sel_ref).all()
            im, islot, mp, ms, nm = lru.step(gl.astype(np.int32), sel_ref, n_sel=ns_ref)
            assert (dec.n_miss[:nl].cpu().numpy() == nm).all()
            assert (dec.item_slot[:nl].cpu().numpy() == islot).all()
            cache = dec.debug_read(0, np.uint8, nl * C_ * UB).reshape(-1, UB)
            got = out.cpu().numpy().reshape(nl, G, 128)
            for a0 in range(0, nl, 16):
                a1 = min(nl, a0 + 16)
                js = np.arange(k)[None] < ns_ref[a0:a1, None]
                sl = np.where(js, islot[a0:a1], 0)
                sel_units = cache[gl[a0:a1, None] * C_ + sl]
                want = units[(gl[a0:a1, None] * N + np.where(js, sel_ref[a0:a1], 0)) % U]
                assert (sel_units[js] == want[js]).all()
                if f8:
                    pages = oracle.e4m3_dequant(sel_units.reshape(-1, UB)).reshape(a1 - a0, k, 4096)
                    ref = oracle.sparse_decode_f32(qn.reshape(nl, G, 128)[a0:a1], pages, ns_ref[a0:a1],
                                                   128 ** -0.5)
                else:
                    ref = oracle.sparse_decode(qn.reshape(nl, G, 128)[a0:a1].view(np.uint16),
                                               sel_units.view(np.uint16), ns_ref[a0:a1], 128 ** -0.5)
                g64, r64 = got[a0:a1].reshape(-1, 128).astype(np.float64), ref.reshape(-1, 128).astype(np.float64)
                err = float((np.abs(g64 - r64).max(1) / np.maximum(np.abs(r64).max(1), 1e-30)).max())
                assert err <= ATTN_RTOL, (step, a0, err)
    finally:
        dec.close()


def test_select_mode_rules(torch_cuda):
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import small

    d = Decoder(small(num_requests=2), 0)
    try:
        with pytest.raises(_abi.FerryError):
            _abi.call("ferry_select_mode", d.ctx, 9)
        d.register_pool()
        with pytest.raises(_abi.FerryError):  # after the pool: summaries already sized
            _abi.call("ferry_select_mode", d.ctx, _abi.SELECT_QUEST)
    finally:
        d.close()
