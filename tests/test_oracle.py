"""Pin the CPU oracle against the reference's own golden numbers, fixtures and
compiled host code (oracle/_ref). No GPU needed."""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _numbers():
    with open(os.path.join(GOLDEN, "reference_numbers.json")) as f:
        return json.load(f)


def test_default_stream_matches_published_numbers(oracle_lib):
    """refill 1242.97 MB, hit 0.865, 79550 misses (mode-B segments), 9216 MB
    mode A (results/wla_7rep_20260930/wla_bursty_balanced_r1.log:2-9)."""
    o = oracle_lib
    g = _numbers()
    blocks, miss, tot = o.replay_miss_stream(o.miss_spec())
    assert int(tot[0]) == 48 * 16 * 12 * 64
    assert int(tot[1]) == g["mode_B_refill_segments"]
    assert round(int(tot[2]) / 2**20, 2) == g["refill_MB"]
    assert round(1 - int(tot[1]) / int(tot[0]), 3) == g["hit_rate"]
    assert round(int(tot[0]) * 16384 / 2**20, 2) == g["mode_A_refill_MB"]


def test_mode_c_gather_plan_segments(oracle_lib):
    """Sort/unique/adaptive-batch/run-merge plan gives the published 59863
    refill segments and unchanged bytes."""
    o = oracle_lib
    sp = o.miss_spec()
    blocks, miss, tot = o.replay_miss_stream(sp)
    segs, nbytes = o.gather_plan_totals(sp, blocks, miss)
    assert segs == _numbers()["mode_C_refill_segments"]
    assert nbytes == int(tot[2])


def test_prefix_sharing_numbers(oracle_lib):
    """prefix group 4 / 8 steps: hit 0.921, trace baseline 731.31 MB
    (results/wla_pathdep_20261018/base_s42.log:12,14)."""
    o = oracle_lib
    sp = o.miss_spec(prefix_group=4, prefix_steps=8)
    blocks, _, _ = o.replay_miss_stream(sp)
    _, tot = o.prefix_share_stats(sp, blocks)
    g = _numbers()["prefix_grp4_stp8"]
    assert round(1 - int(tot[1]) / int(tot[0]), 3) == g["hit_rate"]
    assert round(int(tot[2]) / 2**20, 2) == g["trace_baseline_MB"]


def test_restatement_equals_reference_code(oracle_lib):
    o = oracle_lib
    if o.ref_lib() is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    for kw in [{}, dict(R=5, L=3, S=20, sel=32, hot=40, seed=7), dict(seed=123, hot=64)]:
        sp = o.miss_spec(**kw)
        b, m, t = o.replay_miss_stream(sp)
        rb, rm, rt = o.ref_replay_miss_stream(sp)
        assert (b == rb).all() and (m == rm).all() and (t == rt).all()
    for mb in [0.0, 0.5, 3.9, 4.0, 7.5, 16.0, 100.0]:
        assert o.lib().orc_choose_mb(mb, 1.0, 4.0, 4.0) == o.ref_lib().ref_choose_mb(mb)


def test_fixture_small_stream(oracle_lib):
    """The committed fixture (made by tests/golden/make_golden.py from the
    reference code) equals the restatement."""
    o = oracle_lib
    z = np.load(os.path.join(GOLDEN, "refstream_small.npz"))
    R, L, S, sel, hot, kv, d, seed = [int(x) for x in z["spec"]]
    b, m, t = o.replay_miss_stream(o.miss_spec(R=R, L=L, S=S, sel=sel, hot=hot, kv=kv, d=d, seed=seed))
    assert (b == z["blocks"]).all() and (m == z["is_miss"]).all() and (t == z["totals"]).all()


def test_lru_lanes_reproduce_reference_hits(oracle_lib):
    """The page-table LRU lanes give the reference's is_miss sequence on its
    own block stream, duplicates included."""
    o = oracle_lib
    sp = o.miss_spec()
    blocks, miss, _ = o.replay_miss_stream(sp)
    R, S, L, G = 48, 16, 12, 64
    B = blocks.reshape(R, S, L, G).astype(np.int32)
    M = miss.reshape(R, S, L, G)
    lr = o.LruLanes(R * L, sp.hot_blocks, 64 + 8 * S)
    lanes = np.arange(R * L, dtype=np.int32)
    for s in range(S):
        im, islot, mp, ms, nm = lr.step(lanes, B[:, s].reshape(R * L, G))
        assert (im == M[:, s].reshape(R * L, G)).all()
        assert (nm == im.sum(1)).all()
    # state invariants: size <= cap, page table consistent with the order
    for lane in [0, 5, R * L - 1]:
        ps, order, size = lr.state(lane)
        assert size <= sp.hot_blocks and len(set(order.tolist())) == size
        resident = np.nonzero(ps >= 0)[0]
        assert sorted(ps[resident].tolist()) == sorted(order.tolist())


def test_lru_slot_rule_and_intra_step_eviction(oracle_lib):
    o = oracle_lib
    lr = o.LruLanes(1, 2, 10)
    lane = np.zeros(1, np.int32)
    im, islot, mp, ms, nm = lr.step(lane, np.array([[3, 5]], np.int32))
    assert im.tolist() == [[1, 1]] and islot.tolist() == [[0, 1]]
    # [C, A] on a full cache [A, B]: C evicts A (front), then A misses and evicts B
    lr2 = o.LruLanes(1, 2, 10)
    lr2.step(lane, np.array([[1, 2]], np.int32))            # A=1 -> slot0, B=2 -> slot1
    im, islot, mp, ms, nm = lr2.step(lane, np.array([[7, 1]], np.int32))
    assert im.tolist() == [[1, 1]]
    assert islot.tolist() == [[0, 1]]                       # 7 takes A's slot, A takes B's
    ps, order, size = lr2.state(0)
    assert ps[7] == 0 and ps[1] == 1 and ps[2] == -1 and order.tolist() == [0, 1]
    # reset empties the lane
    im, islot, *_ = lr2.step(lane, np.array([[1, 7]], np.int32), reset=np.ones(1, np.uint8))
    assert im.tolist() == [[1, 1]] and islot.tolist() == [[0, 1]]


def test_kv_gen_is_deterministic_and_standard(oracle_lib):
    o = oracle_lib
    a = o.kv_gen(42, 1000, 8)
    b = o.kv_gen(42, 1000, 8)
    assert (a == b).all()
    x = a.view(np.float16).astype(np.float64).ravel()
    assert abs(x.mean()) < 0.05 and 0.9 < x.std() < 1.1 and np.abs(x).max() <= 6.0
    # values are k / 65536 rounded to fp16: first element pinned across machines
    assert int(o.lib().orc_kv_elem(42, 0, 0)) == int(o.kv_gen(42, 0, 1)[0, 0])


def test_select_topk_ties_and_order(oracle_lib):
    o = oracle_lib
    rng = np.random.default_rng(1)
    summ = rng.standard_normal((2, 40, 128)).astype(np.float32)
    q = np.zeros((2, 1, 128), np.float16).view(np.uint16)
    sel, ns = o.select_topk(q, summ, [40, 10], 8)
    # all-zero q: every score is 0 -> the k lowest page ids, ascending
    assert sel[0].tolist() == list(range(8)) and ns.tolist() == [8, 8]
    sel, ns = o.select_topk(q, summ, [40, 5], 8)
    assert ns.tolist() == [8, 5] and sel[1].tolist() == [0, 1, 2, 3, 4, -1, -1, -1]
    qf = rng.standard_normal((2, 1, 128)).astype(np.float16)
    sel, ns, sc = o.select_topk(qf.view(np.uint16), summ, [40, 40], 8, return_scores=True)
    for i in range(2):
        top = np.argsort(-sc[i, :40], kind="stable")[:8]
        assert sel[i].tolist() == sorted(top.tolist())


def test_attention_oracle_against_numpy(oracle_lib):
    o = oracle_lib
    rng = np.random.default_rng(2)
    pages = rng.standard_normal((3, 4, 2 * 16 * 128)).astype(np.float16)
    q = rng.standard_normal((3, 2, 128)).astype(np.float16)
    n_sel = np.array([4, 2, 1], np.int32)
    out = o.sparse_decode(q.view(np.uint16), pages.view(np.uint16), n_sel, 128 ** -0.5)
    for i in range(3):
        K = pages[i, : n_sel[i], : 2048].reshape(-1, 128).astype(np.float64)
        V = pages[i, : n_sel[i], 2048:].reshape(-1, 128).astype(np.float64)
        for g in range(2):
            lg = K @ q[i, g].astype(np.float64) / np.sqrt(128)
            p = np.exp(lg - lg.max())
            ref = (p / p.sum()) @ V
            np.testing.assert_allclose(out[i, g], ref, rtol=1e-5, atol=1e-6)


def test_cpu_pipeline_runs(oracle_lib):
    o = oracle_lib
    lanes, N, C_, k = 4, 32, 8, 8
    pool = o.kv_gen(5, 0, lanes * N)
    summ = o.page_summary(pool).reshape(lanes, N, 128)
    pipe = o.CpuPipeline(lanes, N, C_, k, 1, pool, summ, threads=2)
    rng = np.random.default_rng(3)
    q = rng.standard_normal((lanes, 1, 128)).astype(np.float16).view(np.uint16)
    out, misses = pipe.step(np.arange(lanes, dtype=np.int32), q)
    assert misses == lanes * k and np.isfinite(out).all()
    out2, misses2 = pipe.step(np.arange(lanes, dtype=np.int32), q)
    assert misses2 == 0 and np.allclose(out, out2)
