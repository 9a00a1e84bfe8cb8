"""Workload B on the CPU: the task-stream generator of the C ABI against the
reference's own (golden fixture, and live where oracle/_ref is built), the
executor's batch plan against the reference's policy, argument checks."""
import ast
import ctypes as C
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "taskb_tasks.npz")


def test_generator_matches_reference_fixture(cuda_lib):
    from ferry_b200 import taskb

    g = np.load(GOLDEN)
    for i, c in enumerate(g["cases"]):
        arrival, sparsity, skew, total, ng, frac, cards, seed = ast.literal_eval(str(c))
        t = taskb.generate(taskb.spec(arrival, sparsity, skew, total, ng, frac, cards), seed)
        assert (t["arrive_t"] == g[f"{i}_arrive_t"]).all(), c
        assert (t["payload"] == g[f"{i}_payload"]).all(), c
        assert (t["work"] == g[f"{i}_work"]).all(), c
        assert (t["dest"] == g[f"{i}_dest"]).all(), c


def test_generator_matches_reference_live(cuda_lib, oracle_lib):
    from ferry_b200 import taskb

    if oracle_lib.ref_lib() is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    for arrival in ("steady", "bursty", "skewed"):
        for sparsity in ("low", "medium", "high"):
            for skew in ("balanced", "imbalanced"):
                for ng in (1, 3, 8):
                    t = taskb.generate(taskb.spec(arrival, sparsity, skew, 2000, ng), 11)
                    a, p, w, d = oracle_lib.ref_generate_tasks(arrival, sparsity, skew, 2000, ng, 0.8, 0, 11)
                    assert (t["arrive_t"] == a).all() and (t["payload"] == p).all()
                    assert (t["work"] == w).all() and (t["dest"] == d).all()


def test_trace_arrivals_taken_as_given(cuda_lib):
    from ferry_b200 import taskb

    ticks = np.cumsum(np.linspace(0.5, 2.0, 300))
    t = taskb.generate(taskb.spec("trace", "low", "imbalanced", 300), 5, trace_ticks=ticks)
    assert (t["arrive_t"] == ticks).all()
    # the work draws are the same as any other arrival mode's with this seed
    s = taskb.generate(taskb.spec("steady", "low", "imbalanced", 300), 5)
    assert (t["work"] == s["work"]).all()


def test_batch_plan_follows_the_adaptive_policy(oracle_lib):
    from ferry_b200 import _abi, taskb

    n, payload = 65536, 16 << 10
    pc = taskb.params("C")
    plan = taskb.plan(pc, n, payload)
    assert sum(c for _, c in plan) == n and plan[0][0] == 0
    assert all(a + c == b for (a, c), (b, _) in zip(plan, plan[1:]))
    # choose_mb of the reference (adaptive_batch.cuh:31-36) with its default
    # policy (1..4 MB, 4 target batches) sets every batch but the last
    R = oracle_lib.ref_lib()
    pol = taskb.params("C", target_batches=4.0)
    off = 0
    for off, cnt in taskb.plan(pol, n, payload)[:-1]:
        mb = (n - off) * payload / (1 << 20)
        g = R.ref_choose_mb(mb) if R is not None else min(max(mb / 4.0, 1.0), 4.0)
        assert cnt == max(int(g * (1 << 20)) // payload, 64)
    assert taskb.plan(taskb.params("A"), n, payload) == [(0, n)]
    b = taskb.plan(taskb.params("B", stride=64), 1000, payload)
    assert len(b) == 16 and b[-1] == (960, 40)
    fixed = taskb.plan(taskb.params("C", adaptive=False, max_mb=2.0), n, payload)
    assert {c for _, c in fixed[:-1]} == {128}
    assert pc.mode == _abi.TASKB_C


def test_bad_arguments_rejected_without_gpu(cuda_lib):
    from ferry_b200 import _abi, taskb

    out = np.zeros(4, taskb.TASK_DTYPE)
    bad = taskb.spec(total=4)
    bad.arrival = 7
    assert cuda_lib.ferry_taskb_generate(C.byref(bad), 1, None, out.ctypes.data_as(C.c_void_p)) == _abi.E_INVAL
    tr = taskb.spec("trace", total=4)
    assert cuda_lib.ferry_taskb_generate(C.byref(tr), 1, None, out.ctypes.data_as(C.c_void_p)) == _abi.E_INVAL
    h = C.c_void_p()
    assert cuda_lib.ferry_taskb_create(0, 0, None, 4, C.byref(h)) == _abi.E_INVAL
    t = taskb.generate(taskb.spec(total=4), 1)
    t["payload"][2] = 4096  # one payload size per stream
    assert cuda_lib.ferry_taskb_create(0, 0, t.ctypes.data_as(C.c_void_p), 4, C.byref(h)) == _abi.E_INVAL
    st = _abi.TaskbStats()
    p = taskb.params("C")
    assert cuda_lib.ferry_taskb_run(None, C.byref(p), C.byref(st)) == _abi.E_INVAL
