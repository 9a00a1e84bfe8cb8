"""Workload B on the GPU (csrc/taskb.cu): every executor (A, B, C and C's
ablations) over both transports leaves exactly the outputs the reference's
executor computes from the same task stream and payload pool -- the CPU
restatement of the task kernel over the same batch plan, bit for bit -- and
moves every payload byte once, in the plan's number of transfers."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


CASES = [("A", "p2p", {}), ("B", "p2p", {}), ("C", "p2p", {}), ("C", "p2p", {"adaptive": False, "max_mb": 1.0}),
         ("C", "p2p", {"overlap": False}), ("A", "host", {}), ("B", "host", {}), ("C", "host", {}),
         ("C", "host", {"overlap": False, "pending_ahead": 2})]


def _check(tb, tasks, p, st):
    import oracle
    from ferry_b200 import taskb

    plan = taskb.plan(p, tb.n, tb.payload)
    exp = oracle.taskb_expected(tasks, plan, p.inner_scale)
    got = tb.results()
    assert (got.view(np.uint32) == exp.view(np.uint32)).all()
    assert st["migrations"] == len(plan)
    assert st["migrated_bytes"] == tb.n * tb.payload
    assert st["makespan_ms"] >= st["arrival_span_ms"]
    assert 0.0 <= st["p50_ms"] <= st["p99_ms"] <= st["makespan_ms"]
    assert st["throughput"] > 0


@pytest.mark.parametrize("mode,transport,kw", CASES)
def test_executor_outputs_match_reference_semantics(torch_cuda, mode, transport, kw):
    from ferry_b200 import taskb

    tasks = taskb.generate(taskb.spec("bursty", "low", "imbalanced", 3000), 42)
    tb = taskb.TaskB(tasks, 0, 0)
    try:
        p = taskb.params(mode, transport, inner_scale=2, tick_ms=0.001, **kw)
        _check(tb, tasks, p, tb.run(p))
        # a second run on the same pool (outputs cleared) gives the same outputs
        tb.reset()
        _check(tb, tasks, p, tb.run(p))
    finally:
        tb.close()


@pytest.mark.parametrize("arrival,sparsity", [("steady", "high"), ("skewed", "medium")])
def test_every_arrival_and_payload_size(torch_cuda, arrival, sparsity):
    from ferry_b200 import taskb

    tasks = taskb.generate(taskb.spec(arrival, sparsity, "balanced", 2048), 7)
    tb = taskb.TaskB(tasks, 0, 0)
    try:
        for mode in ("A", "B", "C"):
            tb.reset()
            p = taskb.params(mode, "p2p", tick_ms=0.0005)
            _check(tb, tasks, p, tb.run(p))
    finally:
        tb.close()


def test_two_gpus_over_nvlink_and_host(torch_cuda):
    """Payloads on GPU 1, compute on GPU 0: the copy kernel reads GPU 1's HBM
    over NVLink; the host-staged ring copies device to host on GPU 1 and host
    to device on GPU 0."""
    from ferry_b200 import taskb

    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    tasks = taskb.generate(taskb.spec("steady", "medium", "imbalanced", 4096, num_gpus=2), 3)
    tb = taskb.TaskB(tasks, 1, 0)
    try:
        for transport in ("p2p", "host"):
            for mode in ("A", "B", "C"):
                tb.reset()
                p = taskb.params(mode, transport, tick_ms=0.0005)
                _check(tb, tasks, p, tb.run(p))
    finally:
        tb.close()


def test_run_synthetic_driver(torch_cuda):
    """The C++ driver (drivers/run_synthetic.cpp, the reference's
    run_synthetic CLI on the C ABI) prints the A / B / C rows and C's
    speed-ups for a scenario."""
    import os
    import subprocess

    from ferry_b200 import build

    exe = [p for p in build.build_drivers() if os.path.basename(p) == "run_synthetic"][0]
    for transport in ("p2p", "host"):
        out = subprocess.run([exe, "--arrival", "bursty", "--sparsity", "low", "--tasks", "4096", "--tick", "0.001",
                              "--transport", transport], capture_output=True, text=True, timeout=300)
        assert out.returncode == 0, out.stderr
        rows = [ln for ln in out.stdout.splitlines() if "makespan=" in ln]
        assert [r.split()[0] for r in rows] == ["baseline-A", "baseline-B", "ferry-C"]
        assert "=> C vs A:" in out.stdout
        # every row moved the whole pool (4096 tasks x 4 KB = 16 MB)
        assert all("bytes=    16.00MB" in r for r in rows), rows
