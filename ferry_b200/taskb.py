"""Workload B host side: the reference's synthetic task stream and its A / B / C
executors (src/benches/run_synthetic.cu, src/workloads/baselines.cuh) on the
C ABI (``ferry_taskb_*``, csrc/taskb.cu).

``generate`` returns the task stream of a spec and seed as a numpy record
array; ``TaskB`` owns the payload pool (source GPU) and the compute buffers
(destination GPU) and runs one executor per ``run`` call, returning the
reference's ExecStats fields. ``plan`` is the executor's batch sequence
(task offset, count), which fixes what every run moves and which outputs its
kernels write.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _abi
from ._abi import call

ARRIVALS = {"steady": _abi.TASKB_STEADY, "bursty": _abi.TASKB_BURSTY, "skewed": _abi.TASKB_SKEWED,
            "trace": _abi.TASKB_TRACE}
SPARSITY = {"low": 0, "medium": 1, "high": 2}
MODES = {"A": _abi.TASKB_A, "B": _abi.TASKB_B, "C": _abi.TASKB_C}
TASK_DTYPE = np.dtype([("arrive_t", np.float64), ("payload", np.uint64), ("work", np.int32), ("dest", np.int32)])


def spec(arrival="steady", sparsity="medium", skew="balanced", total=1 << 16, num_gpus=1, dest_hot_frac=0.8,
         dest_hot_cards=0) -> _abi.TaskbSpec:
    """The reference's ArrivalSpec (synthetic.cuh:34-60) with its defaults."""
    return _abi.TaskbSpec(ARRIVALS[arrival], SPARSITY[sparsity], int(skew == "imbalanced"), num_gpus, total,
                          dest_hot_frac, dest_hot_cards, 0)


def generate(sp: _abi.TaskbSpec, seed: int = 42, trace_ticks: np.ndarray | None = None) -> np.ndarray:
    """generate_tasks (synthetic.cuh:83-173) for `sp` and `seed`."""
    out = np.zeros(sp.total, TASK_DTYPE)
    tr = None
    if trace_ticks is not None:
        trace_ticks = np.ascontiguousarray(trace_ticks, np.float64)
        tr = trace_ticks.ctypes.data_as(C.c_void_p)
    call("ferry_taskb_generate", C.byref(sp), C.c_uint64(seed), tr, out.ctypes.data_as(C.c_void_p))
    return out


def params(mode="C", transport="p2p", inner_scale=1, stride=64, tick_ms=0.01, pending_ahead=4, adaptive=True,
           overlap=True, min_mb=1.0, max_mb=4.0, target_batches=8.0) -> _abi.TaskbParams:
    """Executor parameters; the defaults are run_synthetic's (run_synthetic.cu:65-95:
    tick 0.01 ms, stride 64, pending 4, AdaptiveBatchPolicy 1..4 MB with 8
    target batches)."""
    tr = {"p2p": _abi.TASKB_P2P, "host": _abi.TASKB_HOST_STAGED}[transport]
    return _abi.TaskbParams(MODES[mode], tr, inner_scale, stride, tick_ms, pending_ahead, int(adaptive),
                            int(overlap), min_mb, max_mb, target_batches)


def plan(p: _abi.TaskbParams, n: int, payload: int) -> list[tuple[int, int]]:
    """(first task, tasks) of every batch the executor moves and computes."""
    if p.mode == _abi.TASKB_A:
        return [(0, n)]
    out, off = [], 0
    while off < n:
        if p.mode == _abi.TASKB_B:
            cnt = min(p.stride, n - off)
        elif p.adaptive:  # choose_batch over choose_mb (baselines.cuh:127-137, adaptive_batch.cuh:31-36)
            g = min(max((n - off) * payload / (1 << 20) / p.target_batches, p.min_mb), p.max_mb)
            by_bytes = max(int(g * (1 << 20)), 64 * payload)
            cnt = min(max(by_bytes // payload, 64), n - off)
        else:
            cnt = min(max(int(p.max_mb * (1 << 20)) // payload, 64), n - off)
        out.append((off, cnt))
        off += cnt
    return out


class TaskB:
    """Payload pool on `src`, compute buffers on `dst` (ferry_taskb_create)."""

    def __init__(self, tasks: np.ndarray, src: int = 0, dst: int = 0):
        self.tasks = np.ascontiguousarray(tasks, TASK_DTYPE)
        self.n = len(self.tasks)
        self.payload = int(self.tasks["payload"][0])
        self.h = C.c_void_p()
        call("ferry_taskb_create", src, dst, self.tasks.ctypes.data_as(C.c_void_p), C.c_uint64(self.n),
             C.byref(self.h))

    def run(self, p: _abi.TaskbParams) -> dict:
        st = _abi.TaskbStats()
        call("ferry_taskb_run", self.h, C.byref(p), C.byref(st))
        return {k: getattr(st, k) for k, _ in _abi.TaskbStats._fields_}

    def results(self, n_floats: int | None = None) -> np.ndarray:
        n = self.n * self.payload // 4 if n_floats is None else n_floats
        out = np.empty(n, np.float32)
        call("ferry_taskb_results", self.h, out.ctypes.data_as(C.c_void_p), C.c_uint64(n))
        return out

    def reset(self):
        call("ferry_taskb_reset", self.h)

    def close(self):
        if self.h:
            call("ferry_taskb_destroy", self.h)
            self.h = C.c_void_p()
