"""Regenerate tests/golden/taskb_tasks.npz (run where the reference tree is
present: it drives the reference's own generate_tasks, src/workloads/
synthetic.cuh:83-173, compiled into oracle/_ref by oracle/Makefile).

    python tests/golden/make_taskb_golden.py

For every case of CASES: the task stream's arrival ticks, payload bytes, work
counts and destination GPUs, as the reference generates them.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

# (arrival, sparsity, skew, total, num_gpus, hot_frac, hot_cards, seed)
CASES = [
    ("steady", "medium", "balanced", 1500, 1, 0.8, 0, 42),
    ("bursty", "low", "imbalanced", 1500, 4, 0.8, 0, 42),
    ("skewed", "high", "imbalanced", 1500, 8, 0.5, 2, 7),
    ("bursty", "medium", "balanced", 1500, 2, 0.8, 0, 123),
    ("skewed", "medium", "imbalanced", 1500, 5, 0.0, 0, 2026),
]


def main():
    oracle.build()
    out = {}
    for i, c in enumerate(CASES):
        r = oracle.ref_generate_tasks(*c)
        if r is None:
            raise SystemExit("oracle/_ref is not built: the reference tree is absent")
        for name, a in zip(("arrive_t", "payload", "work", "dest"), r):
            out[f"{i}_{name}"] = a
    out["cases"] = np.array([repr(c) for c in CASES])
    np.savez_compressed(os.path.join(HERE, "taskb_tasks.npz"), **out)
    print("wrote", os.path.join(HERE, "taskb_tasks.npz"))


if __name__ == "__main__":
    main()
