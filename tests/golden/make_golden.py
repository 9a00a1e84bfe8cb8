"""Regenerate the golden fixtures in this folder (run where the reference tree
is present: it drives the reference's own host headers compiled into
oracle/_ref).

    python tests/golden/make_golden.py

Writes:
  refstream_small.npz  replay_miss_stream (src/workloads/missstream.cuh:104-170)
                       of a small spec, straight from the reference code:
                       blocks and is_miss per event, plus totals.
  reference_numbers.json  the reference's published regression numbers for the
                       default synthetic stream, with their sources.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

SMALL = dict(R=4, L=3, S=8, sel=16, hot=32, kv=8, d=128, seed=42)


def main():
    oracle.build()
    sp = oracle.miss_spec(**SMALL)
    out = oracle.ref_replay_miss_stream(sp)
    if out is None:
        raise SystemExit("oracle/_ref is not built (reference tree absent)")
    blocks, miss, tot = out
    np.savez_compressed(os.path.join(HERE, "refstream_small.npz"), blocks=blocks,
                        is_miss=miss, totals=tot, spec=np.array(list(SMALL.values()), np.int64))
    numbers = {
        "default_spec": {"requests": 48, "steps": 16, "layers": 12, "sel": 64, "hot": 128,
                         "kv_heads": 8, "head_dim": 128, "seed": 42},
        "refill_MB": 1242.97, "hit_rate": 0.865,
        "mode_B_refill_segments": 79550, "mode_C_refill_segments": 59863,
        "mode_A_refill_MB": 9216.00,
        "source": "results/wla_7rep_20260930/wla_bursty_balanced_r1.log:3-9; "
                  "results/realtrace_20261021.md:19",
        "prefix_grp4_stp8": {"hit_rate": 0.921, "trace_baseline_MB": 731.31,
                             "source": "results/wla_pathdep_20261018/base_s42.log:12,14"},
    }
    with open(os.path.join(HERE, "reference_numbers.json"), "w") as f:
        json.dump(numbers, f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
