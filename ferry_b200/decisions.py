"""Steal-decision logs of the executor and their counterfactual pricing.

The B200 counterpart of the reference's decision snapshots
(FERRY_WLA_SNAPSHOT, src/runtime/wla_multigpu.cuh:667-788) and of its offline
tool src/tools/wla_counterfact.cpp, which enumerates for every decision point
"a0" (no migration), single-request carry / drop and the batch actually taken,
prices bytes exactly and time with a linear model. Here every rank's executor
writes its steals (``ferry_exec_log``); this module reads the logs and prices,
per stolen request, the migration modes of this path:

  a0     the request stays on the victim and waits there: no bytes move; the
         thief's idle share of the tick is the cost (value_ms forgone)
  delta  resident pages over NVLink (what FERRY_MIGRATE_DELTA moves)
  full   every cache slot of the request's lanes over NVLink
  drop   nothing over NVLink; the thief refills the resident pages by misses
         over the host link when they are reselected (an upper bound: all of
         them)

Time is bytes / link rate + a fixed cost per migration (the reference's
kMigDeltaFixedMs, 0.06 ms, wla_multigpu.cuh:146); value is the remaining
decode steps times the thief's step time (policy E's value, :942-1061).

    python -m ferry_b200.decisions rank0.log [rank1.log ...] [--nvlink-gbs G]
        [--host-gbs H] [--fixed-ms F]   -> CSV on stdout
"""
from __future__ import annotations

import argparse
import dataclasses
import struct
import sys

HEADER = struct.Struct("<4sI14i")          # 64 bytes
RECORD = struct.Struct("<qiiqqqiidffq")    # fixed part of a decision record
TASK = struct.Struct("<iiiiq")             # per stolen request
FIELDS = ("rank", "world", "num_requests", "num_layers", "kv_heads", "max_pages", "cache_pages", "top_k",
          "unit_bytes", "steps_per_req", "migrate_mode", "steal_batch", "max_batch", "cost_filter")
MODES = {0: "full", 1: "delta", 2: "drop"}


@dataclasses.dataclass
class Task:
    request: int
    step: int
    victim_slot: int
    thief_slot: int
    resident_units: int


@dataclasses.dataclass
class Decision:
    rank: int
    tick: int
    victim: int
    forced: bool
    fair: int
    own_occupancy: int
    victim_size: int
    planned: int
    taken: int
    step_ms: float
    mig_ms: float
    mig_bytes: int
    tasks: list


def read_log(path: str):
    """(header dict, [Decision]) of one executor's log."""
    with open(path, "rb") as f:
        raw = f.read()
    if len(raw) < HEADER.size:
        raise ValueError(f"{path}: truncated header")
    magic, version, *vals = HEADER.unpack_from(raw, 0)
    if magic != b"FRYD" or version != 1:
        raise ValueError(f"{path}: not a decision log (magic {magic!r}, version {version})")
    hdr = dict(zip(FIELDS, vals))
    out, o = [], HEADER.size
    while o < len(raw):
        if o + RECORD.size > len(raw):
            raise ValueError(f"{path}: truncated record at byte {o}")
        tick, victim, forced, fair, occ, vsize, planned, got, step_ms, mig_ms, _, mig_bytes = RECORD.unpack_from(raw, o)
        o += RECORD.size
        if got < 0 or o + got * TASK.size > len(raw):
            raise ValueError(f"{path}: corrupt record at tick {tick}")
        tasks = [Task(*TASK.unpack_from(raw, o + i * TASK.size)) for i in range(got)]
        o += got * TASK.size
        out.append(Decision(hdr["rank"], tick, victim, bool(forced), fair, occ, vsize, planned, got, step_ms,
                            mig_ms, mig_bytes, tasks))
    return hdr, out


def price(hdr: dict, d: Decision, nvlink_gbs: float, host_gbs: float, fixed_ms: float = 0.06):
    """Rows of (mode, request, nvlink_bytes, host_bytes, cost_ms, value_ms) for
    every stolen request of one decision and every alternative."""
    ub, LH = hdr["unit_bytes"], hdr["num_layers"] * hdr["kv_heads"]
    full_units = LH * hdr["cache_pages"]
    rows = []
    for t in d.tasks:
        remain = hdr["steps_per_req"] - t.step
        value = remain * d.step_ms
        res = t.resident_units * ub
        alts = {
            "a0": (0, 0, value),  # staying put forgoes the thief's share of the work
            "delta": (res, 0, res / (nvlink_gbs * 1e6) + fixed_ms),
            "full": (full_units * ub, 0, full_units * ub / (nvlink_gbs * 1e6) + fixed_ms),
            "drop": (0, res, res / (host_gbs * 1e6)),
        }
        for mode, (nv, host, cost) in alts.items():
            rows.append((mode, t.request, nv, host, cost, value))
    return rows


def counterfactuals(paths, nvlink_gbs: float, host_gbs: float, fixed_ms: float = 0.06):
    """CSV rows over every decision of every log: decision id, rank, tick,
    victim, taken, actual mode, its measured bytes / ms, then per request and
    alternative the priced bytes and time, and whether the alternative is the
    cheapest for that request."""
    rows = [("decision", "rank", "tick", "victim", "taken", "actual_mode", "actual_bytes", "actual_ms",
             "request", "alt", "nvlink_bytes", "host_bytes", "cost_ms", "value_ms", "cheapest")]
    did = 0
    for p in paths:
        hdr, ds = read_log(p)
        for d in ds:
            priced = price(hdr, d, nvlink_gbs, host_gbs, fixed_ms)
            best = {}
            for mode, req, nv, host, cost, value in priced:
                if req not in best or cost < best[req][1]:
                    best[req] = (mode, cost)
            for mode, req, nv, host, cost, value in priced:
                rows.append((did, d.rank, d.tick, d.victim, d.taken, MODES.get(hdr["migrate_mode"], "?"),
                             d.mig_bytes, round(d.mig_ms, 4), req, mode, nv, host, round(cost, 4),
                             round(value, 4), int(best[req][0] == mode)))
            did += 1
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("logs", nargs="+")
    ap.add_argument("--nvlink-gbs", type=float, default=770.0, help="peer-copy rate (measure: ferry_probe_link)")
    ap.add_argument("--host-gbs", type=float, default=55.0, help="host-link rate (measure: ferry_probe_link)")
    ap.add_argument("--fixed-ms", type=float, default=0.06)
    a = ap.parse_args(argv)
    for r in counterfactuals(a.logs, a.nvlink_gbs, a.host_gbs, a.fixed_ms):
        sys.stdout.write(",".join(str(x) for x in r) + "\n")


if __name__ == "__main__":
    main()
