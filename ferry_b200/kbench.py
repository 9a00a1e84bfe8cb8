"""Per-kernel timing of the decode path at a workload's full batch.

    python -m ferry_b200.kbench [--workload cfg1] [--iters 50]

Fills the cache with a few decode steps, then times each kernel alone with
CUDA events over back-to-back launches on the same inputs (selected KV larger
than L2, so each attention launch streams from HBM). Prints one JSON line:
microseconds, algorithmic bytes and GB/s per kernel. ``-k regex:<kernel>``
under ncu captures the same launches.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .engine import Decoder
from .workload import WORKLOADS, q_stream


def _time(fn, iters: int, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / iters  # us


def migrate_bench(w, iters: int) -> dict:
    """Request migration over NVLink (the reference's run_mig_path axis,
    src/benches/run_mig_path.cu:176-320): warm every request on GPU 1 (GPU 0
    when only one exists), then time ferry_migrate_requests pulling all of
    them into GPU 0 (delta: resident slots only)."""
    import ctypes as C

    from . import _abi

    src_dev = 1 if torch.cuda.device_count() > 1 else 0
    R = w.num_requests
    src, dst = Decoder(w, src_dev), Decoder(w, 0)
    try:
        for dec, d in ((src, src_dev), (dst, 0)):
            dec.register_pool()
            dd = torch.device("cuda", d)
            ids = torch.arange(R, dtype=torch.int32, device=dd)
            dec.begin(ids, torch.full((R,), w.init_pages, dtype=torch.int32, device=dd))
        sd = torch.device("cuda", src_dev)
        ids = torch.arange(R, dtype=torch.int32, device=sd)
        out = torch.empty((R, w.num_layers, w.q_heads, 128), dtype=torch.float32, device=sd)
        for s in range(2):
            q = torch.from_numpy(np.stack([q_stream(w, r, steps=s + 1)[s] for r in range(R)])).to(sd)
            src.step(q, ids, out)
        torch.cuda.synchronize(sd)
        src.check()
        _abi.call("ferry_ctx_link", dst.ctx, 0, src.ctx)
        d0 = torch.device("cuda", 0)
        s_ids = torch.arange(R, dtype=torch.int32, device=d0)
        st = C.c_void_p(torch.cuda.current_stream(d0).cuda_stream)
        fn = lambda: _abi.call("ferry_migrate_requests", dst.ctx, st, 0, C.c_void_p(s_ids.data_ptr()),
                               C.c_void_p(s_ids.data_ptr()), R, _abi.MIGRATE_DELTA)
        dst.all_stats(reset=True)
        with torch.cuda.device(d0):
            t = _time(fn, iters)
        units, _, mu, mb = dst.all_stats()[:4]
        dst.check()
        per = mb / (iters + 3)
        peak = None
        if src_dev != 0:  # the peer-read copy peak of the same link, measured now
            g = C.c_double()
            _abi.call("ferry_probe_link", src_dev, 0, C.c_size_t(256 << 20), 3, C.byref(g))
            peak = g.value
        return {"src_device": src_dev, "requests": R, "bytes_per_call": per, "us": t,
                "GB_s": per / t / 1e3, "nvlink_peak_GB_s": peak,
                "frac": per / t / 1e3 / peak if peak else None}
    finally:
        dst.close()
        src.close()


def migrate_many(w, iters: int, thieves: int) -> dict:
    """Several thieves pulling from one victim at once (the skewed job's
    steals: every idle GPU takes from the busiest): requests warmed on GPU 0,
    GPU j (1..thieves) migrates its share [j-1 of thieves] of them with
    ferry_migrate_requests (delta), all launched together; each thief's
    calls timed with CUDA events on its own stream. Returns per-thief GB/s
    and the victim's egress = all bytes / the slowest thief's time."""
    import ctypes as C

    from . import _abi

    n = torch.cuda.device_count()
    if n < thieves + 1:
        raise SystemExit(f"needs {thieves + 1} GPUs")
    R = w.num_requests
    vic = Decoder(w, 0)
    th = [Decoder(w, d) for d in range(1, thieves + 1)]
    try:
        for dec, d in [(vic, 0)] + [(t, i + 1) for i, t in enumerate(th)]:
            dec.register_pool()
            dd = torch.device("cuda", d)
            ids = torch.arange(R, dtype=torch.int32, device=dd)
            dec.begin(ids, torch.full((R,), w.init_pages, dtype=torch.int32, device=dd))
        d0 = torch.device("cuda", 0)
        ids = torch.arange(R, dtype=torch.int32, device=d0)
        out = torch.empty((R, w.num_layers, w.q_heads, 128), dtype=torch.float32, device=d0)
        for s in range(2):
            q = torch.from_numpy(np.stack([q_stream(w, r, steps=s + 1)[s] for r in range(R)])).to(d0)
            vic.step(q, ids, out)
        torch.cuda.synchronize(d0)
        vic.check()
        share = R // thieves
        calls = []
        for j, t in enumerate(th):
            dev = torch.device("cuda", j + 1)
            _abi.call("ferry_ctx_link", t.ctx, 0, vic.ctx)
            sub = torch.arange(j * share, (j + 1) * share, dtype=torch.int32, device=dev)
            st = torch.cuda.Stream(dev)
            calls.append((t, dev, sub, st))

        def launch(t, dev, sub, st):
            _abi.call("ferry_migrate_requests", t.ctx, C.c_void_p(st.cuda_stream), 0, C.c_void_p(sub.data_ptr()),
                      C.c_void_p(sub.data_ptr()), share, _abi.MIGRATE_DELTA)

        for c in calls:  # warm-up
            for _ in range(2):
                launch(*c)
        for d in range(thieves + 1):
            torch.cuda.synchronize(d)
        for t, *_ in calls:
            t.all_stats(reset=True)
        evs = []
        for t, dev, sub, st in calls:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.device(dev):
                a.record(st)
            evs.append((a, b))
        for _ in range(iters):
            for c in calls:
                launch(*c)
        for (t, dev, sub, st), (a, b) in zip(calls, evs):
            with torch.cuda.device(dev):
                b.record(st)
        for d in range(thieves + 1):
            torch.cuda.synchronize(d)
        per, ms = [], []
        for (t, *_), (a, b) in zip(calls, evs):
            t.check()
            per.append(t.all_stats()[3])
            ms.append(a.elapsed_time(b))
        g = C.c_double()
        _abi.call("ferry_probe_link", 1, 0, C.c_size_t(256 << 20), 3, C.byref(g))
        rates = [b_ / (m / 1e3) / 1e9 for b_, m in zip(per, ms)]
        egress = sum(per) / (max(ms) / 1e3) / 1e9
        return {"thieves": thieves, "requests_each": share, "bytes_each_per_call": per[0] / iters,
                "thief_GB_s": rates, "victim_egress_GB_s": egress, "nvlink_peak_GB_s": g.value,
                "thief_frac": [r / g.value for r in rates], "egress_frac": egress / g.value}
    finally:
        for t in th:
            t.close()
        vic.close()


def probe() -> dict:
    """Devices, P2P access / native peer atomics, and the two link peaks the
    decode path uses (host -> device 0, and every peer -> device 0)."""
    import ctypes as C

    from . import _abi

    n = C.c_int()
    _abi.call("ferry_probe_topology", C.byref(n), None, None, 0)
    cap = max(1, n.value)
    p2p = (C.c_int32 * (cap * cap))()
    at = (C.c_int32 * (cap * cap))()
    _abi.call("ferry_probe_topology", C.byref(n), p2p, at, cap)
    g = C.c_double()
    _abi.call("ferry_probe_link", -1, 0, C.c_size_t(1 << 30), 5, C.byref(g))
    res = {"devices": n.value, "p2p": [[p2p[i * cap + j] for j in range(n.value)] for i in range(n.value)],
           "peer_atomics": [[at[i * cap + j] for j in range(n.value)] for i in range(n.value)],
           "host_to_dev0_GB_s": g.value, "peer_to_dev0_GB_s": {}}
    for s in range(1, n.value):
        if p2p[0 * cap + s]:
            _abi.call("ferry_probe_link", s, 0, C.c_size_t(1 << 30), 5, C.byref(g))
            res["peer_to_dev0_GB_s"][s] = g.value
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="cfg1")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--migrate", action="store_true", help="time request migration over NVLink")
    ap.add_argument("--probe", action="store_true", help="topology and link peaks")
    ap.add_argument("--thieves", type=int, default=0,
                    help="with --migrate: this many GPUs pull from GPU 0 at once")
    ap.add_argument("--requests", type=int, default=0, help="override the batch (a smaller case to profile)")
    ap.add_argument("--only", default="", help="comma list of kernels to time (gather,attention,select,detect)")
    ap.add_argument("--select", default="mean", help="selection rule: mean (the benchmark's) or quest")
    ap.add_argument("--store-world", type=int, default=0,
                    help="serve misses from page-owner stores of W ranks (rank r on GPU r mod count)")
    ap.add_argument("--host-bulk", action="store_true",
                    help="host-pool misses by TMA bulk copies (FERRY_SRC_HOST_BULK) instead of SM loads")
    args = ap.parse_args()
    if args.probe:
        print(json.dumps({"probe": probe()}))
        return
    if args.migrate:
        w = WORKLOADS[args.workload]
        if args.requests:
            import dataclasses

            w = dataclasses.replace(w, num_requests=args.requests)
        if args.thieves:
            print(json.dumps({"migrate_many": migrate_many(w, args.iters, args.thieves)}))
        else:
            print(json.dumps({"migrate": migrate_bench(w, args.iters)}))
        return
    w = WORKLOADS[args.workload]
    if args.requests:
        import dataclasses

        w = dataclasses.replace(w, num_requests=args.requests)
    only = set(args.only.split(",")) if args.only else {"gather", "attention", "select", "detect"}
    torch.cuda.set_device(args.device)
    dev = torch.device("cuda", args.device)
    from . import _abi as _a

    dec = Decoder(w, args.device, select_mode=_a.SELECT_QUEST if args.select == "quest" else _a.SELECT_MEAN)
    dec.register_pool()
    peers = []
    if args.store_world:
        from . import _abi

        W = args.store_world
        ndev = torch.cuda.device_count()
        dec.store_create(W, 0)
        dec.store_fill()
        for r in range(1, W):
            p = Decoder(w, (args.device + r) % ndev)
            p.store_create(W, r)
            p.store_fill(pool_units=w.pool_units)
            peers.append(p)
        for i, p in enumerate(peers):
            _abi.call("ferry_ctx_link", dec.ctx, i, p.ctx)
        for d in range(ndev):
            torch.cuda.synchronize(d)
        dec.gather_source(_abi.SRC_OWNER)
    elif args.host_bulk:
        dec.gather_source(_a.SRC_HOST_BULK)
    R = w.num_requests
    ids = torch.arange(R, dtype=torch.int32, device=dev)
    dec.begin(ids, torch.full((R,), w.init_pages, dtype=torch.int32, device=dev))
    qs = [torch.from_numpy(np.stack([q_stream(w, r, steps=s + 1)[s] for r in range(R)])).to(dev)
          for s in range(4)]
    out = torch.empty((R, w.num_layers, w.q_heads, 128), dtype=torch.float32, device=dev)
    for s in range(3):
        dec.select(qs[s], ids)
        dec.detect(ids)
        dec.gather(ids)
        dec.attention(qs[s], ids, out)
    q = qs[3]
    dec.select(q, ids)
    dec.detect(ids)  # leaves this step's misses in the miss list
    torch.cuda.synchronize()
    dec.check()
    units = int(dec.n_miss.sum().item())
    res = {"workload": w.name, "batch_requests": R, "kv_dtype": w.kv_dtype}
    # gather re-copies the same miss list each launch (idempotent)
    if "gather" in only:
        dec.all_stats(reset=True)
        t = _time(lambda: dec.gather(ids), max(3, args.iters // 5))
        ub = w.unit_bytes
        st = dec.all_stats()
        res["gather"] = {"us": t, "units": units, "bytes": units * ub, "GB_s": units * ub / t / 1e3,
                         "source": ("owner stores, world %d" % args.store_world) if args.store_world else
                         ("host pool, bulk copies" if args.host_bulk else "host pool, SM loads"),
                         "share_peer": st[4] / max(1, st[0]), "share_local_store": st[6] / max(1, st[0])}
    dec.gather(ids)
    if "attention" in only:
        t = _time(lambda: dec.attention(q, ids, out), args.iters)
        b = R * w.attn_bytes_per_token() + R * w.qo_bytes_per_token()
        res["attention"] = {"us": t, "bytes": b, "GB_s": b / t / 1e3}
    if "select" in only:
        t = _time(lambda: dec.select(q, ids), args.iters)
        # summaries read: mean rows (512 B per page and lane) or Quest bounds (1 KiB)
        b = R * w.select_bytes_per_token() * (2 if args.select == "quest" else 1)
        res["select"] = {"us": t, "bytes": b, "GB_s": b / t / 1e3, "rule": args.select}
    if "detect" in only:
        # as in a decode step: each launch follows its step's selection (which
        # streams the summaries through L2) and sees that step's drift, so the
        # LRU evicts; repeating one selection would time an all-hit replay
        n_det = max(3, args.iters // 5)
        qd = np.stack([q_stream(w, r, steps=4 + n_det) for r in range(R)], 1)[4:]
        evs = []
        for s in range(n_det):
            dec.select(torch.from_numpy(np.ascontiguousarray(qd[s])).to(dev), ids)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            dec.detect(ids)
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        t = float(np.mean([a.elapsed_time(b) for a, b in evs])) * 1e3
        res["detect"] = {"us": t, "steps": n_det, "misses_last_step": int(dec.n_miss.sum().item())}
    dec.check()
    dec.close()
    for p in peers:
        p.close()
    print(json.dumps(res))


if __name__ == "__main__":
    main()
