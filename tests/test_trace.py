"""FMT1 trace ingestion: the library's reader against the reference's own
load_miss_trace (compiled into oracle/_ref), error reporting, and the device
LRU replaying the trace with the reference's hit/miss flags."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

SPEC = dict(requests=6, steps=5, layers=3, sel_blocks=16, kv_heads=8, head_dim=128)


def _ref_load(oracle, path, hot=32):
    R = oracle.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    s = SPEC
    n = s["requests"] * s["steps"] * s["layers"] * s["sel_blocks"]
    blocks = np.zeros(n, np.int64)
    miss = np.zeros(n, np.uint8)
    tot = np.zeros(3, np.uint64)
    slab = C.c_int()
    R.ref_load_miss_trace(path.encode(), s["requests"], s["layers"], s["steps"], s["sel_blocks"], hot,
                          s["kv_heads"], s["head_dim"], blocks.ctypes.data, miss.ctypes.data, tot.ctypes.data,
                          C.byref(slab))
    return blocks, miss, tot, slab.value


def _write(tmp_path, name="t.bin", **kw):
    from ferry_b200 import trace

    s = SPEC
    ids = trace.synthetic_ids(s["requests"], s["steps"], s["layers"], s["sel_blocks"], seed=3)
    path = str(tmp_path / name)
    trace.write_fmt1(path, ids, **kw)
    return path, ids


def test_reader_matches_reference(tmp_path, oracle_lib, cuda_lib):
    from ferry_b200 import trace

    path, raw = _write(tmp_path)
    blocks, uniq, slab = trace.load(path, **SPEC)
    rb, rm, rt, rslab = _ref_load(oracle_lib, path)
    assert (blocks.ravel() == rb).all()
    assert slab == rslab and uniq == len(np.unique(raw))
    # dense ids follow first-seen order
    first = {}
    for x in raw.ravel():
        first.setdefault(int(x), len(first))
    assert (blocks.ravel() == np.array([first[int(x)] for x in raw.ravel()])).all()


@pytest.mark.parametrize("bad", [dict(header_override={"layers": 4}), dict(header_override={"version": 2}),
                                 dict(header_override={"block_tokens": 8}), dict(kv_heads=4),
                                 dict(counts="short"), dict(truncate=True)])
def test_reader_reports_mismatch_like_reference_exits(tmp_path, oracle_lib, cuda_lib, bad):
    from ferry_b200 import FerryError, trace

    s = SPEC
    kw = dict(bad)
    counts = None
    if kw.pop("counts", None) == "short":
        counts = np.full((s["requests"], s["steps"], s["layers"]), s["sel_blocks"])
        counts[2, 1, 0] -= 4
    trunc = kw.pop("truncate", False)
    path, _ = _write(tmp_path, counts=counts, **kw)
    if trunc:
        with open(path, "r+b") as f:
            f.truncate(os.path.getsize(path) - 10)
    with pytest.raises(FerryError) as e:
        trace.load(path, **s)
    assert e.value.code == 1 and str(e.value)
    if os.path.exists(oracle_lib.REF_TRACE_CHECK):
        r = subprocess.run([oracle_lib.REF_TRACE_CHECK, path, str(s["requests"]), str(s["layers"]),
                            str(s["steps"]), str(s["sel_blocks"]), "32", str(s["kv_heads"]), str(s["head_dim"])],
                           capture_output=True, text=True)
        assert r.returncode == 1 and "miss_trace" in r.stderr


def test_reader_accepts_reference_valid_file(tmp_path, oracle_lib, cuda_lib):
    path, _ = _write(tmp_path)
    if os.path.exists(oracle_lib.REF_TRACE_CHECK):
        s = SPEC
        r = subprocess.run([oracle_lib.REF_TRACE_CHECK, path, str(s["requests"]), str(s["layers"]),
                            str(s["steps"]), str(s["sel_blocks"]), "32", str(s["kv_heads"]), str(s["head_dim"])],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


@pytest.mark.gpu
def test_device_lru_replays_trace_like_reference(tmp_path, oracle_lib, cuda_lib):
    import torch

    from ferry_b200 import _abi, trace

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    path, _ = _write(tmp_path)
    blocks, uniq, _ = trace.load(path, **SPEC)
    rb, rmiss, rt, _ = _ref_load(oracle_lib, path, hot=32)
    s = SPEC
    R, S, L, G = s["requests"], s["steps"], s["layers"], s["sel_blocks"]
    M = rmiss.reshape(R, S, L, G)
    h = C.c_void_p()
    _abi.call("ferry_lru_create", 0, R * L, 32, uniq, C.byref(h))
    try:
        dev = torch.device("cuda", 0)
        lanes = torch.arange(R * L, dtype=torch.int32, device=dev)
        ns = torch.full((R * L,), G, dtype=torch.int32, device=dev)
        p = lambda t: C.c_void_p(t.data_ptr())
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        total = 0
        for step in range(S):
            sel = torch.from_numpy(np.ascontiguousarray(blocks[:, step].reshape(R * L, G), np.int32)).to(dev)
            im = torch.zeros((R * L, G), dtype=torch.uint8, device=dev)
            isl, mp, ms = (torch.zeros((R * L, G), dtype=torch.int32, device=dev) for _ in range(3))
            nm = torch.zeros(R * L, dtype=torch.int32, device=dev)
            _abi.call("ferry_lru_touch", h, st, p(lanes), None, R * L, p(sel), G, p(ns), 0, p(im), p(isl),
                      p(mp), p(ms), p(nm))
            torch.cuda.synchronize()
            assert (im.cpu().numpy() == M[:, step].reshape(R * L, G)).all()
            total += int(nm.sum())
        assert total == int(rt[1])
    finally:
        _abi.call("ferry_lru_destroy", h)
