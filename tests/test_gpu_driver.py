"""The C++ driver (ferry_b200/drivers/run_missstream.cpp, the counterpart of
the reference's src/benches/run_missstream.cu) links only include/ferry_cuda.h
and the library. Run on the configs[0] job's arrivals and queries (cut to 12
decode steps per request), its per-tick attention outputs must be
bit-identical to the Python path's (Decoder.step over the same ticks), and its
refill count must equal the gathered page units."""
import os
import re
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.mark.parametrize("select", ["mean", "quest"])
def test_cpp_driver_matches_python_path(torch_cuda, tmp_path, select):
    import dataclasses

    from ferry_b200 import _abi, build
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import WORKLOADS, Schedule, arrival_ticks, q_stream

    t = torch_cuda
    exe = build.build_drivers()[0]
    w = dataclasses.replace(WORKLOADS["cfg1"], steps=12)
    qs = np.stack([q_stream(w, r) for r in range(w.num_requests)])  # R S L H 128
    qf, jf, of = tmp_path / "q.bin", tmp_path / "join.bin", tmp_path / "out.bin"
    qs.view(np.uint16).tofile(qf)
    arrival_ticks(w).astype(np.int64).tofile(jf)
    res = subprocess.run([exe, "--requests", str(w.num_requests), "--ctx", str(w.ctx_tokens), "--layers", "1",
                          "--heads", "32", "--kv-heads", "32", "--top-k", str(w.top_k), "--cache-frac", "0.25",
                          "--steps", str(w.steps), "--seed", str(w.seed), "--q-file", str(qf),
                          "--join-file", str(jf), "--out-file", str(of), "--select", select],
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr
    refill = int(re.search(r"refill=\s*(\d+)", res.stdout).group(1))
    got = np.fromfile(of, np.float32)

    dev = t.device("cuda", 0)
    dec = Decoder(w, 0, select_mode=_abi.SELECT_QUEST if select == "quest" else _abi.SELECT_MEAN)
    try:
        dec.register_pool()
        sch = Schedule(w)
        n_pages = t.full((w.num_requests,), w.max_pages, dtype=t.int32, device=dev)
        outs = []
        dec.stats(reset=True)
        for i in range(sch.length):
            active, steps, _ = sch.tick(i)
            if len(active) == 0:
                continue
            new = active[steps == 0]
            if len(new):
                dec.begin(t.from_numpy(new).to(dev), n_pages[: len(new)])
            q = t.from_numpy(qs[active, steps]).to(dev)
            out = t.zeros((len(active), 1, 32, 128), dtype=t.float32, device=dev)
            dec.step(q, t.from_numpy(active).to(dev), out)
            outs.append(out.cpu().numpy().ravel())
        t.cuda.synchronize()
        dec.check()
        units = dec.stats()[0]
    finally:
        dec.close()
    want = np.concatenate(outs)
    assert got.size == want.size
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    assert refill == units > 0


@pytest.mark.parametrize("gpus,mode", [("0,0", "delta"), ("0,0", "drop"), ("0,1", "full")])
def test_cpp_multigpu_driver_decodes_every_step_once(torch_cuda, gpus, mode):
    """ferry_b200/drivers/run_wla_multigpu.cpp (the reference's
    run_wla_multigpu counterpart): one host thread per GPU, peers linked in
    process, 80% of the requests homed on the first GPU; the idle executor
    steals and migrates, and every (request, step) is decoded exactly once.

    The owner pops its deque LIFO (Chase-Lev), so it runs its newest batch to
    completion while the older tasks wait; with a batch of 2 the homes (12 on
    the first GPU, 4 on the second) leave the first GPU's deque above the
    water level for whole ticks once the second GPU's work is done, so the
    steal does not hinge on reading the deque between two of the owner's
    ticks."""
    from ferry_b200 import build

    t = torch_cuda
    if max(int(g) for g in gpus.split(",")) >= t.cuda.device_count():
        pytest.skip("needs two GPUs")
    exe = [p for p in build.build_drivers() if p.endswith("run_wla_multigpu")][0]
    res = subprocess.run([exe, "--gpus", gpus, "--requests-per-gpu", "8", "--steps", "12", "--ctx", "1024",
                          "--heads", "4", "--top-k", "16", "--max-batch", "2", "--skew", "imbalanced",
                          "--kv-mode", mode], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "exactly_once=yes" in res.stdout
    stolen = sum(int(m) for m in re.findall(r"stolen=(\d+)", res.stdout))
    assert stolen > 0, res.stdout
