"""Topology and link probes (ferry_probe_topology / ferry_probe_link), the
counterparts of the reference's probe_topology / probe_host_staged_bandwidth
(src/topo/topo.cpp:68-215, src/probe/main.cu:12-52): the device count and P2P
matrix agree with the CUDA runtime's own answers, and the host -> GPU probe
(a copy kernel reading pinned host memory, the miss gather's access) reports
a finite rate of the same order as a plain copy-engine copy timed here."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def test_probe_topology(torch_cuda):
    from ferry_b200 import _abi

    t = torch_cuda
    n = C.c_int()
    _abi.call("ferry_probe_topology", C.byref(n), None, None, 0)
    assert n.value == t.cuda.device_count()
    cap = n.value
    p2p = np.full((cap, cap), -1, np.int32)
    at = np.full((cap, cap), -1, np.int32)
    _abi.call("ferry_probe_topology", C.byref(n), p2p.ctypes.data_as(C.c_void_p),
              at.ctypes.data_as(C.c_void_p), cap)
    for i in range(cap):
        assert p2p[i, i] == 0 and at[i, i] == 0
        for j in range(cap):
            if i != j:
                assert p2p[i, j] == int(t.cuda.can_device_access_peer(i, j))
                assert at[i, j] in (0, 1) and (at[i, j] <= p2p[i, j])


def _ce_h2d_gbs(t, nbytes):
    src = t.empty(nbytes, dtype=t.uint8).pin_memory()
    dst = t.empty(nbytes, dtype=t.uint8, device="cuda:0")
    st = t.cuda.current_stream(0)
    dst.copy_(src, non_blocking=True)
    t.cuda.synchronize(0)
    a, b = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(3):
        dst.copy_(src, non_blocking=True)
    b.record(st)
    t.cuda.synchronize(0)
    return 3 * nbytes / (a.elapsed_time(b) / 1e3) / 1e9


def test_probe_link_host_to_gpu(torch_cuda):
    from ferry_b200 import _abi

    t = torch_cuda
    g = C.c_double()
    nbytes = 256 << 20
    _abi.call("ferry_probe_link", -1, 0, C.c_size_t(nbytes), 3, C.byref(g))
    ce = _ce_h2d_gbs(t, nbytes)
    assert np.isfinite(g.value) and g.value > 0
    # the same host link: the copy kernel lands within a factor of 2 of the copy engine
    assert 0.5 * ce < g.value < 2.0 * ce, (g.value, ce)
    with pytest.raises(_abi.FerryError):
        _abi.call("ferry_probe_link", 0, 0, C.c_size_t(nbytes), 1, C.byref(g))  # src == dst
    with pytest.raises(_abi.FerryError):
        _abi.call("ferry_probe_link", -1, 0, C.c_size_t(16), 1, C.byref(g))  # below one page unit


def test_probe_link_peer(torch_cuda):
    from ferry_b200 import _abi

    t = torch_cuda
    if t.cuda.device_count() < 2 or not t.cuda.can_device_access_peer(1, 0):
        pytest.skip("needs two GPUs with peer access")
    g = C.c_double()
    _abi.call("ferry_probe_link", 0, 1, C.c_size_t(256 << 20), 3, C.byref(g))
    assert np.isfinite(g.value) and g.value > 50.0  # NVLink: far above any host link
