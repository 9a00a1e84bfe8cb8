"""Failure detection without a GPU fault: a device wait on a flag that nothing
sets runs out after its poll budget, the ctx reports FERRY_E_TIMEOUT, and the
same ctx keeps decoding afterwards."""
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


def test_bounded_wait_times_out_and_ctx_stays_usable(torch_cuda):
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import q_stream, small

    t = torch_cuda
    dev = t.device("cuda", 0)
    w = small(num_requests=2)
    dec = Decoder(w, 0)
    try:
        dec.register_pool()
        st = C.c_void_p(t.cuda.current_stream().cuda_stream)
        flag = t.zeros(1, dtype=t.int32, device=dev)
        # nothing ever sets the flag: ~20k polls, then the kernel gives up
        _abi.call("ferry_wait_flag", dec.ctx, st, C.c_void_p(flag.data_ptr()), 1, 20000)
        t.cuda.synchronize()
        with pytest.raises(_abi.FerryError) as e:
            dec.check()
        assert e.value.code == _abi.E_TIMEOUT
        dec.check()  # reported once, then cleared
        # the ctx still decodes
        ids = t.arange(2, dtype=t.int32, device=dev)
        dec.begin(ids, t.full((2,), w.max_pages, dtype=t.int32, device=dev))
        q = t.from_numpy(np.stack([q_stream(w, r, steps=1)[0] for r in range(2)])).to(dev)
        out = t.zeros((2, w.num_layers, w.q_heads, 128), dtype=t.float32, device=dev)
        dec.step(q, ids, out)
        t.cuda.synchronize()
        dec.check()
        assert t.isfinite(out).all() and out.abs().sum() > 0
        # a flag that is set returns at once
        flag.fill_(1)
        _abi.call("ferry_wait_flag", dec.ctx, st, C.c_void_p(flag.data_ptr()), 1, 20000)
        t.cuda.synchronize()
        dec.check()
    finally:
        dec.close()
