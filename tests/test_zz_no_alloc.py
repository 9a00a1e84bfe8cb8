"""The allocation-free attention entry point (ferry_sparse_decode_noalloc).

It serves callers that cannot call cudaMalloc -- an engine whose caching
allocator or KV arena already owns all of HBM, or a latency-critical decode
loop that cannot afford cudaMalloc's implicit synchronisation -- by keeping
its split-K scratch in a fixed array inside the library. This file is named
so that pytest collects it last; it must pass alone in a fresh process and
after the other tests. Output is compared with ferry_sparse_decode (the ctx
entry point) at the attention tolerance of the parity tests: 2e-3 relative per
output row.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATTN_RTOL = 2e-3


def _rel_err(a, b):
    a = a.reshape(-1, 128).astype(np.float64)
    b = b.reshape(-1, 128).astype(np.float64)
    return float((np.abs(a - b).max(1) / np.maximum(np.abs(b).max(1), 1e-30)).max())


def test_noalloc_matches_ctx_attention_two_calls_in_a_row():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import q_stream, small

    w = small(num_requests=3, num_layers=2, q_heads=8, kv_heads=4, ctx_tokens=1024, top_k=16,
              cache_frac=0.25)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dec = Decoder(w, 0)
    try:
        dec.register_pool()
        reqs = np.array([2, 0, 1], np.int32)
        ids = torch.from_numpy(reqs).to(dev)
        dec.begin(ids, torch.full((3,), w.max_pages, dtype=torch.int32, device=dev))
        units = w.num_requests * w.lanes_per_req * w.cache_pages
        for step in range(2):
            q = torch.from_numpy(np.stack([q_stream(w, int(r), steps=step + 1)[step] for r in reqs])).to(dev)
            dec.select(q, ids)
            dec.detect(ids)
            dec.gather(ids)
            ref = torch.zeros((3, w.num_layers, w.q_heads, 128), dtype=torch.float32, device=dev)
            dec.attention(q, ids, ref)
            torch.cuda.synchronize()
            dec.check()
            # the same cache contents in a caller-owned buffer
            cache = torch.from_numpy(dec.debug_read(0, np.uint8, units * 8192)).to(dev)
            st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
            p = lambda t: C.c_void_p(t.data_ptr())
            for _ in range(2):  # two calls in a row share (and re-clear) the fixed scratch
                out = torch.full_like(ref, float("nan"))
                _abi.call("ferry_sparse_decode_noalloc", st, p(cache), w.cache_pages,
                          w.num_requests, w.lanes_per_req, w.group, w.top_k, p(q), p(ids), 3,
                          p(dec.item_slot), p(dec.n_sel), p(out))
                torch.cuda.synchronize()
                got = out.cpu().numpy()
                assert np.isfinite(got).all()
                assert _rel_err(got, ref.cpu().numpy()) <= ATTN_RTOL
    finally:
        dec.close()


def test_noalloc_rejects_batches_beyond_the_fixed_scratch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from ferry_b200 import _abi

    L = _abi.lib()
    dummy = C.c_void_p(16)  # never dereferenced: both calls are rejected before any launch
    rc = L.ferry_sparse_decode_noalloc(None, dummy, 64, 2, 20000, 1, 64, dummy, dummy, 1, dummy,
                                       dummy, dummy)
    assert rc == _abi.E_INVAL and b"maximum" in L.ferry_last_error()
    rc = L.ferry_sparse_decode_noalloc(None, dummy, 4096, 1, 16000, 8, 4096, dummy, dummy, 1,
                                       dummy, dummy, dummy)
    assert rc == _abi.E_INVAL and b"fixed scratch" in L.ferry_last_error()
