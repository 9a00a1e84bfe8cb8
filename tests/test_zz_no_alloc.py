"""The allocation-free attention entry point (ferry_sparse_decode_noalloc).

It serves callers that cannot call cudaMalloc -- an engine whose caching
allocator or KV arena already owns all of HBM, or a latency-critical decode
loop that cannot afford cudaMalloc's implicit synchronisation -- by keeping
its split-K scratch and its error word in a fixed array inside the library.
This file is named so that pytest collects it last; it must pass alone in a
fresh process and after the other tests. Output is compared with
ferry_sparse_decode (the ctx entry point) at the attention tolerance of the
parity tests: 2e-3 relative per output row.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATTN_RTOL = 2e-3
# the fixed array: 4 MiB = 64 KiB of lane counters | partials | 256-B error word
SCRATCH_BYTES, COUNTER_BYTES, ERR_BYTES = 4 << 20, 64 << 10, 256
PART_STRIDE = 132  # floats per (lane, head) partial: o[128], m, l, pad


def _rel_err(a, b):
    a = a.reshape(-1, 128).astype(np.float64)
    b = b.reshape(-1, 128).astype(np.float64)
    return float((np.abs(a - b).max(1) / np.maximum(np.abs(b).max(1), 1e-30)).max())


def _warps_fit(n_lanes, group, top_k, sms):
    """(warps the ctx path would use, partial slots the fixed array leaves)."""
    T = n_lanes * top_k
    nw = min(sms * 12, max(1, T // 4), max(1, 31 * n_lanes))
    nw = nw // 4 * 4 if nw >= 4 else nw
    fit = (SCRATCH_BYTES - COUNTER_BYTES - ERR_BYTES) // (group * PART_STRIDE * 4) - n_lanes
    return nw, fit


def _run_case(w, reqs, bad_req=None):
    """Decode one step through the ctx (select -> detect -> gather ->
    ferry_sparse_decode), then call the allocation-free entry point twice in
    a row on a copy of the cache and compare. bad_req: a batch position whose
    request id is replaced by an out-of-range one for the no-alloc calls."""
    import torch

    from ferry_b200 import _abi
    from ferry_b200.engine import Decoder
    from ferry_b200.workload import q_stream

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = len(reqs)
    dec = Decoder(w, 0)
    try:
        dec.register_pool()
        ids = torch.from_numpy(np.asarray(reqs, np.int32)).to(dev)
        dec.begin(ids, torch.full((n,), w.max_pages, dtype=torch.int32, device=dev))
        units = w.num_requests * w.lanes_per_req * w.cache_pages
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        p = lambda t: C.c_void_p(t.data_ptr())
        for step in range(2):
            q = torch.from_numpy(np.stack([q_stream(w, int(r), steps=step + 1)[step] for r in reqs])).to(dev)
            dec.select(q, ids)
            dec.detect(ids)
            dec.gather(ids)
            ref = torch.zeros((n, w.num_layers, w.q_heads, 128), dtype=torch.float32, device=dev)
            dec.attention(q, ids, ref)
            torch.cuda.synchronize()
            dec.check()
            ref = ref.cpu().numpy()
            # the same cache contents in a caller-owned buffer
            cache = torch.from_numpy(dec.debug_read(0, np.uint8, units * 8192)).to(dev)
            nids = ids.clone()
            if bad_req is not None:
                nids[bad_req] = w.num_requests  # one past the last request slot
                ref[bad_req] = 0.0  # a skipped lane decodes to zero rows
            for _ in range(2):  # two calls in a row share (and re-clear) the fixed scratch
                out = torch.full((n, w.num_layers, w.q_heads, 128), float("nan"), device=dev)
                _abi.call("ferry_sparse_decode_noalloc", st, p(cache), w.cache_pages,
                          w.num_requests, w.lanes_per_req, w.group, w.top_k, p(q), p(nids), n,
                          p(dec.item_slot), p(dec.n_sel), p(out))
                rc = _abi.lib().ferry_sparse_decode_noalloc_status(st)
                got = out.cpu().numpy()
                assert np.isfinite(got).all()
                assert _rel_err(got, ref) <= ATTN_RTOL
                if bad_req is None:
                    assert rc == _abi.OK, _abi.lib().ferry_last_error()
                else:
                    assert rc == _abi.E_RANGE
                    # the status read cleared the word
                    assert _abi.lib().ferry_sparse_decode_noalloc_status(st) == _abi.OK
    finally:
        dec.close()


def _need_gpu():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_noalloc_matches_ctx_attention_two_calls_in_a_row():
    _need_gpu()
    from ferry_b200.workload import small

    w = small(num_requests=3, num_layers=2, q_heads=8, kv_heads=4, ctx_tokens=1024, top_k=16,
              cache_frac=0.25)
    _run_case(w, [2, 0, 1])


def test_noalloc_group1():
    _need_gpu()
    from ferry_b200.workload import small

    w = small(num_requests=3, num_layers=2, q_heads=4, kv_heads=4, ctx_tokens=1024, top_k=16,
              cache_frac=0.25)
    _run_case(w, [1, 2, 0])


def test_noalloc_group8_with_warps_capped_by_the_fixed_scratch():
    """128 lanes of G = 8: the ctx path would run 1776 warps (one per resident
    warp slot on 148 SMs), but the array holds partials for fewer, so the
    entry point runs with the capped warp count."""
    _need_gpu()
    import torch

    from ferry_b200.workload import small

    w = small(num_requests=8, num_layers=2, q_heads=64, kv_heads=8, ctx_tokens=2048, top_k=64,
              cache_frac=0.5)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    nw, fit = _warps_fit(8 * w.lanes_per_req, w.group, w.top_k, sms)
    assert fit < nw, (nw, fit)
    _run_case(w, [5, 0, 7, 1, 2, 6, 3, 4])


def test_noalloc_reports_out_of_range_request_ids():
    _need_gpu()
    from ferry_b200.workload import small

    w = small(num_requests=3, num_layers=1, q_heads=8, kv_heads=4, ctx_tokens=1024, top_k=16,
              cache_frac=0.25)
    _run_case(w, [0, 1, 2], bad_req=1)


def test_noalloc_rejects_batches_beyond_the_fixed_scratch():
    _need_gpu()
    from ferry_b200 import _abi

    L = _abi.lib()
    dummy = C.c_void_p(16)  # never dereferenced: both calls are rejected before any launch
    rc = L.ferry_sparse_decode_noalloc(None, dummy, 64, 2, 20000, 1, 64, dummy, dummy, 1, dummy,
                                       dummy, dummy)
    assert rc == _abi.E_INVAL and b"maximum" in L.ferry_last_error()
    rc = L.ferry_sparse_decode_noalloc(None, dummy, 4096, 1, 16000, 8, 4096, dummy, dummy, 1,
                                       dummy, dummy, dummy)
    assert rc == _abi.E_INVAL and b"fixed scratch" in L.ferry_last_error()
