"""The C-ABI library loads, exports every symbol include/ferry_cuda.h declares,
and rejects bad configurations before touching a GPU. No compute calls."""
import ctypes as C
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    src = open(os.path.join(ROOT, "include", "ferry_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ferry_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported(cuda_lib):
    from ferry_b200 import _abi

    names = _header_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(cuda_lib, n), n
    assert sorted(_abi.EXPORTS) == names


def test_version_and_error_string(cuda_lib):
    assert cuda_lib.ferry_version() == 100
    assert isinstance(cuda_lib.ferry_last_error(), bytes)


def test_invalid_configs_rejected_without_gpu(cuda_lib):
    from ferry_b200 import _abi

    base = dict(num_requests=2, num_layers=1, q_heads=4, kv_heads=4, head_dim=128, page_tokens=16,
                max_pages=64, cache_pages=16, top_k=8, kv_dtype=0)
    bad = [dict(head_dim=64), dict(page_tokens=8), dict(q_heads=6), dict(q_heads=48, kv_heads=4),
           dict(top_k=17), dict(top_k=0), dict(max_pages=20000), dict(kv_dtype=3),
           dict(num_requests=0),
           dict(max_pages=16384, cache_pages=16384, top_k=8192)]  # LRU lane past 227 KiB of smem
    for b in bad:
        cfg = _abi.Cfg(**{**base, **b})
        h = C.c_void_p()
        rc = cuda_lib.ferry_ctx_create(0, C.byref(cfg), C.byref(h))
        assert rc == _abi.E_INVAL, (b, rc)
        assert cuda_lib.ferry_last_error()
        assert not h.value


def test_null_arguments_rejected(cuda_lib):
    from ferry_b200 import _abi

    assert cuda_lib.ferry_ctx_create(0, None, None) == _abi.E_INVAL
    assert cuda_lib.ferry_select_topk(None, None, None, None, 0, None, None) == _abi.E_INVAL
    assert cuda_lib.ferry_ctx_check(None) == _abi.E_INVAL
    assert cuda_lib.ferry_ctx_destroy(None) == _abi.OK
    assert cuda_lib.ferry_kv_register(None, None, 0) == _abi.E_INVAL
    assert cuda_lib.ferry_store_create(None, 2, 0, 16) == _abi.E_INVAL
    assert cuda_lib.ferry_store_fill(None, None, 1, 16) == _abi.E_INVAL
    assert cuda_lib.ferry_gather_source(None, _abi.SRC_OWNER) == _abi.E_INVAL
    assert cuda_lib.ferry_comm_unique_id(None) == _abi.E_INVAL
    assert cuda_lib.ferry_comm_create(0, 0, 0, None, None) == _abi.E_INVAL
    assert cuda_lib.ferry_comm_destroy(None) == _abi.OK
    assert cuda_lib.ferry_comm_abort(None) == _abi.E_INVAL
    assert cuda_lib.ferry_exchange_ownership(None, None, None, 4, None) == _abi.E_INVAL


def test_product_never_imports_oracle():
    """The shipped package and kernels never reach the test oracle."""
    pkg = os.path.join(ROOT, "ferry_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                src = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f
                assert "liboracle" not in src and "orc_" not in src, f


def test_workload_schedule_is_deterministic():
    from ferry_b200 import CFG1, Schedule, q_stream, small

    s1, s2 = Schedule(CFG1), Schedule(CFG1)
    assert s1.length == s2.length and (s1.join == s2.join).all()
    seen = np.zeros(CFG1.num_requests, int)
    for i in range(s1.length):
        active, steps, job = s1.tick(i)
        assert job == 0
        seen[active] += 1
        assert ((steps >= 0) & (steps < CFG1.steps)).all()
    assert (seen == CFG1.steps).all()
    assert s1.tick(s1.length)[2] == 1
    w = small()
    a, b = q_stream(w, 1), q_stream(w, 1)
    assert a.shape == (w.steps, w.num_layers, w.q_heads, 128) and (a == b).all()
    assert not (q_stream(w, 2) == a).all()


def test_cfg1_shapes():
    from ferry_b200 import CFG1

    assert CFG1.max_pages == 256 and CFG1.cache_pages == 64 and CFG1.top_k == 64
    assert CFG1.attn_bytes_per_token() == 32 * 64 * 16 * 128 * 4 == 16 * 2**20
    assert CFG1.select_bytes_per_token() == 32 * 256 * 128 * 4 == 4 * 2**20
    assert CFG1.pool_units * 8192 == 2**30
