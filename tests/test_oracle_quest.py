"""The oracle's Quest selection against the reference's own selector.

tests/golden/quest_selector.npz holds page sets that the reference's
Selector.on_layer(method="quest") (tools/capture_miss_trace.py:128-159)
chose on CPU torch for keys from the procedural pool and seeded fp16 queries
(tests/golden/make_quest_golden.py). The oracle restatement must choose the
same pages; it also checks its own key bounds against numpy."""
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quest_selector.npz")
CASES = ["cfg1_shape", "gqa8", "ragged", "few_pages"]


def quest_inputs(z, name):
    """(q bits [R*L, Hq, 128], key bounds [R*L, Hkv, N, 256], n_pages, k, shape)."""
    R, L, Hq, Hkv, N, T, k = [int(x) for x in z[f"{name}_shape"]]
    units = oracle.kv_gen(int(z["kv_seed"]), 0, R * L * Hkv * N)
    mm = oracle.page_minmax(units).reshape(R * L, Hkv, N, 256)
    q = z[f"{name}_q"].reshape(R * L, Hq, 128)
    return q, mm, np.full(R * L, T // 16, np.int32), k, (R, L, Hq, Hkv, N, T, k)


@pytest.mark.parametrize("name", CASES)
def test_oracle_quest_matches_reference_selector(name):
    z = np.load(GOLDEN)
    q, mm, n_pages, k, (R, L, Hq, Hkv, N, T, _) = quest_inputs(z, name)
    sel, ns = oracle.select_quest(q, Hkv, mm, n_pages, k)
    ref = z[f"{name}_sel"].reshape(R * L, k)
    assert (ns == np.minimum(T // 16, k)).all()
    assert (sel == ref).all()


def test_page_minmax_is_the_key_min_and_max():
    units = oracle.kv_gen(7, 100, 5)
    K = units.reshape(5, 2, 16, 128)[:, 0].view(np.float16).astype(np.float32)
    mm = oracle.page_minmax(units)
    assert (mm[:, :128] == K.min(1)).all() and (mm[:, 128:] == K.max(1)).all()
    u8 = oracle.kv_gen_e4m3(7, 100, 5)
    Kf = oracle.e4m3_dequant(u8).reshape(5, 2, 16, 128)[:, 0]
    mm8 = oracle.page_minmax_e4m3(u8)
    assert (mm8[:, :128] == Kf.min(1)).all() and (mm8[:, 128:] == Kf.max(1)).all()
