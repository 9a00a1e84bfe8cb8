"""CPU checks of the e4m3 KV oracle: codec against torch's float8_e4m3fn,
page-unit structure (4112 B: K | V | k_scale | v_scale | pad), dequantisation
and summaries against numpy restatements, and the fp16 input guard."""
import numpy as np
import pytest
import torch

import oracle

UB = oracle.UNIT_BYTES_E4M3


@pytest.fixture(scope="module")
def o():
    oracle.lib()
    return oracle


def test_decode_table_matches_torch(o):
    tab = o.e4m3_decode_table()
    ref = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    nan = np.isnan(ref)
    assert nan.sum() == 2 and nan[0x7F] and nan[0xFF]
    assert np.isnan(tab[nan]).all()
    assert (tab[~nan].view(np.uint32) == ref[~nan].view(np.uint32)).all()


def test_encode_matches_torch_rne(o):
    tab = o.e4m3_decode_table()
    fin = np.sort(np.unique(tab[np.isfinite(tab)]))
    mids = (fin[:-1].astype(np.float64) + fin[1:]) / 2  # exact ties
    rng = np.random.default_rng(11)
    x = np.concatenate([fin, mids.astype(np.float32), -mids.astype(np.float32),
                        rng.uniform(-447, 447, 4000).astype(np.float32),
                        (rng.standard_normal(2000) * 2.0 ** rng.integers(-12, 4, 2000)).astype(np.float32),
                        np.float32([0.0, -0.0, 2.0 ** -10, 2.0 ** -11, 447.9])])
    got = o.e4m3_encode(x)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert (got == ref).all(), x[got != ref][:8]


def test_encode_saturates(o):
    x = np.float32([448.0, 460.0, 1e6, np.inf, -500.0, -np.inf])
    assert o.e4m3_encode(x).tolist() == [0x7E, 0x7E, 0x7E, 0x7E, 0xFE, 0xFE]


def test_units_structure_and_determinism(o):
    u = o.kv_gen_e4m3(7, 100, 12)
    assert u.shape == (12, UB)
    assert (u == o.kv_gen_e4m3(7, 100, 12, threads=3)).all()
    assert (u[5] == o.kv_gen_e4m3(7, 105, 1)[0]).all()
    assert not (u == o.kv_gen_e4m3(8, 100, 12)).all()
    assert (u[:, 4104:] == 0).all()
    sc = u[:, 4096:4104].copy().view(np.float32)
    assert (sc > 0).all() and np.isfinite(sc).all()
    tab = o.e4m3_decode_table()
    codes = u[:, :4096].reshape(12, 2, 2048)
    assert not ((codes & 0x7F) == 0x7F).any()  # no NaN codes
    # scale = amax / 448: each half's largest code decodes to 448
    assert (np.abs(tab[codes]).max(axis=2) == 448.0).all()


def test_units_follow_the_fp16_stream(o):
    """Quantised value * scale stays within e4m3 rounding of the fp16 stream
    (both derive from the same exact fp32 Irwin-Hall values)."""
    u = o.kv_gen_e4m3(3, 0, 4)
    f16 = o.kv_gen(3, 0, 4).view(np.float16).astype(np.float64)
    dq = o.e4m3_dequant(u).astype(np.float64)
    sc = u[:, 4096:4104].copy().view(np.float32).astype(np.float64)
    step = np.repeat(sc, 2048, axis=1) * 2.0 ** -9  # subnormal spacing, absolute
    err = np.abs(dq - f16)
    bound = np.abs(f16) * (2.0 ** -4 + 2.0 ** -10) + step
    assert (err <= bound).all()


def test_dequant_and_summary_restatement(o):
    u = o.kv_gen_e4m3(9, 40, 6)
    tab = o.e4m3_decode_table()
    sc = u[:, 4096:4104].copy().view(np.float32)
    dq = (tab[u[:, :4096]].reshape(6, 2, 2048) * sc[:, :, None]).astype(np.float32).reshape(6, 4096)
    assert (o.e4m3_dequant(u).view(np.uint32) == dq.view(np.uint32)).all()
    k = dq[:, :2048].reshape(6, 16, 128)
    acc = k[:, 0].copy()
    for t in range(1, 16):
        acc = (acc + k[:, t]).astype(np.float32)
    ref = (acc * np.float32(0.0625)).astype(np.float32)
    assert (o.page_summary_e4m3(u).view(np.uint32) == ref.view(np.uint32)).all()


def test_fp16_inputs_are_reinterpreted_not_cast(o):
    rng = np.random.default_rng(4)
    q = rng.standard_normal((2, 4, 128)).astype(np.float16)
    pages = rng.standard_normal((2, 3, 4096)).astype(np.float32)
    n = np.array([3, 2], np.int32)
    a = o.sparse_decode_f32(q, pages, n, 128 ** -0.5)
    b = o.sparse_decode_f32(q.view(np.uint16), pages, n, 128 ** -0.5)
    assert np.isfinite(a).all() and (a == b).all()
    with pytest.raises(TypeError):
        o.sparse_decode_f32(q.astype(np.float32), pages, n, 128 ** -0.5)
