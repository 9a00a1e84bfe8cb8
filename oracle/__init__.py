"""CPU oracle for the sparse KV-cache miss-stream decode path -- TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline``
leg and ``--impl reference`` arm) may import this package, and only as the
checker or the timed CPU baseline. The product (``ferry_b200``) never imports it.

Two native libraries back it (``oracle/Makefile``):

* ``liboracle.so`` -- the C++ restatement (``ferry_oracle.cpp``), each function
  citing the reference file:line it follows;
* ``_ref/libferry_ref.so`` -- the reference's own host headers
  (``src/workloads/missstream.cuh``, ``miss_trace.cuh``,
  ``src/runtime/adaptive_batch.cuh``) compiled in place, used to pin the
  restatement. Absent on machines without the reference tree unless prebuilt.

Parity status: LRU miss stream, prefix sharing and the mode-C gather plan are
pinned to the reference's golden numbers and to ``_ref``. Selection scores and
attention have no reference vectors ("parity unpinned"); they follow the
benchmark definition stated in ``ferry_oracle.cpp``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None


def build(quiet: bool = True) -> None:
    """Compile liboracle.so (and _ref when the reference tree exists)."""
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


class MissSpec(C.Structure):
    _fields_ = [("num_requests", C.c_int), ("num_layers", C.c_int), ("steps", C.c_int),
                ("sel_blocks", C.c_int), ("hot_blocks", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("prefix_group", C.c_int), ("prefix_steps", C.c_int),
                ("cap_mode", C.c_int), ("seed", C.c_uint64)]


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.orc_replay_miss_stream.argtypes = [C.POINTER(MissSpec), C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_prefix_share_stats.argtypes = [C.POINTER(MissSpec), C.c_void_p, C.c_void_p]
        L.orc_choose_mb.restype = C.c_double
        L.orc_choose_mb.argtypes = [C.c_double] * 4
        L.orc_gather_plan.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_uint64,
                                      C.c_void_p, C.c_void_p]
        L.orc_lru_create.restype = C.c_void_p
        L.orc_lru_create.argtypes = [C.c_int, C.c_int, C.c_int]
        L.orc_lru_destroy.argtypes = [C.c_void_p]
        L.orc_lru_step.argtypes = [C.c_void_p, C.c_int] + [C.c_void_p] * 3 + [C.c_int] + [C.c_void_p] * 6
        L.orc_lru_state.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_lru_group_enable.argtypes = [C.c_void_p]
        L.orc_lru_touch_owned.argtypes = ([C.c_void_p, C.c_int] + [C.c_void_p] * 3 + [C.c_int]
                                          + [C.c_void_p] * 7)
        L.orc_lru_set_capacity.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_lru_release.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_uint32]
        L.orc_lru_count_owned.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_uint32, C.c_void_p]
        L.orc_lru_handoff.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                      C.c_uint32]
        L.orc_lru_owned_state.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_kv_elem.restype = C.c_uint16
        L.orc_kv_elem.argtypes = [C.c_uint64, C.c_uint64, C.c_uint32]
        L.orc_kv_gen.argtypes = [C.c_uint64, C.c_uint64, C.c_int64, C.c_void_p]
        L.orc_kv_gen_mt.argtypes = [C.c_uint64, C.c_uint64, C.c_int64, C.c_void_p, C.c_int]
        L.orc_page_summary.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        L.orc_select_topk.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                      C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_sparse_decode.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                        C.c_int, C.c_float, C.c_void_p]
        L.orc_e4m3_encode.restype = C.c_uint8
        L.orc_e4m3_encode.argtypes = [C.c_float]
        L.orc_e4m3_decode.restype = C.c_float
        L.orc_e4m3_decode.argtypes = [C.c_uint8]
        L.orc_kv_gen_e4m3_mt.argtypes = [C.c_uint64, C.c_uint64, C.c_int64, C.c_void_p, C.c_int]
        L.orc_e4m3_unit_dequant.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        L.orc_page_summary_e4m3.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        L.orc_page_minmax.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        L.orc_page_minmax_e4m3.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        L.orc_select_quest.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                       C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_pipe_create.restype = C.c_void_p
        L.orc_pipe_create.argtypes = [C.c_int] * 5 + [C.c_void_p, C.c_void_p, C.c_int]
        L.orc_pipe_destroy.argtypes = [C.c_void_p]
        L.orc_pipe_step.restype = C.c_int64
        L.orc_pipe_step.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_float, C.c_void_p, C.c_void_p]
        L.orc_taskb_payload.argtypes = [C.c_uint64, C.c_void_p]
        L.orc_taskb_compute.argtypes = [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p, C.c_int]
        _LIB = L
    return _LIB


def ref_lib():
    """The reference's own headers compiled in place (None when unavailable)."""
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libferry_ref.so")
        if not os.path.exists(path):
            return None
        R = C.CDLL(path)
        R.ref_replay_miss_stream.argtypes = [C.c_int] * 7 + [C.c_uint64] + [C.c_void_p] * 3
        R.ref_choose_mb.restype = C.c_double
        R.ref_choose_mb.argtypes = [C.c_double]
        R.ref_load_miss_trace.argtypes = [C.c_char_p] + [C.c_int] * 7 + [C.c_void_p] * 4
        R.ref_generate_tasks.argtypes = ([C.c_char_p] * 3 + [C.c_uint64, C.c_int, C.c_double, C.c_int, C.c_uint64]
                                         + [C.c_void_p] * 4)
        _REF = R
    return _REF


REF_TRACE_CHECK = os.path.join(HERE, "_ref", "ref_trace_check")

# --------------------------------------------------------------------------- miss stream


def miss_spec(R=48, L=12, S=16, sel=64, hot=128, kv=8, d=128, seed=42,
              prefix_group=1, prefix_steps=8, cap_mode=0) -> MissSpec:
    """Defaults = the reference's regression configuration
    (results/wla_7rep_20260930/wla_bursty_balanced_r1.log:1)."""
    return MissSpec(R, L, S, sel, hot, kv, d, prefix_group, prefix_steps, cap_mode, seed)


def replay_miss_stream(sp: MissSpec):
    n = sp.num_requests * sp.steps * sp.num_layers * sp.sel_blocks
    blocks = np.zeros(n, np.int64)
    miss = np.zeros(n, np.uint8)
    tot = np.zeros(3, np.uint64)
    lib().orc_replay_miss_stream(C.byref(sp), blocks.ctypes.data, miss.ctypes.data, tot.ctypes.data)
    return blocks, miss, tot


def ref_replay_miss_stream(sp: MissSpec):
    R = ref_lib()
    if R is None:
        return None
    n = sp.num_requests * sp.steps * sp.num_layers * sp.sel_blocks
    blocks = np.zeros(n, np.int64)
    miss = np.zeros(n, np.uint8)
    tot = np.zeros(3, np.uint64)
    R.ref_replay_miss_stream(sp.num_requests, sp.num_layers, sp.steps, sp.sel_blocks,
                             sp.hot_blocks, sp.kv_heads, sp.head_dim, sp.seed,
                             blocks.ctypes.data, miss.ctypes.data, tot.ctypes.data)
    return blocks, miss, tot


def prefix_share_stats(sp: MissSpec, blocks: np.ndarray):
    b = blocks.copy()
    tot = np.zeros(3, np.uint64)
    rc = lib().orc_prefix_share_stats(C.byref(sp), b.ctypes.data, tot.ctypes.data)
    if rc != 0:
        raise ValueError("prefix_group must be > 1")
    return b, tot


def gather_plan_totals(sp: MissSpec, blocks: np.ndarray, miss: np.ndarray):
    """Mode-C refill segments and bytes summed over every (request, step)."""
    L, S, G = sp.num_layers, sp.steps, sp.sel_blocks
    c4 = 4 * 2 * sp.kv_heads * sp.head_dim * 2
    b = blocks.reshape(sp.num_requests, S, L, G)
    m = miss.reshape(sp.num_requests, S, L, G).astype(bool)
    lay = np.broadcast_to(np.arange(L, dtype=np.int32)[:, None], (L, G))
    segs = bytes_ = 0
    s_out = np.zeros(1, np.uint64)
    b_out = np.zeros(1, np.uint64)
    for r in range(sp.num_requests):
        for s in range(S):
            mm = m[r, s]
            ls = np.ascontiguousarray(lay[mm], np.int32)
            bs = np.ascontiguousarray(b[r, s][mm], np.int64)
            lib().orc_gather_plan(ls.ctypes.data, bs.ctypes.data, len(bs), sp.hot_blocks, c4,
                                  s_out.ctypes.data, b_out.ctypes.data)
            segs += int(s_out[0])
            bytes_ += int(b_out[0])
    return segs, bytes_


# --------------------------------------------------------------------------- LRU lanes


class LruLanes:
    """Page-table LRU lanes (the miss-detect definition)."""

    def __init__(self, lanes: int, capacity: int, ids: int):
        self.lanes, self.cap, self.ids = lanes, capacity, ids
        self.h = lib().orc_lru_create(lanes, capacity, ids)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_lru_destroy(self.h)
            self.h = None

    def step(self, lane_ids, sel, n_sel=None, reset=None):
        lane_ids = np.ascontiguousarray(lane_ids, np.int32)
        sel = np.ascontiguousarray(sel, np.int32)
        n, k = sel.shape
        n_sel = np.full(n, k, np.int32) if n_sel is None else np.ascontiguousarray(n_sel, np.int32)
        reset = np.zeros(n, np.uint8) if reset is None else np.ascontiguousarray(reset, np.uint8)
        is_miss = np.zeros((n, k), np.uint8)
        item_slot = np.full((n, k), -1, np.int32)
        mp = np.full((n, k), -1, np.int32)
        ms = np.full((n, k), -1, np.int32)
        nm = np.zeros(n, np.int32)
        rc = lib().orc_lru_step(self.h, n, lane_ids.ctypes.data, reset.ctypes.data, sel.ctypes.data,
                                k, n_sel.ctypes.data, is_miss.ctypes.data, item_slot.ctypes.data,
                                mp.ctypes.data, ms.ctypes.data, nm.ctypes.data)
        if rc != 0:
            raise ValueError(f"orc_lru_step rc={rc}")
        return is_miss, item_slot, mp, ms, nm

    def state(self, lane: int):
        ps = np.zeros(self.ids, np.int32)
        order = np.zeros(self.cap, np.int32)
        size = np.zeros(1, np.int32)
        lib().orc_lru_state(self.h, lane, ps.ctypes.data, order.ctypes.data, size.ctypes.data)
        return ps, order[: size[0]].copy(), int(size[0])

    # ---- group lanes: the reference's kv_touch / grp_trim / own_* / kv_handoff
    def group_enable(self):
        lib().orc_lru_group_enable(self.h)

    def step_owned(self, lane_ids, sel, bits, n_sel=None, reset=None):
        lane_ids = np.ascontiguousarray(lane_ids, np.int32)
        sel = np.ascontiguousarray(sel, np.int32)
        bits = np.ascontiguousarray(bits, np.uint32)
        n, k = sel.shape
        n_sel = np.full(n, k, np.int32) if n_sel is None else np.ascontiguousarray(n_sel, np.int32)
        reset = np.zeros(n, np.uint8) if reset is None else np.ascontiguousarray(reset, np.uint8)
        is_miss = np.zeros((n, k), np.uint8)
        item_slot = np.full((n, k), -1, np.int32)
        mp = np.full((n, k), -1, np.int32)
        ms = np.full((n, k), -1, np.int32)
        nm = np.zeros(n, np.int32)
        rc = lib().orc_lru_touch_owned(self.h, n, lane_ids.ctypes.data, reset.ctypes.data, sel.ctypes.data, k,
                                       n_sel.ctypes.data, bits.ctypes.data, is_miss.ctypes.data,
                                       item_slot.ctypes.data, mp.ctypes.data, ms.ctypes.data, nm.ctypes.data)
        if rc != 0:
            raise ValueError(f"orc_lru_touch_owned rc={rc}")
        return is_miss, item_slot, mp, ms, nm

    def set_capacity(self, lane_ids, caps):
        lane_ids = np.ascontiguousarray(lane_ids, np.int32)
        caps = np.ascontiguousarray(caps, np.int32)
        rc = lib().orc_lru_set_capacity(self.h, len(lane_ids), lane_ids.ctypes.data, caps.ctypes.data)
        if rc != 0:
            raise ValueError(f"orc_lru_set_capacity rc={rc}")

    def release(self, lane_ids, bit: int):
        lane_ids = np.ascontiguousarray(lane_ids, np.int32)
        if lib().orc_lru_release(self.h, len(lane_ids), lane_ids.ctypes.data, bit) != 0:
            raise ValueError("orc_lru_release")

    def count_owned(self, lane_ids, bit: int) -> np.ndarray:
        lane_ids = np.ascontiguousarray(lane_ids, np.int32)
        out = np.zeros(len(lane_ids), np.int32)
        if lib().orc_lru_count_owned(self.h, len(lane_ids), lane_ids.ctypes.data, bit, out.ctypes.data) != 0:
            raise ValueError("orc_lru_count_owned")
        return out

    def handoff(self, src: "LruLanes", src_lanes, dst_lanes, mode: int, bit: int = 0):
        """mode 0 drop, 1 carry, 2 owned (into this object's dst lanes)."""
        dst_lanes = np.ascontiguousarray(dst_lanes, np.int32)
        src_lanes = np.ascontiguousarray(src_lanes if src_lanes is not None else dst_lanes, np.int32)
        rc = lib().orc_lru_handoff(self.h, src.h, len(dst_lanes), src_lanes.ctypes.data, dst_lanes.ctypes.data,
                                   mode, bit)
        if rc != 0:
            raise ValueError(f"orc_lru_handoff rc={rc}")

    def owned_state(self, lane: int):
        masks = np.zeros(self.cap, np.uint32)
        cap = np.zeros(1, np.int32)
        if lib().orc_lru_owned_state(self.h, lane, masks.ctypes.data, cap.ctypes.data) != 0:
            raise ValueError("orc_lru_owned_state")
        return masks, int(cap[0])


# --------------------------------------------------------------------------- KV, selection, attention

UNIT_ELEMS = 2 * 16 * 128


def _f16bits(x) -> np.ndarray:
    """fp16 data as contiguous uint16 bit patterns: float16 arrays are
    reinterpreted (never value-cast), integer arrays are taken as bits."""
    x = np.asarray(x)
    if x.dtype == np.float16:
        return np.ascontiguousarray(x).view(np.uint16)
    if x.dtype != np.uint16 and x.dtype.kind == "f":
        raise TypeError(f"fp16 bits expected, got {x.dtype}")
    return np.ascontiguousarray(x, np.uint16)


def kv_gen(seed: int, unit0: int, n_units: int, threads: int = 1) -> np.ndarray:
    out = np.zeros((n_units, UNIT_ELEMS), np.uint16)
    lib().orc_kv_gen_mt(seed, unit0, n_units, out.ctypes.data, threads)
    return out


UNIT_BYTES_E4M3 = 4112


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    f = lib().orc_e4m3_encode
    return np.array([f(float(v)) for v in np.asarray(x, np.float32).ravel()], np.uint8).reshape(np.shape(x))


def e4m3_decode_table() -> np.ndarray:
    return np.array([lib().orc_e4m3_decode(b) for b in range(256)], np.float32)


def kv_gen_e4m3(seed: int, unit0: int, n_units: int, threads: int = 1) -> np.ndarray:
    out = np.zeros((n_units, UNIT_BYTES_E4M3), np.uint8)
    lib().orc_kv_gen_e4m3_mt(seed, unit0, n_units, out.ctypes.data, threads)
    return out


def e4m3_dequant(units: np.ndarray) -> np.ndarray:
    """[n][4112] fp8 units -> [n][4096] fp32 (K then V, scales applied)."""
    units = np.ascontiguousarray(units, np.uint8).reshape(-1, UNIT_BYTES_E4M3)
    out = np.zeros((units.shape[0], 4096), np.float32)
    lib().orc_e4m3_unit_dequant(units.ctypes.data, units.shape[0], out.ctypes.data)
    return out


def page_summary_e4m3(units: np.ndarray) -> np.ndarray:
    units = np.ascontiguousarray(units, np.uint8).reshape(-1, UNIT_BYTES_E4M3)
    out = np.zeros((units.shape[0], 128), np.float32)
    lib().orc_page_summary_e4m3(units.ctypes.data, units.shape[0], out.ctypes.data)
    return out


def sparse_decode_f32(q_f16bits: np.ndarray, pages_f32: np.ndarray, n_sel, scale: float) -> np.ndarray:
    """Attention in float64 over already-dequantised pages [lanes][k][4096].
    q: [lanes, G, 128] as float16 values or their uint16 bit patterns."""
    q = _f16bits(q_f16bits).view(np.float16).astype(np.float64)
    lanes, G, _ = q.shape
    out = np.zeros((lanes, G, 128), np.float32)
    for i in range(lanes):
        n = int(n_sel[i])
        K = pages_f32[i, :n, :2048].reshape(-1, 128).astype(np.float64)
        V = pages_f32[i, :n, 2048:].reshape(-1, 128).astype(np.float64)
        for g in range(G):
            if n == 0:
                continue
            lg = K @ q[i, g] * scale
            p = np.exp(lg - lg.max())
            out[i, g] = (p / p.sum()) @ V
    return out


def page_summary(units: np.ndarray) -> np.ndarray:
    units = _f16bits(units).reshape(-1, UNIT_ELEMS)
    out = np.zeros((units.shape[0], 128), np.float32)
    lib().orc_page_summary(units.ctypes.data, units.shape[0], out.ctypes.data)
    return out


def select_topk(q_f16bits: np.ndarray, summ: np.ndarray, n_pages, k: int, return_scores=False):
    """q: [lanes, G, 128] uint16 (fp16 bits); summ: [lanes, N, 128] fp32."""
    q = _f16bits(q_f16bits)
    lanes, G, _ = q.shape
    summ = np.ascontiguousarray(summ, np.float32)
    N = summ.shape[1]
    n_pages = np.ascontiguousarray(n_pages, np.int32)
    sel = np.full((lanes, k), -1, np.int32)
    ns = np.zeros(lanes, np.int32)
    sc = np.zeros((lanes, N), np.float32)
    lib().orc_select_topk(q.ctypes.data, G, summ.ctypes.data, N, n_pages.ctypes.data, lanes, k,
                          sel.ctypes.data, ns.ctypes.data, sc.ctypes.data)
    return (sel, ns, sc) if return_scores else (sel, ns)


def sparse_decode(q_f16bits: np.ndarray, pages: np.ndarray, n_sel, scale: float) -> np.ndarray:
    """pages: [lanes, k, UNIT_ELEMS] uint16 -- the selected pages' contents."""
    q = _f16bits(q_f16bits)
    lanes, G, _ = q.shape
    pages = _f16bits(pages)
    k = pages.shape[1]
    n_sel = np.ascontiguousarray(n_sel, np.int32)
    out = np.zeros((lanes, G, 128), np.float32)
    lib().orc_sparse_decode(q.ctypes.data, G, pages.ctypes.data, n_sel.ctypes.data, lanes, k,
                            C.c_float(scale), out.ctypes.data)
    return out


def page_minmax(units: np.ndarray) -> np.ndarray:
    """Quest page bounds of fp16 units: rows [kmin[128] | kmax[128]] fp32."""
    units = _f16bits(units).reshape(-1, UNIT_ELEMS)
    out = np.zeros((units.shape[0], 256), np.float32)
    lib().orc_page_minmax(units.ctypes.data, units.shape[0], out.ctypes.data)
    return out


def page_minmax_e4m3(units: np.ndarray) -> np.ndarray:
    """Quest page bounds of e4m3 units (dequantised keys)."""
    units = np.ascontiguousarray(units, np.uint8).reshape(-1, UNIT_BYTES_E4M3)
    out = np.zeros((units.shape[0], 256), np.float32)
    lib().orc_page_minmax_e4m3(units.ctypes.data, units.shape[0], out.ctypes.data)
    return out


def select_quest(q_f16bits: np.ndarray, kv_heads: int, mm: np.ndarray, n_pages, k: int,
                 return_scores=False):
    """The reference's Quest selection (one page set per request and layer).
    q: [n_grp, Hkv * G, 128] fp16 (bits or values); mm: [n_grp, Hkv, N, 256]."""
    q = _f16bits(q_f16bits)
    n_grp, Hq, _ = q.shape
    G = Hq // kv_heads
    mm = np.ascontiguousarray(mm, np.float32)
    N = mm.shape[2]
    n_pages = np.ascontiguousarray(n_pages, np.int32)
    sel = np.full((n_grp, k), -1, np.int32)
    ns = np.zeros(n_grp, np.int32)
    sc = np.zeros((n_grp, N), np.float32)
    lib().orc_select_quest(q.ctypes.data, kv_heads, G, mm.ctypes.data, N, n_pages.ctypes.data, n_grp, k,
                           sel.ctypes.data, ns.ctypes.data, sc.ctypes.data)
    return (sel, ns, sc) if return_scores else (sel, ns)


class CpuPipeline:
    """Multi-threaded CPU path (select -> LRU -> memcpy gather -> fp32 attention)."""

    def __init__(self, lanes, N, C_, k, G, pool: np.ndarray, summ: np.ndarray, threads: int):
        self.pool = _f16bits(pool)
        self.summ = np.ascontiguousarray(summ, np.float32)
        self.G = G
        self.h = lib().orc_pipe_create(lanes, N, C_, k, G, self.pool.ctypes.data,
                                       self.summ.ctypes.data, threads)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_pipe_destroy(self.h)
            self.h = None

    def step(self, lane_ids, q_f16bits, reset=None, scale=128 ** -0.5, n_pages=None):
        """One step of the lanes; n_pages (per lane, optional): whole pages of
        each lane's context (default: all N)."""
        lane_ids = np.ascontiguousarray(lane_ids, np.int32)
        n = len(lane_ids)
        reset = np.zeros(n, np.uint8) if reset is None else np.ascontiguousarray(reset, np.uint8)
        q = _f16bits(q_f16bits)
        out = np.zeros((n, self.G, 128), np.float32)
        npg = None if n_pages is None else np.ascontiguousarray(n_pages, np.int32)
        misses = lib().orc_pipe_step(self.h, n, lane_ids.ctypes.data, reset.ctypes.data,
                                     q.ctypes.data, C.c_float(scale), out.ctypes.data,
                                     None if npg is None else npg.ctypes.data)
        return out, int(misses)


# --------------------------------------------------------------------------- Workload B

def taskb_payload(n_floats: int) -> np.ndarray:
    """The reference's payload pool content (baselines.cuh:86-89)."""
    out = np.empty(n_floats, np.float32)
    lib().orc_taskb_payload(C.c_uint64(n_floats), out.ctypes.data_as(C.c_void_p))
    return out


def taskb_expected(tasks: np.ndarray, batches, inner: int) -> np.ndarray:
    """Outputs an executor leaves: for a batch (off, cnt) the task kernel reads
    the cnt floats from the batch's first payload float on, element j with
    task off + j's work (baselines.cuh:40-48, 176-178, 220-223, 332-335)."""
    payload = int(tasks["payload"][0])
    pf = payload // 4
    n_floats = len(tasks) * pf
    pool = taskb_payload(n_floats)
    works = np.ascontiguousarray(tasks["work"], np.int32)
    out = np.zeros(n_floats, np.float32)
    for off, cnt in batches:
        seg = np.empty(cnt, np.float32)
        lib().orc_taskb_compute(pool[off * pf:].ctypes.data_as(C.c_void_p), seg.ctypes.data_as(C.c_void_p),
                                C.c_uint64(cnt), works[off:].ctypes.data_as(C.c_void_p), inner)
        out[off * pf: off * pf + cnt] = seg
    return out


def ref_generate_tasks(arrival: str, sparsity: str, skew: str, total: int, num_gpus: int = 1,
                       hot_frac: float = 0.8, hot_cards: int = 0, seed: int = 42):
    """The reference's own generate_tasks (None when _ref is unavailable):
    (arrive_t, payload, work, dest)."""
    R = ref_lib()
    if R is None:
        return None
    a = np.empty(total, np.float64)
    p = np.empty(total, np.uint64)
    w = np.empty(total, np.int32)
    d = np.empty(total, np.int32)
    R.ref_generate_tasks(arrival.encode(), sparsity.encode(), skew.encode(), C.c_uint64(total), num_gpus,
                         hot_frac, hot_cards, C.c_uint64(seed), a.ctypes.data_as(C.c_void_p),
                         p.ctypes.data_as(C.c_void_p), w.ctypes.data_as(C.c_void_p), d.ctypes.data_as(C.c_void_p))
    return a, p, w, d
