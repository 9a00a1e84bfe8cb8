"""Host-side decoder over the C ABI (one instance per GPU).

``Decoder`` owns one ``ferry_ctx`` (HBM page cache, page tables, LRU state,
summaries, scratch) and the pinned host KV pool. It exposes the four hot-path
steps separately (select / detect / gather / attention) and fused
(``step``), plus ``step_host`` -- the end-to-end call a user makes with host
buffers. ``run_miss_workload`` drives a whole job the way the reference's
single-GPU executor does (src/workloads/kv_exec.cuh:64-315, mode C), but every
step runs on the device: selection, miss detection, gather and attention.
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import numpy as np
import torch

from . import _abi
from ._abi import call
from .workload import Schedule, Workload, q_stream

UNIT_BYTES = 8192


def _ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream=None, device=None):
    """The stream handle for a call on `device`: the given stream, else that
    device's current stream (never another device's: the library launches on
    the ctx's device with the stream it is handed)."""
    s = torch.cuda.current_stream(device) if stream is None else stream
    return C.c_void_p(s.cuda_stream)


class PinnedPool:
    """Pinned, device-mapped host memory from ferry_host_alloc (caller-owned)."""

    def __init__(self, nbytes: int):
        p = C.c_void_p()
        call("ferry_host_alloc", C.c_size_t(nbytes), C.byref(p))
        self.ptr, self.nbytes = p, nbytes

    def numpy(self, dtype=np.uint8) -> np.ndarray:
        buf = (C.c_uint8 * self.nbytes).from_address(self.ptr.value)
        return np.frombuffer(buf, dtype=dtype)

    def close(self):
        if self.ptr:
            call("ferry_host_free", self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Decoder:
    def __init__(self, w: Workload, device: int = 0, select_mode: int = _abi.SELECT_MEAN):
        self.w = w
        self.device = device
        self.dev = torch.device("cuda", device)
        self.kv_dtype = _abi.KV_E4M3 if w.kv_dtype == "e4m3" else _abi.KV_F16
        cfg = _abi.Cfg(kv_dtype=self.kv_dtype, **w.cfg_dict())
        h = C.c_void_p()
        call("ferry_ctx_create", device, C.byref(cfg), C.byref(h))
        self.ctx = h
        if select_mode != _abi.SELECT_MEAN:
            call("ferry_select_mode", h, select_mode)
        self.select_mode = select_mode
        if w.append:
            call("ferry_decode_appends", h, w.append)  # every fused step grows its requests' contexts
        self.pool: PinnedPool | None = None
        LH, k = w.lanes_per_req, w.top_k
        n = w.num_requests * LH
        i32 = dict(dtype=torch.int32, device=self.dev)
        # buffers for the separately-called steps (the fused step uses ctx workspace)
        self.sel = torch.empty((n, k), **i32)
        self.n_sel = torch.empty(n, **i32)
        self.item_slot = torch.empty((n, k), **i32)
        self.miss_page = torch.empty((n, k), **i32)
        self.miss_slot = torch.empty((n, k), **i32)
        self.n_miss = torch.empty(n, **i32)
        self.is_miss = torch.empty((n, k), dtype=torch.uint8, device=self.dev)

    # ------------------------------------------------------------------ setup
    def register_pool(self, seed: int | None = None, units: int | None = None, unit0: int = 0) -> PinnedPool:
        """Allocate the pinned pool, fill it with the procedural KV (content of
        units unit0 .. unit0 + units - 1) and compute every unit's page summary
        on the device."""
        w = self.w
        units = w.pool_units if units is None else units
        pool = PinnedPool(units * w.unit_bytes)
        s = _stream(None, self.dev)
        # ferry_kv_generate runs on the current device: make it this ctx's
        with torch.cuda.device(self.dev):
            call("ferry_kv_generate", s, C.c_uint64(w.seed if seed is None else seed), C.c_uint64(unit0),
                 C.c_int64(units), pool.ptr, self.kv_dtype)
        torch.cuda.synchronize(self.dev)
        call("ferry_kv_register", self.ctx, pool.ptr, C.c_size_t(pool.nbytes))
        call("ferry_page_summary_update", self.ctx, s, C.c_int64(0), C.c_int64(units))
        torch.cuda.synchronize(self.dev)
        self.pool = pool
        return pool

    def begin(self, req_ids: torch.Tensor, n_pages: torch.Tensor, stream=None,
              pool_base: torch.Tensor | None = None):
        """Start requests (cold lanes). pool_base (int64, optional): each
        request's first unit in the host pool; default slot * L * Hkv * N."""
        call("ferry_requests_begin", self.ctx, _stream(stream, self.dev), _ptr(req_ids), _ptr(n_pages),
             _ptr(pool_base), int(req_ids.numel()))

    def append(self, req_ids: torch.Tensor, tokens: int | None = None, stream=None):
        """Grow the requests' contexts by `tokens` tokens (default: the
        workload's per-step append); pages that become full turn selectable."""
        call("ferry_requests_append", self.ctx, _stream(stream, self.dev), _ptr(req_ids), int(req_ids.numel()),
             self.w.append if tokens is None else tokens)

    # ------------------------------------------------------------------ steps
    def select(self, q: torch.Tensor, req_ids: torch.Tensor, stream=None):
        call("ferry_select_topk", self.ctx, _stream(stream, self.dev), _ptr(q), _ptr(req_ids),
             int(req_ids.numel()), _ptr(self.sel), _ptr(self.n_sel))

    def detect(self, req_ids: torch.Tensor, stream=None):
        call("ferry_detect_misses", self.ctx, _stream(stream, self.dev), _ptr(req_ids), int(req_ids.numel()),
             _ptr(self.sel), _ptr(self.n_sel), _ptr(self.item_slot), _ptr(self.miss_page),
             _ptr(self.miss_slot), _ptr(self.n_miss), _ptr(self.is_miss))

    def gather(self, req_ids: torch.Tensor, stream=None):
        call("ferry_gather_misses", self.ctx, _stream(stream, self.dev), _ptr(req_ids), int(req_ids.numel()),
             _ptr(self.miss_page), _ptr(self.miss_slot), _ptr(self.n_miss))

    def attention(self, q: torch.Tensor, req_ids: torch.Tensor, out: torch.Tensor, stream=None):
        call("ferry_sparse_decode", self.ctx, _stream(stream, self.dev), _ptr(q), _ptr(req_ids),
             int(req_ids.numel()), _ptr(self.item_slot), _ptr(self.n_sel), _ptr(out))

    def step(self, q: torch.Tensor, req_ids: torch.Tensor, out: torch.Tensor, stream=None):
        """Fused decode step on device-resident q / req_ids / out."""
        call("ferry_decode_step", self.ctx, _stream(stream, self.dev), _ptr(q), _ptr(req_ids),
             int(req_ids.numel()), _ptr(out))

    # ------------------------------------------------------------------ inspection
    def check(self):
        call("ferry_ctx_check", self.ctx)

    def stats(self, reset: bool = False) -> tuple[int, int]:
        """(page units gathered, gather bytes) since the last reset."""
        return self.all_stats(reset)[:2]

    def all_stats(self, reset: bool = False) -> tuple[int, ...]:
        """(units gathered, gather bytes, units migrated in, migration bytes,
        units / bytes gathered from peer owner stores, units / bytes gathered
        from this GPU's own store)."""
        s = (C.c_uint64 * _abi.NUM_STATS)()
        call("ferry_stats_read", self.ctx, s, int(reset))
        return tuple(int(v) for v in s)

    # ------------------------------------------------------------------ page-owner stores
    def store_create(self, world: int, rank: int, global_lanes: int | None = None):
        """Keep the pages with page id % world == rank of global lanes
        [0, global_lanes) in this GPU's HBM (default: this ctx's lanes)."""
        gl = self.w.num_requests * self.w.lanes_per_req if global_lanes is None else global_lanes
        call("ferry_store_create", self.ctx, world, rank, C.c_int64(gl))

    def store_fill(self, seed: int | None = None, pool_units: int | None = None, stream=None):
        """Procedural content of the owned units: the bytes of pool unit
        (lane * N + p) mod pool_units (default: the registered pool's size)."""
        if pool_units is None:
            pool_units = self.pool.nbytes // self.w.unit_bytes if self.pool is not None else self.w.pool_units
        call("ferry_store_fill", self.ctx, _stream(stream, self.dev), C.c_uint64(self.w.seed if seed is None else seed),
             C.c_uint64(pool_units))

    def gather_source(self, source: int):
        call("ferry_gather_source", self.ctx, source)

    def step_chunks(self, chunks: int):
        """Pipeline step(): chunk i's selection overlaps chunk i-1's detect,
        gather and attention (1 = no pipelining)."""
        call("ferry_step_chunks", self.ctx, chunks)

    def register_stores(self, units: int):
        """No host pool: summary rows for `units` pool units, misses from the
        owner stores only (after store_create)."""
        call("ferry_kv_register_stores", self.ctx, C.c_uint64(units))

    def summaries_from_stores(self, req_ids: torch.Tensor, stream=None):
        """Summaries of every page of the requests (after begin), read from
        their owners' stores; every owner's store filled and linked first."""
        call("ferry_page_summary_from_stores", self.ctx, _stream(stream, self.dev), _ptr(req_ids),
             int(req_ids.numel()))

    def debug_read(self, which: int, dtype, count: int, offset_elems: int = 0) -> np.ndarray:
        out = np.empty(count, dtype)
        call("ferry_debug_read", self.ctx, which, C.c_size_t(offset_elems * out.itemsize),
             C.c_size_t(out.nbytes), out.ctypes.data_as(C.c_void_p))
        return out

    def close(self):
        if self.ctx:
            call("ferry_ctx_destroy", self.ctx)
            self.ctx = None
        if self.pool is not None:
            self.pool.close()
            self.pool = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclasses.dataclass
class WorkloadStats:
    """Mirrors the reference's WlAStats (src/workloads/kv_exec.cuh:39-45)."""
    makespan_ms: float
    p50_step_ms: float
    p99_step_ms: float
    refill_events: int
    refill_bytes: int
    tokens: int
    throughput_tokens: float


def run_miss_workload(dec: Decoder, ticks: int | None = None, stream=None) -> WorkloadStats:
    """Run a job tick by tick on one GPU (device-resident queries), timing each
    tick with CUDA events -- the device twin of run_miss_workload mode C
    (src/workloads/kv_exec.cuh:187-292)."""
    w = dec.w
    sch = Schedule(w)
    ticks = sch.length if ticks is None else ticks
    qs = torch.from_numpy(np.stack([q_stream(w, r) for r in range(w.num_requests)])).to(dec.dev)
    out = torch.empty((w.num_requests, w.num_layers, w.q_heads, w.head_dim), dtype=torch.float32,
                      device=dec.dev)
    n_pages = torch.full((w.num_requests,), w.init_pages, dtype=torch.int32, device=dec.dev)
    st = torch.cuda.current_stream(dec.dev) if stream is None else stream
    dec.stats(reset=True)
    evs = []
    tokens = 0
    for i in range(ticks):
        active, steps, _ = sch.tick(i)
        if len(active) == 0:
            continue
        ids = torch.from_numpy(active).to(dec.dev, non_blocking=True)
        new = active[steps == 0]
        if len(new):
            nid = torch.from_numpy(new).to(dec.dev)
            dec.begin(nid, n_pages[: len(new)], stream=st)
        q = qs[torch.from_numpy(active).long(), torch.from_numpy(steps).long()].contiguous()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        dec.step(q, ids, out[: len(active)], stream=st)
        e1.record(st)
        evs.append((e0, e1, len(active)))
        tokens += len(active)
    torch.cuda.synchronize(dec.dev)
    dec.check()
    ms = np.array([a.elapsed_time(b) for a, b, _ in evs])
    units, nbytes = dec.stats()
    span = float(ms.sum())
    srt = np.sort(ms)
    return WorkloadStats(makespan_ms=span, p50_step_ms=float(srt[len(srt) // 2]),
                         p99_step_ms=float(srt[int(0.99 * (len(srt) - 1))]),
                         refill_events=units, refill_bytes=nbytes, tokens=tokens,
                         throughput_tokens=tokens / (span / 1000.0) if span > 0 else 0.0)
