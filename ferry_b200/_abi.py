"""ctypes binding of libferry_cuda.so (the C ABI declared in include/ferry_cuda.h).

The library is required: importing this module on a machine where it was not
built raises immediately -- there is no CPU fallback for the decode path.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libferry_cuda.so")

OK, E_INVAL, E_OOM, E_TIMEOUT, E_CUDA, E_STATE, E_RANGE = range(7)
_NAMES = {E_INVAL: "FERRY_E_INVAL", E_OOM: "FERRY_E_OOM", E_TIMEOUT: "FERRY_E_TIMEOUT",
          E_CUDA: "FERRY_E_CUDA", E_STATE: "FERRY_E_STATE", E_RANGE: "FERRY_E_RANGE"}
KV_F16 = 0
KV_E4M3 = 1
UNIT_BYTES = {KV_F16: 8192, KV_E4M3: 4112}
LRU_DISTINCT = 1
SELECT_MEAN, SELECT_QUEST = 0, 1

# every symbol include/ferry_cuda.h declares
EXPORTS = [
    "ferry_last_error", "ferry_version", "ferry_ctx_create", "ferry_ctx_destroy",
    "ferry_ctx_check", "ferry_host_alloc", "ferry_host_free", "ferry_kv_register",
    "ferry_kv_generate", "ferry_page_summary_update", "ferry_requests_begin",
    "ferry_requests_append", "ferry_decode_appends", "ferry_step_chunks",
    "ferry_select_mode", "ferry_select_topk", "ferry_detect_misses", "ferry_gather_misses", "ferry_sparse_decode",
    "ferry_sparse_decode_noalloc", "ferry_sparse_decode_noalloc_status", "ferry_decode_step", "ferry_wait_flag", "ferry_stats_read", "ferry_debug_read",
    "ferry_ctx_export", "ferry_store_create", "ferry_store_fill", "ferry_gather_source",
    "ferry_kv_register_stores", "ferry_page_summary_from_stores",
    "ferry_ctx_import", "ferry_ctx_link", "ferry_migrate_requests",
    "ferry_slot_states", "ferry_deque_create", "ferry_deque_destroy", "ferry_deque_push",
    "ferry_deque_pop", "ferry_deque_steal", "ferry_deque_size", "ferry_deque_peek", "ferry_deque_export",
    "ferry_deque_import", "ferry_deque_peer_view", "ferry_deque_stress",
    "ferry_exec_create", "ferry_exec_destroy", "ferry_exec_link_peer", "ferry_exec_admit",
    "ferry_exec_set_global", "ferry_exec_owned", "ferry_exec_tick", "ferry_exec_output", "ferry_exec_log", "ferry_exec_policy",
    "ferry_exec_usage", "ferry_exec_rebalance",
    "ferry_steal_filter",
    "ferry_comm_unique_id", "ferry_comm_create", "ferry_comm_destroy", "ferry_comm_abort",
    "ferry_exchange_ownership",
    "ferry_trace_load", "ferry_probe_topology", "ferry_probe_link",
    "ferry_lru_create", "ferry_lru_destroy", "ferry_lru_touch", "ferry_lru_read",
    "ferry_lru_group_enable", "ferry_lru_touch_owned", "ferry_lru_set_capacity", "ferry_lru_release",
    "ferry_lru_count_owned", "ferry_lru_handoff", "ferry_lru_read_owned",
    "ferry_taskb_generate", "ferry_taskb_create", "ferry_taskb_run", "ferry_taskb_results",
    "ferry_taskb_reset", "ferry_taskb_destroy",
]
MAX_PEERS = 8
CTX_HANDLE_BYTES = 1024
COMM_ID_BYTES = 128
MIGRATE_FULL, MIGRATE_DELTA, MIGRATE_DROP = 0, 1, 2
HANDOFF_DROP, HANDOFF_CARRY, HANDOFF_OWNED = 0, 1, 2
SRC_HOST, SRC_OWNER, SRC_HOST_BULK = 0, 1, 2
NUM_STATS = 8


class FerryError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{_NAMES.get(code, code)}: {msg}")
        self.code = code


class Cfg(C.Structure):
    _fields_ = [("num_requests", C.c_int), ("num_layers", C.c_int), ("q_heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("page_tokens", C.c_int),
                ("max_pages", C.c_int), ("cache_pages", C.c_int), ("top_k", C.c_int),
                ("kv_dtype", C.c_int)]


class ExecCfg(C.Structure):
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("max_batch", C.c_int),
                ("steal_batch", C.c_int), ("migrate_mode", C.c_int), ("steps_per_req", C.c_int),
                ("total_requests", C.c_int), ("q_table_steps", C.c_int)]


class StealPolicy(C.Structure):
    """ferry_steal_policy: cost_filter 0 = water-level steal (policy C),
    1 = plus the value/cost filter (policy E)."""
    _fields_ = [("cost_filter", C.c_int), ("margin", C.c_double), ("cost_scale", C.c_double),
                ("link_gbs", C.c_double), ("fixed_ms", C.c_double)]


TASKB_STEADY, TASKB_BURSTY, TASKB_SKEWED, TASKB_TRACE = 0, 1, 2, 3
TASKB_A, TASKB_B, TASKB_C = 0, 1, 2
TASKB_P2P, TASKB_HOST_STAGED = 0, 1


class TaskbSpec(C.Structure):
    _fields_ = [("arrival", C.c_int), ("sparsity", C.c_int), ("imbalanced", C.c_int), ("num_gpus", C.c_int),
                ("total", C.c_uint64), ("dest_hot_frac", C.c_double), ("dest_hot_cards", C.c_int),
                ("pad", C.c_int)]


class TaskbTask(C.Structure):
    _fields_ = [("arrive_t", C.c_double), ("payload", C.c_uint64), ("work", C.c_int32), ("dest", C.c_int32)]


class TaskbParams(C.Structure):
    _fields_ = [("mode", C.c_int), ("transport", C.c_int), ("inner_scale", C.c_int), ("stride", C.c_int),
                ("tick_ms", C.c_double), ("pending_ahead", C.c_uint64), ("adaptive", C.c_int),
                ("overlap", C.c_int), ("min_mb", C.c_double), ("max_mb", C.c_double),
                ("target_batches", C.c_double)]


class TaskbStats(C.Structure):
    _fields_ = [("makespan_ms", C.c_double), ("p50_ms", C.c_double), ("p99_ms", C.c_double),
                ("throughput", C.c_double), ("backlog_max", C.c_double), ("arrival_span_ms", C.c_double),
                ("migrated_bytes", C.c_uint64), ("migrations", C.c_uint64)]


class TickStats(C.Structure):
    _fields_ = [("decoded", C.c_int), ("finished", C.c_int), ("stolen", C.c_int),
                ("stolen_from", C.c_int), ("queued", C.c_int), ("tick_ms", C.c_float),
                ("mig_ms", C.c_float), ("mig_bytes", C.c_int64)]


_lib = None

V = C.c_void_p
I = C.c_int
_SIGS = {
    "ferry_last_error": (C.c_char_p, []),
    "ferry_version": (I, []),
    "ferry_ctx_create": (I, [I, C.POINTER(Cfg), C.POINTER(V)]),
    "ferry_ctx_destroy": (I, [V]),
    "ferry_ctx_check": (I, [V]),
    "ferry_host_alloc": (I, [C.c_size_t, C.POINTER(V)]),
    "ferry_host_free": (I, [V]),
    "ferry_kv_register": (I, [V, V, C.c_size_t]),
    "ferry_kv_generate": (I, [V, C.c_uint64, C.c_uint64, C.c_int64, V, I]),
    "ferry_page_summary_update": (I, [V, V, C.c_int64, C.c_int64]),
    "ferry_requests_begin": (I, [V, V, V, V, V, I]),
    "ferry_select_mode": (I, [V, I]),
    "ferry_requests_append": (I, [V, V, V, I, I]),
    "ferry_decode_appends": (I, [V, I]),
    "ferry_step_chunks": (I, [V, I]),
    "ferry_select_topk": (I, [V, V, V, V, I, V, V]),
    "ferry_detect_misses": (I, [V, V, V, I, V, V, V, V, V, V, V]),
    "ferry_gather_misses": (I, [V, V, V, I, V, V, V]),
    "ferry_sparse_decode": (I, [V, V, V, V, I, V, V, V]),
    "ferry_sparse_decode_noalloc": (I, [V, V, I, I, I, I, I, V, V, I, V, V, V]),
    "ferry_sparse_decode_noalloc_status": (I, [V]),
    "ferry_decode_step": (I, [V, V, V, V, I, V]),
    "ferry_wait_flag": (I, [V, V, V, C.c_uint32, C.c_uint32]),
    "ferry_stats_read": (I, [V, V, I]),
    "ferry_debug_read": (I, [V, I, C.c_size_t, C.c_size_t, V]),
    "ferry_ctx_export": (I, [V, V]),
    "ferry_store_create": (I, [V, I, I, C.c_int64]),
    "ferry_store_fill": (I, [V, V, C.c_uint64, C.c_uint64]),
    "ferry_gather_source": (I, [V, I]),
    "ferry_kv_register_stores": (I, [V, C.c_uint64]),
    "ferry_page_summary_from_stores": (I, [V, V, V, I]),
    "ferry_ctx_import": (I, [V, I, V]),
    "ferry_ctx_link": (I, [V, I, V]),
    "ferry_migrate_requests": (I, [V, V, I, V, V, I, I]),
    "ferry_slot_states": (I, [V, V, I]),
    "ferry_deque_create": (I, [I, C.c_uint64, C.POINTER(V)]),
    "ferry_deque_destroy": (I, [V]),
    "ferry_deque_push": (I, [V, V, V, I, V]),
    "ferry_deque_pop": (I, [V, V, V, I, V]),
    "ferry_deque_steal": (I, [V, V, V, I, V]),
    "ferry_deque_size": (I, [V, V, V]),
    "ferry_deque_peek": (I, [V, V, V, I, V]),
    "ferry_deque_export": (I, [V, V]),
    "ferry_deque_import": (I, [I, V, C.c_uint64, C.POINTER(V)]),
    "ferry_deque_peer_view": (I, [I, V, C.POINTER(V)]),
    "ferry_deque_stress": (I, [I, C.c_uint64, I, I, I, V, V]),
    "ferry_exec_create": (I, [V, V, C.POINTER(ExecCfg), V, C.POINTER(V)]),
    "ferry_exec_destroy": (I, [V]),
    "ferry_exec_link_peer": (I, [V, I, I, V]),
    "ferry_exec_admit": (I, [V, V, V, I]),
    "ferry_exec_set_global": (I, [V, C.c_int64]),
    "ferry_exec_owned": (I, [V, V, I, C.POINTER(I)]),
    "ferry_exec_tick": (I, [V, V, C.POINTER(TickStats)]),
    "ferry_exec_output": (I, [V, V, V, V, I, V]),
    "ferry_exec_log": (I, [V, C.c_char_p]),
    "ferry_exec_policy": (I, [V, C.POINTER(StealPolicy)]),
    "ferry_exec_usage": (I, [V, C.POINTER(C.c_int64), C.POINTER(C.c_int32)]),
    "ferry_exec_rebalance": (I, [V, I, I]),
    "ferry_steal_filter": (I, [C.POINTER(StealPolicy), I, V, V, C.c_double, V, V, C.POINTER(I)]),
    "ferry_comm_unique_id": (I, [V]),
    "ferry_comm_create": (I, [I, I, I, V, C.POINTER(V)]),
    "ferry_comm_destroy": (I, [V]),
    "ferry_comm_abort": (I, [V]),
    "ferry_exchange_ownership": (I, [V, V, V, I, V]),
    "ferry_trace_load": (I, [C.c_char_p, I, I, I, I, I, I, V, C.c_int64, V, V]),
    "ferry_probe_topology": (I, [C.POINTER(I), V, V, I]),
    "ferry_probe_link": (I, [I, I, C.c_size_t, I, C.POINTER(C.c_double)]),
    "ferry_lru_create": (I, [I, I, I, I, C.POINTER(V)]),
    "ferry_lru_destroy": (I, [V]),
    "ferry_lru_touch": (I, [V, V, V, V, I, V, I, V, I, V, V, V, V, V]),
    "ferry_lru_read": (I, [V, I, V, V, V]),
    "ferry_lru_group_enable": (I, [V]),
    "ferry_lru_touch_owned": (I, [V, V, V, V, I, V, I, V, I, V, V, V, V, V, V]),
    "ferry_lru_set_capacity": (I, [V, V, V, V, I]),
    "ferry_lru_release": (I, [V, V, V, I, C.c_uint32]),
    "ferry_lru_count_owned": (I, [V, V, V, I, C.c_uint32, V]),
    "ferry_lru_handoff": (I, [V, V, V, V, V, I, I, C.c_uint32]),
    "ferry_lru_read_owned": (I, [V, I, V, V]),
    "ferry_taskb_generate": (I, [C.POINTER(TaskbSpec), C.c_uint64, V, V]),
    "ferry_taskb_create": (I, [I, I, V, C.c_uint64, C.POINTER(V)]),
    "ferry_taskb_run": (I, [V, C.POINTER(TaskbParams), C.POINTER(TaskbStats)]),
    "ferry_taskb_results": (I, [V, V, C.c_uint64]),
    "ferry_taskb_reset": (I, [V]),
    "ferry_taskb_destroy": (I, [V]),
}


def lib() -> C.CDLL:
    """Load libferry_cuda.so; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m ferry_b200.build` "
                              "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        raise FerryError(rc, lib().ferry_last_error().decode())


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
