"""Multi-GPU miss-stream decode: one process per GPU, work stealing, NVLink
migration, and the page-ownership exchange over NCCL.

Each rank owns a ``ferry_ctx`` (its HBM page cache and page tables), a device
work-stealing deque of decode tasks and a ``ferry_exec`` (the C++ tick loop,
``include/ferry_cuda.h``). At start-up the ranks swap CUDA IPC handles of
their ctx and deque (``all_gather_object``), so every executor can steal from
any peer's deque and pull a stolen request's state straight out of the peer's
HBM. Every ``epoch`` ticks the ranks exchange their ownership rows -- which
requests each GPU holds, how many it admitted and finished -- with one
``all_gather`` (NCCL on GPU tensors; gloo on CPU). That table gives every rank
the global pending count behind the fair-share steal threshold and the
termination test; the data path itself never goes through a collective.

The reference runs the same protocol with host threads, a mutex-guarded
std::deque per GPU and host-staged copies (src/runtime/wla_multigpu.cuh:
793-806 dispatch, :1063-1506 steal_from, :2291-2775 run_wla_multigpu).
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import math

import numpy as np

from . import _abi
from ._abi import call
from .workload import Workload, arrival_ticks, q_stream

# ---------------------------------------------------------------- host logic (CPU-testable)


def assign_ranks(n_req: int, world: int, policy: str = "rr", seed: int = 42,
                 zipf_a: float = 1.5) -> np.ndarray:
    """Home GPU of every request. 'rr': round-robin (the reference's RR
    dispatch); 'zipf': P(rank i) proportional to 1/(i+1)^a, which with a = 1.5
    puts ~80% of requests on two of eight GPUs (the benchmark's skewed config;
    the reference's own skew is 80% on half the GPUs,
    src/runtime/wla_multigpu.cuh:483-492)."""
    if policy == "rr":
        return (np.arange(n_req) % world).astype(np.int32)
    if policy == "zipf":
        p = 1.0 / np.arange(1, world + 1) ** zipf_a
        p /= p.sum()
        rng = np.random.default_rng([seed, 1501])
        return rng.choice(world, size=n_req, p=p).astype(np.int32)
    raise ValueError(f"unknown policy {policy!r}")


ROW_HEAD = 4  # finished, admitted, count, remaining steps (usage)


def ownership_row(finished: int, admitted: int, owned: np.ndarray, cap: int, usage: int = 0) -> np.ndarray:
    row = np.full(cap + ROW_HEAD, -1, np.int64)
    row[0], row[1], row[2], row[3] = finished, admitted, len(owned), usage
    row[ROW_HEAD:ROW_HEAD + len(owned)] = owned[:cap]
    return row


def merge_ownership(rows: np.ndarray, total_requests: int):
    """rows: [world][cap + 4] gathered ownership rows -> (owner_of[total],
    finished_total, admitted_total). A request absent from every row is -1."""
    owner = np.full(total_requests, -1, np.int32)
    cap = rows.shape[1] - ROW_HEAD
    for rank, row in enumerate(rows):
        n = int(row[2])
        if not (0 <= n <= cap) or row[0] < 0 or row[1] < 0 or row[3] < 0:
            raise ValueError(f"ownership row of rank {rank} is corrupt (count {n}, cap {cap})")
        ids = row[ROW_HEAD:ROW_HEAD + n]
        ids = ids[(ids >= 0) & (ids < total_requests)]
        owner[ids] = rank
    return owner, int(rows[:, 0].sum()), int(rows[:, 1].sum())


def llx_plan(usage: np.ndarray, counts: np.ndarray, threshold: float = 0.25, cap: int = 4):
    """The rebalancer's decision (rebalance_llumnix, wla_multigpu.cuh:2084-2112):
    usage[g] = remaining decode steps on GPU g, counts[g] = its requests.
    Act when the max-min spread exceeds `threshold` x the mean: the least
    loaded GPU pulls k requests from the most loaded one, k = the excess over
    the mean divided by the source's mean steps per request (+1), clamped to
    [1, cap]. Returns (src, dst, k) or None."""
    usage = np.asarray(usage, np.int64)
    counts = np.asarray(counts, np.int64)
    n = len(usage)
    if n < 2:
        return None
    src, dst = int(np.argmax(usage)), int(np.argmin(usage))
    mean = float(usage.sum()) / n
    if src == dst or mean == 0.0 or (usage[src] - usage[dst]) / mean <= threshold:
        return None
    over = int(usage[src] - int(mean))
    per = int(mean / max(1, counts[src])) + 1 if mean > 0 else 1
    k = max(1, min(over // max(per, 1), cap))
    return src, dst, k


class OwnershipComm:
    """The ownership exchange's own NCCL communicator, through the C ABI
    (ferry_comm_create / ferry_exchange_ownership). Collective: every rank of
    the default process group constructs it (ranks on distinct GPUs); rank 0's
    NCCL id reaches the others through that process group."""

    def __init__(self, device: int):
        import torch
        import torch.distributed as dist

        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        self.dev = torch.device("cuda", device)
        uid = (C.c_uint8 * _abi.COMM_ID_BYTES)()
        if self.rank == 0:
            call("ferry_comm_unique_id", uid)
        box = [bytes(uid)]
        dist.broadcast_object_list(box, src=0)
        uid = (C.c_uint8 * _abi.COMM_ID_BYTES).from_buffer_copy(box[0])
        self.h = C.c_void_p()
        call("ferry_comm_create", device, self.world, self.rank, uid, C.byref(self.h))
        # NCCL connects the ranks on a communicator's first collective (hundreds
        # of ms): do that here, outside any timed region
        self.all_gather(np.zeros(ROW_HEAD, np.int32))

    def all_gather(self, row: np.ndarray, timeout_s: float = 60.0) -> np.ndarray:
        """[world][len(row)] int32 rows of every rank (returns after the copy
        back). A collective not done within timeout_s (a peer rank gone) is
        aborted -- the communicator with it -- and raises TimeoutError at the
        deadline, the way a process group's timeout ends its collective. The
        abort (ncclCommAbort: it ends the kernel in flight, then tears the
        communicator down, which takes seconds) runs on a helper thread;
        wait_aborted() joins it, and every later exchange raises FerryError
        (FERRY_E_STATE)."""
        import threading
        import time

        import torch

        self.wait_aborted()
        # the copy, the collective and the completion event all on this
        # communicator's device and its current stream, whatever device the
        # caller has current
        with torch.cuda.device(self.dev):
            st = torch.cuda.current_stream(self.dev)
            with torch.cuda.stream(st):
                d_row = torch.from_numpy(np.ascontiguousarray(row, np.int32)).to(self.dev)
                d_all = torch.empty((self.world, len(row)), dtype=torch.int32, device=self.dev)
            call("ferry_exchange_ownership", self.h, C.c_void_p(st.cuda_stream), C.c_void_p(d_row.data_ptr()),
                 len(row), C.c_void_p(d_all.data_ptr()))
            done = torch.cuda.Event()
            done.record(st)
        deadline = time.monotonic() + timeout_s
        while not done.query():
            if time.monotonic() > deadline:
                h = self.h
                self._abort = threading.Thread(target=lambda: _abi.lib().ferry_comm_abort(h), daemon=True)
                self._abort.start()
                raise TimeoutError(f"ownership exchange on rank {self.rank} not done within {timeout_s} s")
            time.sleep(5e-5)
        return d_all.cpu().numpy()

    def wait_aborted(self, timeout_s: float = 120.0) -> None:
        """Join the abort a missed deadline started (no-op without one)."""
        t = getattr(self, "_abort", None)
        if t is not None:
            t.join(timeout_s)
            self._abort = None

    def close(self):
        self.wait_aborted()
        if self.h:
            call("ferry_comm_destroy", self.h)
            self.h = None


def exchange_ownership(finished: int, admitted: int, owned: np.ndarray, cap: int, total_requests: int,
                       device=None, usage: int = 0, with_rows: bool = False, comm: "OwnershipComm | None" = None):
    """The page-ownership exchange: one all_gather of fixed-size rows -- over
    ``comm`` (the C ABI's NCCL exchange) when given, else the default process
    group (NCCL when ``device`` is a CUDA device, else its backend)."""
    row = ownership_row(finished, admitted, owned, cap, usage)
    if comm is not None:
        rows = comm.all_gather(row).astype(np.int64)
    else:
        import torch
        import torch.distributed as dist

        t = torch.from_numpy(row)
        if device is not None:
            t = t.to(device)
        out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
        dist.all_gather(out, t)
        rows = torch.stack(out).cpu().numpy()
    merged = merge_ownership(rows, total_requests)
    return (merged, rows) if with_rows else merged


@dataclasses.dataclass
class ClusterStats:
    rank: int
    tokens: int
    ticks: int
    device_ms: float
    steals: int
    stolen_tasks: int
    migrated_units: int
    migrated_bytes: int
    gathered_bytes: int
    tick_ms: list
    mig_ms: float = 0.0          # device time of the migration kernels
    mig_event_bytes: int = 0     # bytes those kernels moved
    rebalances: int = 0          # rebalance orders this rank executed (LLX)
    window_ms: float = 0.0       # device time of the timed tick window (run(window=...))
    window_tokens: int = 0       # tokens decoded inside it
    window_gathered_bytes: int = 0  # miss-gather bytes inside it
    h2d_bytes: int = 0           # host -> device query bytes of the window (host_q)
    d2h_bytes: int = 0           # device -> host output bytes of the window (outputs)


# ---------------------------------------------------------------- per-rank runner (GPU)


class RankRunner:
    """One GPU's share of a multi-GPU job."""

    def __init__(self, w: Workload, total_requests: int, world: int, rank: int, device: int,
                 slots: int, max_batch: int, steal_batch: int = 4,
                 migrate_mode: int = _abi.MIGRATE_DELTA, pool_units: int | None = None,
                 policy: "_abi.StealPolicy | None" = None, host_q: bool = False,
                 q_steps: int | None = None, log_path: str | None = None, step_chunks: int = 1):
        import torch
        import torch.distributed as dist

        from .engine import Decoder

        self.w, self.world, self.rank, self.total = w, world, rank, total_requests
        self.dev = torch.device("cuda", device)
        torch.cuda.set_device(self.dev)
        wl = dataclasses.replace(w, num_requests=slots)
        self.dec = Decoder(wl, device)
        self.dec.register_pool(units=pool_units or min(total_requests * w.lanes_per_req * w.max_pages, 1 << 17))
        # the executor's ferry_decode_step pipelined over request chunks (ferry_step_chunks)
        self.dec.step_chunks(step_chunks)
        # query table [total][steps][L][Hq][128]: resident in HBM, or (host_q)
        # in pinned, device-mapped host memory that the executor's query
        # gather reads over the host link every tick
        # (q_steps: rows per request; later steps reuse them cyclically)
        q_steps = w.steps if q_steps is None else min(q_steps, w.steps)
        q = np.stack([q_stream(w, r, steps=q_steps) for r in range(total_requests)])
        self.host_q = host_q
        if host_q:
            from .engine import PinnedPool

            self.q_pool = PinnedPool(q.nbytes)
            self.q_pool.numpy(np.uint16)[:] = q.view(np.uint16).ravel()
            q_ptr = self.q_pool.ptr
        else:
            self.q_table = torch.from_numpy(q).to(self.dev)
            q_ptr = C.c_void_p(self.q_table.data_ptr())
        self.row_elems = w.num_layers * w.q_heads * w.head_dim
        self.deque = C.c_void_p()
        call("ferry_deque_create", device, max(slots, 1), C.byref(self.deque))
        cfg = _abi.ExecCfg(rank=rank, world=world, max_batch=max_batch, steal_batch=steal_batch,
                           migrate_mode=migrate_mode, steps_per_req=w.steps, total_requests=total_requests,
                           q_table_steps=q_steps)
        self.exec = C.c_void_p()
        call("ferry_exec_create", self.dec.ctx, self.deque, C.byref(cfg), q_ptr, C.byref(self.exec))
        if policy is not None:
            call("ferry_exec_policy", self.exec, C.byref(policy))
        if log_path is not None:  # one record per steal (ferry_b200.decisions reads it)
            call("ferry_exec_log", self.exec, log_path.encode())
        self.slots = slots
        self.peer_deques = []
        self.comm = None
        if world > 1:
            h = (C.c_uint8 * _abi.CTX_HANDLE_BYTES)()
            call("ferry_ctx_export", self.dec.ctx, h)
            dh = (C.c_uint8 * 64)()
            call("ferry_deque_export", self.deque, dh)
            mine = (bytes(h), bytes(dh), slots)
            allh = [None] * world
            dist.all_gather_object(allh, mine)
            slot = 0
            for p in range(world):
                if p == rank:
                    continue
                ch, qh, pslots = allh[p]
                call("ferry_ctx_import", self.dec.ctx, slot, (C.c_uint8 * _abi.CTX_HANDLE_BYTES).from_buffer_copy(ch))
                pq = C.c_void_p()
                call("ferry_deque_import", device, (C.c_uint8 * 64).from_buffer_copy(qh), pslots, C.byref(pq))
                self.peer_deques.append(pq)
                call("ferry_exec_link_peer", self.exec, p, slot, pq)
                slot += 1

    def run(self, home: np.ndarray, join: np.ndarray, epoch: int = 4, max_ticks: int = 100000,
            exchange_device=None, llx: float | None = None, window: tuple | None = None,
            n_pages: np.ndarray | None = None, outputs: bool = False, barrier=None) -> ClusterStats:
        """Tick until every request of the job finished on some GPU. home/join:
        each request's home rank and arrival tick; n_pages: each request's
        context in pages (default: the workload's). With ``exchange_device`` set
        (ranks on distinct GPUs) the ownership exchange runs over the C ABI's
        NCCL communicator, created here before the timed region.

        window=(w0, w1): run exactly w1 ticks (every rank the same count, so
        the ranks take the same exchanges) and time ticks [w0, w1) with CUDA
        events, bracketed by ``barrier()`` and a synchronize on both sides.
        outputs: copy every tick's attention output to pinned host memory
        (ferry_exec_output) -- the device -> host read of an end-to-end step."""
        import torch

        if exchange_device is not None and self.comm is None:
            self.comm = OwnershipComm(self.dev.index)
        comm = self.comm if exchange_device is not None else None
        st = torch.cuda.current_stream(self.dev)
        mine = np.nonzero(home == self.rank)[0]
        pages_of = np.full(len(home), self.w.init_pages, np.int32) if n_pages is None else np.asarray(n_pages, np.int32)
        admitted = finished = tokens = ticks = steals = stolen = 0
        mig_ms, mig_b = 0.0, 0
        tick_ms = []
        self.dec.all_stats(reset=True)
        s = _abi.TickStats()
        owned = np.zeros(self.slots, np.int32)
        n_owned = C.c_int()
        u_steps, u_reqs = C.c_int64(), C.c_int32()
        rebalances = 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0, w1 = window if window is not None else (0, max_ticks)
        last = w1 if window is not None else max_ticks
        win_tokens = win_h2d = win_d2h = 0
        g0 = 0
        host_out = n_out = None
        if outputs:
            host_out = torch.empty((self.slots, self.row_elems), dtype=torch.float32).pin_memory()
            n_out = C.c_int()
        started = False
        if w0 == 0:
            if barrier is not None:
                torch.cuda.synchronize(self.dev)
                barrier()
                torch.cuda.synchronize(self.dev)
            e0.record(st)
            started = True
        t = 0
        while t < last:
            if window is not None and t == w0 and w0 > 0:
                torch.cuda.synchronize(self.dev)
                if barrier is not None:
                    barrier()
                    torch.cuda.synchronize(self.dev)
                g0 = self.dec.all_stats()[1]
                e0.record(st)
                started = True
            arr = mine[join[mine] == t].astype(np.int32)
            if len(arr):
                pages = pages_of[arr]
                call("ferry_exec_admit", self.exec, arr.ctypes.data_as(C.c_void_p),
                     pages.ctypes.data_as(C.c_void_p), len(arr))
                admitted += len(arr)
            call("ferry_exec_tick", self.exec, C.c_void_p(st.cuda_stream), C.byref(s))
            tokens += s.decoded
            finished += s.finished
            if w0 <= t < w1:
                win_tokens += s.decoded
                if self.host_q:
                    win_h2d += s.decoded * self.row_elems * 2
            if outputs and s.decoded:
                call("ferry_exec_output", self.exec, C.c_void_p(st.cuda_stream), C.c_void_p(host_out.data_ptr()),
                     None, self.slots, C.byref(n_out))
                if w0 <= t < w1:
                    win_d2h += n_out.value * self.row_elems * 4
            if s.stolen:
                steals += 1
                stolen += s.stolen
                mig_ms += s.mig_ms
                mig_b += s.mig_bytes
            tick_ms.append(s.tick_ms)
            t += 1
            if t % epoch == 0:
                call("ferry_exec_owned", self.exec, owned.ctypes.data_as(C.c_void_p), self.slots,
                     C.byref(n_owned))
                call("ferry_exec_usage", self.exec, C.byref(u_steps), C.byref(u_reqs))
                (_, fin_all, adm_all), rows = exchange_ownership(
                    finished, admitted, owned[:n_owned.value], self.slots, self.total, exchange_device,
                    usage=u_steps.value, with_rows=True, comm=comm)
                call("ferry_exec_set_global", self.exec, adm_all - fin_all)
                if llx is not None and fin_all < self.total:
                    plan = llx_plan(rows[:, 3], rows[:, 2], llx)
                    if plan is not None and plan[1] == self.rank:
                        call("ferry_exec_rebalance", self.exec, plan[0], plan[2])
                        rebalances += 1
                if fin_all >= self.total:
                    break
        if not started:  # the job ended before the window opened: an empty window
            e0.record(st)
            if barrier is not None:  # the barrier the window's start would have taken
                torch.cuda.synchronize(self.dev)
                barrier()
        e1.record(st)
        torch.cuda.synchronize(self.dev)
        if window is not None and barrier is not None:
            barrier()
        self.dec.check()
        g_units, g_bytes, m_units, m_bytes = self.dec.all_stats()[:4]
        dev_ms = e0.elapsed_time(e1)
        return ClusterStats(rank=self.rank, tokens=tokens, ticks=t, device_ms=dev_ms,
                            steals=steals, stolen_tasks=stolen, migrated_units=m_units,
                            migrated_bytes=m_bytes, gathered_bytes=g_bytes, tick_ms=tick_ms,
                            mig_ms=mig_ms, mig_event_bytes=mig_b, rebalances=rebalances,
                            window_ms=dev_ms if window is not None else 0.0, window_tokens=win_tokens,
                            window_gathered_bytes=g_bytes - g0 if window is not None else g_bytes,
                            h2d_bytes=win_h2d, d2h_bytes=win_d2h)

    def close(self):
        if self.comm is not None:
            self.comm.close()
            self.comm = None
        for pq in self.peer_deques:
            call("ferry_deque_destroy", pq)
        self.peer_deques = []
        if self.exec:
            call("ferry_exec_destroy", self.exec)
            self.exec = None
        if self.deque:
            call("ferry_deque_destroy", self.deque)
            self.deque = None
        self.dec.close()
        if getattr(self, "q_pool", None) is not None:
            self.q_pool.close()
            self.q_pool = None


def job_schedule(w: Workload, total_requests: int, world: int, policy: str, rate: float | None = None):
    """Arrival tick and home rank of each request of a multi-GPU job (Poisson
    arrivals at ``rate`` requests/s box-wide, default the workload's)."""
    wj = dataclasses.replace(w, num_requests=total_requests, arrival_rate=rate or w.arrival_rate)
    join = arrival_ticks(wj)
    join = join - join.min()
    home = assign_ranks(total_requests, world, policy, w.seed)
    return home, join


def slots_needed(home: np.ndarray, world: int, max_batch: int) -> int:
    """Request slots per GPU: enough for the busiest home plus stolen work."""
    return int(max(np.bincount(home, minlength=world).max(), max_batch) + max_batch)


def ceil_div(a: int, b: int) -> int:
    return int(math.ceil(a / b))
