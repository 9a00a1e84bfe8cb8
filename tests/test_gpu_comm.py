"""The page-ownership exchange through the C ABI (ferry_comm_* /
ferry_exchange_ownership, an NCCL all_gather of fixed-size int32 rows): one
rank on one GPU, and two ranks on two GPUs with the rows merged the way the
cluster runner merges them."""
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


def test_exchange_single_rank(torch_cuda):
    from ferry_b200 import _abi

    t = torch_cuda
    uid = (C.c_uint8 * _abi.COMM_ID_BYTES)()
    _abi.call("ferry_comm_unique_id", uid)
    h = C.c_void_p()
    _abi.call("ferry_comm_create", 0, 1, 0, uid, C.byref(h))
    try:
        dev = t.device("cuda", 0)
        row = t.arange(37, dtype=t.int32, device=dev) * 3 - 5
        out = t.full((1, 37), -9, dtype=t.int32, device=dev)
        st = t.cuda.current_stream(dev)
        for _ in range(2):
            _abi.call("ferry_exchange_ownership", h, C.c_void_p(st.cuda_stream), C.c_void_p(row.data_ptr()), 37,
                      C.c_void_p(out.data_ptr()))
            assert (out.cpu()[0] == row.cpu()).all()
        with pytest.raises(_abi.FerryError):
            _abi.call("ferry_exchange_ownership", h, None, C.c_void_p(row.data_ptr()), 0, C.c_void_p(out.data_ptr()))
        with pytest.raises(_abi.FerryError):
            _abi.call("ferry_comm_create", 0, 2, 2, uid, C.byref(C.c_void_p()))  # rank outside world
        t.cuda.synchronize(dev)
        _abi.call("ferry_comm_abort", h)  # nothing in flight: the comm just becomes unusable
        with pytest.raises(_abi.FerryError):
            _abi.call("ferry_exchange_ownership", h, C.c_void_p(st.cuda_stream), C.c_void_p(row.data_ptr()), 37,
                      C.c_void_p(out.data_ptr()))
    finally:
        _abi.call("ferry_comm_destroy", h)


def _pair_worker(rank, port, out):
    import os

    import torch
    import torch.distributed as dist

    from ferry_b200.cluster import OwnershipComm, merge_ownership, ownership_row

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    comm = OwnershipComm(rank)
    try:
        owned = np.array([rank, 2 + rank, 10 + rank], np.int32)  # requests this rank holds
        rows = comm.all_gather(ownership_row(5 * rank, 7 + rank, owned, cap=6, usage=100 + rank))
        owner, fin, adm = merge_ownership(rows.astype(np.int64), 12)
        out.put((rank, rows.tolist(), owner.tolist(), fin, adm))
    finally:
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


def test_exchange_two_gpus(torch_cuda):
    import multiprocessing as mp
    import socket

    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_pair_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1] == res[1][1]  # both ranks hold every row
    rows = np.array(res[0][1])
    assert rows.shape == (2, 10) and rows[:, 3].tolist() == [100, 101]
    for rank, _, owner, fin, adm in res:
        assert fin == 5 and adm == 15
        assert [owner[i] for i in (0, 2, 10)] == [0, 0, 0] and [owner[i] for i in (1, 3, 11)] == [1, 1, 1]
        assert owner[5] == -1


def _deadline_worker(rank, port, out, gone):
    """Rank 1 joins the first exchange, then never joins the second (it stays
    alive, its memory intact, until rank 0 has given up). Rank 0's second
    exchange must reach its deadline, abort the communicator (ncclCommAbort
    ends the collective in flight) and raise."""
    import os
    import time

    import torch
    import torch.distributed as dist

    from ferry_b200 import _abi
    from ferry_b200.cluster import OwnershipComm, ownership_row

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    comm = OwnershipComm(rank)
    try:
        comm.all_gather(ownership_row(0, 1, np.array([rank], np.int32), cap=4))  # epoch 1: both ranks
        if rank == 1:
            gone.wait(120)  # never joins epoch 2; leaves once rank 0 has given up
            _abi.call("ferry_comm_abort", comm.h)  # its peer is gone: no collective teardown
            out.put((1, "left", 0.0, 0))
            return
        deadline = 2.0
        t0 = time.monotonic()
        try:
            comm.all_gather(ownership_row(0, 1, np.array([0], np.int32), cap=4), timeout_s=deadline)
            out.put((0, "no timeout", time.monotonic() - t0, 0))
        except TimeoutError:
            waited = time.monotonic() - t0
            comm.wait_aborted()  # the abort's teardown, on its helper thread
            torch.cuda.synchronize(rank)  # the aborted collective has left the stream
            try:  # the communicator is unusable after the abort
                comm.all_gather(np.zeros(8, np.int32), timeout_s=1.0)
                rc = 0
            except _abi.FerryError as e:
                rc = e.code
            out.put((0, "timeout", waited - deadline, rc))
        finally:
            gone.set()
    finally:
        comm.close()


def test_exchange_deadline_aborts_when_a_rank_never_joins(torch_cuda):
    """Failure detection on the ownership exchange without a GPU fault: a peer
    that never joins a collective (it stays alive and idle) ends the other
    rank's exchange at its deadline; NVLS is off, as for every test of a
    departed rank."""
    import multiprocessing as mp
    import os
    import socket

    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # inherited by the spawned ranks
    ctx = mp.get_context("spawn")
    q, gone = ctx.Queue(), ctx.Event()
    ps = [ctx.Process(target=_deadline_worker, args=(r, port, q, gone)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=240) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, what, late, rc), (_, left, _, _) = res
    assert what == "timeout" and left == "left"
    assert 0.0 <= late <= 1.0  # raised within the deadline plus 1 s
    from ferry_b200 import _abi

    assert rc == _abi.E_STATE
