"""Host-side logic of the multi-GPU runtime on CPU: rank assignment, the
ownership table, and the ownership exchange across two gloo ranks."""
import os
import socket

import numpy as np
import torch.multiprocessing as mp


def test_assign_ranks_policies():
    from ferry_b200.cluster import assign_ranks

    rr = assign_ranks(10, 4, "rr")
    assert rr.tolist() == [0, 1, 2, 3, 0, 1, 2, 3, 0, 1]
    z = assign_ranks(4000, 8, "zipf", seed=42)
    assert (z == assign_ranks(4000, 8, "zipf", seed=42)).all()
    share = np.bincount(z, minlength=8) / len(z)
    assert share[:2].sum() > 0.7 and share[0] > share[1] > share[7]


def test_merge_ownership():
    from ferry_b200.cluster import merge_ownership, ownership_row

    rows = np.stack([ownership_row(3, 7, np.array([0, 5, 6]), 4),
                     ownership_row(1, 2, np.array([2]), 4)])
    owner, fin, adm = merge_ownership(rows, 8)
    assert owner.tolist() == [0, -1, 1, -1, -1, 0, 0, -1] and fin == 4 and adm == 9


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _exchange_worker(rank, world, port, out):
    import torch.distributed as dist

    from ferry_b200.cluster import exchange_ownership

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    owned = np.array([rank, rank + 2], np.int32)
    owner, fin, adm = exchange_ownership(finished=rank + 1, admitted=10 * (rank + 1), owned=owned,
                                         cap=4, total_requests=6)
    out.put((rank, owner.tolist(), fin, adm))
    dist.destroy_process_group()


def test_exchange_ownership_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    for rank, owner, fin, adm in res:
        assert owner == [0, 1, 0, 1, -1, -1] and fin == 3 and adm == 30
