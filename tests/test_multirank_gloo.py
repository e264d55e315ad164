"""Multi-rank host logic on CPU (gloo, world size 2): slice sharding covers
every slice exactly once, per-rank results assemble into the single-process
result, and the step time reported is the max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import importlib
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch

    import oracle
    from tests import cases as C

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shard = importlib.import_module("not-cute-zig_b200.shard")
    bh, s, d = 5, 37, 16
    p = C.normal_problem(bh, s, d, True, 21, oracle)
    lo, hi = shard.slice_range(bh, world, rank)
    n = s * d
    sub = C.Problem(hi - lo, s, d, (n,) * 4, True, p.scale)
    sub.q, sub.k, sub.v = p.q[lo * n:hi * n], p.k[lo * n:hi * n], p.v[lo * n:hi * n]
    local = torch.from_numpy(C.reference(sub, oracle)) if hi > lo else torch.zeros(0)
    parts = [None] * world
    dist.all_gather_object(parts, (lo, hi, local.numpy()))
    t = torch.tensor([10.0 + rank])  # fake per-rank step times
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        full = np.concatenate([a for (_, _, a) in sorted(parts, key=lambda x: x[0])])
        np.save(result_path, np.concatenate([[t.item()], full]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_shards_reassemble(tmp_path, oracle_mod):
    from tests import cases as C

    path = str(tmp_path / "out.npy")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    res = np.load(path)
    assert res[0] == 11.0  # max over ranks
    p = C.normal_problem(5, 37, 16, True, 21, oracle_mod)
    assert np.array_equal(res[1:].astype(np.float32), C.reference(p, oracle_mod))
