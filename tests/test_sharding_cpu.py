"""(batch x head) sharding host logic on a 2-rank gloo world (CPU): shard
boundaries, the gather, and that a rank failing between steps surfaces as an
error on its peer instead of a hang.  The per-shard compute is the oracle
(CPU), injected in place of the CUDA kernel."""

import datetime
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from python import sharding, workloads


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_attention(q, k, v, mask):
    from oracle import oracle

    D = q.shape[-1]
    return torch.from_numpy(oracle.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                             mask.numpy(), 1.0 / math.sqrt(D)))


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_gather(rank, world, port, result_dir):
    import sys

    _init(rank, world, port)
    cfg = dict(workloads.CONFIGS["c2"], B=1, H=7, N=64)  # 7 heads: uneven over 2 ranks
    lo, hi = sharding.shard_range(7, world, rank)
    q, k, v, m = workloads.make_inputs(cfg, seed=4, heads=(lo, hi))
    out = sharding.sharded_sparse_attention(q, k, v, m, gather=True, total_heads=7, attention=_oracle_attention)
    np.save(os.path.join(result_dir, f"out{rank}.npy"), out.numpy())
    dist.barrier()
    dist.destroy_process_group()


def _worker_fail(rank, world, port, result_dir):
    _init(rank, world, port, timeout_s=10)
    q, k, v, m = workloads.make_inputs(dict(workloads.CONFIGS["c2"], B=1, H=2, N=32), seed=1, heads=(rank, rank + 1))
    out = _oracle_attention(q, k, v, m)
    if rank == 1:
        # This rank dies between steps, before the collective.
        os._exit(3)
    try:
        sharding.gather_heads(out, 2)
        status = "no error"
    except Exception as e:  # the peer's death must surface as an error
        status = "error: " + type(e).__name__
    with open(os.path.join(result_dir, "status0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_shard_range_partitions():
    for total in (0, 1, 7, 192, 4096):
        for world in (1, 2, 3, 4, 8):
            ranges = [sharding.shard_range(total, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            for (a, b), (c, d) in zip(ranges, ranges[1:]):
                assert b == c
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(8, 2, 2)


def test_shard_heads_matches_make_inputs_slices():
    q, k, v, m = workloads.make_inputs("c2", seed=2, B=3, H=5, N=32)
    for rank in range(4):
        lo, hi = sharding.shard_range(15, 4, rank)
        qs, _, _, ms = workloads.make_inputs("c2", seed=2, B=3, H=5, N=32, heads=(lo, hi))
        assert torch.equal(sharding.shard_heads(q, 4, rank), qs)
        assert torch.equal(sharding.shard_heads(m, 4, rank), ms)


def test_two_rank_gather_equals_single_process(tmp_path):
    port = _free_port()
    mp.start_processes(_worker_gather, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    cfg = dict(workloads.CONFIGS["c2"], B=1, H=7, N=64)
    q, k, v, m = workloads.make_inputs(cfg, seed=4)
    want = _oracle_attention(q, k, v, m).numpy()
    for r in range(2):
        got = np.load(tmp_path / f"out{r}.npy")
        assert np.array_equal(got, want)


def test_dead_rank_surfaces_as_error(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_worker_fail, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=False)
    for p in ctx.processes:
        p.join(timeout=60)
        assert not p.is_alive(), "a rank hung"
    status = (tmp_path / "status0.txt").read_text()
    assert status.startswith("error"), status
