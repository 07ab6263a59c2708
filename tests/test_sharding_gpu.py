"""(batch x head) sharding on two GPUs over NCCL: each rank runs the CUDA
kernels on its contiguous block of the flattened B*H range and the output
blocks are all-gathered over NVLink (python/sharding.py, the NCCL branch of
gather_heads).  Every rank's gathered output must equal, bit for bit, the
one-GPU sparse_attention() over all heads, including an uneven split.

Two processes (one per GPU) are spawned; the test is skipped on a machine
with fewer than two GPUs."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from python import sharding, workloads

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_dir, name, heads_total, overrides):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    from python import sparse_attention, sparse_attn_cuda

    lo, hi = sharding.shard_range(heads_total, world, rank)
    q, k, v, m = workloads.make_inputs(name, seed=11, device=dev, heads=(lo, hi), **overrides)
    out = sharding.sharded_sparse_attention(q, k, v, m, gather=True, total_heads=heads_total)
    sparse_attn_cuda.device_status()
    np.save(os.path.join(result_dir, f"gathered{rank}.npy"), out.view(torch.int16).cpu().numpy())
    if rank == 0:
        # One GPU over every head: the same inputs, unsharded.
        qa, ka, va, ma = workloads.make_inputs(name, seed=11, device=dev, heads=(0, heads_total), **overrides)
        ref = sparse_attention(qa, ka, va, ma)
        sparse_attn_cuda.device_status()
        np.save(os.path.join(result_dir, "one_gpu.npy"), ref.view(torch.int16).cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name,heads_total,overrides", [
    ("c5", 4096, {}),                       # the large-batch workload, 2048 heads per rank
    ("c1", 23, {"B": 1, "H": 23}),          # uneven split: 12 + 11 heads
    ("c3", 6, {"B": 1, "H": 6}),            # bf16, head dim 128, block-sparse
])
def test_nccl_gather_matches_one_gpu(tmp_path, name, heads_total, overrides):
    world = 2
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path), name, heads_total, overrides), nprocs=world,
                       join=True, start_method="spawn")
    ref = np.load(tmp_path / "one_gpu.npy")
    for r in range(world):
        got = np.load(tmp_path / f"gathered{r}.npy")
        assert got.shape == ref.shape, (got.shape, ref.shape)
        assert np.array_equal(got, ref), f"rank {r}: gathered output differs from the one-GPU output"
