"""Multi-GPU host logic on the CPU: head sharding, the output gather over gloo ranks.

Each rank runs the forward on its own head block; here the CPU oracle stands in for
the kernel, so the check is that sharding, per-rank computation and the gather give
exactly the single-process result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from hyperion_b200 import sharding as S
from hyperion_b200 import workloads as W


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_head_range_partitions_heads(world):
    for n_heads in (1, 7, 8, 32, 33, 64):
        if n_heads < world:
            continue
        ranges = [S.head_range(n_heads, world, r) for r in range(world)]
        assert ranges[0].start == 0 and ranges[-1].stop == n_heads
        assert all(a.stop == b.start for a, b in zip(ranges, ranges[1:]))
        sizes = [len(r) for r in ranges]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        S.head_range(8, 2, 2)


def _small_workloads():
    return [
        W.make_dense("d", 2, 5, 40, 40, causal=True, scale_mode="head", o_dtype=torch.float32, seed=31),
        W.make_dense("b", 2, 3, 1, 300, scale_mode="bh", o_dtype=torch.float32, seed=32),
        W.make_paged("p", 3, 4, [17, 64, 130], page=16, seed=33, o_dtype=torch.float32),
    ]


@pytest.mark.parametrize("world", [2, 3])
def test_shard_then_assemble_matches_full(oracle, world):
    for wk in _small_workloads():
        full, _, err, _ = oracle.forward_workload_c(wk)
        assert err == 0
        parts = []
        for r in range(world):
            sub = S.shard_workload(wk, S.head_range(wk.heads, world, r))
            o, _, err, _ = oracle.forward_workload_c(sub)
            assert err == 0
            parts.append(torch.from_numpy(o))
        got = S.assemble_heads(parts, wk.batch, wk.heads, wk.seq_q, world).numpy()
        assert np.array_equal(got, full), wk.name


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist

    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for i, wk in enumerate(_small_workloads()):
            sub = S.shard_workload(wk, S.head_range(wk.heads, world, rank))
            o, _, err, _ = O.forward_workload_c(sub, nthreads=1)
            full = S.gather_output(torch.from_numpy(o), wk.batch, wk.heads, wk.seq_q)
            np.save(os.path.join(out_dir, f"r{rank}_w{i}.npy"), full.numpy())
            np.save(os.path.join(out_dir, f"r{rank}_w{i}_err.npy"), np.array([err]))
    finally:
        dist.destroy_process_group()


def test_gather_over_two_gloo_ranks(oracle, tmp_path):
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for i, wk in enumerate(_small_workloads()):
        full, _, _, _ = oracle.forward_workload_c(wk)
        for r in range(world):
            assert np.load(tmp_path / f"r{r}_w{i}_err.npy")[0] == 0
            assert np.array_equal(np.load(tmp_path / f"r{r}_w{i}.npy"), full), (wk.name, r)
