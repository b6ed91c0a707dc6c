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
        # grouped-query heads: 12 query heads over 3 KV heads, and 8 over 2 (paged)
        W.make_dense("gqa_d", 2, 12, 1, 200, scale_mode="bh", o_dtype=torch.float32, seed=34, kv_heads=3),
        W.make_paged("gqa_p", 2, 8, [40, 150], page=16, seed=35, o_dtype=torch.float32, kv_heads=2),
    ]


def _shard(wk, world, rank):
    return S.shard_workload(wk, S.head_range(wk.heads, world, rank, wk.kv_group))


def test_head_range_keeps_kv_groups_whole():
    for n_heads, g, world in ((32, 4, 8), (32, 4, 3), (12, 3, 2), (8, 8, 1)):
        ranges = [S.head_range(n_heads, world, r, g) for r in range(world)]
        assert ranges[0].start == 0 and ranges[-1].stop == n_heads
        assert all(a.stop == b.start for a, b in zip(ranges, ranges[1:]))
        assert all(r.start % g == 0 and len(r) % g == 0 for r in ranges)
        sizes = [len(r) // g for r in ranges]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        S.head_range(30, 2, 0, 4)
    wk = W.make_dense("g", 1, 8, 1, 32, o_dtype=torch.float32, kv_heads=2)
    with pytest.raises(ValueError):
        S.shard_workload(wk, range(0, 2))  # half a KV group


@pytest.mark.parametrize("world", [2, 3])
def test_shard_then_assemble_matches_full(oracle, world):
    for wk in _small_workloads():
        if wk.heads // wk.kv_group < world:
            continue
        full, _, err, _ = oracle.forward_workload_c(wk)
        assert err == 0
        parts = []
        for r in range(world):
            sub = _shard(wk, world, r)
            assert sub.kv_group == wk.kv_group
            o, _, err, _ = oracle.forward_workload_c(sub)
            assert err == 0
            parts.append(torch.from_numpy(o))
        got = S.assemble_heads(parts, wk.batch, wk.heads, wk.seq_q, world, wk.kv_group).numpy()
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
            sub = _shard(wk, world, rank)
            o, _, err, _ = O.forward_workload_c(sub, nthreads=1)
            full = S.gather_output(torch.from_numpy(o), wk.batch, wk.heads, wk.seq_q, kv_group=wk.kv_group)
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


def _idle_rank_main(rank, world, port, out_dir):
    """A world larger than the KV heads: the last rank owns no head.  It still takes
    part in the gather (with an empty block) and computes nothing."""
    import torch.distributed as dist

    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wk = W.make_paged("gqa_p", 2, 8, [40, 150], page=16, seed=35, o_dtype=torch.float32, kv_heads=2)
        sub = _shard(wk, world, rank)
        if sub.total_work:
            o, _, _, _ = O.forward_workload_c(sub, nthreads=1)
            o = torch.from_numpy(o)
        else:
            o = torch.zeros(0, wk.head_dim)
        np.save(os.path.join(out_dir, f"idle_r{rank}_n.npy"), np.array([sub.total_work, sub.n_bh]))
        full = S.gather_output(o, wk.batch, wk.heads, wk.seq_q, kv_group=wk.kv_group)
        np.save(os.path.join(out_dir, f"idle_r{rank}.npy"), full.numpy())
    finally:
        dist.destroy_process_group()


def test_world_larger_than_kv_heads_leaves_a_rank_idle(oracle, tmp_path):
    wk = W.make_paged("gqa_p", 2, 8, [40, 150], page=16, seed=35, o_dtype=torch.float32, kv_heads=2)
    assert len(S.head_range(8, 3, 2, 4)) == 0
    world = 3
    mp.spawn(_idle_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    full, _, _, _ = oracle.forward_workload_c(wk)
    assert np.load(tmp_path / "idle_r2_n.npy").tolist() == [0, 0]
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"idle_r{r}.npy"), full), r


def _chunked_rank_main(rank, world, port, out_dir):
    """Each rank computes its head block one batch entry at a time and all-gathers
    each entry's O as it is done (forward_and_gather); the oracle stands in for the
    kernel."""
    import torch.distributed as dist

    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wk = W.make_dense("c", 3, 4, 20, 20, causal=True, o_dtype=torch.float32, seed=37)
        sub = _shard(wk, world, rank)
        o_local = torch.zeros(sub.n_bh * sub.seq_q, sub.head_dim)
        done = []

        def forward_chunk(items):
            piece = W.Workload(**{**sub.__dict__, "worklist": sub.worklist[items]})
            o, written, _, _ = O.forward_workload_c(piece, nthreads=1)
            rows = (piece.worklist[:, 1].long() * sub.seq_q + piece.worklist[:, 0].long())
            o_local[rows] = torch.from_numpy(o)[rows]
            done.append(items)

        chunks = S.row_chunks(sub, 3)
        rows_c = chunks[0][1].stop - chunks[0][1].start
        out = torch.empty(len(chunks), world, rows_c, sub.head_dim)
        S.forward_and_gather(forward_chunk, chunks, o_local, out)
        parts = list(out.transpose(0, 1).reshape(world, -1, sub.head_dim))
        full = S.assemble_heads(parts, wk.batch, wk.heads, wk.seq_q, world)
        np.save(os.path.join(out_dir, f"chunked_r{rank}.npy"), full.numpy())
        np.save(os.path.join(out_dir, f"chunked_r{rank}_n.npy"), np.array([len(done)]))
    finally:
        dist.destroy_process_group()


def test_chunked_forward_and_gather_over_two_gloo_ranks(oracle, tmp_path):
    """The overlapped gather's bookkeeping: chunks of (batch, head) rows, out[c, r] holding
    rank r's chunk c, and out.transpose(0, 1) giving each rank's head block in order,
    which assemble into the single-process result."""
    world = 2
    mp.spawn(_chunked_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    wk = W.make_dense("c", 3, 4, 20, 20, causal=True, o_dtype=torch.float32, seed=37)
    full, _, _, _ = oracle.forward_workload_c(wk)
    for r in range(world):
        assert np.load(tmp_path / f"chunked_r{r}_n.npy")[0] == 3
        assert np.array_equal(np.load(tmp_path / f"chunked_r{r}.npy"), full), r


def _peer_fail_main(rank, world, port, out_dir, fail_at):
    """PeerOutput's setup with the IPC calls faked: the step named by fail_at fails
    on rank 1 only, and every rank must raise the same error and release what it
    allocated and opened."""
    import json

    import torch.distributed as dist

    import hyperion_b200 as H

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    log = {"freed": [], "closed": [], "opened": []}

    def alloc(nbytes):
        if fail_at == "alloc" and rank == 1:
            raise RuntimeError("hyperion_ipc_alloc failed (status 5): out of memory")
        return 1000 + rank, bytes([rank]) * 64

    def open_(handle):
        if fail_at == "open" and rank == 1:
            raise RuntimeError("hyperion_ipc_open failed (status 5): peer access refused")
        log["opened"].append(handle[0])
        return 2000 + handle[0]

    H.ipc_alloc, H.ipc_open = alloc, open_
    H.ipc_close = lambda p: log["closed"].append(p)
    H.ipc_free = lambda p: log["freed"].append(p)
    try:
        try:
            S.PeerOutput(16, 128, torch.bfloat16, None)
            log["error"] = None
        except RuntimeError as e:
            log["error"] = str(e)
        with open(os.path.join(out_dir, f"peer_{fail_at}_r{rank}.json"), "w") as f:
            json.dump(log, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_at", ["alloc", "open"])
def test_peer_output_setup_fails_on_every_rank_together(tmp_path, fail_at):
    import json

    world = 3
    mp.spawn(_peer_fail_main, args=(world, _free_port(), str(tmp_path), fail_at), nprocs=world, join=True)
    logs = [json.load(open(tmp_path / f"peer_{fail_at}_r{r}.json")) for r in range(world)]
    errors = {log["error"] for log in logs}
    assert len(errors) == 1 and None not in errors, errors
    assert "rank 1" in errors.pop()
    for r, log in enumerate(logs):
        if fail_at == "alloc":
            assert log["opened"] == [] and log["freed"] == ([] if r == 1 else [1000 + r])
        else:
            assert log["freed"] == [1000 + r]
            assert sorted(log["closed"]) == sorted(2000 + h for h in log["opened"])
            if r != 1:
                assert sorted(log["opened"]) == [q for q in range(world) if q != r]
