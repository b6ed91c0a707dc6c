"""The output written to peer buffers as well as O (hyperion_apex_kernel o_peers).

On one GPU the "peers" are other buffers of the same device: every kernel (tile,
row with and without KV splits, both grouped kernels) must leave each of them equal
to O, bit for bit, and O itself must still meet the oracle bar.  On two GPUs,
PeerOutput maps each rank's gathered buffer into the other rank and the forward
stores its head block into both; the result must equal the NCCL all-gather of the
same blocks, bit for bit.  The same blocks moved by the copy engines
(sharding.forward_and_push: the forward in runs, each run's rows pushed into the
other rank's buffer) must meet the oracle bar on every rank.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from hyperion_b200 import sharding as S
from hyperion_b200 import workloads as W

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _workload(kind, o_dtype):
    if kind == "prefill":
        return W.make_dense("po_pre", 2, 3, 300, 300, causal=True, o_dtype=o_dtype, seed=81)
    if kind == "decode":
        return W.make_dense("po_dec", 3, 4, 1, 5000, o_dtype=o_dtype, seed=82)
    if kind == "paged":
        return W.make_paged("po_paged", 4, 4, [17, 300, 1000, 2500], page=16, seed=83, o_dtype=o_dtype)
    if kind == "gqa":
        return W.make_dense("po_gqa", 3, 8, 1, 3000, o_dtype=o_dtype, seed=84, kv_heads=2)
    raise ValueError(kind)


CASES = [
    ("prefill", "tile", "auto", 0, torch.bfloat16),
    ("prefill", "tile", "auto", 0, torch.float16),
    ("prefill", "tile", "auto", 0, torch.float32),
    ("prefill", "row", "auto", 0, torch.bfloat16),
    ("decode", "row", "auto", 1, torch.bfloat16),
    ("decode", "row", "auto", 3, torch.float32),
    ("paged", "auto", "auto", 0, torch.bfloat16),
    ("gqa", "row", "cuda", 0, torch.bfloat16),
    ("gqa", "row", "mma", 0, torch.float32),
    ("gqa", "row", "mma", 2, torch.bfloat16),
]


@pytest.mark.parametrize("kind,path,group_kernel,num_splits,o_dtype", CASES)
@pytest.mark.parametrize("n_peers", [1, 7])
def test_peer_copies_equal_output(hyperion, oracle, kind, path, group_kernel, num_splits, o_dtype, n_peers):
    dev = torch.device("cuda", 0)
    wk = _workload(kind, o_dtype)
    g = wk.to(dev)
    shape = (g.n_bh * g.seq_q, g.head_dim)
    o = torch.full(shape, float("nan"), dtype=o_dtype, device=dev)
    peers = [torch.full(shape, float("nan"), dtype=o_dtype, device=dev) for _ in range(n_peers)]
    hyperion.read_device_errors(dev, clear=True)
    hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens,
                                  g.block_tables, o, g.seq_q, g.head_dim, g.head_dim // 8, g.block_size,
                                  g.num_blocks, g.inv_sqrt_d, g.causal, path=path, num_splits=num_splits,
                                  kv_group=wk.kv_group, group_kernel=group_kernel,
                                  o_peers=[t.data_ptr() for t in peers])
    torch.cuda.synchronize()
    assert hyperion.read_device_errors(dev, clear=True) == 0
    for t in peers:
        assert torch.equal(t.view(torch.int8) if o_dtype != torch.float32 else t.view(torch.int32),
                           o.view(torch.int8) if o_dtype != torch.float32 else o.view(torch.int32))
    o_ref, _, _, _ = oracle.forward_workload_c(wk)
    ok, mx, mn = oracle.tolerance_check(o.float().cpu().numpy(), o_ref, MAX_ABS, MEAN_ABS)
    assert ok, f"max {mx:.3e} mean {mn:.3e}"


def test_peer_argument_errors(hyperion):
    dev = torch.device("cuda", 0)
    g = _workload("decode", torch.bfloat16).to(dev)
    o = torch.empty(g.n_bh * g.seq_q, g.head_dim, dtype=torch.bfloat16, device=dev)
    args = (g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens, g.block_tables, o,
            g.seq_q, g.head_dim, g.head_dim // 8, g.block_size, g.num_blocks, g.inv_sqrt_d, g.causal)
    spare = torch.empty(o.numel() + 64, dtype=torch.bfloat16, device=dev)
    with pytest.raises(RuntimeError, match="at most 7"):
        hyperion.hyperion_apex_kernel(*args, o_peers=[spare.data_ptr()] * 8)
    with pytest.raises(RuntimeError, match="16-byte"):
        hyperion.hyperion_apex_kernel(*args, o_peers=[spare.data_ptr() + 2])
    with pytest.raises(RuntimeError, match="NULL"):
        hyperion.hyperion_apex_kernel(*args, o_peers=[0])
    torch.cuda.synchronize()


def test_copy_async_moves_bytes(hyperion):
    # hyperion_copy_async between two buffers of this device, at offsets and sizes
    # that are not multiples of anything, on a side stream; a NULL address is refused.
    dev = torch.device("cuda", 0)
    src = torch.randint(0, 256, (1 << 20,), dtype=torch.uint8, device=dev)
    dst = torch.zeros_like(src)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    for off, n in ((0, 1 << 20), (7, 1000), (4097, 65531), (1 << 19, 0)):
        hyperion.copy_async(dst.data_ptr() + off, src.data_ptr() + off, n, st)
    torch.cuda.current_stream(dev).wait_stream(st)
    torch.cuda.synchronize()
    assert torch.equal(dst, src)
    with pytest.raises(RuntimeError):
        hyperion.copy_async(0, src.data_ptr(), 16)


class _LocalPeers:
    """The attributes of sharding.PeerOutput that forward_and_push reads, with
    buffers of this device standing in for the other ranks' gathered outputs."""

    def __init__(self, rows, d, dtype, n_peers, dev):
        self.local = torch.full((rows, d), float("nan"), dtype=dtype, device=dev)
        self.peers = [torch.full((rows, d), float("nan"), dtype=dtype, device=dev) for _ in range(n_peers)]
        self.row_bytes = d * self.local.element_size()
        self.local_ptr = self.local.data_ptr()
        self.o_peers = [t.data_ptr() for t in self.peers]

    push_rows = S.PeerOutput.push_rows


@pytest.mark.parametrize("kind,path,n_chunks,n_peers,n_streams", [
    ("prefill", "tile", 3, 7, 7), ("prefill", "row", 2, 1, 1), ("decode", "row", 4, 3, 2), ("gqa", "row", 3, 2, 2)])
def test_forward_and_push_on_one_gpu(hyperion, oracle, kind, path, n_chunks, n_peers, n_streams):
    # The forward in runs of (batch, head) rows, each run's rows copied into every
    # "peer" buffer by the copy engines while the next run computes: every peer
    # buffer ends equal to the local output, which meets the oracle bar.
    dev = torch.device("cuda", 0)
    wk = _workload(kind, torch.bfloat16)
    g = wk.to(dev)
    peer = _LocalPeers(g.n_bh * g.seq_q, g.head_dim, torch.bfloat16, n_peers, dev)

    def fwd(items):
        wl = g.worklist[items]
        hyperion.hyperion_apex_kernel(wl, wl.shape[0], g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens,
                                      g.block_tables, peer.local, g.seq_q, g.head_dim, g.head_dim // 8, g.block_size,
                                      g.num_blocks, g.inv_sqrt_d, g.causal, path=path, kv_group=wk.kv_group)

    hyperion.read_device_errors(dev, clear=True)
    streams = [torch.cuda.Stream(dev) for _ in range(n_streams)]
    S.forward_and_push(fwd, S.row_chunks(g, n_chunks), peer, streams)
    torch.cuda.synchronize()
    assert hyperion.read_device_errors(dev, clear=True) == 0
    for t in peer.peers:
        assert torch.equal(t.view(torch.int16), peer.local.view(torch.int16))
    o_ref, _, _, _ = oracle.forward_workload_c(wk)
    ok, mx, mn = oracle.tolerance_check(peer.local.float().cpu().numpy(), o_ref, MAX_ABS, MEAN_ABS)
    assert ok, f"max {mx:.3e} mean {mn:.3e}"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_workloads():
    return [
        W.make_dense("po2_pre", 2, 4, 256, 256, causal=True, o_dtype=torch.bfloat16, seed=91),
        W.make_dense("po2_gqa", 2, 8, 1, 2000, o_dtype=torch.float32, seed=92, kv_heads=2),
        W.make_paged("po2_paged", 3, 5, [40, 900, 3000], page=16, seed=93, o_dtype=torch.bfloat16),
    ]


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist

    import hyperion_b200 as hyperion

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        for i, wk in enumerate(_two_gpu_workloads()):
            hr = S.head_range(wk.heads, world, rank, wk.kv_group)
            sub = S.shard_workload(wk, hr).to(dev)
            rows_max = wk.batch * len(S.head_range(wk.heads, world, 0, wk.kv_group)) * wk.seq_q
            peer = S.PeerOutput(rows_max, wk.head_dim, wk.o_dtype, dev)
            try:
                peer.out.fill_(float("nan"))
                torch.cuda.synchronize()
                dist.barrier()
                o = peer.local[: sub.n_bh * sub.seq_q]
                hyperion.hyperion_apex_kernel(sub.worklist, sub.total_work, sub.q, None, sub.k, None, sub.v,
                                              sub.v_scale, sub.ctx_lens, sub.block_tables, o, sub.seq_q,
                                              sub.head_dim, sub.head_dim // 8, sub.block_size, sub.num_blocks,
                                              sub.inv_sqrt_d, sub.causal, kv_group=wk.kv_group,
                                              o_peers=peer.o_peers)
                dist.barrier()
                torch.cuda.synchronize()
                parts = [peer.out[r][: wk.batch * len(S.head_range(wk.heads, world, r, wk.kv_group)) * wk.seq_q]
                         for r in range(world)]
                fused = S.assemble_heads(parts, wk.batch, wk.heads, wk.seq_q, world, wk.kv_group)
                gathered = S.gather_output(o.clone(), wk.batch, wk.heads, wk.seq_q, kv_group=wk.kv_group)
                same = torch.equal(fused.float(), gathered.float())
                np.save(os.path.join(out_dir, f"r{rank}_w{i}.npy"), fused.float().cpu().numpy())
                np.save(os.path.join(out_dir, f"r{rank}_w{i}_same.npy"), np.array([same]))
                # The same blocks through the copy engines: the forward in runs of
                # (batch, head) rows into `local`, each run pushed into the other
                # rank's buffer while the next computes (sharding.forward_and_push).
                peer.out.fill_(float("nan"))
                torch.cuda.synchronize()
                dist.barrier()
                n_chunks = next(c for c in (3, 2, 1) if sub.n_bh % c == 0)

                def fwd(items):
                    wl = sub.worklist[items]
                    hyperion.hyperion_apex_kernel(wl, wl.shape[0], sub.q, None, sub.k, None, sub.v, sub.v_scale,
                                                  sub.ctx_lens, sub.block_tables, o, sub.seq_q, sub.head_dim,
                                                  sub.head_dim // 8, sub.block_size, sub.num_blocks, sub.inv_sqrt_d,
                                                  sub.causal, kv_group=wk.kv_group)

                streams = [torch.cuda.Stream(dev) for _ in range(world - 1)]
                S.forward_and_push(fwd, S.row_chunks(sub, n_chunks), peer, streams)
                dist.barrier()
                torch.cuda.synchronize()
                parts = [peer.out[r][: wk.batch * len(S.head_range(wk.heads, world, r, wk.kv_group)) * wk.seq_q]
                         for r in range(world)]
                pushed = S.assemble_heads(parts, wk.batch, wk.heads, wk.seq_q, world, wk.kv_group)
                np.save(os.path.join(out_dir, f"r{rank}_w{i}_pushed.npy"), pushed.float().cpu().numpy())
                np.save(os.path.join(out_dir, f"r{rank}_w{i}_err.npy"),
                        np.array([hyperion.read_device_errors(dev, clear=True)]))
            finally:
                peer.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_output_over_two_gpus(oracle, tmp_path):
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for i, wk in enumerate(_two_gpu_workloads()):
        o_ref, _, _, _ = oracle.forward_workload_c(wk)
        for r in range(world):
            assert np.load(tmp_path / f"r{r}_w{i}_err.npy")[0] == 0
            assert np.load(tmp_path / f"r{r}_w{i}_same.npy")[0], (wk.name, r)
            got = np.load(tmp_path / f"r{r}_w{i}.npy")
            ok, mx, mn = oracle.tolerance_check(got, o_ref, MAX_ABS, MEAN_ABS)
            assert ok, f"{wk.name} rank {r}: max {mx:.3e} mean {mn:.3e}"
            pushed = np.load(tmp_path / f"r{r}_w{i}_pushed.npy")
            assert not np.isnan(pushed).any(), (wk.name, r)
            ok, mx, mn = oracle.tolerance_check(pushed, o_ref, MAX_ABS, MEAN_ABS)
            assert ok, f"{wk.name} rank {r} pushed: max {mx:.3e} mean {mn:.3e}"
