"""(batch, head) sharding of the forward over ranks, one process per GPU.

The forward's units are independent per (batch, head) row: a row reads only its own
Q rows, its own keys (its block-table row) and writes only its own O rows
(hyperion_fa3_production_final.py:342-354, :582-593).  Ranks therefore split the
rows and each runs the forward on its share with no data exchange.  The one
collective is an optional gather of O for a caller that wants the whole output on
every rank; a tensor-parallel consumer keeps its head block instead.

Heads are split in contiguous blocks (the first H % world ranks take one extra), so
a rank's rows are the same head block in every batch entry.  With grouped-query
heads (kv_group > 1) the KV heads are split instead and a rank owns the query heads
of its KV heads, so no KV head is read on two ranks.
"""
from __future__ import annotations

from typing import List

import torch

from .workloads import Workload, dense_worklist


def head_range(n_heads: int, world: int, rank: int, kv_group: int = 1) -> range:
    """Contiguous block of query heads owned by `rank`.  The n_heads / kv_group KV
    heads are split in blocks that differ in size by at most one, and a rank owns the
    kv_group query heads of each of its KV heads."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if kv_group < 1 or n_heads % kv_group:
        raise ValueError(f"{n_heads} heads do not split into groups of {kv_group}")
    base, extra = divmod(n_heads // kv_group, world)
    lo = rank * base + min(rank, extra)
    return range(lo * kv_group, (lo + base + (1 if rank < extra else 0)) * kv_group)


def shard_bh(batch: int, n_heads: int, heads: range) -> torch.Tensor:
    """(batch, head) row ids b*H + h of a head block, in (b, h) order (int64)."""
    b = torch.arange(batch, dtype=torch.int64).repeat_interleave(len(heads))
    h = torch.tensor(list(heads), dtype=torch.int64).repeat(batch)
    return b * n_heads + h


def shard_workload(wk: Workload, heads: range) -> Workload:
    """The rows of `heads` of a workload, as a workload of its own.

    Q rows are sliced by query head; context lengths, per-(batch, head) V scales and
    block-table rows by KV head (the same thing without grouped-query heads).  A paged
    pool stays whole (the table rows point into it), a contiguous cache is cut to the
    selected KV rows.  The worklist is rebuilt over the local query rows."""
    H, g = wk.heads, wk.kv_group
    if heads.start % g or len(heads) % g:
        raise ValueError(f"heads {heads.start}-{heads.stop - 1} are not whole groups of {g}")
    Hkv = H // g
    kv_heads = range(heads.start // g, heads.stop // g)
    dev = wk.q.device
    rows = shard_bh(wk.batch, H, heads).to(dev)
    kv_rows = shard_bh(wk.batch, Hkv, kv_heads).to(dev)
    nb, nkv = len(rows), len(kv_rows)
    # Explicit row widths: a rank that owns no head (more ranks than KV heads) gets
    # empty tensors of the right width.
    qw, kw_, vw = wk.q.shape[-1], wk.k.shape[-1], wk.v.shape[-1]
    q = wk.q.view(wk.n_bh, wk.seq_q, qw)[rows].reshape(nb * wk.seq_q, qw)
    ctx = wk.ctx_lens[kv_rows]
    vs = wk.v_scale
    pool_rows = wk.v.shape[0]
    per_slot = vs.numel() == pool_rows and vs.numel() > 1
    if not per_slot and vs.numel() == wk.n_kv_bh:
        vs = vs[kv_rows]
    elif not per_slot and vs.numel() == Hkv:
        vs = vs[torch.tensor(list(kv_heads), dtype=torch.int64, device=vs.device)]
    if wk.block_tables.numel():
        bt = wk.block_tables.view(wk.n_kv_bh, -1)[kv_rows].contiguous()
        k, v = wk.k, wk.v
    else:
        span = wk.num_blocks * wk.block_size
        k = wk.k.view(wk.n_kv_bh, span, kw_)[kv_rows].reshape(nkv * span, kw_)
        v = wk.v.view(wk.n_kv_bh, span, vw)[kv_rows].reshape(nkv * span, vw)
        if per_slot:
            vs = vs.view(wk.n_kv_bh, span)[kv_rows].reshape(-1)
        bt = wk.block_tables
    wl = dense_worklist(nb, wk.seq_q, wk.q.device)
    if wk.seq_q == 1:
        wl[:, 0] = 0
    return Workload(name=f"{wk.name}[heads {heads.start}-{heads.stop - 1}]", worklist=wl, q=q.contiguous(),
                    k=k.contiguous(), v=v.contiguous(), v_scale=vs.contiguous(), ctx_lens=ctx.contiguous(),
                    block_tables=bt, seq_q=wk.seq_q, head_dim=wk.head_dim, block_size=wk.block_size,
                    num_blocks=wk.num_blocks, causal=wk.causal, o_dtype=wk.o_dtype, batch=wk.batch,
                    heads=len(heads), inv_sqrt_d=wk.inv_sqrt_d, meta=dict(wk.meta), kv_group=g)


def assemble_heads(parts: List[torch.Tensor], batch: int, n_heads: int, seq_q: int, world: int,
                   kv_group: int = 1) -> torch.Tensor:
    """Full O [batch*H*seq_q, D] from the ranks' head-block outputs, in rank order."""
    d = parts[0].shape[-1]
    out = torch.empty(batch, n_heads, seq_q, d, dtype=parts[0].dtype, device=parts[0].device)
    for r, part in enumerate(parts):
        hr = head_range(n_heads, world, r, kv_group)
        out[:, hr.start:hr.stop] = part.reshape(batch, len(hr), seq_q, d)
    return out.reshape(batch * n_heads * seq_q, d)


def row_chunks(wk: Workload, n_chunks: int) -> List[tuple]:
    """(work items, O rows) of n_chunks equal runs of (batch, head) rows of a workload
    whose worklist is the dense one in (bh, q_idx) order: each run's items and O rows
    are then each one contiguous range."""
    per = wk.seq_q
    if wk.total_work != wk.n_bh * per:
        raise ValueError("row_chunks needs the dense (bh, q_idx) worklist")
    if n_chunks < 1 or wk.n_bh % n_chunks:
        raise ValueError(f"{wk.n_bh} (batch, head) rows do not split into {n_chunks} equal chunks")
    step = wk.n_bh // n_chunks * per
    return [(slice(c * step, (c + 1) * step), slice(c * step, (c + 1) * step)) for c in range(n_chunks)]


def forward_and_gather(forward_chunk, chunks, o_local: torch.Tensor, out: torch.Tensor, group=None,
                       comm_stream=None) -> None:
    """Runs the forward chunk by chunk and all-gathers each chunk's O while the next
    chunk computes.

    forward_chunk(items) enqueues the forward of the work items `items` (a slice of the
    worklist) on the current stream; chunks is a list of equal (items, O rows) slices
    in row order, such as row_chunks gives.  out: [n_chunks, world, rows of a chunk,
    D]: out[c, r] receives rank r's O rows of chunk c, so rank r's whole output is
    out[:, r] in chunk order (out.transpose(0, 1), without a copy).  The
    gathers run on comm_stream (a new stream when None) once their chunk is computed;
    the current stream waits for the last one before this returns.  Every rank of
    `group` must call this with the same chunk sizes, in the same order of
    collectives."""
    import torch.distributed as dist

    if not o_local.is_cuda:  # host tensors (a CPU process group): one chunk after the other
        for c, (items, rows) in enumerate(chunks):
            forward_chunk(items)
            dist.all_gather_into_tensor(out[c].view(-1, *o_local.shape[1:]), o_local[rows], group=group)
        return
    cur = torch.cuda.current_stream(o_local.device)
    comm = comm_stream or torch.cuda.Stream(o_local.device)
    for c, (items, rows) in enumerate(chunks):
        forward_chunk(items)
        done = torch.cuda.Event()
        done.record(cur)
        comm.wait_event(done)
        with torch.cuda.stream(comm):
            dist.all_gather_into_tensor(out[c].view(-1, *o_local.shape[1:]), o_local[rows], group=group)
    cur.wait_stream(comm)


def forward_and_push(forward_chunk, chunks, peer: "PeerOutput", streams) -> None:
    """Runs the forward chunk by chunk into peer.local and copies each finished
    chunk's O rows into every other rank's gathered output on the copy engines
    (PeerOutput.push_rows) while the next chunk computes.

    forward_chunk(items) enqueues the forward of the work items `items` on the
    current stream with O = peer.local; chunks is a list of (items, O rows) slices
    such as row_chunks gives.  The copies of a chunk start once its forward is done
    and run on `streams` (one per peer at most is useful); the current stream waits
    for all of them before this returns.  Then, as for the fused form, a collective
    on the current stream of every rank is the barrier after which peer.out holds
    every rank's rows.  The forward keeps every SM: the copy engines, not kernels,
    move the rows."""
    cur = torch.cuda.current_stream(peer.local.device)
    for items, rows in chunks:
        forward_chunk(items)
        done = torch.cuda.Event()
        done.record(cur)
        for st in streams:
            st.wait_event(done)
        peer.push_rows(rows, streams)
    for st in streams:
        cur.wait_stream(st)


def gather_output(o_local: torch.Tensor, batch: int, n_heads: int, seq_q: int, group=None,
                  kv_group: int = 1) -> torch.Tensor:
    """All-gathers the head-block outputs of every rank into the full O on each rank.

    Blocks of unequal size are padded to the largest for the collective.  Every rank
    of `group` must call this with its own block, in the same order of collectives."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    d = o_local.shape[-1]
    rows_max = batch * len(head_range(n_heads, world, 0, kv_group)) * seq_q
    buf = torch.zeros(rows_max, d, dtype=o_local.dtype, device=o_local.device)
    buf[: o_local.shape[0]] = o_local
    bufs = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(bufs, buf, group=group)
    parts = [bufs[r][: batch * len(head_range(n_heads, world, r, kv_group)) * seq_q] for r in range(world)]
    return assemble_heads(parts, batch, n_heads, seq_q, world, kv_group)


class _DeviceArray:
    """A plain device address, shape and numpy type string in the CUDA array
    interface, so that torch.as_tensor wraps memory this package allocated."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


_TYPESTR = {torch.float32: ("<f4", torch.float32), torch.float16: ("<f2", torch.float16),
            torch.bfloat16: ("<i2", torch.bfloat16)}


def _on(device):
    """The CUDA device context of `device`, or none for None (the current device)."""
    import contextlib

    return contextlib.nullcontext() if device is None else torch.cuda.device(device)


class PeerOutput:
    """The gathered output [world, rows, D] held in IPC memory on every rank, with
    the other ranks' copies mapped into this process.

    The forward writes its O rows into `local` (this rank's slot, out[rank]) and,
    through `o_peers` (hyperion_apex_kernel's o_peers argument), the same rows into
    slot `rank` of every other rank's copy over NVLink: when the forward on every
    rank has finished, each rank holds the whole output and no gather collective
    has run.  Stores only: no peer memory is read, and nothing is loaded through a
    tensor map from it.

    A step is forward(o=local, o_peers=o_peers) then a collective barrier (any
    collective the ranks run after the forward on the same stream): a rank reads
    `out` only after it, and a rank must not start the next forward until every
    rank is done reading the last output (a second barrier, or the next step's
    collective).  rows is the largest block of any rank (shards of unequal size are
    padded to it); every rank of `group` constructs this with the same rows, D and
    dtype, in the same order of collectives.  close() unmaps the peers and frees
    the buffer after a barrier."""

    def __init__(self, rows: int, d: int, dtype: torch.dtype, device, group=None):
        import torch.distributed as dist

        from . import ipc_alloc, ipc_open

        if dtype not in _TYPESTR:
            raise ValueError(f"unsupported output dtype {dtype}")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world - 1 > 7:
            raise ValueError(f"a world of {self.world} needs more than 7 output peers")
        typestr, view = _TYPESTR[dtype]
        esize = torch.tensor([], dtype=dtype).element_size()
        slot = rows * d * esize
        # Every step below that can fail on one rank is followed by an exchange of
        # its outcome, so that all ranks fail together instead of leaving the others
        # waiting in a collective.
        self.ptr, handle, why = None, None, None
        try:
            with _on(device):
                self.ptr, handle = ipc_alloc(self.world * slot)
        except RuntimeError as e:
            why = str(e)
        handles = [None] * self.world
        dist.all_gather_object(handles, (handle, why), group=group)
        self._opened = []
        failed = [(r, w) for r, (_, w) in enumerate(handles) if w is not None]
        if not failed:  # the same decision on every rank: they all hold the same list
            try:
                with _on(device):
                    for r in range(self.world):
                        if r != self.rank:
                            self._opened.append(ipc_open(handles[r][0]))
            except RuntimeError as e:
                why = str(e)
            whys = [None] * self.world
            dist.all_gather_object(whys, why, group=group)
            failed = [(r, w) for r, w in enumerate(whys) if w is not None]
        if failed:
            self._release(barrier=True)  # every rank takes this branch
            raise RuntimeError(f"PeerOutput: rank {failed[0][0]}: {failed[0][1]}")
        self.o_peers = [base + self.rank * slot for base in self._opened]
        self.row_bytes = d * esize
        self.local_ptr = self.ptr + self.rank * slot
        raw = torch.as_tensor(_DeviceArray(self.ptr, (self.world, rows, d), typestr), device=device)
        self.out = raw.view(view)
        self.local = self.out[self.rank]

    def push_rows(self, rows: slice, streams) -> None:
        """Copies rows `rows` of `local` into slot `rank` of every other rank's
        gathered output on the copy engines (hyperion_copy_async over the peer
        mappings), the peers spread over `streams` (torch.cuda.Stream objects), with
        no kernel and no SM taken from a forward running beside the copies.  The
        caller orders each stream after the writes of those rows (an event); the
        copies are done when the streams are."""
        from . import copy_async

        n = (rows.stop - rows.start) * self.row_bytes
        off = rows.start * self.row_bytes
        for j, dst in enumerate(self.o_peers):
            copy_async(dst + off, self.local_ptr + off, n, streams[j % len(streams)])

    def close(self) -> None:
        import torch.distributed as dist

        if self.ptr is None:
            return
        torch.cuda.synchronize(self.out.device)
        dist.barrier(group=self.group)
        self._release(barrier=True)

    def _release(self, barrier: bool = False) -> None:
        """Unmaps the peers this rank opened and frees its buffer (after a barrier
        when the peers may still hold mappings of it)."""
        import torch.distributed as dist

        from . import ipc_close, ipc_free

        for base in self._opened:
            ipc_close(base)
        self._opened = []
        self.o_peers = []
        if barrier:
            dist.barrier(group=self.group)
        self.out = self.local = None
        if self.ptr is not None:
            ipc_free(self.ptr)
            self.ptr = None
