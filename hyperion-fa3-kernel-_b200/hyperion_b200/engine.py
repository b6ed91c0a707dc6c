"""The kernel-facing half of the reference engine's batch loop, with real tensors.

The reference's HyperionApexEngine._batch_loop (hyperion_fa3_production_final.py:1062-1117)
takes a batch from KVAwareSchedulerV2.get_next_batch (:793-823), resets the work
counter (:1072), builds the worklist with PersistentKernelManager.prepare_worklist
(:914-929) and calls the kernel.  As written it cannot compute attention: every
work item has bh = 0 (:926), Q and O are [1, head_dim] placeholders (:1082-1096),
the block tables are all zeros, and decode runs with causal=True (:1112).

`BatchLauncher.launch` is that step for the sign-bit path, taking the scheduler's
output unchanged (its PrioritizedRequest objects and prefetch blocks):
  * the work items of prepare_worklist, with the real (batch, head) row in field 1
    and the reference's kv_signature hash and prefetch-hint bits in fields 2 and 3;
  * Q and O of shape [batch * num_heads * seq_q, ...], one block of seq_q rows per
    (request, query head), seq_q the longest request;
  * per-KV-head context lengths and block tables, from each request's ctx_len and
    block_table, into a pool whose pages hold one KV head each (KVPool), read with
    kv_group = num_heads // num_kv_heads;
  * causal masking for prompts (several query rows, keys of the prompt itself), none
    for decode steps (one query row against the whole cache), in two calls;
  * the launch hints of get_launch_config (:907-912), which the forward treats as
    hints only.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import glue


@dataclass
class KVPool:
    """The engine's paged cache (hyperion_fa3_production_final.py:1017-1032) in the
    forward's format: num_kv_heads * num_blocks pages of block_size slots, page
    h * num_blocks + p holding page p of KV head h; sign-bit K words, e4m3 V codes,
    one V scale per KV head."""
    k: torch.Tensor        # int32 [num_kv_heads * num_blocks * block_size, head_dim // 32]
    v: torch.Tensor        # uint8 [num_kv_heads * num_blocks * block_size, head_dim]
    v_scale: torch.Tensor  # float32 [num_kv_heads]
    num_kv_heads: int
    num_blocks: int
    block_size: int
    head_dim: int

    @staticmethod
    def allocate(num_kv_heads: int, num_blocks: int, block_size: int, head_dim: int, device) -> "KVPool":
        rows = num_kv_heads * num_blocks * block_size
        return KVPool(k=torch.zeros(rows, head_dim // 32, dtype=torch.int32, device=device),
                      v=torch.zeros(rows, head_dim, dtype=torch.uint8, device=device),
                      v_scale=torch.ones(num_kv_heads, dtype=torch.float32, device=device),
                      num_kv_heads=num_kv_heads, num_blocks=num_blocks, block_size=block_size, head_dim=head_dim)

    def page_id(self, kv_head: int, page: int) -> int:
        return kv_head * self.num_blocks + page


def prefetch_hint(block_table: Sequence[int], prefetch_blocks: Sequence[int]) -> int:
    """Bit i set when the request's first 8 pages hold prefetch block i
    (hyperion_fa3_production_final.py:916-924)."""
    where = {b: i for i, b in enumerate(list(prefetch_blocks)[:8])}
    hint = 0
    for b in list(block_table)[:8]:
        if b in where:
            hint |= 1 << where[b]
    return hint


@dataclass
class LaunchedBatch:
    worklist: torch.Tensor
    q: torch.Tensor
    o: torch.Tensor
    ctx_lens: torch.Tensor
    block_tables: torch.Tensor
    seq_q: int
    causal: bool
    rows: Dict[str, Tuple[int, int]]  # req_id -> (first (batch, head) row, query rows)


class BatchLauncher:
    """Runs scheduler batches through the drop-in forward with real Q, O and tables."""

    def __init__(self, hyperion, pool: KVPool, num_heads: int, o_dtype=torch.bfloat16, grid=None, block=None,
                 shared=None):
        if num_heads % pool.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.hyperion = hyperion
        self.pool = pool
        self.num_heads = num_heads
        self.kv_group = num_heads // pool.num_kv_heads
        self.o_dtype = o_dtype
        self.hints = (grid, block, shared)

    def launch(self, batch: Sequence, prefetch_blocks: Sequence[int],
               q_words: Dict[str, torch.Tensor]) -> List[LaunchedBatch]:
        """One scheduler batch.  q_words[req_id]: int32 [num_heads, L, head_dim // 32]
        sign-bit query rows of that request (L = its query rows).

        Prompts (L > 1: causal over their own L keys, so ctx_len must equal L) and
        decode steps (L == 1: the newest token against all ctx_len cached keys, no
        mask) go to the forward as two calls: the reference's causal rule masks key t
        of query row q_idx when t > q_idx, which is right for a prompt whose rows are
        its tokens 0..L-1 and wrong for a decode row.  Asynchronous on the current
        stream; returns, per call, the tensors the forward read and wrote."""
        prompts = [r for r in batch if int(q_words[r.req_id].shape[1]) > 1]
        steps = [r for r in batch if int(q_words[r.req_id].shape[1]) == 1]
        for r in prompts:
            if int(r.ctx_len) != int(q_words[r.req_id].shape[1]):
                raise ValueError(f"{r.req_id}: a prompt's ctx_len must equal its query rows (causal from key 0)")
        return [self._launch(reqs, prefetch_blocks, q_words, causal)
                for reqs, causal in ((prompts, True), (steps, False)) if reqs]

    def _launch(self, batch, prefetch_blocks, q_words, causal: bool) -> LaunchedBatch:
        pool, H, Hkv = self.pool, self.num_heads, self.pool.num_kv_heads
        dev = pool.k.device
        W = pool.head_dim // 32
        q_lens = [int(q_words[r.req_id].shape[1]) for r in batch]
        seq_q = max(q_lens)
        B = len(batch)
        sigs = [hash(r.kv_signature) & 0x7FFFFFFF for r in batch]
        hints = [prefetch_hint(r.block_table, prefetch_blocks) for r in batch]
        wl = glue.build_worklist(torch.tensor(q_lens, dtype=torch.int32, device=dev), H, kv_signatures=sigs,
                                 prefetch_hints=torch.tensor(hints, dtype=torch.int32))
        q = torch.zeros(B * H * seq_q, W, dtype=torch.int32, device=dev)
        qv = q.view(B, H, seq_q, W)
        ctx, tables, rows = [], [], {}
        for i, r in enumerate(batch):
            qv[i, :, :q_lens[i]] = q_words[r.req_id].to(dev)
            pages = list(r.block_table)
            if int(r.ctx_len) > len(pages) * pool.block_size:
                raise ValueError(f"{r.req_id}: ctx_len {r.ctx_len} exceeds its block table")
            for h in range(Hkv):
                ctx.append(int(r.ctx_len))
                tables.append([pool.page_id(h, p) for p in pages])
            rows[r.req_id] = (i * H, q_lens[i])
        nb = max((len(t) for t in tables), default=1)
        bt = torch.zeros(B * Hkv, nb, dtype=torch.int32)
        for j, t in enumerate(tables):
            bt[j, :len(t)] = torch.tensor(t, dtype=torch.int32)
        bt = bt.to(dev)
        ctx_t = torch.tensor(ctx, dtype=torch.int32, device=dev)
        o = torch.zeros(B * H * seq_q, pool.head_dim, dtype=self.o_dtype, device=dev)
        grid, block, shared = self.hints
        self.hyperion.hyperion_reset_counter(grid=(1, 1, 1), block=(1, 1, 1))
        self.hyperion.hyperion_apex_kernel(wl, wl.shape[0], q, None, pool.k, None, pool.v, pool.v_scale, ctx_t, bt, o,
                                           seq_q, pool.head_dim, pool.head_dim // 8, pool.block_size, nb,
                                           1.0 / pool.head_dim ** 0.5, causal, grid=grid, block=block, shared=shared,
                                           kv_group=self.kv_group)
        return LaunchedBatch(worklist=wl, q=q, o=o, ctx_lens=ctx_t, block_tables=bt, seq_q=seq_q, causal=causal,
                             rows=rows)
