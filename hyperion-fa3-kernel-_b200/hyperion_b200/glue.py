"""Glue the reference's engine wraps around the forward, for the sign-bit path.

* build_worklist: the work items of PersistentKernelManager.prepare_worklist
  (hyperion_fa3_production_final.py:914-929), built with tensor ops on the device
  instead of a Python loop over batch x seq_q, and with the real (batch, head) row in
  the second field -- the reference writes 0 there (:926), so every item would read
  head 0 of sequence 0.
* launch_config: the (grid, block, shared) triple of get_launch_config (:907-912),
  derived from the device; the forward treats it as a hint only.
* memory_requirements: SystemProfiler.calculate_memory_requirements (:957-977) with
  the same signature and keys, for a sign-bit K (head_dim/8 bytes, no per-token
  scale) and an FP8 V (head_dim bytes) per token and KV head.
"""
from __future__ import annotations

import zlib
from typing import Dict, Optional, Sequence, Tuple

import torch


def build_worklist(q_lens: torch.Tensor, n_heads: int, kv_signatures: Optional[Sequence] = None,
                   prefetch_hints: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Work items int32 [n, 4] = {q_idx, bh, kv_signature, prefetch_hint} on q_lens' device.

    q_lens[b] query rows of sequence b, for each of its n_heads heads; items are
    ordered by (bh = b*n_heads + h, q_idx), the order the forward's tile path reads
    in 256-item chunks.  kv_signatures holds one value per sequence: an int is kept
    (its low 31 bits: the reference's hash(kv_signature) & 0x7FFFFFFF of a tuple of
    ints, :923, is the same in every process), a string becomes its 31-bit CRC32
    (Python's hash of a string is salted per process); prefetch_hints is an optional
    int32 [B] bit mask per sequence.  Neither field is read by the forward."""
    if q_lens.dim() != 1:
        raise ValueError("q_lens must be 1-D (one length per sequence)")
    dev = q_lens.device
    lens = q_lens.to(torch.int64).clamp_min(0)
    B = lens.numel()
    per_bh = lens.repeat_interleave(n_heads)  # [B*H]
    n = int(per_bh.sum())
    if n == 0:
        return torch.zeros((0, 4), dtype=torch.int32, device=dev)
    bh = torch.repeat_interleave(torch.arange(B * n_heads, device=dev), per_bh)
    starts = torch.cumsum(per_bh, 0) - per_bh
    q_idx = torch.arange(n, device=dev) - starts[bh]
    wl = torch.zeros((n, 4), dtype=torch.int32, device=dev)
    wl[:, 0] = q_idx.to(torch.int32)
    wl[:, 1] = bh.to(torch.int32)
    b_of = bh // n_heads
    if kv_signatures is not None:
        if len(kv_signatures) != B:
            raise ValueError("one kv_signature per sequence")
        sig = torch.tensor([(int(s) if isinstance(s, int) else zlib.crc32(s.encode())) & 0x7FFFFFFF
                            for s in kv_signatures], dtype=torch.int64, device=dev)
        wl[:, 2] = sig[b_of].to(torch.int32)
    if prefetch_hints is not None:
        wl[:, 3] = prefetch_hints.to(dev, torch.int32)[b_of]
    return wl


def launch_config(device=None, seq_q: int = 1, kv_group: int = 1,
                  head_dim: int = 128) -> Tuple[Tuple[int, int, int], Tuple[int, int, int], int]:
    """(grid, block, shared) of the kernel the forward launches for `seq_q` query rows per
    (batch, head) and `kv_group` query heads per KV head, as the library sized it on
    `device`: the row kernel for decode (seq_q 1), the grouped kernel for grouped-query
    decode or short prefill rows (on the tensor core at head_dim 128), the tcgen05
    tile kernel for prefill (seq_q >= 64) -- its resident CTAs, its block size and its
    dynamic shared memory.  The forward treats the triple it is given as a hint only."""
    from . import launch_info

    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    with torch.cuda.device(dev):
        info = launch_info()
    if seq_q >= 64 and info["tile_available"] and head_dim == 128:
        return (info["sm_count"] * info["tile_ctas_per_sm"], 1, 1), (info["tile_threads"], 1, 1), \
            int(info["tile_smem_bytes"])
    if (seq_q > 1 or kv_group > 1) and head_dim == 128 and info["group_mma_threads"]:
        return (info["sm_count"] * info["group_mma_ctas_per_sm"], 1, 1), (info["group_mma_threads"], 1, 1), \
            int(info["group_mma_smem_bytes"])
    if seq_q > 1 or kv_group > 1:
        return (info["sm_count"] * info["group_ctas_per_sm"], 1, 1), (info["group_threads"], 1, 1), \
            int(info["group_smem_bytes"])
    return (info["sm_count"] * info["row_ctas_per_sm"], 1, 1), (info["row_threads"], 1, 1), \
        int(info["row_smem_bytes"])


def memory_requirements(model_size_b: float, context_len: int, batch_size: int, num_layers: int, num_heads: int,
                        num_kv_heads: int, head_dim: int) -> Dict[str, float]:
    """calculate_memory_requirements for the sign-bit cache: K is head_dim/8 bytes of
    sign bits (no per-token scale) and V head_dim FP8 bytes per token and KV head.
    The weight, activation and headroom terms are the reference's."""
    per_token_bytes = head_dim // 8 + head_dim
    weights_gb = model_size_b * (1.25 / 8) * 1.15 + 1.0
    total_tokens = batch_size * context_len * num_layers * num_kv_heads
    kv_cache_gb = (total_tokens * per_token_bytes) / (1024 ** 3) * 1.1
    activations_gb = weights_gb * 0.2
    total_gb = weights_gb + kv_cache_gb + activations_gb + 2.0
    return {
        "weights_gb": weights_gb,
        "kv_cache_gb": kv_cache_gb,
        "activations_gb": activations_gb,
        "total_gb": total_gb,
        "fits_on_3090": total_gb < 24.0,
        "fits_on_b200": total_gb < 180.0,
    }
