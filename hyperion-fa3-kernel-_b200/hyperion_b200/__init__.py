"""B200 (sm_100a) drop-in for the reference's `hyperion` extension module.

The reference builds its forward with `load_inline` and uses the module object
as `hyperion` (hyperion_fa3_production_final.py:613-634):

    hyperion.hyperion_reset_counter(grid=(1, 1, 1), block=(1, 1, 1))          # :905
    hyperion.hyperion_apex_kernel(worklist, n, Q, Q_scale, K, K_scale, V, V_scale,
        ctx_lens, block_tables, O, seq_q, D, k_packed_bytes, block_size,
        num_blocks, inv_sqrt_d, causal, grid=grid, block=block, shared=smem)  # :1099-1114

This package exposes the same two names with the same argument order and
meaning, so a caller swaps the module object and nothing else:

    import hyperion_b200 as hyperion
    HYPERION_LOADED = hyperion.HYPERION_LOADED

Tensors are torch CUDA tensors (PyTorch is plumbing here: device memory and the
current stream); every call goes through the C ABI of libhyperion_b200.so.
Differences from the reference's boundary, all forced by the sign-bit path:
  * Q and K_cache hold sign bits packed into uint32 words (int32 / uint32 / uint8
    storage of the same bytes); k_packed_bytes must be head_dim // 8;
  * Q_scale and K_scale are accepted and ignored;
  * V_scale may be per tensor (numel 1), per slot (numel == pool rows) or per
    head / per (batch, head) (index bh % numel);
  * O may be float16 (the reference's type), bfloat16 or float32;
  * grid / block / shared are accepted as hints: the library sizes its own launch;
  * a block_tables tensor with numel 0 selects the contiguous KV layout.
Errors in arguments raise RuntimeError (the reference's TORCH_CHECK would);
errors found on the device (bad block ids, out-of-range work items) are
accumulated in the error word of the calling stream's workspace:
`read_device_errors()`.  Each (device, stream) has its own workspace, so forwards
on different streams never share a work counter or split-KV partials.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional

import torch

from . import _capi
from ._capi import (  # noqa: F401
    DEVERR_BAD_BLOCK,
    DEVERR_BAD_ITEM,
    DEVERR_CTX_OVERFLOW,
    DEVERR_NEG_CTX,
    DEVERR_WAIT_TIMEOUT,
    PATH_AUTO,
    PATH_ROW,
    PATH_TILE,
)

HYPERION_LOADED = True
__version__ = "1.4.0"

_O_DTYPES = {torch.float16: _capi.DTYPE_F16, torch.bfloat16: _capi.DTYPE_BF16, torch.float32: _capi.DTYPE_F32}
_PATHS = {"auto": _capi.PATH_AUTO, "row": _capi.PATH_ROW, "tile": _capi.PATH_TILE}
_GROUP_KERNELS = {"auto": 0, "cuda": 1, "mma": 2}
_KERNELS = {1: "row", 2: "group", 3: "group_mma", 4: "tile"}

_ws_lock = threading.Lock()
_workspaces: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Workspace (work counter, error word, split-KV partials) of the current stream of
    `device`, grown on demand.

    One workspace per (device, stream): forwards on two streams then never share a
    work counter or split-KV partials, and the calls that use one workspace are
    ordered by its stream.  It is allocated on that stream as well, so when it grows
    the caching allocator hands the old block out again only after the work already
    queued on the stream."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    dev = torch.device("cuda", idx)
    key = (idx, torch.cuda.current_stream(dev).cuda_stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            new = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=dev)
            if ws is not None:
                new[:256].copy_(ws[:256])  # keep the sticky error word
            ws = new
            _workspaces[key] = ws
        return ws


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(f"hyperion_apex_kernel: {msg}")


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def hyperion_apex_kernel(
    worklist: torch.Tensor,
    total_work: int,
    Q: torch.Tensor,
    Q_scale: Optional[torch.Tensor],
    K_cache: torch.Tensor,
    K_scale: Optional[torch.Tensor],
    V_cache: torch.Tensor,
    V_scale: torch.Tensor,
    context_lens: torch.Tensor,
    block_tables: Optional[torch.Tensor],
    O: torch.Tensor,
    seq_q: int,
    head_dim: int,
    k_packed_bytes: int,
    block_size: int,
    num_blocks: int,
    inv_sqrt_d: float,
    causal: bool,
    *,
    grid=None,
    block=None,
    shared=None,
    path: str = "auto",
    num_splits: int = 0,
    debug_scores: Optional[torch.Tensor] = None,
    kv_group: int = 1,
    sm_budget: int = 0,
    group_kernel: str = "auto",
    o_peers=None,
) -> None:
    """Enqueues the forward on the current CUDA stream of O's device (asynchronous).

    Same positional signature as the reference's kernel entry
    (hyperion_fa3_production_final.py:268-288).  `path`, `num_splits` and
    `debug_scores` (int32 [total_work, L]: receives head_dim - 2*popcount for
    every attended key) are extensions for tests and tuning.

    `kv_group` (grouped-query attention): query heads per KV head.  Work items,
    Q and O are indexed by the query row bh in [0, numel(context_lens) * kv_group);
    context_lens, the block-table rows, the contiguous layout and a per-head
    V_scale by the KV row bh // kv_group.  The row path streams each KV stage once
    for up to 4 consecutive work items on the same KV row.

    `sm_budget` (0: all): SMs the persistent kernels may occupy, for a caller that
    overlaps a collective on another stream with the forward.

    `group_kernel` ("auto", "cuda" or "mma"): the kernel of the row path's grouped
    runs (kv_group > 1 or seq_q > 1): the P.V products on the tensor core where it
    applies (head_dim 128, a per-tensor or per-head V scale), else on the CUDA cores.

    `o_peers` (up to 7 device addresses, ints): every output element is also written
    there, at O's own index -- the other ranks' gathered outputs for a head-sharded
    forward (`sharding.PeerOutput`), so that the forward also does the all-gather of
    O by peer stores while it computes.  The caller synchronises the ranks before
    any of them reads its gathered output.
    """
    total_work = int(total_work)
    _check(int(kv_group) >= 1, "kv_group must be >= 1")
    _check(O.is_cuda, "O must be a CUDA tensor")
    dev = O.device
    for name, t in (("worklist", worklist), ("Q", Q), ("K_cache", K_cache), ("V_cache", V_cache),
                    ("V_scale", V_scale), ("context_lens", context_lens)):
        _check(t.is_cuda and t.device == dev, f"{name} must be on {dev}")
        _check(t.is_contiguous(), f"{name} must be contiguous")
    _check(worklist.dtype == torch.int32 and worklist.dim() == 2 and worklist.size(1) == 4,
           "worklist must be int32 [n, 4]")
    _check(0 <= total_work <= worklist.size(0), "total_work must be in [0, worklist.size(0)]")
    _check(context_lens.dtype == torch.int32, "context_lens must be int32")
    # An empty call (a rank that owns no (batch, head) row) may pass empty tensors.
    _check(V_scale.dtype == torch.float32 and (V_scale.numel() >= 1 or total_work == 0),
           "V_scale must be a non-empty float32 tensor")
    _check(V_cache.element_size() == 1, "V_cache must hold one byte per element (FP8 e4m3 codes)")
    _check(O.dtype in _O_DTYPES, "O must be float16, bfloat16 or float32")
    _check(O.is_contiguous(), "O must be contiguous")
    _check(head_dim in (128, 256), "head_dim must be 128 or 256")
    _check(k_packed_bytes == head_dim // 8, "k_packed_bytes must be head_dim // 8 (sign-bit K)")
    n_kv = context_lens.numel()
    n_bh = n_kv * int(kv_group)
    row_bytes = head_dim // 8
    _check(_nbytes(Q) >= n_bh * seq_q * row_bytes, "Q smaller than n_bh * seq_q rows of head_dim/8 bytes")
    _check(_nbytes(K_cache) % row_bytes == 0, "K_cache bytes must be a multiple of head_dim/8")
    _check(V_cache.numel() % head_dim == 0, "V_cache numel must be a multiple of head_dim")
    pool_rows = min(_nbytes(K_cache) // row_bytes, V_cache.numel() // head_dim)
    _check(O.numel() >= n_bh * seq_q * head_dim, "O smaller than n_bh * seq_q * head_dim")
    bt_numel = 0
    if block_tables is not None and block_tables.numel() > 0:
        _check(block_tables.is_cuda and block_tables.device == dev and block_tables.is_contiguous(),
               "block_tables must be a contiguous CUDA tensor on O's device")
        _check(block_tables.dtype == torch.int32, "block_tables must be int32")
        bt_numel = block_tables.numel()
        _check(bt_numel >= n_kv * num_blocks, "block_tables numel < numel(context_lens) * num_blocks")
    if debug_scores is not None:
        _check(debug_scores.is_cuda and debug_scores.dtype == torch.int32 and debug_scores.dim() == 2
               and debug_scores.is_contiguous() and debug_scores.size(0) >= total_work,
               "debug_scores must be a contiguous int32 CUDA tensor [>= total_work, L]")
    _check(path in _PATHS, f"path must be one of {sorted(_PATHS)}")
    _check(group_kernel in _GROUP_KERNELS, f"group_kernel must be one of {sorted(_GROUP_KERNELS)}")

    def _hint(x, i=0):
        if x is None:
            return 0
        if isinstance(x, (tuple, list)):
            return int(x[i]) if len(x) > i else 0
        return int(x)

    ext = _capi.Extents(n_kv, pool_rows, V_scale.numel(), bt_numel, _O_DTYPES[O.dtype],
                        _hint(grid), _hint(block), _hint(shared))
    peers = list(o_peers or [])
    _check(len(peers) <= _capi.MAX_OUT_PEERS, f"at most {_capi.MAX_OUT_PEERS} o_peers")
    peer_arr = (ctypes.c_void_p * max(len(peers), 1))(*[int(x) for x in peers])
    opt = _capi.Options(_PATHS[path], int(num_splits),
                        debug_scores.data_ptr() if debug_scores is not None else None,
                        debug_scores.size(1) if debug_scores is not None else 0, int(kv_group), int(sm_budget),
                        _GROUP_KERNELS[group_kernel],
                        ctypes.cast(peer_arr, ctypes.POINTER(ctypes.c_void_p)) if peers else None, len(peers))
    with torch.cuda.device(dev):
        need = _capi.lib.hyperion_workspace_bytes(total_work, head_dim, block_size, num_blocks)
        _check(need > 0, f"hyperion_workspace_bytes failed: {_capi.last_error()}")
        if num_splits > 1:  # a forced split count: its partials, (m, l, acc[head_dim]) f32 per unit
            need = max(need, 256 + total_work * min(int(num_splits), 16) * (2 + head_dim) * 4)
        ws = _workspace(dev, need)
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = _capi.lib.hyperion_apex_kernel_ex(
            _ptr(worklist), total_work, _ptr(Q), _ptr(Q_scale), _ptr(K_cache), _ptr(K_scale),
            _ptr(V_cache), _ptr(V_scale), _ptr(context_lens),
            block_tables.data_ptr() if bt_numel else None, _ptr(O),
            int(seq_q), int(head_dim), int(k_packed_bytes), int(block_size), int(num_blocks),
            float(inv_sqrt_d), 1 if causal else 0, ctypes.byref(ext), ctypes.byref(opt),
            ws.data_ptr(), ws.numel(), stream)
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_apex_kernel failed (status {rc}): {_capi.last_error()}")


def kv_cache_write(K_new: torch.Tensor, V_new: torch.Tensor, seq_ids: torch.Tensor, positions: torch.Tensor,
                   block_tables: Optional[torch.Tensor], block_size: int, num_blocks: int, V_scale: torch.Tensor,
                   K_cache: torch.Tensor, V_cache: torch.Tensor) -> None:
    """Writes new keys and values into the cache the forward reads (asynchronous on
    the current stream of K_cache's device).

    K_new, V_new: [n_tokens, n_heads, head_dim] float16 / bfloat16 / float32; token i
    belongs to sequence seq_ids[i] (int32) at position positions[i] (int32).  Each
    (token, head) row lands in the slot the forward reads it from (block_tables row
    seq*n_heads + head, or the contiguous layout when block_tables is None / empty):
    K as sign bits into K_cache [pool_rows, head_dim/32] (int32 / uint32 storage), V
    as e4m3 codes of clamp(v / scale, -448, 448) into V_cache [pool_rows, head_dim]
    uint8, with the scale the forward decodes that slot with: V_scale[0] (numel 1),
    V_scale[slot] (numel == pool rows) or V_scale[(seq*n_heads + head) % numel].  Rows whose
    position or page falls outside the pool are skipped and flagged
    (read_device_errors)."""
    dtypes = {torch.float16: _capi.DTYPE_F16, torch.bfloat16: _capi.DTYPE_BF16, torch.float32: _capi.DTYPE_F32}
    _check(K_cache.is_cuda and K_cache.is_contiguous(), "K_cache must be a contiguous CUDA tensor")
    dev = K_cache.device
    for name, t in (("K_new", K_new), ("V_new", V_new), ("seq_ids", seq_ids), ("positions", positions),
                    ("V_scale", V_scale), ("V_cache", V_cache)):
        _check(t.is_cuda and t.device == dev and t.is_contiguous(), f"{name} must be a contiguous tensor on {dev}")
    _check(K_new.dtype in dtypes and V_new.dtype == K_new.dtype, "K_new / V_new must share a float16, bfloat16 or "
                                                                  "float32 dtype")
    _check(K_new.dim() == 3 and V_new.shape == K_new.shape, "K_new / V_new must be [n_tokens, n_heads, head_dim]")
    n_tokens, n_heads, head_dim = K_new.shape
    _check(head_dim in (128, 256), "head_dim must be 128 or 256")
    _check(seq_ids.dtype == torch.int32 and positions.dtype == torch.int32 and seq_ids.numel() == n_tokens
           and positions.numel() == n_tokens, "seq_ids / positions must be int32 [n_tokens]")
    _check(V_scale.dtype == torch.float32 and V_scale.numel() >= 1, "V_scale must be a non-empty float32 tensor")
    _check(V_cache.element_size() == 1 and V_cache.numel() % head_dim == 0, "V_cache must be uint8 [pool_rows, head_dim]")
    pool_rows = V_cache.numel() // head_dim
    _check(_nbytes(K_cache) >= pool_rows * head_dim // 8, "K_cache smaller than pool_rows rows of head_dim/8 bytes")
    bt_numel = 0
    if block_tables is not None and block_tables.numel() > 0:
        _check(block_tables.is_cuda and block_tables.device == dev and block_tables.is_contiguous()
               and block_tables.dtype == torch.int32, "block_tables must be a contiguous int32 CUDA tensor")
        bt_numel = block_tables.numel()
    with torch.cuda.device(dev):
        ws = _workspace(dev, 1 << 16)
        rc = _capi.lib.hyperion_kv_cache_write(
            K_new.data_ptr(), V_new.data_ptr(), dtypes[K_new.dtype], n_tokens, n_heads, head_dim,
            seq_ids.data_ptr(), positions.data_ptr(), block_tables.data_ptr() if bt_numel else None, bt_numel,
            int(block_size), int(num_blocks), V_scale.data_ptr(), V_scale.numel(), K_cache.data_ptr(),
            V_cache.data_ptr(), pool_rows, ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"kv_cache_write failed (status {rc}): {_capi.last_error()}")


def hyperion_reset_counter(*, grid=None, block=None, device=None) -> None:
    """Reference call site hyperion_fa3_production_final.py:905.  Zeroes the work
    counter of the workspace of the current stream of the current device, on that
    stream.  The forward also zeroes it itself, so calling this is optional."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    with torch.cuda.device(dev):
        ws = _workspace(dev, 1 << 16)
        rc = _capi.lib.hyperion_reset_counter(ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_reset_counter failed (status {rc}): {_capi.last_error()}")


def read_device_errors(device=None, clear: bool = True) -> int:
    """Synchronises the current stream of `device` and returns the DEVERR_* flags that
    the calls issued on that stream raised (each stream has its own workspace and so
    its own error word)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    with torch.cuda.device(dev):
        ws = _workspace(dev, 1 << 16)
        flags = ctypes.c_uint32(0)
        rc = _capi.lib.hyperion_read_device_errors(ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream,
                                                   ctypes.byref(flags), 1 if clear else 0)
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_read_device_errors failed (status {rc}): {_capi.last_error()}")
    return int(flags.value)


def debug_fault(wait_cycles: int, stage: int = -1) -> None:
    """Test hook of the bounded device waits (hyperion_debug_fault): the next forward
    on this thread bounds every device wait by `wait_cycles` SM clocks and, for
    stage >= 0, leaves that KV stage of its key stream unarmed so the first wait on
    it runs out.  That forward then raises DEVERR_WAIT_TIMEOUT (read_device_errors)
    and leaves its output incomplete; the device stays usable."""
    rc = _capi.lib.hyperion_debug_fault(int(wait_cycles), int(stage))
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_debug_fault failed (status {rc}): {_capi.last_error()}")


def launch_info() -> dict:
    """Launch facts derived from the current device (SM count, CTAs per SM, shared memory)."""
    keys = ("sm_count", "row_ctas_per_sm", "row_smem_bytes", "tile_ctas_per_sm", "tile_smem_bytes",
            "row_ctas_per_sm_d256", "tile_available", "row_threads", "group_threads", "group_ctas_per_sm",
            "group_smem_bytes", "tile_threads", "group_mma_threads", "group_mma_ctas_per_sm",
            "group_mma_smem_bytes")
    out = (ctypes.c_int32 * len(keys))()
    rc = _capi.lib.hyperion_launch_info(out, len(keys))
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_launch_info failed: {_capi.last_error()}")
    return dict(zip(keys, list(out)))


def last_call_info() -> dict:
    """What the last forward on this thread launched: path ('row' / 'tile' / None),
    KV splits per item, number of kernels, the main kernel's grid and the main
    kernel ('row', 'group' on the CUDA cores, 'group_mma' on the tensor core, 'tile'
    or None)."""
    out = (ctypes.c_int32 * 5)()
    _capi.lib.hyperion_last_call_info(out, 5)
    path = {_capi.PATH_ROW: "row", _capi.PATH_TILE: "tile"}.get(out[0])
    return {"path": path, "splits": out[1], "kernels": out[2], "grid": out[3], "kernel": _KERNELS.get(out[4])}


def library_path() -> str:
    return _capi.LIB_PATH


def ipc_alloc(nbytes: int):
    """Device memory other processes may map: (address, 64-byte IPC handle)."""
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * _capi.IPC_HANDLE_BYTES)()
    rc = _capi.lib.hyperion_ipc_alloc(int(nbytes), ctypes.byref(ptr), handle)
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_ipc_alloc failed (status {rc}): {_capi.last_error()}")
    return int(ptr.value), bytes(handle)


def ipc_open(handle: bytes) -> int:
    """Maps another process's ipc_alloc memory into this one; returns its address here."""
    _check(len(handle) == _capi.IPC_HANDLE_BYTES, "an IPC handle is 64 bytes")
    ptr = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * _capi.IPC_HANDLE_BYTES)(*handle)
    rc = _capi.lib.hyperion_ipc_open(buf, ctypes.byref(ptr))
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_ipc_open failed (status {rc}): {_capi.last_error()}")
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    rc = _capi.lib.hyperion_ipc_close(ctypes.c_void_p(ptr))
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_ipc_close failed (status {rc}): {_capi.last_error()}")


def ipc_free(ptr: int) -> None:
    rc = _capi.lib.hyperion_ipc_free(ctypes.c_void_p(ptr))
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_ipc_free failed (status {rc}): {_capi.last_error()}")


def copy_async(dst: int, src: int, nbytes: int, stream=None) -> None:
    """Copies nbytes from device address src to dst on the copy engines,
    asynchronously on `stream` (a torch.cuda.Stream; the current stream when None).
    Either address may be a peer mapping from ipc_open."""
    st = stream if stream is not None else torch.cuda.current_stream()
    rc = _capi.lib.hyperion_copy_async(ctypes.c_void_p(dst), ctypes.c_void_p(src), int(nbytes),
                                       ctypes.c_void_p(st.cuda_stream))
    if rc != _capi.HYPERION_OK:
        raise RuntimeError(f"hyperion_copy_async failed (status {rc}): {_capi.last_error()}")
