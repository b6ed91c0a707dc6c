"""ctypes binding of the C ABI in include/hyperion_b200.h.

This is the binding a maintainer adds in place of the reference's
`load_inline(...)` module (hyperion_fa3_production_final.py:613-628).  It loads
the in-tree libhyperion_b200.so; if the library is missing the import fails
loudly: there is no CPU or eager fallback for the forward.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("HYPERION_B200_LIB", os.path.join(_HERE, "libhyperion_b200.so"))

HYPERION_OK = 0
HYPERION_ERR_INVALID_ARG = 1
HYPERION_ERR_UNSUPPORTED = 2
HYPERION_ERR_WORKSPACE = 3
HYPERION_ERR_CUDA = 4

DEVERR_BAD_ITEM = 0x1
DEVERR_BAD_BLOCK = 0x2
DEVERR_CTX_OVERFLOW = 0x4
DEVERR_NEG_CTX = 0x8
DEVERR_WAIT_TIMEOUT = 0x10

DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_F32 = 2

PATH_AUTO = 0
PATH_ROW = 1
PATH_TILE = 2

# Every symbol include/hyperion_b200.h declares.
EXPORTED = (
    "hyperion_workspace_bytes",
    "hyperion_apex_kernel",
    "hyperion_apex_kernel_ex",
    "hyperion_reset_counter",
    "hyperion_read_device_errors",
    "hyperion_launch_info",
    "hyperion_last_call_info",
    "hyperion_last_error_string",
    "hyperion_version",
    "hyperion_apex_kernel_noalloc",
    "hyperion_kv_cache_write",
    "hyperion_debug_fault",
    "hyperion_ipc_alloc",
    "hyperion_ipc_open",
    "hyperion_ipc_close",
    "hyperion_ipc_free",
    "hyperion_copy_async",
)

IPC_HANDLE_BYTES = 64  # HYPERION_IPC_HANDLE_BYTES
MAX_OUT_PEERS = 7

# Fixed per-device scratch of hyperion_apex_kernel_noalloc (HYPERION_NOALLOC_SCRATCH_BYTES).
NOALLOC_SCRATCH_BYTES = 32 << 20


class Extents(ctypes.Structure):
    _fields_ = [
        ("n_bh", ctypes.c_int32),
        ("pool_rows", ctypes.c_int64),
        ("v_scale_numel", ctypes.c_int64),
        ("block_tables_numel", ctypes.c_int64),
        ("o_dtype", ctypes.c_int32),
        ("grid_hint", ctypes.c_int32),
        ("block_hint", ctypes.c_int32),
        ("shared_hint", ctypes.c_int32),
    ]


class Options(ctypes.Structure):
    _fields_ = [
        ("path", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
        ("debug_scores", ctypes.c_void_p),
        ("debug_ld", ctypes.c_int64),
        ("kv_group", ctypes.c_int32),
        ("sm_budget", ctypes.c_int32),
        ("group_kernel", ctypes.c_int32),
        ("o_peers", ctypes.POINTER(ctypes.c_void_p)),
        ("n_o_peers", ctypes.c_int32),
    ]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_FWD_ARGS = [
    _vp, _i32,  # worklist, total_work
    _vp, _vp,  # Q, Q_scale
    _vp, _vp,  # K_cache, K_scale
    _vp, _vp,  # V_cache, V_scale
    _vp, _vp,  # context_lens, block_tables
    _vp,  # O
    _i32, _i32, _i32, _i32, _i32,  # seq_q, head_dim, k_packed_bytes, block_size, num_blocks
    ctypes.c_float, _i32,  # inv_sqrt_d, causal
    ctypes.POINTER(Extents),
]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libhyperion_b200.so not found at {LIB_PATH}; build it with "
            "`python hyperion-fa3-kernel-_b200/build.py` (nvcc, sm_100a)"
        )
    lib = ctypes.CDLL(LIB_PATH)
    lib.hyperion_workspace_bytes.restype = ctypes.c_size_t
    lib.hyperion_workspace_bytes.argtypes = [_i32, _i32, _i32, _i32]
    lib.hyperion_apex_kernel.restype = ctypes.c_int
    lib.hyperion_apex_kernel.argtypes = _FWD_ARGS + [_vp, ctypes.c_size_t, _vp]
    lib.hyperion_apex_kernel_ex.restype = ctypes.c_int
    lib.hyperion_apex_kernel_ex.argtypes = _FWD_ARGS + [ctypes.POINTER(Options), _vp, ctypes.c_size_t, _vp]
    lib.hyperion_reset_counter.restype = ctypes.c_int
    lib.hyperion_reset_counter.argtypes = [_vp, ctypes.c_size_t, _vp]
    lib.hyperion_read_device_errors.restype = ctypes.c_int
    lib.hyperion_read_device_errors.argtypes = [_vp, ctypes.c_size_t, _vp, ctypes.POINTER(ctypes.c_uint32), _i32]
    lib.hyperion_launch_info.restype = ctypes.c_int
    lib.hyperion_launch_info.argtypes = [ctypes.POINTER(_i32), _i32]
    lib.hyperion_last_call_info.restype = ctypes.c_int
    lib.hyperion_last_call_info.argtypes = [ctypes.POINTER(_i32), _i32]
    lib.hyperion_last_error_string.restype = ctypes.c_char_p
    lib.hyperion_last_error_string.argtypes = []
    lib.hyperion_version.restype = _i32
    lib.hyperion_version.argtypes = []
    lib.hyperion_apex_kernel_noalloc.restype = ctypes.c_int
    lib.hyperion_apex_kernel_noalloc.argtypes = _FWD_ARGS + [_vp]
    _i64 = ctypes.c_int64
    lib.hyperion_kv_cache_write.restype = ctypes.c_int
    lib.hyperion_kv_cache_write.argtypes = [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _i64,
                                            _vp, _vp, _i64, _vp, ctypes.c_size_t, _vp]
    lib.hyperion_debug_fault.restype = ctypes.c_int
    lib.hyperion_debug_fault.argtypes = [_i64, _i32]
    _u8p = ctypes.POINTER(ctypes.c_uint8)
    lib.hyperion_ipc_alloc.restype = ctypes.c_int
    lib.hyperion_ipc_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(_vp), _u8p]
    lib.hyperion_ipc_open.restype = ctypes.c_int
    lib.hyperion_ipc_open.argtypes = [_u8p, ctypes.POINTER(_vp)]
    lib.hyperion_ipc_close.restype = ctypes.c_int
    lib.hyperion_ipc_close.argtypes = [_vp]
    lib.hyperion_ipc_free.restype = ctypes.c_int
    lib.hyperion_ipc_free.argtypes = [_vp]
    lib.hyperion_copy_async.restype = ctypes.c_int
    lib.hyperion_copy_async.argtypes = [_vp, _vp, ctypes.c_size_t, _vp]
    return lib


lib = _load()


def last_error() -> str:
    s = lib.hyperion_last_error_string()
    return s.decode() if s else ""
