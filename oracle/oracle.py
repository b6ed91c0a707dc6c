"""CPU oracle of the Hyperion sign-bit / FP8 attention forward.

TEST INFRASTRUCTURE.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg import this module, and only to check or to time the CPU path; the
product (hyperion_b200, libhyperion_b200.so) never calls it.

Two independent restatements of the reference (hyperion_fa3_production_final.py,
REF below, and README.md):
  * `forward_c`: the C restatement in hyperion_oracle.c, one key at a time in the
    reference's order with its online (m, l) update (REF:544-572), threaded over
    work items.  This is the oracle the GPU parity tests compare with, and the
    timed CPU baseline.
  * `forward_numpy`: a vectorised numpy restatement per work item: integer scores
    by popcount (numpy.bitwise_count), the clamped softmax as one exact two-pass
    softmax (equal to the online form up to rounding; the -80 clamp only differs
    for weights below e^-80), the reference's FP8 decode.  Used to cross-check
    the C oracle on small cases.

Parity status: partially pinned (the FP8 decode against the reference's own
compiled code; scoring and softmax by known-answer cases only: the reference
has no runnable attention and no test vectors).
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
EXP_CLAMP = -80.0  # REF:59

ERR_BAD_ITEM = 0x1
ERR_BAD_BLOCK = 0x2
ERR_CTX_OVERFLOW = 0x4
ERR_NEG_CTX = 0x8

_lib = None
_ref = None


def lib() -> ctypes.CDLL:
    """The C oracle, built on first use when missing (oracle/build.py)."""
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            import importlib.util

            spec = importlib.util.spec_from_file_location("_oracle_build", os.path.join(HERE, "build.py"))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mod.build_oracle()
        L = ctypes.CDLL(path)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        L.oracle_apex_forward.restype = ctypes.c_int
        L.oracle_apex_forward.argtypes = [vp, i32, vp, vp, vp, vp, i64, vp, i32, vp, i64, i64, vp, vp, i32, i32, i32,
                                          i32, ctypes.c_float, i32, vp, i64, ctypes.POINTER(ctypes.c_uint32), i32]
        L.oracle_fp8_e4m3_to_f32.restype = ctypes.c_float
        L.oracle_fp8_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.oracle_sign_score.restype = ctypes.c_int
        L.oracle_sign_score.argtypes = [vp, vp, ctypes.c_int]
        L.oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def reference_fp8_lib():
    """The reference's own fp8_e4m3_to_fp32 compiled from its source (oracle/_ref), or None."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libref_fp8.so")
        if not os.path.exists(path):
            return None
        R = ctypes.CDLL(path)
        R.ref_fp8_e4m3_to_fp32.restype = ctypes.c_float
        R.ref_fp8_e4m3_to_fp32.argtypes = [ctypes.c_uint8]
        _ref = R
    return _ref


def _np(t):
    """numpy view of a CPU tensor or array (no copy when contiguous)."""
    try:
        import torch

        if isinstance(t, torch.Tensor):
            return np.ascontiguousarray(t.detach().cpu().numpy())
    except ImportError:  # pragma: no cover
        pass
    return np.ascontiguousarray(t)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None and a.size else None


def forward_c(worklist, q, k, v, v_scale, ctx_lens, block_tables, seq_q, head_dim, block_size, num_blocks,
              inv_sqrt_d, causal, scores_ld=0, nthreads=0, total_work=None):
    """Runs the C oracle.  Returns (O fp32 [n_bh*seq_q, D], written[total_work] bool,
    err_flags, scores int32 [total_work, scores_ld] or None)."""
    wl = _np(worklist).astype(np.int32, copy=False)
    qa = _np(q).view(np.uint32) if _np(q).dtype != np.uint8 else _np(q).view(np.uint32)
    ka = _np(k).view(np.uint32) if _np(k).dtype != np.uint8 else _np(k).view(np.uint32)
    va = _np(v).view(np.uint8)
    vs = _np(v_scale).astype(np.float32, copy=False)
    ctx = _np(ctx_lens).astype(np.int32, copy=False)
    bt = _np(block_tables).astype(np.int32, copy=False) if block_tables is not None else np.zeros(0, np.int32)
    n_bh = ctx.size
    tw = wl.shape[0] if total_work is None else total_work
    pool_rows = min(ka.size // (head_dim // 32), va.size // head_dim)
    o = np.zeros((n_bh * seq_q, head_dim), np.float32)
    written = np.zeros(max(tw, 1), np.uint8)
    scores = np.zeros((tw, scores_ld), np.int32) if scores_ld else None
    err = ctypes.c_uint32(0)
    rc = lib().oracle_apex_forward(_ptr(wl), tw, _ptr(qa), _ptr(ka), _ptr(va), _ptr(vs), vs.size, _ptr(ctx), n_bh,
                                   _ptr(bt), bt.size, pool_rows, _ptr(o), _ptr(written), seq_q, head_dim, block_size,
                                   num_blocks, float(inv_sqrt_d), 1 if causal else 0,
                                   _ptr(scores) if scores is not None else None, scores_ld, ctypes.byref(err),
                                   int(nthreads))
    if rc != 0:
        raise ValueError("oracle_apex_forward rejected its arguments")
    return o, written[:tw].astype(bool), int(err.value), scores


def expand_kv_group(ctx_lens, block_tables, v_scale, kv_group, num_blocks, pool_rows):
    """Grouped-query attention restated as the plain problem: query row bh reads KV
    row bh // kv_group, so the KV-side index arrays are repeated per query row.

    Returns (context_lens, block_tables, v_scale) over n_kv * kv_group rows.  The
    contiguous layout (empty table) becomes the explicit table kv * num_blocks + j.
    A per-tensor or per-slot V scale is unchanged; a per-head / per-(batch, head)
    one is indexed kv % numel, as the kernels do."""
    g = int(kv_group)
    ctx = _np(ctx_lens).astype(np.int32).reshape(-1)
    n_kv = ctx.size
    kv_of_bh = np.arange(n_kv * g, dtype=np.int64) // g
    ctx_q = np.ascontiguousarray(ctx[kv_of_bh])
    bt = _np(block_tables).astype(np.int32).reshape(-1) if block_tables is not None else np.zeros(0, np.int32)
    if bt.size == 0:
        table = kv_of_bh[:, None] * num_blocks + np.arange(num_blocks, dtype=np.int64)[None, :]
        bt_q = np.ascontiguousarray(table.astype(np.int32))
    else:
        bt_q = np.ascontiguousarray(bt[: n_kv * num_blocks].reshape(n_kv, num_blocks)[kv_of_bh])
    vs = _np(v_scale).astype(np.float32).reshape(-1)
    if vs.size in (1, pool_rows):
        vs_q = vs
    else:
        vs_q = np.ascontiguousarray(vs[kv_of_bh % vs.size])
        if vs_q.size == pool_rows:
            raise ValueError("expanded per-head V scale would read as per-slot: pick other sizes")
    return ctx_q, bt_q, vs_q


def _workload_arrays(wk):
    """(v_scale, context_lens, block_tables) of a workload as the plain problem sees them."""
    g = getattr(wk, "kv_group", 1)
    if g == 1:
        return wk.v_scale, wk.ctx_lens, wk.block_tables
    W = wk.head_dim // 32
    pool_rows = min(_np(wk.k).size // W, _np(wk.v).size // wk.head_dim)
    ctx_q, bt_q, vs_q = expand_kv_group(wk.ctx_lens, wk.block_tables, wk.v_scale, g, wk.num_blocks, pool_rows)
    return vs_q, ctx_q, bt_q


def forward_workload_c(wk, nthreads=0, scores_ld=0, total_work=None):
    """forward_c over a hyperion_b200.workloads.Workload (moved to the CPU)."""
    vs, ctx, bt = _workload_arrays(wk)
    return forward_c(wk.worklist, wk.q, wk.k, wk.v, vs, ctx, bt, wk.seq_q,
                     wk.head_dim, wk.block_size, wk.num_blocks, wk.inv_sqrt_d, wk.causal, scores_ld=scores_ld,
                     nthreads=nthreads, total_work=total_work)


# ---------------------------------------------------------------------------- numpy restatement
def fp8_e4m3_decode_table() -> np.ndarray:
    """REF:122-141: the 256 decoded values (bias 7, subnormal mant*2^-9, exponent 15 finite)."""
    out = np.zeros(256, np.float32)
    for c in range(256):
        if c in (0x00, 0x80):
            out[c] = -0.0 if c == 0x80 else 0.0
            continue
        sign = -1.0 if c & 0x80 else 1.0
        e = (c >> 3) & 0xF
        m = c & 7
        out[c] = sign * (m * 2.0**-9 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7))
    return out


def sign_scores_np(qrow_words: np.ndarray, krows_words: np.ndarray, head_dim: int) -> np.ndarray:
    """README.md:22: D - 2*popcount(q XOR k) for each key row (uint32 words)."""
    x = np.bitwise_xor(krows_words.astype(np.uint32), qrow_words.astype(np.uint32)[None, :])
    return head_dim - 2 * np.bitwise_count(x).sum(axis=1).astype(np.int64)


def forward_numpy(worklist, q, k, v, v_scale, ctx_lens, block_tables, seq_q, head_dim, block_size, num_blocks,
                  inv_sqrt_d, causal):
    """Per-item vectorised restatement; returns (O fp32, written bool[total_work])."""
    wl = _np(worklist).astype(np.int64)
    W = head_dim // 32
    qa = _np(q).view(np.uint32).reshape(-1, W)
    ka = _np(k).view(np.uint32).reshape(-1, W)
    va = _np(v).view(np.uint8).reshape(-1, head_dim)
    vs = _np(v_scale).astype(np.float32).reshape(-1)
    ctx = _np(ctx_lens).astype(np.int64)
    bt = _np(block_tables).astype(np.int64).reshape(-1) if block_tables is not None else np.zeros(0, np.int64)
    pool_rows = min(ka.shape[0], va.shape[0])
    pool_blocks = pool_rows // block_size
    lut = fp8_e4m3_decode_table()
    n_bh = ctx.size
    o = np.zeros((n_bh * seq_q, head_dim), np.float32)
    written = np.zeros(wl.shape[0], bool)
    for i, (q_idx, bh, _, _) in enumerate(wl):
        if not (0 <= bh < n_bh and 0 <= q_idx < seq_q):
            continue
        L = int(min(max(ctx[bh], 0), num_blocks * block_size))
        t = np.arange(L, dtype=np.int64)
        if causal:
            t = t[t <= q_idx]
        page = t // block_size
        ids = (bh * num_blocks + page) if bt.size == 0 else bt[bh * num_blocks + page]
        ok = (ids >= 0) & (ids < pool_blocks)
        t, ids = t[ok], ids[ok]
        slots = ids * block_size + t % block_size
        row = bh * seq_q + q_idx
        written[i] = True
        if slots.size == 0:
            continue  # nothing attended: acc = 0, O = 0 (REF:584)
        s = sign_scores_np(qa[row], ka[slots], head_dim).astype(np.float32) * np.float32(inv_sqrt_d)
        m = s.max()
        w = np.exp(np.maximum(s - m, EXP_CLAMP)).astype(np.float32)
        if vs.size == 1:
            scale = np.full(slots.size, vs[0], np.float32)
        elif vs.size == pool_rows:
            scale = vs[slots]
        else:
            scale = np.full(slots.size, vs[bh % vs.size], np.float32)
        vals = lut[va[slots]] * scale[:, None]
        acc = (w[:, None].astype(np.float64) * vals).sum(0)
        l = float(w.astype(np.float64).sum())
        o[row] = (acc * (1.0 / l if l > 1e-6 else 1.0)).astype(np.float32)
    return o, written


def forward_workload_numpy(wk):
    vs, ctx, bt = _workload_arrays(wk)
    return forward_numpy(wk.worklist, wk.q, wk.k, wk.v, vs, ctx, bt, wk.seq_q,
                         wk.head_dim, wk.block_size, wk.num_blocks, wk.inv_sqrt_d, wk.causal)


def tolerance_check(o_gpu: np.ndarray, o_ref: np.ndarray, max_abs: float = 2e-2, mean_abs: float = 2e-3):
    """The parity bar: max |diff| <= 2e-2 and mean |diff| <= 2e-3 in fp32."""
    d = np.abs(o_gpu.astype(np.float32) - o_ref.astype(np.float32))
    mx = float(d.max()) if d.size else 0.0
    mn = float(d.mean()) if d.size else 0.0
    return (mx <= max_abs and mn <= mean_abs and math.isfinite(mx)), mx, mn
