"""GPU test of hyperion_apex_kernel_noalloc, the forward that allocates nothing.

Callers that cannot allocate device memory use this entry point. Examples are a
plugin whose host framework owns the allocator, or an engine that reserved all
device memory at start-up. Its scratch is a fixed per-device array inside the
library instead of a caller workspace.

The test calls it through the C ABI, several times in a row, on different inputs.
Each output is compared with the workspace entry point hyperion_apex_kernel on the
same inputs, within the tolerance of the parity tests. A later call must not see
stale state from an earlier one, because every call shares the one array.

The file sorts last so that a run stopping at its first failure has run every
other test before this one. It passes alone in a fresh process too: the first
call on the device does the scratch look-up.
"""
import ctypes

import numpy as np
import pytest
import torch

from hyperion_b200 import workloads as W

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
_DTYPES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def _args(g, o):
    """Positional arguments shared by both entry points, plus the extents struct."""
    from hyperion_b200 import _capi

    bt = g.block_tables
    ext = _capi.Extents(g.n_bh, g.k.size(0), g.v_scale.numel(), bt.numel(), _DTYPES[o.dtype], 0, 0, 0)
    pos = (g.worklist.data_ptr(), g.total_work, g.q.data_ptr(), None, g.k.data_ptr(), None, g.v.data_ptr(),
           g.v_scale.data_ptr(), g.ctx_lens.data_ptr(), bt.data_ptr() if bt.numel() else None, o.data_ptr(),
           g.seq_q, g.head_dim, g.head_dim // 8, g.block_size, g.num_blocks, g.inv_sqrt_d, 1 if g.causal else 0)
    return pos, ext


def _with_workspace(g, o):
    from hyperion_b200 import _capi

    pos, ext = _args(g, o)
    need = _capi.lib.hyperion_workspace_bytes(g.total_work, g.head_dim, g.block_size, g.num_blocks)
    ws = torch.zeros(max(int(need), 256), dtype=torch.uint8, device=o.device)
    rc = _capi.lib.hyperion_apex_kernel(*pos, ctypes.byref(ext), ws.data_ptr(), ws.numel(),
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == _capi.HYPERION_OK, _capi.last_error()
    torch.cuda.synchronize()
    return ws


def _no_alloc(g, o):
    from hyperion_b200 import _capi

    pos, ext = _args(g, o)
    rc = _capi.lib.hyperion_apex_kernel_noalloc(*pos, ctypes.byref(ext), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc


def _last_call():
    from hyperion_b200 import _capi

    out = (ctypes.c_int32 * 4)()
    _capi.lib.hyperion_last_call_info(out, 4)
    return list(out)


def _compare(a, b):
    a = a.float().cpu().numpy()
    b = b.float().cpu().numpy()
    assert np.isfinite(a).all() and np.isfinite(b).all()
    d = np.abs(a - b)
    assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, f"max {d.max():.3e} mean {d.mean():.3e}"


WORKLOADS = [
    # decode, 2 x 4 heads over 3000 keys: the row kernel with split-KV partials
    dict(name="decode_a", B=2, H=4, S_q=1, S_kv=3000, seed=21, o_dtype=torch.float32),
    # a second decode with other sizes: partials of a different shape over the same array
    dict(name="decode_b", B=3, H=2, S_q=1, S_kv=5000, seed=22, o_dtype=torch.bfloat16),
    # causal prefill, 1 x 2 heads of 256 rows: the tile kernel (work counter only)
    dict(name="prefill", B=1, H=2, S_q=256, S_kv=256, seed=23, o_dtype=torch.float32, causal=True),
]


def test_no_alloc_matches_workspace_entry_point_on_consecutive_calls(hyperion):
    from hyperion_b200 import _capi

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    seen_splits = []
    for spec in WORKLOADS:
        spec = dict(spec)
        wk = W.make_dense(spec.pop("name"), spec.pop("B"), spec.pop("H"), spec.pop("S_q"), spec.pop("S_kv"),
                          scale_mode="head", **spec)
        g = wk.to(dev)
        o_ref = torch.full((g.n_bh * g.seq_q, g.head_dim), float("nan"), dtype=g.o_dtype, device=dev)
        _with_workspace(g, o_ref)
        for _ in range(2):  # two calls in a row on the same inputs, then the next workload
            o = torch.full_like(o_ref, float("nan"))
            rc = _no_alloc(g, o)
            assert rc == _capi.HYPERION_OK, _capi.last_error()
            seen_splits.append(_last_call()[1])
            _compare(o, o_ref)
    assert max(seen_splits) > 1, "no call used split-KV partials in the scratch array"


def test_no_alloc_rejects_calls_beyond_its_scratch(hyperion):
    """16384 decode items over a 131072-key table take 16 KV splits: 136 MB of
    partials, above the fixed 32 MiB. The call is refused on the host before any
    kernel is launched. Every buffer is still sized for the call, with
    one-key contexts, so the inputs stay in bounds whatever happens. A normal
    call afterwards still works."""
    from hyperion_b200 import _capi

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_bh, bs, nb = 16384, 16, 8192
    wl = torch.zeros(n_bh, 4, dtype=torch.int32, device=dev)
    wl[:, 1] = torch.arange(n_bh, dtype=torch.int32, device=dev)
    q = torch.zeros(n_bh, 4, dtype=torch.int32, device=dev)
    k = torch.zeros(bs, 4, dtype=torch.int32, device=dev)
    v = torch.zeros(bs, 128, dtype=torch.uint8, device=dev)
    vs = torch.ones(1, dtype=torch.float32, device=dev)
    ctx = torch.ones(n_bh, dtype=torch.int32, device=dev)
    o = torch.zeros(n_bh, 128, dtype=torch.float32, device=dev)
    ext = _capi.Extents(n_bh, bs, 1, 0, _DTYPES[torch.float32], 0, 0, 0)
    rc = _capi.lib.hyperion_apex_kernel_noalloc(
        wl.data_ptr(), n_bh, q.data_ptr(), None, k.data_ptr(), None, v.data_ptr(), vs.data_ptr(), ctx.data_ptr(),
        None, o.data_ptr(), 1, 128, 16, bs, nb, 128 ** -0.5, 0, ctypes.byref(ext),
        torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == _capi.HYPERION_ERR_WORKSPACE
    msg = _capi.last_error()
    assert "hyperion_apex_kernel_noalloc" in msg and str(_capi.NOALLOC_SCRATCH_BYTES) in msg, msg
    assert _last_call()[2] == 0, "a kernel was launched for a refused call"

    wk = W.make_dense("after", 1, 2, 1, 2048, scale_mode="head", o_dtype=torch.float32, seed=24).to(dev)
    o_ref = torch.zeros(wk.n_bh, 128, dtype=torch.float32, device=dev)
    _with_workspace(wk, o_ref)
    o2 = torch.full_like(o_ref, float("nan"))
    assert _no_alloc(wk, o2) == _capi.HYPERION_OK, _capi.last_error()
    _compare(o2, o_ref)
