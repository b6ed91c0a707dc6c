"""Failure detection on the GPU without a GPU fault: bounded waits that run out.

Every mbarrier wait in the kernels is bounded.  hyperion_debug_fault shortens the
bound for the next forward and makes the warp that streams the keys leave one KV
stage unarmed (no copy in flight on it), so the first wait on that stage runs out.
The call must come back, raise DEVERR_WAIT_TIMEOUT, free its tensor memory and
leave the device, the workspace and the library usable: the next normal call on
every path is checked against the oracle.  Nothing here faults, traps or hangs a
GPU: the wait that runs out is one no copy will ever complete, and the bound is
about a millisecond.
"""
import numpy as np
import pytest
import torch

from hyperion_b200 import workloads as W

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
SHORT = 2_000_000  # SM clock cycles, about a millisecond


def _forward(hyperion, g, o, path, kv_group=1, group_kernel="auto"):
    hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens,
                                  g.block_tables, o, g.seq_q, g.head_dim, g.head_dim // 8, g.block_size,
                                  g.num_blocks, g.inv_sqrt_d, g.causal, path=path, kv_group=kv_group,
                                  group_kernel=group_kernel)


def _cases():
    return [
        ("tile", W.make_dense("f_tile", 1, 4, 512, 512, causal=True, o_dtype=torch.float32, seed=81), 1, "auto"),
        ("row", W.make_dense("f_row", 2, 4, 1, 2000, o_dtype=torch.float32, seed=82), 1, "auto"),
        ("row", W.make_dense("f_gqa", 2, 8, 1, 2000, kv_heads=2, o_dtype=torch.float32, seed=83), 4, "cuda"),
        # 128-key stages: 8000 keys in 8 pieces leave every CTA 8 stages, so the
        # fourth exists to be left unarmed
        ("row", W.make_dense("f_gqa_mma", 2, 8, 1, 8000, kv_heads=2, o_dtype=torch.float32, seed=84), 4, "mma"),
    ]


@pytest.mark.parametrize("case", range(4), ids=["tile", "row", "grouped_row", "grouped_mma"])
@pytest.mark.parametrize("stage", [0, 3])
def test_a_wait_that_runs_out_unwinds_and_the_next_call_is_correct(hyperion, oracle, case, stage):
    path, wk, kv_group, group_kernel = _cases()[case]
    g = wk.to(DEV)
    ref, _, _, _ = oracle.forward_workload_c(wk)
    for rep in range(2):
        o = torch.full((g.n_bh * g.seq_q, g.head_dim), float("nan"), dtype=torch.float32, device=DEV)
        hyperion.read_device_errors(DEV, clear=True)
        hyperion.debug_fault(SHORT, stage)
        _forward(hyperion, g, o, path, kv_group, group_kernel)
        torch.cuda.synchronize()  # the call came back: the unwind ended every wait
        err = hyperion.read_device_errors(DEV, clear=True)
        assert err & hyperion.DEVERR_WAIT_TIMEOUT, (path, err)
        assert hyperion.last_call_info()["path"] == path
        # The same device, workspace and library: a normal call is correct.
        o2 = g.new_output()
        _forward(hyperion, g, o2, path, kv_group, group_kernel)
        assert hyperion.read_device_errors(DEV, clear=True) == 0
        ok, mx, mn = oracle.tolerance_check(o2.cpu().numpy(), ref, 2e-2, 2e-3)
        assert ok, (path, rep, mx, mn)


def test_the_hook_is_consumed_by_one_call(hyperion, oracle):
    """A short bound with no unarmed stage changes nothing for a healthy call, and the
    hook does not outlive the call it was armed for."""
    _, wk, _, _ = _cases()[0]
    g = wk.to(DEV)
    ref, _, _, _ = oracle.forward_workload_c(wk)
    hyperion.read_device_errors(DEV, clear=True)
    hyperion.debug_fault(SHORT, -1)
    o = g.new_output()
    _forward(hyperion, g, o, "tile")
    assert hyperion.read_device_errors(DEV, clear=True) == 0
    assert oracle.tolerance_check(o.cpu().numpy(), ref, 2e-2, 2e-3)[0]
    with pytest.raises(RuntimeError):
        hyperion.debug_fault(0, 1)


def test_negative_context_length_is_flagged_on_both_paths(hyperion, oracle):
    """A negative context length is treated as 0 (the row attends nothing, O = 0) and
    raises DEVERR_NEG_CTX, on the row path and on the tile path; the other rows are
    unaffected."""
    for path, seq_q in (("row", 1), ("tile", 128)):
        wk = W.make_dense("neg", 1, 3, seq_q, 300, causal=seq_q > 1, o_dtype=torch.float32, seed=84)
        wk.ctx_lens[1] = -5
        g = wk.to(DEV)
        o = torch.full((g.n_bh * g.seq_q, 128), float("nan"), dtype=torch.float32, device=DEV)
        hyperion.read_device_errors(DEV, clear=True)
        _forward(hyperion, g, o, path)
        err = hyperion.read_device_errors(DEV, clear=True)
        assert err & hyperion.DEVERR_NEG_CTX, (path, err)
        got = o.cpu().numpy()
        assert np.all(got[seq_q:2 * seq_q] == 0.0), path
        ref, _, oerr, _ = oracle.forward_workload_c(wk)
        assert oerr & 0x8
        ok, mx, mn = oracle.tolerance_check(got, ref, 2e-2, 2e-3)
        assert ok, (path, mx, mn)
