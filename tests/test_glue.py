"""Engine glue: the device worklist builder, launch hints and the memory estimator."""
import zlib

import numpy as np
import pytest
import torch

from hyperion_b200 import glue
from hyperion_b200 import workloads as W


def _loop_worklist(q_lens, H, sigs=None, hints=None):
    """The work items written out one by one (the reference's loop, with the real bh)."""
    out = []
    for b, L in enumerate(q_lens):
        for h in range(H):
            for q in range(L):
                sig = (zlib.crc32(sigs[b].encode()) & 0x7FFFFFFF) if sigs else 0
                out.append([q, b * H + h, sig, hints[b] if hints else 0])
    return np.array(out, dtype=np.int32).reshape(-1, 4)


@pytest.mark.parametrize("q_lens", [[1, 1, 1], [5, 0, 17, 3], [256, 1]])
def test_build_worklist_matches_loop(q_lens):
    H = 3
    sigs = [f"seq-{i}" for i in range(len(q_lens))]
    hints = [i * 7 + 1 for i in range(len(q_lens))]
    wl = glue.build_worklist(torch.tensor(q_lens, dtype=torch.int32), H, kv_signatures=sigs,
                             prefetch_hints=torch.tensor(hints, dtype=torch.int32))
    assert wl.dtype == torch.int32 and wl.shape[1] == 4
    assert np.array_equal(wl.numpy(), _loop_worklist(q_lens, H, sigs, hints))


def test_build_worklist_dense_equals_generator_worklist():
    wl = glue.build_worklist(torch.full((4,), 64, dtype=torch.int32), 2)
    assert torch.equal(wl, W.dense_worklist(8, 64, "cpu"))
    assert glue.build_worklist(torch.zeros(3, dtype=torch.int32), 4).shape == (0, 4)


def test_memory_requirements_sign_bit_sizes():
    r = glue.memory_requirements(7.0, 8192, 4, 32, 32, 8, 128)
    tokens = 4 * 8192 * 32 * 8
    assert r["kv_cache_gb"] == pytest.approx(tokens * (16 + 128) / 1024 ** 3 * 1.1)
    assert set(r) >= {"weights_gb", "kv_cache_gb", "activations_gb", "total_gb", "fits_on_3090"}
    assert r["total_gb"] == pytest.approx(r["weights_gb"] + r["kv_cache_gb"] + r["activations_gb"] + 2.0)


@pytest.mark.gpu
def test_device_worklist_drives_the_forward(hyperion, oracle):
    """A ragged prefill worklist built on the device runs through the forward and
    matches the oracle on the same items."""
    wk = W.make_dense("g", 2, 2, 96, 96, causal=True, scale_mode="head", o_dtype=torch.float32, seed=41)
    q_lens = torch.tensor([96, 70], dtype=torch.int32)
    dev = torch.device("cuda", 0)
    wl = glue.build_worklist(q_lens.to(dev), 2)
    g = wk.to(dev)
    o = torch.zeros(g.n_bh * g.seq_q, 128, dtype=torch.float32, device=dev)
    hyperion.read_device_errors(dev, clear=True)
    hyperion.hyperion_apex_kernel(wl, wl.shape[0], g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens, g.block_tables,
                                  o, g.seq_q, 128, 16, g.block_size, g.num_blocks, g.inv_sqrt_d, True)
    assert hyperion.read_device_errors(dev, clear=True) == 0
    ref_wk = W.Workload(**{**wk.__dict__, "worklist": wl.cpu()})
    ref, written, err, _ = oracle.forward_workload_c(ref_wk)
    assert err == 0
    rows = (wl[:, 1].long() * g.seq_q + wl[:, 0].long()).cpu().numpy()
    ok, mx, mn = oracle.tolerance_check(o.cpu().numpy()[rows], ref[rows], 2e-2, 2e-3)
    assert ok, (mx, mn)
    # The launch hints describe the kernel the forward really launched for this
    # worklist (the tile kernel for 64+ query rows per (batch, head)).
    info = hyperion.launch_info()
    grid, block, shared = glue.launch_config(dev, seq_q=g.seq_q)
    assert hyperion.last_call_info()["path"] == "tile"
    assert block == (info["tile_threads"], 1, 1) == (512, 1, 1)
    assert grid[0] == info["sm_count"] * info["tile_ctas_per_sm"] and shared == info["tile_smem_bytes"]
    # Decode: the row kernel's 96-thread CTAs (a producer warp and two consumer warps).
    grid, block, shared = glue.launch_config(dev)
    assert block == (info["row_threads"], 1, 1) == (96, 1, 1)
    assert grid[0] == info["sm_count"] * info["row_ctas_per_sm"] >= 148 and shared == info["row_smem_bytes"] > 0
    d = W.make_dense("lc_decode", 2, 2, 1, 300, o_dtype=torch.float32, seed=5).to(dev)
    od = d.new_output()
    hyperion.hyperion_apex_kernel(d.worklist, d.total_work, d.q, None, d.k, None, d.v, d.v_scale, d.ctx_lens,
                                  d.block_tables, od, 1, 128, 16, d.block_size, d.num_blocks, d.inv_sqrt_d, False,
                                  grid=grid, block=block, shared=shared)
    assert hyperion.last_call_info()["path"] == "row"
    assert hyperion.last_call_info()["grid"] <= grid[0]
    # Grouped-query decode (4 query heads per KV head): the tensor-core grouped
    # kernel's 192-thread CTAs (producer, four query warps, MMA issuer).
    grid, block, shared = glue.launch_config(dev, kv_group=4)
    if info["group_mma_threads"]:
        assert block == (info["group_mma_threads"], 1, 1) == (192, 1, 1)
        assert grid[0] == info["sm_count"] * info["group_mma_ctas_per_sm"] and shared == info["group_mma_smem_bytes"]
        gq = W.make_dense("lc_gqa", 2, 8, 1, 300, kv_heads=2, o_dtype=torch.float32, seed=6).to(dev)
        og = gq.new_output()
        hyperion.hyperion_apex_kernel(gq.worklist, gq.total_work, gq.q, None, gq.k, None, gq.v, gq.v_scale,
                                      gq.ctx_lens, gq.block_tables, og, 1, 128, 16, gq.block_size, gq.num_blocks,
                                      gq.inv_sqrt_d, False, kv_group=gq.kv_group, grid=grid, block=block, shared=shared)
        assert hyperion.last_call_info()["kernel"] == "group_mma"
        assert hyperion.last_call_info()["grid"] <= grid[0]
