"""GPU parity of the grouped kernel with the P.V products on the tensor core.

Grouped runs (kv_group > 1, or several query rows of one (batch, head) on the row
path) take row_mma_kernel at head_dim 128 with a per-tensor or per-head V scale:
O^T = V^T P^T on tcgen05 with an f32 accumulator in TMEM, a lazy running max whose
moves open new accumulator columns (epochs), and an exact CUDA-core redo of a run
whose accumulator met an FP8 code 0x7F / 0xFF.  Every case is checked against the
CPU oracle at the bar of every parity test: integer scores bit-exact, outputs
within max-abs 2e-2 and mean-abs 2e-3 in fp32.
"""
import numpy as np
import pytest
import torch

from hyperion_b200 import workloads as W

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def run(hyperion, wk, group_kernel="auto", num_splits=0, debug_ld=0, path="row"):
    g = wk.to(DEV)
    o = torch.full((g.n_bh * g.seq_q, g.head_dim), float("nan"), dtype=torch.float32, device=DEV)
    dbg = torch.zeros(g.total_work, debug_ld, dtype=torch.int32, device=DEV) if debug_ld else None
    hyperion.read_device_errors(DEV, clear=True)
    hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens,
                                  g.block_tables, o, g.seq_q, g.head_dim, g.head_dim // 8, g.block_size,
                                  g.num_blocks, g.inv_sqrt_d, g.causal, path=path, num_splits=num_splits,
                                  debug_scores=dbg, kv_group=wk.kv_group, group_kernel=group_kernel)
    info = hyperion.last_call_info()
    err = hyperion.read_device_errors(DEV, clear=True)
    return o.cpu().numpy(), err, (dbg.cpu().numpy() if dbg is not None else None), info


def check(oracle, wk, o_gpu, rows=None):
    o_ref, _, _, _ = oracle.forward_workload_c(wk)
    if rows is not None:
        o_ref, o_gpu = o_ref[rows], o_gpu[rows]
    ok, mx, mn = oracle.tolerance_check(o_gpu, o_ref, MAX_ABS, MEAN_ABS)
    assert ok, f"max {mx:.3e} mean {mn:.3e}"


@pytest.fixture(autouse=True)
def _needs_the_kernel(hyperion):
    if not hyperion.launch_info()["group_mma_threads"]:
        pytest.skip("the tensor-core grouped kernel did not load on this device")


@pytest.mark.parametrize("num_splits", [0, 1, 2, 5, 16])
def test_engine_layout_decode_takes_the_tensor_core_kernel(hyperion, oracle, num_splits):
    """32 query heads over 8 KV heads (the reference engine's layout), contexts that
    end inside a 64-key stage, every split count from none to 16."""
    wk = W.make_dense("mma_dec", 2, 32, 1, 2100, kv_heads=8, o_dtype=torch.float32, seed=201)
    o, err, _, info = run(hyperion, wk, num_splits=num_splits)
    assert err == 0 and info["kernel"] == "group_mma", info
    assert np.isfinite(o).all()
    check(oracle, wk, o)
    o_cuda, err2, _, info2 = run(hyperion, wk, group_kernel="cuda", num_splits=num_splits)
    assert err2 == 0 and info2["kernel"] == "group"
    assert np.abs(o - o_cuda).max() <= 2e-2


@pytest.mark.parametrize("kv_heads,H", [(2, 8), (2, 6), (1, 8), (4, 8)])
def test_runs_of_every_length(hyperion, oracle, kv_heads, H):
    """kv_group 4 (full runs), 3 (a run stops inside the unit), 8 (two runs per KV
    head), 2 (two runs per unit)."""
    wk = W.make_paged("mma_runs", 3, H, [65, 700, 1999], page=16, seed=202, o_dtype=torch.float32,
                      kv_heads=kv_heads)
    o, err, _, info = run(hyperion, wk, num_splits=3)
    assert err == 0 and info["kernel"] == "group_mma"
    check(oracle, wk, o)


def test_scores_bit_exact(hyperion, oracle):
    wk = W.make_paged("mma_sc", 2, 8, [70, 500], page=16, seed=203, o_dtype=torch.float32, kv_heads=2)
    L = 500
    _, _, _, sc_ref = oracle.forward_workload_c(wk, scores_ld=L)
    _, err, sc, info = run(hyperion, wk, debug_ld=L, num_splits=2)
    assert err == 0 and info["kernel"] == "group_mma"
    assert np.array_equal(sc, sc_ref)


@pytest.mark.parametrize("num_splits", [1, 3])
def test_every_fp8_code_redoes_the_run_exactly(hyperion, oracle, num_splits):
    """Random V bytes include 0x7F / 0xFF, which the hardware conversion makes NaN and
    the reference decodes as +-480: the runs that meet one are redone on the CUDA
    cores with the exact decode."""
    wk = W.make_dense("mma_codes", 1, 8, 1, 1500, scale_mode="head", o_dtype=torch.float32, seed=204, kv_heads=2)
    gen = torch.Generator().manual_seed(205)
    wk.v = torch.randint(0, 256, tuple(wk.v.shape), dtype=torch.uint8, generator=gen)
    wk.v_scale = torch.tensor([0.004, 0.006], dtype=torch.float32)
    o, err, _, info = run(hyperion, wk, num_splits=num_splits)
    assert err == 0 and info["kernel"] == "group_mma"
    assert np.isfinite(o).all()
    check(oracle, wk, o)


def test_a_nan_code_outside_every_context_does_not_matter(hyperion, oracle):
    """0x7F codes on keys past every query's context (read into the stage but
    attended by nobody) are zeroed before the tensor core sees them."""
    wk = W.make_dense("mma_tail", 1, 4, 1, 256, kv_heads=1, o_dtype=torch.float32, seed=206)
    wk.ctx_lens[0] = 100
    wk.v[100:256] = 0x7F
    o, err, _, info = run(hyperion, wk, num_splits=1)
    assert err == 0 and info["kernel"] == "group_mma"
    check(oracle, wk, o)


def _staged_keys(levels, inv_sqrt_d):
    """4 query heads over one KV head, all four queries equal, one 128-key stage per
    entry of `levels`, every key of stage i scoring levels[i] (its sign bits differ
    from the query's in (128 - level) / 2 places)."""
    wk = W.make_dense("mma_epochs", 1, 4, 1, 128 * len(levels), kv_heads=1, o_dtype=torch.float32, seed=207)
    q = wk.q[0].clone()
    wk.q[:] = q
    for st, level in enumerate(levels):
        nd = (128 - level) // 2
        bits = torch.zeros(128, dtype=torch.int64)
        bits[:nd] = 1
        flip = (bits.view(4, 32) << torch.arange(32)).sum(1)
        flip = torch.where(flip >= 2**31, flip - 2**32, flip).to(torch.int32)
        wk.k[128 * st:128 * (st + 1)] = q ^ flip
    wk.inv_sqrt_d = inv_sqrt_d
    return wk


@pytest.mark.parametrize("inv_sqrt_d", [0.117, -0.1, 0.088])
def test_running_max_moves_open_new_epochs(hyperion, oracle, inv_sqrt_d):
    """Scaled scores that climb stage by stage by more than ln 4 (the levels reversed
    for a negative inv_sqrt_d): the running max moves at every stage and each query
    uses all four epochs; one split or two."""
    levels = [-128, -64, 0, 128] if inv_sqrt_d > 0 else [128, 64, 0, -128]
    wk = _staged_keys(levels, inv_sqrt_d)
    for splits in (1, 2):
        o, err, _, info = run(hyperion, wk, num_splits=splits)
        assert err == 0 and info["kernel"] == "group_mma"
        check(oracle, wk, o)


def test_a_fifth_move_redoes_the_run_exactly(hyperion, oracle):
    """Five climbing stages need a fifth epoch: the run is redone on the CUDA cores."""
    wk = _staged_keys([-128, -64, 0, 64, 128], 0.117)
    o, err, _, info = run(hyperion, wk, num_splits=1)
    assert err == 0 and info["kernel"] == "group_mma"
    check(oracle, wk, o)


def test_flat_weights(hyperion, oracle):
    """inv_sqrt_d = 0: every weight is 1, all keys count the same."""
    wk = W.make_dense("mma_flat", 2, 8, 1, 3000, kv_heads=2, o_dtype=torch.float32, seed=208)
    wk.inv_sqrt_d = 0.0
    o, err, _, info = run(hyperion, wk)
    assert err == 0 and info["kernel"] == "group_mma"
    check(oracle, wk, o)


def test_calls_outside_its_bounds_take_the_cuda_core_kernel(hyperion, oracle):
    """|inv_sqrt_d| above 0.117, a per-slot V scale or head_dim 256 take the grouped
    kernel with the products on the CUDA cores; forcing the tensor-core kernel there
    is refused."""
    big = W.make_dense("mma_big_c", 1, 8, 1, 600, kv_heads=2, o_dtype=torch.float32, seed=209)
    big.inv_sqrt_d = 0.5
    o, err, _, info = run(hyperion, big)
    assert err == 0 and info["kernel"] == "group"
    check(oracle, big, o)
    with pytest.raises(RuntimeError, match="tensor-core grouped kernel"):
        run(hyperion, big, group_kernel="mma")
    slot = W.make_paged("mma_slot", 2, 4, [64, 700], page=16, seed=210, o_dtype=torch.float32, kv_heads=2)
    gen = torch.Generator().manual_seed(211)
    slot.v_scale = torch.rand(slot.v.shape[0], generator=gen) * 0.01 + 1e-3
    o, err, _, info = run(hyperion, slot, num_splits=2)
    assert err == 0 and info["kernel"] == "group"
    check(oracle, slot, o)
    d256 = W.make_dense("mma_d256", 1, 8, 1, 500, D=256, kv_heads=2, o_dtype=torch.float32, seed=212)
    o, err, _, info = run(hyperion, d256)
    assert err == 0 and info["kernel"] == "group"
    check(oracle, d256, o)


def test_row_path_causal_prefill_rows(hyperion, oracle):
    """Four neighbouring query rows of one (batch, head) share a run and each keeps
    its own causal key range."""
    wk = W.make_dense("mma_pre", 1, 4, 150, 150, causal=True, o_dtype=torch.float32, seed=213, kv_heads=2)
    o, err, _, info = run(hyperion, wk)
    assert err == 0 and info["kernel"] == "group_mma"
    check(oracle, wk, o)


def test_bad_pages_and_items_are_flagged(hyperion, oracle):
    wk = W.make_paged("mma_bad", 2, 8, [300, 640], page=16, seed=214, o_dtype=torch.float32, kv_heads=2)
    wk.block_tables[1, 3] = 1 << 30   # KV row 1: page 3 outside the pool, its keys skipped
    wl = wk.worklist.clone()
    wl[5, 1] = 10_000                 # item 5: bh out of range, row left unwritten
    wk.worklist = wl
    o, err, _, info = run(hyperion, wk, num_splits=2)
    assert info["kernel"] == "group_mma"
    assert err & hyperion.DEVERR_BAD_BLOCK and err & hyperion.DEVERR_BAD_ITEM
    assert np.isnan(o[5]).all()
    rows = [r for r in range(wk.n_bh) if r != 5]
    check(oracle, wk, o, rows=rows)


@pytest.mark.parametrize("page,kernel", [(8, "group_mma"), (32, "group_mma"), (64, "group_mma"), (128, "group_mma"),
                                         (256, "group_mma"), (24, "group"), (4, "group")])
def test_page_sizes(hyperion, oracle, page, kernel):
    """A tensor-map box per page for pages of 8 to 128 keys dividing a 128-key stage,
    one box per stage for pages of a multiple of 128 keys; other page sizes take the
    CUDA-core grouped kernel.  Contexts end mid-page and mid-stage."""
    wk = W.make_paged("mma_pages", 3, 8, [77, 1000, 2431], page=page, seed=215, o_dtype=torch.float32,
                      kv_heads=2)
    o, err, _, info = run(hyperion, wk, num_splits=3)
    assert err == 0 and info["kernel"] == kernel, info
    check(oracle, wk, o)


@pytest.mark.parametrize("S_kv", [5, 100, 300])
def test_short_contiguous_rows(hyperion, oracle, S_kv):
    """The contiguous layout (one page per row): a row shorter than a stage is one
    box of its own length; a longer one ends with a box that runs into the next row
    (or past the pool, where the copy fills zeros), whose extra keys are zeroed."""
    wk = W.make_dense("mma_short", 2, 8, 1, S_kv, kv_heads=2, o_dtype=torch.float32, seed=216)
    o, err, _, info = run(hyperion, wk)
    assert err == 0 and info["kernel"] == "group_mma", info
    check(oracle, wk, o)
