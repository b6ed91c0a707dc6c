"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bar (the reference's own tolerance for this path): integer QK scores bit-exact;
outputs within max-abs 2e-2 and mean-abs 2e-3 of the oracle in fp32.  Every test
here is marked gpu; none of them makes a GPU fault or hang: bad inputs are
host-built and the kernels turn them into error flags.
"""
import numpy as np
import pytest
import torch

from hyperion_b200 import workloads as W

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def run(hyperion, wk, path="auto", num_splits=0, debug_ld=0, o_dtype=None):
    dev = torch.device("cuda", 0)
    g = wk.to(dev)
    o = torch.full((g.n_bh * g.seq_q, g.head_dim), float("nan"), dtype=o_dtype or g.o_dtype, device=dev)
    dbg = torch.zeros(g.total_work, debug_ld, dtype=torch.int32, device=dev) if debug_ld else None
    hyperion.read_device_errors(dev, clear=True)
    hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens,
                                  g.block_tables, o, g.seq_q, g.head_dim, g.head_dim // 8, g.block_size,
                                  g.num_blocks, g.inv_sqrt_d, g.causal, path=path, num_splits=num_splits,
                                  debug_scores=dbg)
    err = hyperion.read_device_errors(dev, clear=True)
    return o.float().cpu().numpy(), err, (dbg.cpu().numpy() if dbg is not None else None)


def check(oracle, wk, o_gpu, rows=None):
    o_ref, written, err, _ = oracle.forward_workload_c(wk)
    if rows is not None:
        o_ref, o_gpu = o_ref[rows], o_gpu[rows]
    ok, mx, mn = oracle.tolerance_check(o_gpu, o_ref, MAX_ABS, MEAN_ABS)
    assert ok, f"max {mx:.3e} mean {mn:.3e}"
    return mx, mn


def written_rows(wk):
    wl = wk.worklist.cpu().numpy()
    return (wl[:, 1].astype(np.int64) * wk.seq_q + wl[:, 0]).tolist()


# ----------------------------------------------------------------------------- row path
@pytest.mark.parametrize("o_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_cpu_ref_config_row_path(hyperion, oracle, o_dtype):
    wk = W.make_config("cpu_ref", device="cpu", exact=True)
    o, err, _ = run(hyperion, wk, path="row", o_dtype=o_dtype)
    assert err == 0
    check(oracle, wk, o)


@pytest.mark.parametrize("num_splits", [1, 3, 7, 16])
def test_row_path_split_kv(hyperion, oracle, num_splits):
    wk = W.make_dense("d", 2, 4, 1, 3000, scale_mode="head", o_dtype=torch.float32, seed=3)
    o, err, _ = run(hyperion, wk, path="row", num_splits=num_splits)
    assert err == 0
    check(oracle, wk, o)


@pytest.mark.parametrize("scale_mode", ["tensor", "head", "bh"])
def test_row_path_causal_ragged_prefill(hyperion, oracle, scale_mode):
    wk = W.make_dense("c", 2, 3, 157, 157, causal=True, scale_mode=scale_mode, o_dtype=torch.float32, seed=5)
    o, err, _ = run(hyperion, wk, path="row")
    assert err == 0
    check(oracle, wk, o)


def test_row_path_paged_decode_ragged(hyperion, oracle):
    lens = [1, 15, 16, 17, 100, 511, 2000, 4097]
    wk = W.make_paged("p", len(lens), 4, lens, page=16, seed=6, o_dtype=torch.float32)
    o, err, _ = run(hyperion, wk, path="row")
    assert err == 0
    check(oracle, wk, o)


@pytest.mark.parametrize("page", [1, 8, 64, 256])
def test_row_path_page_sizes(hyperion, oracle, page):
    wk = W.make_paged("p", 3, 2, [300, 77, 1000], page=page, seed=8, o_dtype=torch.float32)
    o, err, _ = run(hyperion, wk, path="row")
    assert err == 0
    check(oracle, wk, o)


def test_row_path_per_slot_scale(hyperion, oracle):
    wk = W.make_paged("p", 2, 2, [200, 333], page=16, seed=9, o_dtype=torch.float32)
    pool_rows = wk.v.shape[0]
    g = torch.Generator().manual_seed(1)
    wk.v_scale = (torch.rand(pool_rows, generator=g) * 0.02 + 0.001).to(torch.float32)
    o, err, _ = run(hyperion, wk, path="row")
    assert err == 0
    check(oracle, wk, o)


def test_row_path_head_dim_256(hyperion, oracle):
    wk = W.make_dense("d256", 1, 3, 5, 700, D=256, causal=True, scale_mode="head", o_dtype=torch.float32, seed=12)
    o, err, _ = run(hyperion, wk, path="row")
    assert err == 0
    check(oracle, wk, o)


def test_row_path_scores_bit_exact(hyperion, oracle):
    wk = W.make_paged("p", 3, 2, [50, 129, 700], page=16, seed=13, o_dtype=torch.float32)
    L = 700
    _, _, _, sc_ref = oracle.forward_workload_c(wk, scores_ld=L)
    _, err, sc = run(hyperion, wk, path="row", debug_ld=L)
    assert err == 0
    assert np.array_equal(sc, sc_ref)


def test_row_path_fully_masked_rows_are_zero(hyperion, oracle):
    wk = W.make_dense("m", 1, 4, 1, 64, o_dtype=torch.float32, seed=14)
    wk.ctx_lens[1] = 0
    wk.ctx_lens[3] = 0
    o, err, _ = run(hyperion, wk, path="row", num_splits=2)
    assert err == 0
    assert np.all(o[1] == 0) and np.all(o[3] == 0)
    check(oracle, wk, o)


def test_row_path_bad_block_and_item_raise_flags(hyperion, oracle):
    wk = W.make_paged("p", 2, 2, [64, 64], page=16, seed=15, o_dtype=torch.float32)
    wk.block_tables[1, 2] = 1 << 30
    wk.block_tables[2, 0] = -7
    wl = wk.worklist.clone()
    wl[3, 1] = 1000
    wk.worklist = wl
    o, err, _ = run(hyperion, wk, path="row")
    assert err & hyperion.DEVERR_BAD_BLOCK and err & hyperion.DEVERR_BAD_ITEM
    assert np.isnan(o[3]).all()  # the out-of-range item's row is never written
    check(oracle, wk, o, rows=[0, 1, 2])


def test_row_path_context_overflow_flag(hyperion, oracle):
    wk = W.make_dense("o", 1, 2, 1, 128, o_dtype=torch.float32, seed=16)
    wk.ctx_lens[0] = 5000  # beyond num_blocks * block_size = 128
    o, err, _ = run(hyperion, wk, path="row")
    assert err & hyperion.DEVERR_CTX_OVERFLOW
    check(oracle, wk, o)


def test_empty_worklist_is_a_no_op(hyperion):
    dev = torch.device("cuda", 0)
    wl = torch.zeros(0, 4, dtype=torch.int32, device=dev)
    o = torch.full((4, 128), 7.0, device=dev)
    z = torch.zeros(4, 4, dtype=torch.int32, device=dev)
    hyperion.hyperion_apex_kernel(wl, 0, z, None, z, None, torch.zeros(4, 128, dtype=torch.uint8, device=dev),
                                  torch.ones(1, device=dev), torch.ones(1, dtype=torch.int32, device=dev), None, o,
                                  4, 128, 16, 4, 1, 0.088, False)
    torch.cuda.synchronize()
    assert torch.all(o == 7.0)


def test_reset_counter_and_repeat_calls_are_stable(hyperion, oracle):
    wk = W.make_dense("r", 2, 2, 1, 999, o_dtype=torch.float32, seed=17)
    o1, _, _ = run(hyperion, wk, path="row")
    hyperion.hyperion_reset_counter(grid=(1, 1, 1), block=(1, 1, 1))
    o2, _, _ = run(hyperion, wk, path="row")
    assert np.array_equal(o1, o2)


# ----------------------------------------------------------------------------- full-size, sampled rows
def _sampled_check(hyperion, oracle, name, n_rows=24, path="auto"):
    dev = torch.device("cuda", 0)
    wk = W.make_config(name, device=dev, exact=False)
    o = wk.new_output()
    hyperion.read_device_errors(dev, clear=True)
    hyperion.hyperion_apex_kernel(wk.worklist, wk.total_work, wk.q, None, wk.k, None, wk.v, wk.v_scale,
                                  wk.ctx_lens, wk.block_tables, o, wk.seq_q, wk.head_dim, wk.head_dim // 8,
                                  wk.block_size, wk.num_blocks, wk.inv_sqrt_d, wk.causal, path=path)
    assert hyperion.read_device_errors(dev, clear=True) == 0
    assert torch.isfinite(o.float()).all()
    g = torch.Generator().manual_seed(0)
    items = torch.randperm(wk.total_work, generator=g)[:n_rows].sort().values.tolist()
    sub, rows = compact_subset(wk, items)
    o_ref, _, _, _ = oracle.forward_workload_c(sub)
    ok, mx, mn = oracle.tolerance_check(o.float().cpu().numpy()[rows], o_ref, MAX_ABS, MEAN_ABS)
    assert ok, (mx, mn)


def compact_subset(wk, items):
    """The keys the listed work items attend, gathered on the device into a small
    contiguous CPU workload (one bh per item, non-causal with the causal bound
    folded into its length).  Returns (workload, output rows of the items in wk)."""
    wl = wk.worklist.cpu()
    ctx = wk.ctx_lens.cpu()
    W_ = wk.head_dim // 32
    qs, ks, vs_rows, lens, scales, rows = [], [], [], [], [], []
    vsc = wk.v_scale.cpu()
    for it in items:
        q_idx, bh = int(wl[it, 0]), int(wl[it, 1])
        L = min(int(ctx[bh]), wk.num_blocks * wk.block_size)
        if wk.causal:
            L = min(L, q_idx + 1)
        t = torch.arange(L, device=wk.k.device)
        page = t // wk.block_size
        if wk.block_tables.numel():
            ids = wk.block_tables[bh].to(torch.int64)[page]
        else:
            ids = bh * wk.num_blocks + page
        slots = ids * wk.block_size + t % wk.block_size
        ks.append(wk.k[slots].cpu())
        vs_rows.append(wk.v[slots].cpu())
        qs.append(wk.q[bh * wk.seq_q + q_idx].cpu().view(1, W_))
        lens.append(L)
        scales.append(float(vsc[0] if vsc.numel() == 1 else vsc[bh % vsc.numel()]))
        rows.append(bh * wk.seq_q + q_idx)
    n = len(items)
    Lmax = max(lens)
    kk = torch.zeros(n * Lmax, W_, dtype=torch.int32)
    vv = torch.zeros(n * Lmax, wk.head_dim, dtype=torch.uint8)
    for i in range(n):
        kk[i * Lmax: i * Lmax + lens[i]] = ks[i]
        vv[i * Lmax: i * Lmax + lens[i]] = vs_rows[i]
    sc = torch.tensor(scales, dtype=torch.float32)
    if sc.numel() == kk.shape[0]:  # keep the per-(item) scale mode unambiguous
        sc = torch.cat([sc, sc[:1]])
    wl2 = W.dense_worklist(n, 1, "cpu")
    wl2[:, 0] = 0
    sub = W.Workload(name=wk.name + "_subset", worklist=wl2, q=torch.cat(qs), k=kk, v=vv, v_scale=sc,
                     ctx_lens=torch.tensor(lens, dtype=torch.int32), block_tables=torch.zeros(0, dtype=torch.int32),
                     seq_q=1, head_dim=wk.head_dim, block_size=Lmax, num_blocks=1, causal=False,
                     o_dtype=torch.float32, batch=1, heads=n, inv_sqrt_d=wk.inv_sqrt_d)
    return sub, rows


def test_decode_config_full_size_sampled_rows(hyperion, oracle):
    _sampled_check(hyperion, oracle, "decode")


def test_paged_decode_config_full_size_sampled_rows(hyperion, oracle):
    _sampled_check(hyperion, oracle, "paged_decode")


# ----------------------------------------------------------------------------- tile path (tcgen05)
def paged_copy(wk, page=16, seed=0):
    """The same keys as a contiguous workload, moved into a shuffled pool of pages."""
    n_bh = wk.n_bh
    S = wk.block_size
    pages = (S + page - 1) // page
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n_bh * pages, generator=g)
    k = torch.zeros(n_bh * pages * page, wk.k.shape[1], dtype=wk.k.dtype)
    v = torch.zeros(n_bh * pages * page, wk.head_dim, dtype=wk.v.dtype)
    bt = torch.zeros(n_bh, pages, dtype=torch.int32)
    for bh in range(n_bh):
        for pg in range(pages):
            blk = int(perm[bh * pages + pg])
            lo, hi = pg * page, min(S, (pg + 1) * page)
            k[blk * page: blk * page + hi - lo] = wk.k[bh * S + lo: bh * S + hi]
            v[blk * page: blk * page + hi - lo] = wk.v[bh * S + lo: bh * S + hi]
            bt[bh, pg] = blk
    return W.Workload(**{**wk.__dict__, "k": k, "v": v, "block_tables": bt, "block_size": page,
                         "num_blocks": pages})


def test_tile_path_is_available(hyperion):
    assert hyperion.launch_info()["tile_available"] == 1


@pytest.mark.parametrize("o_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_tile_path_cpu_ref_config(hyperion, oracle, o_dtype):
    wk = W.make_config("cpu_ref", device="cpu", exact=True)
    o, err, _ = run(hyperion, wk, path="tile", o_dtype=o_dtype)
    assert err == 0 and hyperion.last_call_info()["path"] == "tile"
    check(oracle, wk, o)


@pytest.mark.parametrize("scale_mode", ["tensor", "head", "bh"])
def test_tile_path_causal_ragged_multisegment(hyperion, oracle, scale_mode):
    # 300 rows per bh: chunks of 256 work items straddle (batch, head) rows.
    wk = W.make_dense("c", 2, 3, 300, 300, causal=True, scale_mode=scale_mode, o_dtype=torch.float32, seed=21)
    o, err, _ = run(hyperion, wk, path="tile")
    assert err == 0
    check(oracle, wk, o)


def test_tile_path_noncausal_kv_longer_than_q(hyperion, oracle):
    wk = W.make_dense("n", 1, 4, 130, 1000, causal=False, o_dtype=torch.float32, seed=22)
    o, err, _ = run(hyperion, wk, path="tile")
    assert err == 0
    check(oracle, wk, o)


def test_tile_path_scores_bit_exact(hyperion, oracle):
    wk = W.make_dense("s", 1, 2, 256, 384, causal=True, o_dtype=torch.float32, seed=23)
    L = 384
    _, _, _, sc_ref = oracle.forward_workload_c(wk, scores_ld=L)
    _, err, sc = run(hyperion, wk, path="tile", debug_ld=L)
    assert err == 0
    assert np.array_equal(sc, sc_ref)


def test_tile_path_paged_prefill(hyperion, oracle):
    dense = W.make_dense("pp", 2, 2, 200, 200, causal=True, o_dtype=torch.float32, seed=24)
    wk = paged_copy(dense, page=16, seed=3)
    o, err, _ = run(hyperion, wk, path="tile")
    assert err == 0
    check(oracle, wk, o)
    check(oracle, dense, o)


def test_tile_path_large_scores_force_rescale(hyperion, oracle):
    # inv_sqrt_d = 1: scores span +-128, the running max moves by more than 2^8
    # many times and O is rescaled in TMEM.
    wk = W.make_dense("r", 1, 2, 256, 1024, causal=False, o_dtype=torch.float32, seed=25)
    wk.inv_sqrt_d = 1.0
    o, err, _ = run(hyperion, wk, path="tile")
    assert err == 0
    check(oracle, wk, o)


@pytest.mark.parametrize("path", ["row", "tile"])
def test_negative_inv_sqrt_d(hyperion, oracle, path):
    # A negative scale turns the scores around: the tile path flips Q's bits, the row
    # path takes the integer minimum as the group maximum.
    wk = W.make_dense("n", 1, 2, 256, 512, causal=True, o_dtype=torch.float32, seed=27)
    wk.inv_sqrt_d = -1.0 / 128 ** 0.5
    o, err, dbg = run(hyperion, wk, path=path, debug_ld=512)
    assert err == 0 and hyperion.last_call_info()["path"] == path
    check(oracle, wk, o)
    _, _, _, ref_scores = oracle.forward_workload_c(wk, scores_ld=512)
    assert np.array_equal(dbg, ref_scores)  # the integer scores D - 2*popc, unscaled


@pytest.mark.parametrize("path", ["row", "tile"])
def test_shuffled_worklist(hyperion, oracle, path):
    # Items in random order: every 256-item chunk mixes many (batch, head) rows, so the
    # tile path runs many short segments per chunk.
    wk = W.make_dense("s", 2, 3, 96, 96, causal=True, o_dtype=torch.float32, seed=28)
    perm = torch.randperm(wk.total_work, generator=torch.Generator().manual_seed(9))
    wk.worklist = wk.worklist[perm].contiguous()
    o, err, _ = run(hyperion, wk, path=path)
    assert err == 0 and hyperion.last_call_info()["path"] == path
    check(oracle, wk, o)


def test_row_path_large_scores_force_rescale(hyperion, oracle):
    wk = W.make_dense("rr", 1, 2, 8, 3000, causal=False, o_dtype=torch.float32, seed=29)
    wk.inv_sqrt_d = 1.0
    o, err, _ = run(hyperion, wk, path="row", num_splits=3)
    assert err == 0
    check(oracle, wk, o)


@pytest.mark.parametrize("path,D", [("row", 128), ("row", 256), ("tile", 128)])
def test_every_fp8_code_in_the_cache(hyperion, oracle, path, D):
    """V bytes drawn from all 256 codes, so 0x7F / 0xFF (+-480 in the reference's
    decode, NaN to the hardware e4m3 conversion the row kernel's fast decode uses)
    land in most groups: the row kernel must redo those groups exactly, and every
    output must match the oracle."""
    S_q = 3 if path == "row" else 150
    wk = W.make_dense("codes", 1, 2, S_q, 1100, D=D, causal=(path == "tile"), scale_mode="head",
                      o_dtype=torch.float32, seed=33)
    gen = torch.Generator().manual_seed(34)
    wk.v = torch.randint(0, 256, tuple(wk.v.shape), dtype=torch.uint8, generator=gen)
    wk.v_scale = torch.tensor([0.004, 0.006], dtype=torch.float32)
    assert int((wk.v == 0x7F).sum()) > 100 and int((wk.v == 0xFF).sum()) > 100
    o, err, _ = run(hyperion, wk, path=path)
    assert err == 0
    assert np.isfinite(o).all()
    check(oracle, wk, o)


def test_row_path_sparse_nan_codes(hyperion, oracle):
    """A cache from the quantiser with a few 0x7F / 0xFF codes planted in it: the
    groups that hold one take the exact redo and the rest the fast decode, across
    split-KV partials."""
    wk = W.make_dense("nan_codes", 2, 2, 1, 5000, scale_mode="head", o_dtype=torch.float32, seed=35)
    gen = torch.Generator().manual_seed(36)
    v = wk.v.clone()
    rows = torch.randint(0, v.shape[0], (40,), generator=gen)
    cols = torch.randint(0, v.shape[1], (40,), generator=gen)
    v[rows[:20], cols[:20]] = 0x7F
    v[rows[20:], cols[20:]] = 0xFF
    wk.v = v
    o, err, _ = run(hyperion, wk, path="row", num_splits=4)
    assert err == 0
    assert np.isfinite(o).all()
    check(oracle, wk, o)


def test_tile_path_short_and_empty_contexts(hyperion, oracle):
    wk = W.make_dense("e", 1, 4, 256, 256, causal=False, o_dtype=torch.float32, seed=26)
    wk.ctx_lens[0] = 0
    wk.ctx_lens[1] = 1
    wk.ctx_lens[2] = 129
    o, err, _ = run(hyperion, wk, path="tile")
    assert err == 0
    assert np.all(o[0:256] == 0)
    check(oracle, wk, o)


def test_tile_path_bad_block_flag(hyperion, oracle):
    dense = W.make_dense("b", 1, 2, 128, 128, causal=True, o_dtype=torch.float32, seed=27)
    wk = paged_copy(dense, page=16, seed=4)
    wk.block_tables[0, 3] = 1 << 29
    o, err, _ = run(hyperion, wk, path="tile")
    assert err & hyperion.DEVERR_BAD_BLOCK
    check(oracle, wk, o)


def test_tile_and_row_paths_agree(hyperion, oracle):
    wk = W.make_dense("a", 2, 2, 384, 384, causal=True, o_dtype=torch.float32, seed=28)
    o_t, e1, _ = run(hyperion, wk, path="tile")
    o_r, e2, _ = run(hyperion, wk, path="row")
    assert e1 == 0 and e2 == 0
    ok, mx, mn = oracle.tolerance_check(o_t, o_r, MAX_ABS, MEAN_ABS)
    assert ok, (mx, mn)


def test_auto_path_picks_tile_for_prefill_and_row_for_decode(hyperion):
    wk = W.make_dense("x", 1, 2, 128, 128, causal=True, o_dtype=torch.float32, seed=29)
    run(hyperion, wk)
    assert hyperion.last_call_info()["path"] == "tile"
    wk2 = W.make_dense("y", 1, 2, 1, 128, o_dtype=torch.float32, seed=29)
    run(hyperion, wk2)
    assert hyperion.last_call_info()["path"] == "row"


def test_prefill_config_full_size_sampled_rows(hyperion, oracle):
    _sampled_check(hyperion, oracle, "prefill", n_rows=32, path="tile")


def test_forwards_on_two_streams_do_not_share_a_workspace(hyperion, oracle):
    """Two split-KV decodes enqueued on two streams at once: each stream has its own
    workspace (work counter, partials), so both results equal the oracle's."""
    dev = torch.device("cuda", 0)
    wks = [W.make_dense(f"s{i}", 2, 4, 1, 3000 + 500 * i, o_dtype=torch.float32, seed=60 + i) for i in range(2)]
    gs = [wk.to(dev) for wk in wks]
    outs = [g.new_output() for g in gs]
    streams = [torch.cuda.Stream(dev) for _ in range(2)]
    torch.cuda.synchronize()
    for rep in range(3):
        for g, o, s in zip(gs, outs, streams):
            with torch.cuda.stream(s):
                hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale,
                                              g.ctx_lens, g.block_tables, o, 1, 128, 16, g.block_size, g.num_blocks,
                                              g.inv_sqrt_d, False, path="row", num_splits=5)
    torch.cuda.synchronize()
    for wk, o, s in zip(wks, outs, streams):
        with torch.cuda.stream(s):
            assert hyperion.read_device_errors(dev, clear=True) == 0
        check(oracle, wk, o.cpu().numpy())


@pytest.mark.parametrize("kv_heads,group_kernel,splits", [(None, "auto", 8), (8, "cuda", 16), (8, "auto", 8)])
def test_split_choice_follows_the_measured_table(hyperion, oracle, kv_heads, group_kernel, splits):
    """On a 148-SM B200 the automatic split count for a shape the launch table
    measured is the table's (128 query rows x 8192 keys: 8 pieces on the row kernel;
    the same with 4 query heads per KV head: 16 pieces on the CUDA-core grouped
    kernel, 8 on the tensor-core one), and the result is still the oracle's."""
    if hyperion.launch_info()["sm_count"] != 148:
        pytest.skip("the launch table was measured on 148 SMs")
    wk = W.make_dense("t", 4, 32, 1, 8192, kv_heads=kv_heads, o_dtype=torch.float32, seed=66)
    dev = torch.device("cuda", 0)
    g = wk.to(dev)
    o = g.new_output()
    hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens,
                                  g.block_tables, o, 1, 128, 16, g.block_size, g.num_blocks, g.inv_sqrt_d, False,
                                  kv_group=g.kv_group, group_kernel=group_kernel)
    info = hyperion.last_call_info()
    assert info["splits"] == splits, info
    rows = list(range(0, g.n_bh, 7))
    check(oracle, wk, o.cpu().numpy(), rows=rows)


@pytest.mark.parametrize("path,seq_q", [("tile", 256), ("row", 1)])
def test_sm_budget_caps_the_persistent_grid(hyperion, oracle, path, seq_q):
    """sm_budget keeps the persistent kernels on that many SMs (the rest stay free for
    a collective on another stream); the result does not change."""
    wk = W.make_dense("b", 4, 16, seq_q, 1024 if seq_q == 1 else seq_q, causal=seq_q > 1, o_dtype=torch.float32,
                      seed=67)
    dev = torch.device("cuda", 0)
    g = wk.to(dev)
    info = hyperion.launch_info()
    o = g.new_output()
    hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens,
                                  g.block_tables, o, g.seq_q, 128, 16, g.block_size, g.num_blocks, g.inv_sqrt_d,
                                  g.causal, path=path, sm_budget=10)
    grid = hyperion.last_call_info()["grid"]
    per_sm = info["tile_ctas_per_sm"] if path == "tile" else info["row_ctas_per_sm"]
    assert grid <= 10 * per_sm, grid
    assert hyperion.read_device_errors(dev, clear=True) == 0
    check(oracle, wk, o.cpu().numpy())
    with pytest.raises(RuntimeError, match="sm_budget"):
        hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens,
                                      g.block_tables, o, g.seq_q, 128, 16, g.block_size, g.num_blocks, g.inv_sqrt_d,
                                      g.causal, path=path, sm_budget=-1)
