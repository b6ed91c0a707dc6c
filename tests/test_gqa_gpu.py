"""GPU parity of grouped-query attention (kv_group > 1) against the CPU oracle.

The oracle restates kv_group by expanding the KV-side index arrays per query row
(pinned on the CPU against materialized KV copies).  Bar as for every parity test:
integer scores bit-exact, outputs within max-abs 2e-2 and mean-abs 2e-3 in fp32.
"""
import numpy as np
import pytest
import torch

from hyperion_b200 import workloads as W

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def run(hyperion, wk, path="auto", num_splits=0, debug_ld=0, kv_group=None, block_tables=None, ctx=None,
        v_scale=None):
    dev = torch.device("cuda", 0)
    g = wk.to(dev)
    o = torch.full((g.n_bh * g.seq_q, g.head_dim), float("nan"), dtype=torch.float32, device=dev)
    dbg = torch.zeros(g.total_work, debug_ld, dtype=torch.int32, device=dev) if debug_ld else None
    bt = g.block_tables if block_tables is None else block_tables.to(dev)
    cl = g.ctx_lens if ctx is None else ctx.to(dev)
    vs = g.v_scale if v_scale is None else v_scale.to(dev)
    hyperion.read_device_errors(dev, clear=True)
    hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, vs, cl, bt, o, g.seq_q,
                                  g.head_dim, g.head_dim // 8, g.block_size, g.num_blocks, g.inv_sqrt_d, g.causal,
                                  path=path, num_splits=num_splits, debug_scores=dbg,
                                  kv_group=wk.kv_group if kv_group is None else kv_group)
    info = hyperion.last_call_info()
    err = hyperion.read_device_errors(dev, clear=True)
    return o.cpu().numpy(), err, (dbg.cpu().numpy() if dbg is not None else None), info


def check(oracle, wk, o_gpu, rows=None):
    o_ref, _, _, _ = oracle.forward_workload_c(wk)
    if rows is not None:
        o_ref, o_gpu = o_ref[rows], o_gpu[rows]
    ok, mx, mn = oracle.tolerance_check(o_gpu, o_ref, MAX_ABS, MEAN_ABS)
    assert ok, f"max {mx:.3e} mean {mn:.3e}"


@pytest.mark.parametrize("H,Hkv,D", [(8, 2, 128), (8, 4, 128), (8, 1, 128), (6, 2, 128), (8, 2, 256)])
def test_gqa_decode_row_path(hyperion, oracle, H, Hkv, D):
    """Decode worklists in (batch, head) order: the run of a unit is the query heads
    of one KV head (kv_group 2 and 4), two runs per KV head (kv_group 8), or a run
    that stops at a group boundary inside the unit (kv_group 3)."""
    wk = W.make_dense("gqa_dec", 3, H, 1, 2100, D=D, scale_mode="head", o_dtype=torch.float32, seed=51,
                      kv_heads=Hkv)
    o, err, _, info = run(hyperion, wk, path="row")
    assert err == 0 and info["path"] == "row"
    assert np.isfinite(o).all()
    check(oracle, wk, o)


@pytest.mark.parametrize("num_splits", [0, 1, 3])
def test_gqa_paged_decode(hyperion, oracle, num_splits):
    wk = W.make_paged("gqa_paged", 4, 8, [17, 300, 1000, 2500], page=16, seed=52, o_dtype=torch.float32,
                      kv_heads=2)
    o, err, _, _ = run(hyperion, wk, num_splits=num_splits)
    assert err == 0
    check(oracle, wk, o)


def test_gqa_equals_block_tables_repeated_per_query_head(hyperion, oracle):
    """The same problem given to the ungrouped kernel, every query head's block-table
    row pointing at its KV head's pages.  Both meet the bar against the oracle, and
    they agree with each other to rounding: the grouped runs take their products on
    the tensor core with f32 sums, the ungrouped kernel sums 32-key groups of f16x2
    products, and the two split the keys differently."""
    wk = W.make_paged("gqa_eq", 3, 8, [100, 999, 3000], page=16, seed=53, o_dtype=torch.float32, kv_heads=2)
    o_g, err, _, _ = run(hyperion, wk, path="row", num_splits=2)
    assert err == 0
    kv_of_bh = torch.arange(wk.n_bh) // wk.kv_group
    o_p, err2, _, _ = run(hyperion, wk, path="row", num_splits=2, kv_group=1,
                          block_tables=wk.block_tables[kv_of_bh].contiguous(),
                          ctx=wk.ctx_lens[kv_of_bh].contiguous(),
                          v_scale=wk.v_scale.repeat_interleave(wk.kv_group))
    assert err2 == 0
    check(oracle, wk, o_g)
    check(oracle, wk, o_p)
    assert np.abs(o_g - o_p).max() <= 2e-3


@pytest.mark.parametrize("path", ["row", "tile"])
def test_gqa_causal_prefill(hyperion, oracle, path):
    """Row path: consecutive items of one (batch, head) at different causal positions
    share a run and each keeps its own key range.  Tile path: KV rows by bh // kv_group."""
    wk = W.make_dense("gqa_pre", 1, 4, 150, 150, causal=True, scale_mode="bh", o_dtype=torch.float32, seed=54,
                      kv_heads=2)
    o, err, _, info = run(hyperion, wk, path=path)
    assert err == 0 and info["path"] == path
    check(oracle, wk, o)


def test_gqa_scores_bit_exact(hyperion, oracle):
    wk = W.make_paged("gqa_sc", 2, 4, [70, 500], page=16, seed=55, o_dtype=torch.float32, kv_heads=1)
    L = 500
    _, _, _, sc_ref = oracle.forward_workload_c(wk, scores_ld=L)
    _, err, sc, _ = run(hyperion, wk, path="row", debug_ld=L)
    assert err == 0
    assert np.array_equal(sc, sc_ref)


def test_gqa_per_slot_scale(hyperion, oracle):
    wk = W.make_paged("gqa_slot", 2, 4, [64, 700], page=16, seed=56, o_dtype=torch.float32, kv_heads=2)
    gen = torch.Generator().manual_seed(57)
    wk.v_scale = torch.rand(wk.v.shape[0], generator=gen) * 0.01 + 1e-3
    o, err, _, _ = run(hyperion, wk, path="row", num_splits=2)
    assert err == 0
    check(oracle, wk, o)


def test_gqa_every_fp8_code(hyperion, oracle):
    wk = W.make_dense("gqa_codes", 1, 8, 1, 1500, scale_mode="head", o_dtype=torch.float32, seed=58, kv_heads=2)
    gen = torch.Generator().manual_seed(59)
    wk.v = torch.randint(0, 256, tuple(wk.v.shape), dtype=torch.uint8, generator=gen)
    wk.v_scale = torch.tensor([0.004, 0.006], dtype=torch.float32)
    o, err, _, _ = run(hyperion, wk, path="row")
    assert err == 0 and np.isfinite(o).all()
    check(oracle, wk, o)


def test_gqa_shuffled_worklist_and_bad_item(hyperion, oracle):
    """Runs break wherever neighbouring items sit on different KV rows; a bad item is
    flagged and left unwritten while the rest of its unit is computed."""
    wk = W.make_paged("gqa_shuf", 3, 8, [200, 900, 1700], page=16, seed=60, o_dtype=torch.float32, kv_heads=2)
    gen = torch.Generator().manual_seed(61)
    wl = wk.worklist[torch.randperm(wk.total_work, generator=gen)].clone()
    wl[5, 1] = wk.n_bh + 3  # query row out of range
    wk.worklist = wl
    o, err, _, _ = run(hyperion, wk, path="row", num_splits=2)
    assert err & 0x1  # HYPERION_DEVERR_BAD_ITEM
    good = [i for i in range(wk.total_work) if i != 5]
    rows = (wl[good, 1].long() * wk.seq_q + wl[good, 0].long()).tolist()
    check(oracle, wk, o, rows=rows)
    # The one query row no valid item names stays as the test filled it (NaN).
    assert np.isnan(np.delete(o, rows, axis=0)).all()


def test_gqa_cache_written_per_kv_head_then_read(hyperion, oracle):
    """kv_cache_write with n_heads = num_kv_heads fills the pool the grouped forward
    reads: a 2-sequence paged decode through both calls against the oracle."""
    dev = torch.device("cuda", 0)
    B, H, Hkv, D, page = 2, 8, 2, 128, 16
    lens = [37, 250]
    nb = max((L + page - 1) // page for L in lens)
    torch.manual_seed(62)
    k_new = [torch.randn(L, Hkv, D) for L in lens]
    v_new = [torch.randn(L, Hkv, D) for L in lens]
    vs = torch.tensor([0.006, 0.008])
    # Pages of sequence b, KV head h: a shuffled pool.
    n_pages = sum((L + page - 1) // page for L in lens) * Hkv
    perm = torch.randperm(n_pages, generator=torch.Generator().manual_seed(63))
    bt = torch.zeros(B * Hkv, nb, dtype=torch.int32)
    c = 0
    for b, L in enumerate(lens):
        for h in range(Hkv):
            for j in range((L + page - 1) // page):
                bt[b * Hkv + h, j] = int(perm[c])
                c += 1
    kc = torch.zeros(n_pages * page, D // 32, dtype=torch.int32, device=dev)
    vc = torch.zeros(n_pages * page, D, dtype=torch.uint8, device=dev)
    for b, L in enumerate(lens):
        hyperion.kv_cache_write(k_new[b].to(dev), v_new[b].to(dev), torch.full((L,), b, dtype=torch.int32, device=dev),
                                torch.arange(L, dtype=torch.int32, device=dev), bt.to(dev), page, nb, vs.to(dev), kc,
                                vc)
    assert hyperion.read_device_errors(dev, clear=True) == 0
    q = W.sign_pack(torch.randn(B * H, D))
    wl = W.dense_worklist(B * H, 1, "cpu")
    wk = W.Workload(name="gqa_e2e", worklist=wl, q=q, k=kc.cpu(), v=vc.cpu(), v_scale=vs,
                    ctx_lens=torch.tensor(lens, dtype=torch.int32).repeat_interleave(Hkv), block_tables=bt, seq_q=1,
                    head_dim=D, block_size=page, num_blocks=nb, causal=False, o_dtype=torch.float32, batch=B,
                    heads=H, kv_group=H // Hkv)
    o, err, _, _ = run(hyperion, wk, path="row")
    assert err == 0
    check(oracle, wk, o)


def _paged_kv_copy(wk, page=16, seed=0):
    """The same keys as a contiguous grouped-query workload, moved into a shuffled
    pool of pages (one block-table row per KV row)."""
    n_kv = wk.n_kv_bh
    S = wk.block_size
    pages = (S + page - 1) // page
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n_kv * pages, generator=g)
    k = torch.zeros(n_kv * pages * page, wk.k.shape[1], dtype=wk.k.dtype)
    v = torch.zeros(n_kv * pages * page, wk.head_dim, dtype=wk.v.dtype)
    bt = torch.zeros(n_kv, pages, dtype=torch.int32)
    for r in range(n_kv):
        for pg in range(pages):
            blk = int(perm[r * pages + pg])
            lo, hi = pg * page, min(S, (pg + 1) * page)
            k[blk * page: blk * page + hi - lo] = wk.k[r * S + lo: r * S + hi]
            v[blk * page: blk * page + hi - lo] = wk.v[r * S + lo: r * S + hi]
            bt[r, pg] = blk
    return W.Workload(**{**wk.__dict__, "k": k, "v": v, "block_tables": bt, "block_size": page,
                         "num_blocks": pages})


@pytest.mark.parametrize("path", ["tile", "row"])
def test_gqa_paged_causal_prefill(hyperion, oracle, path):
    dense = W.make_dense("gqa_pp", 2, 8, 200, 200, causal=True, scale_mode="head", o_dtype=torch.float32, seed=64,
                         kv_heads=2)
    wk = _paged_kv_copy(dense, page=16, seed=3)
    o, err, _, info = run(hyperion, wk, path=path)
    assert err == 0 and info["path"] == path
    check(oracle, wk, o)
    check(oracle, dense, o)


@pytest.mark.parametrize("o_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("path,S_q", [("row", 1), ("tile", 130)])
def test_gqa_half_precision_outputs(hyperion, oracle, o_dtype, path, S_q):
    """bf16 and f16 O (the engine's types) from the grouped row kernel and the tile path."""
    wk = W.make_dense("gqa_o", 2, 8, S_q, 600, causal=(S_q > 1), scale_mode="head", o_dtype=o_dtype, seed=65,
                      kv_heads=2)
    dev = torch.device("cuda", 0)
    g = wk.to(dev)
    o = torch.zeros(g.n_bh * g.seq_q, g.head_dim, dtype=o_dtype, device=dev)
    hyperion.read_device_errors(dev, clear=True)
    hyperion.hyperion_apex_kernel(g.worklist, g.total_work, g.q, None, g.k, None, g.v, g.v_scale, g.ctx_lens,
                                  g.block_tables, o, g.seq_q, g.head_dim, g.head_dim // 8, g.block_size,
                                  g.num_blocks, g.inv_sqrt_d, g.causal, path=path, kv_group=wk.kv_group)
    assert hyperion.last_call_info()["path"] == path
    assert hyperion.read_device_errors(dev, clear=True) == 0
    check(oracle, wk, o.float().cpu().numpy())
