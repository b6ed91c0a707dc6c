"""GPU parity at the measured sizes: whole (batch, head) rows of the full workloads.

The forward runs over the whole workload, as the benchmark runs it; then every
query row of a few chosen (batch, head) rows -- the first, the last and a seeded
interior one, so the last 256-row unit, the causal diagonal and interior units are
all covered -- is checked against the C oracle within max-abs 2e-2 / mean-abs
2e-3, and the integer scores of those rows are checked bit for bit through the
debug score export.  Also here: the 32768-token prefill on one rank's 8 heads, and
adversarial V for the row kernels' f16 partial sums.
"""
import numpy as np
import pytest
import torch

from hyperion_b200 import workloads as W

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
DEV = torch.device("cuda", 0)


def forward(hyperion, wk, o, worklist=None, debug=None, path="auto", num_splits=0):
    wl = wk.worklist if worklist is None else worklist
    hyperion.read_device_errors(DEV, clear=True)
    hyperion.hyperion_apex_kernel(wl, wl.shape[0], wk.q, None, wk.k, None, wk.v, wk.v_scale, wk.ctx_lens,
                                  wk.block_tables, o, wk.seq_q, wk.head_dim, wk.head_dim // 8, wk.block_size,
                                  wk.num_blocks, wk.inv_sqrt_d, wk.causal, path=path, num_splits=num_splits,
                                  debug_scores=debug, kv_group=wk.kv_group)
    return hyperion.read_device_errors(DEV, clear=True)


def bh_subset(wk, bhs, q_lo=0, q_hi=None):
    """Query rows [q_lo, q_hi) of the listed (batch, head) rows of a device workload,
    with each row's keys gathered (from its block table or the contiguous layout)
    into a contiguous CPU workload of the same seq_q, causality and scale.  Returns
    (workload, O rows of those query rows in the full output)."""
    q_hi = wk.seq_q if q_hi is None else q_hi
    g = wk.kv_group
    W_ = wk.head_dim // 32
    cap = wk.num_blocks * wk.block_size
    lens = [min(int(wk.ctx_lens[bh // g]), cap) for bh in bhs]
    Lmax = max(max(lens), 1)
    kk = torch.zeros(len(bhs) * Lmax, W_, dtype=torch.int32)
    vv = torch.zeros(len(bhs) * Lmax, wk.head_dim, dtype=torch.uint8)
    qq, sc, rows = [], [], []
    vsc = wk.v_scale.cpu()
    for i, (bh, L) in enumerate(zip(bhs, lens)):
        t = torch.arange(L, device=wk.k.device)
        page = t // wk.block_size
        kv = bh // g
        ids = wk.block_tables[kv].to(torch.int64)[page] if wk.block_tables.numel() else kv * wk.num_blocks + page
        slots = ids * wk.block_size + t % wk.block_size
        kk[i * Lmax: i * Lmax + L] = wk.k[slots].cpu()
        vv[i * Lmax: i * Lmax + L] = wk.v[slots].cpu()
        qq.append(wk.q[bh * wk.seq_q:(bh + 1) * wk.seq_q].cpu())
        sc.append(float(vsc[0] if vsc.numel() == 1 else vsc[kv % vsc.numel()]))
        rows += [bh * wk.seq_q + q for q in range(q_lo, q_hi)]
    scale = torch.tensor(sc, dtype=torch.float32)
    if scale.numel() == kk.shape[0]:
        scale = torch.cat([scale, scale[:1]])
    wl = W.dense_worklist(len(bhs), wk.seq_q, "cpu").view(len(bhs), wk.seq_q, 4)[:, q_lo:q_hi].reshape(-1, 4)
    if wk.seq_q == 1:
        wl[:, 0] = 0
    sub = W.Workload(name=wk.name + "_rows", worklist=wl.contiguous(), q=torch.cat(qq), k=kk, v=vv, v_scale=scale,
                     ctx_lens=torch.tensor(lens, dtype=torch.int32), block_tables=torch.zeros(0, dtype=torch.int32),
                     seq_q=wk.seq_q, head_dim=wk.head_dim, block_size=Lmax, num_blocks=1, causal=wk.causal,
                     o_dtype=torch.float32, batch=1, heads=len(bhs), inv_sqrt_d=wk.inv_sqrt_d)
    return sub, rows


def items_of(wk, bhs, q_lo=0, q_hi=None):
    """The work items (rows of wk.worklist) of query rows [q_lo, q_hi) of the listed bh,
    in worklist order, as a device worklist."""
    q_hi = wk.seq_q if q_hi is None else q_hi
    wl = wk.worklist
    keep = torch.zeros(wl.shape[0], dtype=torch.bool, device=wl.device)
    for bh in bhs:
        keep |= (wl[:, 1] == bh) & (wl[:, 0] >= q_lo) & (wl[:, 0] < q_hi)
    return wl[keep].contiguous()


def whole_rows_check(hyperion, oracle, wk, bhs, path="auto", debug_q=None):
    """Full-size forward, then every query row of `bhs` against the oracle, then the
    integer scores of query rows debug_q = (lo, hi) of `bhs` bit for bit."""
    o = wk.new_output()
    assert forward(hyperion, wk, o, path=path) == 0
    assert torch.isfinite(o.float()).all()
    sub, rows = bh_subset(wk, bhs)
    ref, written, err, _ = oracle.forward_workload_c(sub)
    assert err == 0 and written.all()
    got = o.float().cpu().numpy()[rows]
    ok, mx, mn = oracle.tolerance_check(got, ref[rows_local(sub)], MAX_ABS, MEAN_ABS)
    assert ok, (wk.name, mx, mn)
    lo, hi = debug_q if debug_q is not None else (0, wk.seq_q)
    L = int(sub.ctx_lens.max())
    wl = items_of(wk, bhs, lo, hi)
    dbg = torch.zeros(wl.shape[0], L, dtype=torch.int32, device=DEV)
    o2 = wk.new_output()
    assert forward(hyperion, wk, o2, worklist=wl, debug=dbg, path=path) == 0
    sub_d, _ = bh_subset(wk, bhs, lo, hi)
    _, _, err, scores = oracle.forward_workload_c(sub_d, scores_ld=L)
    assert err == 0
    assert np.array_equal(dbg.cpu().numpy(), scores), wk.name
    return mx, mn


def rows_local(sub):
    wl = sub.worklist.numpy()
    return (wl[:, 1].astype(np.int64) * sub.seq_q + wl[:, 0]).tolist()


def test_prefill_full_size_whole_rows(hyperion, oracle):
    """B4 H32 S4096 causal on the tile kernel: three whole (batch, head) rows (4096 query
    rows each, all 16 units of 256 rows) against the oracle, and their scores."""
    wk = W.make_config("prefill", device=DEV, exact=False)
    bhs = [0, 77, wk.n_bh - 1]
    whole_rows_check(hyperion, oracle, wk, bhs, path="tile")
    assert hyperion.last_call_info()["path"] == "tile"


def test_decode_full_size_whole_rows(hyperion, oracle):
    """B64 H32 S_kv 8192: every head of the first and the last sequence and 24 seeded
    others (each item is a whole (batch, head) row here)."""
    wk = W.make_config("decode", device=DEV, exact=False)
    g = torch.Generator().manual_seed(1)
    bhs = sorted(set(range(32)) | set(range(wk.n_bh - 32, wk.n_bh)) |
                 set(torch.randperm(wk.n_bh, generator=g)[:24].tolist()))
    whole_rows_check(hyperion, oracle, wk, bhs)


def test_paged_decode_full_size_whole_rows(hyperion, oracle):
    """B256 H32, contexts U[512, 32768], 16-token pages: the longest and the shortest
    sequence's heads (the longest is split over several CTAs) and 16 seeded others."""
    wk = W.make_config("paged_decode", device=DEV, exact=False)
    lens = wk.ctx_lens.cpu()
    b_long, b_short = int(torch.argmax(lens)) // 32, int(torch.argmin(lens)) // 32
    g = torch.Generator().manual_seed(2)
    bhs = sorted(set(range(b_long * 32, b_long * 32 + 32)) | set(range(b_short * 32, b_short * 32 + 8)) |
                 set(torch.randperm(wk.n_bh, generator=g)[:16].tolist()))
    whole_rows_check(hyperion, oracle, wk, bhs)


def test_decode_gqa_full_size_whole_rows(hyperion, oracle):
    """The engine's head layout (32 query heads over 8 KV heads) on the grouped kernel."""
    wk = W.make_config("decode_gqa", device=DEV, exact=False)
    bhs = list(range(32)) + list(range(wk.n_bh - 32, wk.n_bh))
    whole_rows_check(hyperion, oracle, wk, bhs)


def test_prefill_heads_in_l2_groups_whole_rows(hyperion, oracle):
    """B2 H96 S4096 causal: 192 (batch, head) rows whose KV (590 KB each, 113 MB in
    all) does not stay in L2, so the tile kernel's tickets take the rows in groups of
    85 (48 MB of KV), 85 and 22, each group longest units first.  Every output row
    is written (O starts as NaN), and whole rows at the group boundaries and in the
    short last group match the oracle, scores bit for bit."""
    wk = W.make_dense("l2_groups", 2, 96, 4096, 4096, causal=True, o_dtype=torch.float32, seed=241, device=DEV,
                      gen_device=DEV, exact=False)
    assert wk.n_bh * wk.seq_q * 144 > 96 * (1 << 20)
    o = torch.full((wk.n_bh * wk.seq_q, wk.head_dim), float("nan"), dtype=torch.float32, device=DEV)
    assert forward(hyperion, wk, o, path="tile") == 0
    assert hyperion.last_call_info()["path"] == "tile"
    assert torch.isfinite(o).all(), "a chunk of the ticket order was never taken"
    bhs = [0, 84, 85, 170, 191]
    sub, rows = bh_subset(wk, bhs)
    ref, written, err, _ = oracle.forward_workload_c(sub)
    assert err == 0 and written.all()
    ok, mx, mn = oracle.tolerance_check(o.cpu().numpy()[rows], ref[rows_local(sub)], MAX_ABS, MEAN_ABS)
    assert ok, (mx, mn)
    wl = items_of(wk, [85, 191], 4096 - 512, 4096)
    dbg = torch.zeros(wl.shape[0], 4096, dtype=torch.int32, device=DEV)
    assert forward(hyperion, wk, wk.new_output(), worklist=wl, debug=dbg, path="tile") == 0
    sub_d, _ = bh_subset(wk, [85, 191], 4096 - 512, 4096)
    _, _, err, scores = oracle.forward_workload_c(sub_d, scores_ld=4096)
    assert err == 0
    assert np.array_equal(dbg.cpu().numpy(), scores)


def test_longctx_one_rank_heads_whole_row(hyperion, oracle):
    """B1 S32768 causal, the 8 heads one rank owns at world size 8: the last head's
    32768 query rows against the oracle; scores of the last two 256-row units of the
    last head and the first unit of the first head bit for bit."""
    from hyperion_b200.sharding import head_range

    wk = W.make_config("longctx", device=DEV, exact=False, heads=head_range(64, 8, 0))
    assert wk.n_bh == 8 and wk.seq_q == 32768
    whole_rows_check(hyperion, oracle, wk, [7], path="tile", debug_q=(32768 - 512, 32768))
    # the first unit of the first head (its rows attend 1..256 keys)
    o = wk.new_output()
    wl = items_of(wk, [0], 0, 256)
    dbg = torch.zeros(wl.shape[0], 256, dtype=torch.int32, device=DEV)
    assert forward(hyperion, wk, o, worklist=wl, debug=dbg, path="tile") == 0
    sub, rows = bh_subset(wk, [0], 0, 256)
    ref, _, err, scores = oracle.forward_workload_c(sub, scores_ld=256)
    assert err == 0
    assert np.array_equal(dbg.cpu().numpy(), scores)
    ok, mx, mn = oracle.tolerance_check(o.float().cpu().numpy()[rows], ref[rows_local(sub)], MAX_ABS, MEAN_ABS)
    assert ok, (mx, mn)


# ----------------------------------------------------------------------------- adversarial V
def adversarial(n_keys, signed, inv_sqrt_d, seed, n_bh=4):
    """Decode rows whose V codes all lie in |code| in [0x70, 0x7E] (128 .. 448 before the
    scale, the largest finite magnitudes): the row kernels sum 32 products w * v in f16
    before adding them to f32 accumulators, and these codes make those partial sums as
    large as they get (32 * 448 = 14336, where the f16 spacing is 8).  inv_sqrt_d 0
    makes every weight exactly 1; a small inv_sqrt_d makes weights just below 1, whose
    products carry full f16 mantissas."""
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(0x70, 0x7F, (n_bh * n_keys, 128), generator=g, dtype=torch.int32)
    if signed:
        codes |= torch.randint(0, 2, codes.shape, generator=g, dtype=torch.int32) << 7
    wk = W.make_dense("adv", 1, n_bh, 1, n_keys, o_dtype=torch.float32, seed=seed)
    wk.v = codes.to(torch.uint8)
    wk.v_scale = torch.full((n_bh,), 4.5 / 448.0, dtype=torch.float32)
    wk.inv_sqrt_d = inv_sqrt_d
    return wk


@pytest.mark.parametrize("n_keys,num_splits", [(8192, 1), (8192, 4), (32768, 16), (32768, 0)])
@pytest.mark.parametrize("signed", [False, True])
@pytest.mark.parametrize("inv_sqrt_d", [0.0, 0.002, 0.088])
def test_row_kernel_f16_partial_sums_on_adversarial_v(hyperion, oracle, n_keys, num_splits, signed, inv_sqrt_d):
    wk = adversarial(n_keys, signed, inv_sqrt_d, seed=n_keys + num_splits + int(signed))
    assert wk.inv_sqrt_d == inv_sqrt_d
    g = wk.to(DEV)
    o = g.new_output()
    assert forward(hyperion, g, o, path="row", num_splits=num_splits) == 0
    ref, _, err, _ = oracle.forward_workload_c(wk)
    assert err == 0
    ok, mx, mn = oracle.tolerance_check(o.cpu().numpy(), ref, MAX_ABS, MEAN_ABS)
    assert ok, (mx, mn)
    # Far inside the bar: the f16 partial sums lose at most a few f16 spacings of
    # 14336 per 32-key group, divided by the weights' sum.
    assert mx < 2e-3, mx


@pytest.mark.parametrize("signed", [False, True])
def test_grouped_kernel_f16_partial_sums_on_adversarial_v(hyperion, oracle, signed):
    """The same V through the grouped kernel (4 query heads over one KV head)."""
    wk = adversarial(16384, signed, 0.002, seed=5 + int(signed), n_bh=2)
    q = W.sign_pack(torch.randn(8, 128, generator=torch.Generator().manual_seed(9)))
    wk = W.Workload(**{**wk.__dict__, "q": q, "worklist": W.dense_worklist(8, 1, "cpu"), "heads": 8, "kv_group": 4})
    wk.worklist[:, 0] = 0
    g = wk.to(DEV)
    o = g.new_output()
    assert forward(hyperion, g, o, path="row") == 0
    ref, _, err, _ = oracle.forward_workload_c(wk)
    assert err == 0
    ok, mx, mn = oracle.tolerance_check(o.cpu().numpy(), ref, MAX_ABS, MEAN_ABS)
    assert ok and mx < 2e-3, (mx, mn)
