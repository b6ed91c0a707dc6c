"""GPU tests of the cache writer (hyperion_kv_cache_write): bit-exact against the
CPU quantisers (sign bits of K, e4m3 codes of clamp(V / scale, +-448) by torch), at
the slots the forward reads, with untouched slots left alone."""
import numpy as np
import pytest
import torch

from hyperion_b200 import workloads as W

pytestmark = pytest.mark.gpu

SENTINEL = 0xA5


def _paged_layout(lens, H, page, seed):
    """Block tables of a shared pool with pages in a random order (the paged-decode layout)."""
    pages_b = [(L + page - 1) // page for L in lens]
    total = sum(pages_b)
    perm = torch.randperm(total, generator=torch.Generator().manual_seed(seed))
    nb = max(pages_b)
    bt = torch.full((len(lens) * H, nb), -1, dtype=torch.int32)
    off = 0
    for b, npg in enumerate(pages_b):
        for h in range(H):
            bt[b * H + h, :npg] = (perm[off:off + npg] * H + h).to(torch.int32)
        off += npg
    return bt, nb, total * H * page


def _tokens(lens):
    seq = torch.cat([torch.full((L,), b, dtype=torch.int32) for b, L in enumerate(lens)])
    pos = torch.cat([torch.arange(L, dtype=torch.int32) for L in lens])
    return seq, pos


def _crafted(x):
    """Overwrite a few rows with edge values: +-0, ties between e4m3 neighbours, clamp, tiny."""
    special = torch.tensor([0.0, -0.0, 448.0, 500.0, -1000.0, 1.0625, -1.0625, 0.015625 * 1.5, 1e-6, -1e-6,
                            240.0, 232.0, 3.0, -3.25], dtype=torch.float32)
    flat = x.view(-1)
    flat[: special.numel()] = special
    return x


def _reference(k, v, seq, pos, bt, nb, page, scale, H, D, pool_rows):
    """Expected K/V pools on the CPU (sentinel where nothing is written)."""
    kc = torch.full((pool_rows, D // 32), 0, dtype=torch.int32)
    kc.view(torch.uint8).fill_(SENTINEL)
    vc = torch.full((pool_rows, D), SENTINEL, dtype=torch.uint8)
    words = W.sign_pack(k.float())  # [n, H, D/32]
    codes = W.fp8_quantize(v.float(), scale.view(1, -1, 1) if scale.numel() == H else scale.view(1, 1, 1))
    for i in range(seq.numel()):
        b, t = int(seq[i]), int(pos[i])
        for h in range(H):
            bh = b * H + h
            pid = int(bt[bh, t // page]) if bt is not None else bh * nb + t // page
            slot = pid * page + t % page
            kc[slot] = words[i, h]
            vc[slot] = codes[i, h]
    return kc, vc


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_kv_write_paged_matches_cpu_quantisers(hyperion, dtype):
    torch.manual_seed(7)
    H, D, page = 4, 128, 16
    lens = [5, 33, 70]
    bt, nb, pool_rows = _paged_layout(lens, H, page, seed=3)
    seq, pos = _tokens(lens)
    n = seq.numel()
    k = _crafted(torch.randn(n, H, D)).to(dtype)
    v = _crafted(torch.randn(n, H, D) * 3).to(dtype)
    scale = (v.float().abs().amax(dim=(0, 2)) / 448.0).clamp_min(1e-3)  # per head
    dev = torch.device("cuda", 0)
    kc = torch.zeros(pool_rows, D // 32, dtype=torch.int32, device=dev)
    kc.view(torch.uint8).fill_(SENTINEL)
    vc = torch.full((pool_rows, D), SENTINEL, dtype=torch.uint8, device=dev)
    hyperion.read_device_errors(dev, clear=True)
    hyperion.kv_cache_write(k.to(dev), v.to(dev), seq.to(dev), pos.to(dev), bt.to(dev), page, nb, scale.to(dev), kc, vc)
    assert hyperion.read_device_errors(dev, clear=True) == 0
    ek, ev = _reference(k, v, seq, pos, bt, nb, page, scale, H, D, pool_rows)
    assert torch.equal(kc.cpu(), ek)
    assert torch.equal(vc.cpu(), ev)


def test_kv_write_contiguous_d256(hyperion):
    torch.manual_seed(8)
    B, H, D, S = 2, 3, 256, 40
    lens = [S, 17]
    seq, pos = _tokens(lens)
    n = seq.numel()
    k = torch.randn(n, H, D)
    v = torch.randn(n, H, D)
    scale = torch.tensor([0.01], dtype=torch.float32)
    pool_rows = B * H * S
    dev = torch.device("cuda", 0)
    kc = torch.zeros(pool_rows, D // 32, dtype=torch.int32, device=dev)
    kc.view(torch.uint8).fill_(SENTINEL)
    vc = torch.full((pool_rows, D), SENTINEL, dtype=torch.uint8, device=dev)
    hyperion.kv_cache_write(k.to(dev), v.to(dev), seq.to(dev), pos.to(dev), None, S, 1, scale.to(dev), kc, vc)
    assert hyperion.read_device_errors(dev, clear=True) == 0
    ek, ev = _reference(k, v, seq, pos, None, 1, S, scale, H, D, pool_rows)
    assert torch.equal(kc.cpu(), ek)
    assert torch.equal(vc.cpu(), ev)


def test_kv_write_flags_rows_outside_the_pool(hyperion):
    H, D, page = 2, 128, 16
    dev = torch.device("cuda", 0)
    bt = torch.tensor([[0, 5], [1, -1]], dtype=torch.int32)  # seq 0: head 0 -> pages 0, 5; head 1 -> page 1, bad
    seq = torch.tensor([0, 0, 0], dtype=torch.int32)
    pos = torch.tensor([3, 20, 40], dtype=torch.int32)  # 40 is beyond num_blocks * page = 32
    k = torch.randn(3, H, D)
    v = torch.randn(3, H, D)
    pool_rows = 2 * page  # pages 0 and 1 only: page 5 is outside
    kc = torch.zeros(pool_rows, D // 32, dtype=torch.int32, device=dev)
    vc = torch.zeros(pool_rows, D, dtype=torch.uint8, device=dev)
    hyperion.read_device_errors(dev, clear=True)
    hyperion.kv_cache_write(k.to(dev), v.to(dev), seq.to(dev), pos.to(dev), bt.to(dev), page, 2,
                            torch.ones(1, device=dev), kc, vc)
    err = hyperion.read_device_errors(dev, clear=True)
    assert err & hyperion.DEVERR_BAD_ITEM and err & hyperion.DEVERR_BAD_BLOCK
    words = W.sign_pack(k)
    assert torch.equal(kc[3].cpu(), words[0, 0])          # token 0, head 0 -> page 0, slot 3
    assert torch.equal(kc[page + 3].cpu(), words[0, 1])   # token 0, head 1 -> page 1, slot 16 + 3
    assert int(kc[4:page].abs().sum()) == 0 and int(kc[page + 4:].abs().sum()) == 0


def test_written_cache_feeds_the_forward(hyperion, oracle):
    """Round trip: quantise with the writer, then run the forward on that cache; the
    oracle on the same cache bytes must agree within the parity tolerance."""
    torch.manual_seed(9)
    H, D, page = 4, 128, 16
    lens = [100, 257, 31]
    bt, nb, pool_rows = _paged_layout(lens, H, page, seed=5)
    seq, pos = _tokens(lens)
    n = seq.numel()
    dev = torch.device("cuda", 0)
    k = torch.randn(n, H, D, device=dev)
    v = torch.randn(n, H, D, device=dev)
    scale = (v.abs().amax(dim=(0, 2)) / 448.0).float()
    kc = torch.zeros(pool_rows, D // 32, dtype=torch.int32, device=dev)
    vc = torch.zeros(pool_rows, D, dtype=torch.uint8, device=dev)
    hyperion.kv_cache_write(k, v, seq.to(dev), pos.to(dev), bt.to(dev), page, nb, scale, kc, vc)
    n_bh = len(lens) * H
    q = W.sign_pack(torch.randn(n_bh, D, device=dev))
    ctx = torch.tensor([L for L in lens for _ in range(H)], dtype=torch.int32, device=dev)
    wl = W.dense_worklist(n_bh, 1, dev)
    wl[:, 0] = 0
    wk = W.Workload(name="rt", worklist=wl, q=q, k=kc, v=vc, v_scale=scale, ctx_lens=ctx, block_tables=bt.to(dev),
                    seq_q=1, head_dim=D, block_size=page, num_blocks=nb, causal=False, o_dtype=torch.float32,
                    batch=len(lens), heads=H)
    o = torch.zeros(n_bh, D, dtype=torch.float32, device=dev)
    hyperion.read_device_errors(dev, clear=True)
    hyperion.hyperion_apex_kernel(wk.worklist, wk.total_work, wk.q, None, wk.k, None, wk.v, wk.v_scale, wk.ctx_lens,
                                  wk.block_tables, o, 1, D, D // 8, page, nb, wk.inv_sqrt_d, False)
    assert hyperion.read_device_errors(dev, clear=True) == 0
    ref, _, err, _ = oracle.forward_workload_c(wk.to("cpu"))
    assert err == 0
    ok, mx, mn = oracle.tolerance_check(o.cpu().numpy(), ref, 2e-2, 2e-3)
    assert ok, (mx, mn)


def test_per_slot_scale_is_the_one_the_forward_decodes_with(hyperion, oracle):
    """The reference keeps one V scale per cache slot (V_scale[slot]).  The writer must
    quantise each row with the scale of the slot it lands in, which is the one the
    forward decodes it with; the round trip then matches the oracle and the codes match
    the CPU quantiser with per-slot scales bit for bit."""
    torch.manual_seed(13)
    H, D, page = 2, 128, 16
    lens = [70, 33]
    bt, nb, pool_rows = _paged_layout(lens, H, page, seed=8)
    seq, pos = _tokens(lens)
    n = seq.numel()
    dev = torch.device("cuda", 0)
    k = torch.randn(n, H, D)
    v = torch.randn(n, H, D) * torch.rand(n, H, 1) * 4
    slot_scale = (torch.rand(pool_rows) * 0.02 + 0.002).float()
    kc = torch.zeros(pool_rows, D // 32, dtype=torch.int32, device=dev)
    vc = torch.full((pool_rows, D), SENTINEL, dtype=torch.uint8, device=dev)
    hyperion.read_device_errors(dev, clear=True)
    hyperion.kv_cache_write(k.to(dev), v.to(dev), seq.to(dev), pos.to(dev), bt.to(dev), page, nb,
                            slot_scale.to(dev), kc, vc)
    assert hyperion.read_device_errors(dev, clear=True) == 0
    got = vc.cpu()
    for i in range(n):
        b, t = int(seq[i]), int(pos[i])
        for h in range(H):
            slot = int(bt[b * H + h, t // page]) * page + t % page
            assert torch.equal(got[slot], W.fp8_quantize(v[i, h], slot_scale[slot]))
    n_bh = len(lens) * H
    q = W.sign_pack(torch.randn(n_bh, D)).to(dev)
    ctx = torch.tensor([L for L in lens for _ in range(H)], dtype=torch.int32, device=dev)
    wl = W.dense_worklist(n_bh, 1, dev)
    wl[:, 0] = 0
    wk = W.Workload(name="slot", worklist=wl, q=q, k=kc, v=vc, v_scale=slot_scale.to(dev), ctx_lens=ctx,
                    block_tables=bt.to(dev), seq_q=1, head_dim=D, block_size=page, num_blocks=nb, causal=False,
                    o_dtype=torch.float32, batch=len(lens), heads=H)
    o = torch.zeros(n_bh, D, dtype=torch.float32, device=dev)
    hyperion.hyperion_apex_kernel(wk.worklist, wk.total_work, wk.q, None, wk.k, None, wk.v, wk.v_scale, wk.ctx_lens,
                                  wk.block_tables, o, 1, D, D // 8, page, nb, wk.inv_sqrt_d, False)
    assert hyperion.read_device_errors(dev, clear=True) == 0
    ref, _, err, _ = oracle.forward_workload_c(wk.to("cpu"))
    assert err == 0
    ok, mx, mn = oracle.tolerance_check(o.cpu().numpy(), ref, 2e-2, 2e-3)
    assert ok, (mx, mn)
    # The values the forward saw are the clamped V to within e4m3 rounding.
    dec = torch.tensor(oracle.fp8_e4m3_decode_table())[got.long()] * slot_scale[:, None]
    slot0 = int(bt[0, 0]) * page
    s0 = slot_scale[slot0]
    assert torch.allclose(dec[slot0], (v[0, 0] / s0).clamp(-448, 448) * s0, rtol=0.07, atol=s0.item())
