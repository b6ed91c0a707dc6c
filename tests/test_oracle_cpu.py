"""Oracle checks on the CPU: golden FP8 vectors of the reference, known-answer
cases of the sign-bit scoring and the clamped softmax, and agreement of the two
independent restatements (C and numpy) on seeded inputs."""
import json
import os
import struct

import numpy as np
import pytest
import torch

from hyperion_b200 import workloads as W

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "fp8_e4m3_reference.json")


def _golden_fp8():
    with open(GOLDEN) as f:
        bits = json.load(f)["f32_bits_hex"]
    return np.array([struct.unpack("<f", struct.pack("<I", int(b, 16)))[0] for b in bits], np.float32)


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_fp8_decode_c_oracle_matches_reference_golden(oracle):
    gold = _golden_fp8()
    mine = np.array([oracle.lib().oracle_fp8_e4m3_to_f32(c) for c in range(256)], np.float32)
    assert np.array_equal(_bits(mine), _bits(gold))


def test_fp8_decode_numpy_oracle_matches_reference_golden(oracle):
    assert np.array_equal(_bits(oracle.fp8_e4m3_decode_table()), _bits(_golden_fp8()))


def test_fp8_golden_matches_reference_build_here(oracle):
    ref = oracle.reference_fp8_lib()
    if ref is None:
        pytest.skip("oracle/_ref not built (reference checkout absent)")
    vals = np.array([ref.ref_fp8_e4m3_to_fp32(c) for c in range(256)], np.float32)
    assert np.array_equal(_bits(vals), _bits(_golden_fp8()))


def test_fp8_golden_vs_torch_e4m3fn():
    """The reference decodes 0x7F/0xFF as +-480; torch's e4m3fn calls them NaN.
    Every other code agrees, so the quantiser (which never emits 0x7F/0xFF) and the
    reference agree on all values it produces."""
    gold = _golden_fp8()
    tt = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    diff = [c for c in range(256) if not (gold[c] == tt[c] or (np.isnan(tt[c]) and c in (0x7F, 0xFF)))]
    assert diff == []
    assert gold[0x7F] == 480.0 and gold[0xFF] == -480.0
    q = W.fp8_quantize(torch.tensor([1e9, -1e9, 448.0, 500.0]), torch.tensor(1.0))
    assert q.tolist() == [0x7E, 0xFE, 0x7E, 0x7E]


def test_sign_score_known_answers(oracle):
    D = 128
    ones = np.full(4, 0xFFFFFFFF, np.uint32)
    zeros = np.zeros(4, np.uint32)
    L = oracle.lib()
    assert L.oracle_sign_score(ones.ctypes.data, ones.ctypes.data, D) == D
    assert L.oracle_sign_score(ones.ctypes.data, zeros.ctypes.data, D) == -D
    rng = np.random.default_rng(7)
    q = rng.integers(0, 2**32, 4, dtype=np.uint32)
    assert L.oracle_sign_score(q.ctypes.data, (~q).ctypes.data, D) == -D
    ks = rng.integers(0, 2**32, (64, 4), dtype=np.uint32)
    got = [L.oracle_sign_score(q.ctypes.data, np.ascontiguousarray(ks[i]).ctypes.data, D) for i in range(64)]
    assert np.array_equal(np.array(got), oracle.sign_scores_np(q, ks, D))


def test_sign_score_equals_pm1_dot_product():
    """D - 2*popcount(q^k) is the dot product of the +-1 sign vectors."""
    torch.manual_seed(3)
    x = torch.randn(5, 128)
    y = torch.randn(9, 128)
    qa = W.sign_pack(x).numpy().view(np.uint32)
    ka = W.sign_pack(y).numpy().view(np.uint32)
    from oracle.oracle import sign_scores_np

    pm_x = torch.where(x >= 0, 1.0, -1.0)
    pm_y = torch.where(y >= 0, 1.0, -1.0)
    dots = (pm_x @ pm_y.T).numpy().astype(np.int64)
    for i in range(5):
        assert np.array_equal(sign_scores_np(qa[i], ka, 128), dots[i])


def test_sign_pack_bit_order():
    x = -torch.ones(1, 128)
    x[0, 0] = 1.0  # dim 0 -> bit 0 of word 0
    x[0, 33] = 0.0  # >= 0 -> bit 1 of word 1
    x[0, 127] = 2.0  # bit 31 of word 3
    w = W.sign_pack(x).numpy().view(np.uint32)[0]
    assert w.tolist() == [1, 2, 0, 0x80000000]


def _one_case(B=1, H=2, S_q=16, S_kv=40, causal=False, scale_mode="head", seed=0):
    return W.make_dense("t", B, H, S_q, S_kv, causal=causal, scale_mode=scale_mode, o_dtype=torch.float32, seed=seed)


def test_single_key_row_returns_v(oracle):
    wk = _one_case(S_q=1, S_kv=1)
    o, written, err, _ = oracle.forward_workload_c(wk)
    lut = oracle.fp8_e4m3_decode_table()
    for bh in range(wk.n_bh):
        expect = lut[wk.v[bh].numpy()] * wk.v_scale[bh % wk.v_scale.numel()].item()
        assert np.allclose(o[bh], expect, rtol=1e-6, atol=0)
    assert err == 0 and written.all()


def test_fully_masked_row_is_zero(oracle):
    wk = _one_case()
    wk.ctx_lens[:] = 0
    o, written, err, _ = oracle.forward_workload_c(wk)
    assert written.all() and err == 0 and np.all(o == 0)


def test_causal_first_row_attends_key_zero_only(oracle):
    wk = _one_case(causal=True, S_q=8, S_kv=8)
    o, _, _, sc = oracle.forward_workload_c(wk, scores_ld=8)
    lut = oracle.fp8_e4m3_decode_table()
    vs = wk.v_scale[0].item()
    assert np.allclose(o[0], lut[wk.v[0].numpy()] * vs, rtol=1e-6)
    assert np.all(sc[0, 1:] == 0)  # keys 1.. never scored for q_idx 0


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("scale_mode", ["tensor", "head", "bh"])
def test_c_oracle_matches_numpy_oracle(oracle, causal, scale_mode):
    wk = _one_case(B=2, H=3, S_q=33, S_kv=70, causal=causal, scale_mode=scale_mode, seed=11)
    oc, wc, ec, _ = oracle.forward_workload_c(wk)
    on, wn = oracle.forward_workload_numpy(wk)
    assert ec == 0 and np.array_equal(wc, wn)
    ok, mx, mn = oracle.tolerance_check(oc, on, 1e-5, 1e-6)
    assert ok, (mx, mn)


def test_c_oracle_matches_numpy_paged_ragged(oracle):
    wk = W.make_paged("p", 3, 2, [1, 37, 300], page=16, seed=4)
    oc, wc, ec, _ = oracle.forward_workload_c(wk)
    on, wn = oracle.forward_workload_numpy(wk)
    assert ec == 0 and wc.all()
    assert oracle.tolerance_check(oc, on, 1e-5, 1e-6)[0]


def test_cpu_ref_config_c_vs_numpy(oracle):
    wk = W.make_config("cpu_ref", device="cpu", exact=True)
    assert wk.pairs() == 2097152
    oc, _, ec, _ = oracle.forward_workload_c(wk)
    on, _ = oracle.forward_workload_numpy(wk)
    assert ec == 0
    assert oracle.tolerance_check(oc, on, 1e-5, 1e-6)[0]


def test_online_clamp_equals_two_pass_when_clamp_engages(oracle):
    """With inv_sqrt_d = 1 the score range is +-128 and the -80 clamp engages; the
    dropped weights are below e^-80, far under any tolerance."""
    wk = _one_case(B=1, H=2, S_q=12, S_kv=200, seed=9)
    wk.inv_sqrt_d = 1.0
    oc, _, _, _ = oracle.forward_workload_c(wk)
    on, _ = oracle.forward_workload_numpy(wk)
    assert oracle.tolerance_check(oc, on, 1e-5, 1e-6)[0]


def test_error_flags_bad_block_bad_item_overflow_negative(oracle):
    wk = W.make_paged("p", 2, 2, [40, 40], page=16, seed=2)
    bt = wk.block_tables.clone()
    bt[0, 1] = 10**6  # outside the pool: keys 16..31 of bh 0 skipped
    wk.block_tables = bt
    wl = wk.worklist.clone()
    wl[3, 1] = 99  # bh out of range: row not written
    wk.worklist = wl
    o, written, err, _ = oracle.forward_workload_c(wk)
    assert err & oracle.ERR_BAD_BLOCK and err & oracle.ERR_BAD_ITEM
    assert not written[3] and written[:3].all()
    on, wn = oracle.forward_workload_numpy(wk)
    assert np.array_equal(written, wn)
    assert oracle.tolerance_check(o, on, 1e-5, 1e-6)[0]
    wk2 = _one_case()
    wk2.ctx_lens[0] = -5
    wk2.ctx_lens[1] = 10**6
    _, _, err2, _ = oracle.forward_workload_c(wk2)
    assert err2 & oracle.ERR_NEG_CTX and err2 & oracle.ERR_CTX_OVERFLOW


# ----------------------------------------------------------------------------- grouped-query attention
@pytest.mark.parametrize("scale_mode", ["tensor", "head", "bh"])
def test_gqa_oracle_equals_materialized_kv_copies(oracle, scale_mode):
    """kv_group restated by index expansion must give, bit for bit, what the plain
    problem gives when every query head holds its own copy of its KV head's rows."""
    B, H, Hkv, S_q, S_kv, D = 2, 6, 2, 3, 90, 128
    g = H // Hkv
    wk = W.make_dense("gqa", B, H, S_q, S_kv, D=D, causal=True, scale_mode=scale_mode, o_dtype=torch.float32,
                      seed=41, kv_heads=Hkv)
    assert wk.kv_group == g and wk.n_bh == B * H and wk.n_kv_bh == B * Hkv
    o_gqa, wr_gqa, err, _ = oracle.forward_workload_c(wk)
    assert err == 0 and wr_gqa.all()

    kv_of_bh = torch.arange(B * H) // g
    k = wk.k.view(B * Hkv, S_kv, -1)[kv_of_bh].reshape(B * H * S_kv, -1)
    v = wk.v.view(B * Hkv, S_kv, D)[kv_of_bh].reshape(B * H * S_kv, D)
    vs = wk.v_scale
    if scale_mode == "head":
        vs = vs.repeat_interleave(g)  # per query head
    elif scale_mode == "bh":
        vs = vs[kv_of_bh]
    ctx = wk.ctx_lens[kv_of_bh]
    o_copy, wr_copy, err2, _ = oracle.forward_c(wk.worklist, wk.q, k, v, vs, ctx, None, S_q, D, S_kv, 1,
                                                wk.inv_sqrt_d, True)
    assert err2 == 0 and wr_copy.all()
    assert np.array_equal(o_gqa, o_copy)


def test_gqa_oracle_paged_c_vs_numpy(oracle):
    wk = W.make_paged("gqa_p", 3, 8, [40, 333, 1000], page=16, seed=42, o_dtype=torch.float32, kv_heads=2)
    assert wk.kv_group == 4 and wk.block_tables.shape[0] == 6
    o_c, wr, err, _ = oracle.forward_workload_c(wk)
    o_np, wr_np = oracle.forward_workload_numpy(wk)
    assert err == 0 and wr.all() and wr_np.all()
    assert np.abs(o_c - o_np).max() < 1e-5


def test_gqa_expansion_of_index_arrays(oracle):
    ctx = np.array([5, 7], np.int32)
    bt = np.array([[3, 4], [8, 9]], np.int32)
    ctx_q, bt_q, vs_q = oracle.expand_kv_group(ctx, bt, np.array([0.5, 0.25], np.float32), 3, 2, 1000)
    assert ctx_q.tolist() == [5, 5, 5, 7, 7, 7]
    assert bt_q.tolist() == [[3, 4]] * 3 + [[8, 9]] * 3
    assert vs_q.tolist() == [0.5] * 3 + [0.25] * 3
    # The contiguous layout becomes the explicit table kv * num_blocks + j.
    _, bt_c, vs_t = oracle.expand_kv_group(ctx, None, np.array([2.0], np.float32), 2, 3, 1000)
    assert bt_c.tolist() == [[0, 1, 2], [0, 1, 2], [3, 4, 5], [3, 4, 5]]
    assert vs_t.tolist() == [2.0]
