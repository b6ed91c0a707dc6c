"""CPU checks of the measurement logic in bench.py: the algorithmic work the roofline
divides by, the pair counts, and the row sampler of the CPU baseline."""
import numpy as np
import pytest
import torch

import bench
from hyperion_b200 import workloads as W

PEAKS = {"hbm_gbs": 6546.2, "bf16_tflops": 1663.3}


def test_decode_roofline_bytes_are_k_and_v_per_key_plus_q_and_o():
    wk = W.make_dense("d", 2, 4, 1, 300, o_dtype=torch.bfloat16)
    r = bench.roofline_numbers(wk, wk.pairs(), 1.0, PEAKS)
    n = wk.total_work
    assert wk.pairs() == 8 * 300
    assert r["bound"] == "hbm"
    assert r["algorithmic_bytes_per_launch"] == 8 * 300 * (16 + 128) + n * 16 + n * 128 * 2


def test_grouped_query_decode_counts_each_kv_key_once():
    wk = W.make_dense("g", 2, 8, 1, 100, kv_heads=2, o_dtype=torch.float32)
    assert wk.kv_group == 4 and wk.pairs() == 16 * 100 and wk.kv_keys() == 4 * 100
    r = bench.roofline_numbers(wk, wk.pairs(), 1.0, PEAKS)
    assert r["algorithmic_bytes_per_launch"] == 4 * 100 * 144 + 16 * 16 + 16 * 128 * 4


def test_prefill_roofline_flops_and_causal_pairs():
    wk = W.make_dense("p", 1, 2, 64, 64, causal=True, o_dtype=torch.float32)
    assert wk.pairs() == 2 * 64 * 65 // 2
    r = bench.roofline_numbers(wk, wk.pairs(), 1.0, PEAKS)
    assert r["bound"] == "tensor"
    assert r["algorithmic_flops_per_launch"] == 4.0 * 128 * wk.pairs()


@pytest.mark.parametrize("kv_heads", [None, 2])
def test_cpu_baseline_sample_reproduces_its_rows(oracle, kv_heads):
    """The CPU baseline times the oracle on whole (batch, head) rows gathered into a
    contiguous workload; those rows must give what the full workload gives."""
    wk = W.make_paged("s", 2, 4, [40, 170], page=16, seed=71, o_dtype=torch.float32, kv_heads=kv_heads)
    full, _, _, _ = oracle.forward_workload_c(wk)
    rows = [3, 0, 6]
    sub = bench._subset_rows(wk, rows)
    got, _, err, _ = oracle.forward_workload_c(sub)
    assert err == 0
    assert np.array_equal(got, full[rows])


def test_reference_arm_inputs_load_no_device_code_of_this_repository():
    """The reference arm builds its inputs with the workload generators but must not
    map libhyperion_b200.so: it times the CPU restatement alone."""
    import subprocess
    import sys

    code = ("import bench, torch; bench.host_only_package(); "
            "wk, desc, sc = bench.build_workload('cpu_ref', 0, 1, torch.device('cpu')); "
            "print(wk.pairs(), sorted(bench.workload_config(wk, desc, 1, sc))); "
            "print('MAPPED' if 'libhyperion_b200' in open('/proc/self/maps').read() else 'CLEAN')")
    res = subprocess.run([sys.executable, "-c", code], cwd=bench.REPO, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    assert res.stdout.strip().splitlines()[-1] == "CLEAN"
    assert res.stdout.startswith(str(8 * 512 * 512))


def test_config_is_the_same_for_a_workload_on_either_device():
    """Both arms print workload_config(...) of the same workload; it must not depend on
    where the tensors live or on anything a kernel launch reports."""
    wk = W.make_dense("c", 2, 4, 64, 64, causal=True, o_dtype=torch.bfloat16)
    a = bench.workload_config(wk, "desc", 2, "weak")
    b = bench.workload_config(wk.to("cpu"), "desc", 2, "weak")
    assert a == b
    assert set(a) == {"workload", "global_batch", "heads", "seq_len", "head_dim", "causal", "parallelism", "l2"}
    assert a["global_batch"] == 4 and a["seq_len"] == 64
