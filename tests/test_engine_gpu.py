"""The reference's own engine decisions, replayed through the drop-in forward.

tests/golden/engine_batches.json holds what the reference's scheduler and worklist
code produced for a seeded set of requests (KVAwareSchedulerV2.get_next_batch,
PersistentKernelManager.prepare_worklist and get_launch_config,
hyperion_fa3_production_final.py:793-823, :907-929; recorded by
tests/golden/make_engine_batches.py).  Here every recorded batch goes through
hyperion_b200.engine.BatchLauncher with real Q and O, per-KV-head block tables
(32 query heads over 8 KV heads, as the engine is configured) and the recorded
launch hints, and each request's output is checked against the oracle.
"""
import json
import os
import types

import numpy as np
import pytest
import torch

from hyperion_b200 import engine as E
from hyperion_b200 import workloads as W

pytestmark = pytest.mark.gpu

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "engine_batches.json")


def _fixture():
    with open(FIXTURE) as f:
        return json.load(f)


def _pool(m, dev, seed=21):
    pool = E.KVPool.allocate(m["num_kv_heads"], m["num_blocks"], m["block_size"], m["head_dim"], dev)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    pool.k.copy_(torch.randint(-2**31, 2**31 - 1, pool.k.shape, dtype=torch.int32, generator=g, device=dev))
    v = torch.randn(pool.v.shape, generator=g, device=dev).view(m["num_kv_heads"], -1, m["head_dim"])
    scale = v.abs().amax(dim=(1, 2)) / 448.0
    pool.v.copy_(W.fp8_quantize(v, scale.view(-1, 1, 1)).view(pool.v.shape))
    pool.v_scale.copy_(scale)
    return pool


def _requests(fx):
    by_id = {}
    for r in fx["requests"]:
        by_id[r["req_id"]] = r
    return by_id


def test_recorded_batches_run_through_the_drop_in(hyperion, oracle):
    fx = _fixture()
    m = fx["model"]
    dev = torch.device("cuda", 0)
    pool = _pool(m, dev)
    lc = fx["launch_config"]
    launcher = E.BatchLauncher(hyperion, pool, m["num_heads"], o_dtype=torch.float32, grid=tuple(lc["grid"]),
                               block=tuple(lc["block"]), shared=lc["shared"])
    reqs = _requests(fx)
    g = torch.Generator().manual_seed(3)
    assert len(fx["batches"]) >= 2
    kinds = set()
    for bi, b in enumerate(fx["batches"]):
        batch = []
        q_words = {}
        for rid, sig in zip(b["req_ids"], b["kv_signature_hash"]):
            r = reqs[rid]
            # the scheduler's request object: the fields the batch step reads
            batch.append(types.SimpleNamespace(req_id=rid, kv_signature=sig, block_table=r["block_table"],
                                               ctx_len=r["ctx_len"]))
            q_words[rid] = W.sign_pack(torch.randn(m["num_heads"], r["seq_len"], m["head_dim"], generator=g))
        hyperion.read_device_errors(dev, clear=True)
        launched = launcher.launch(batch, b["prefetch_blocks"], q_words)
        assert hyperion.read_device_errors(dev, clear=True) == 0
        # Work items: the reference's (q_idx, kv_signature hash, prefetch hint) of every
        # request, once per query head, with the real (batch, head) row.
        ref_wl = np.array(b["worklist"], dtype=np.int64)
        ref_items, pos = {}, 0
        for rid in b["req_ids"]:
            n = min(b["seq_q"], reqs[rid]["seq_len"])
            ref_items[rid] = ref_wl[pos:pos + n]
            pos += n
        assert pos == len(ref_wl) and (ref_wl[:, 1] == 0).all()  # the reference writes bh = 0 (:926)
        for lb in launched:
            kinds.add(lb.causal)
            wl = lb.worklist.cpu().numpy().astype(np.int64)
            for rid, (row0, L) in lb.rows.items():
                for h in range(m["num_heads"]):
                    mine = wl[wl[:, 1] == row0 + h]
                    assert np.array_equal(mine[:, [0, 2, 3]], ref_items[rid][:, [0, 2, 3]]), (bi, rid, h)
            wk = W.Workload(name=f"engine_b{bi}", worklist=lb.worklist.cpu(), q=lb.q.cpu(), k=pool.k.cpu(),
                            v=pool.v.cpu(), v_scale=pool.v_scale.cpu(), ctx_lens=lb.ctx_lens.cpu(),
                            block_tables=lb.block_tables.cpu(), seq_q=lb.seq_q, head_dim=m["head_dim"],
                            block_size=m["block_size"], num_blocks=lb.block_tables.shape[1], causal=lb.causal,
                            o_dtype=torch.float32, batch=len(lb.rows), heads=m["num_heads"],
                            kv_group=m["num_heads"] // m["num_kv_heads"])
            ref, written, err, _ = oracle.forward_workload_c(wk)
            assert err == 0 and written.all()
            rows = (wl[:, 1] * lb.seq_q + wl[:, 0]).tolist()
            ok, mx, mn = oracle.tolerance_check(lb.o.cpu().numpy()[rows], ref[rows], 2e-2, 2e-3)
            assert ok, (bi, lb.causal, mx, mn)
    # Both kinds of call ran: prompts (causal, tile path for 64+ rows) and decode steps.
    assert kinds == {True, False}
