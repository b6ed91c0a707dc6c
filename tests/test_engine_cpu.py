"""The reference's callers against the drop-in, on the CPU.

tests/golden/engine_batches.json records, from the reference's own code, how it
calls its module object `hyperion` (every call site's positional arguments and
keywords) and what its scheduler and worklist builder produce for a seeded set of
requests (tests/golden/make_engine_batches.py).  These tests check that the
drop-in's entry points accept those calls unchanged, that the engine glue
rebuilds the reference's work-item fields, and -- where the reference checkout is
available (HYPERION_REFERENCE_DIR) -- that re-recording gives the committed file.
"""
import importlib.util
import inspect
import json
import os
import types

import numpy as np
import pytest
import torch

from hyperion_b200 import engine as E
from hyperion_b200 import glue

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "engine_batches.json")


def _fixture():
    with open(FIXTURE) as f:
        return json.load(f)


def _recorder():
    spec = importlib.util.spec_from_file_location("make_engine_batches",
                                                  os.path.join(HERE, "golden", "make_engine_batches.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_call_sites_bind_to_the_drop_in(hyperion):
    """Every hyperion.<name>(...) call in the reference binds to the drop-in function
    of the same name: same positional count, same keywords (grid / block / shared)."""
    sites = _fixture()["call_sites"]
    assert set(sites) == {"hyperion_apex_kernel", "hyperion_reset_counter"}
    for name, calls in sites.items():
        fn = getattr(hyperion, name)
        sig = inspect.signature(fn)
        for c in calls:
            bound = sig.bind(*[object()] * len(c["positional"]), **{k: None for k in c["keywords"]})
            assert len(bound.args) == len(c["positional"])
    kernel = sites["hyperion_apex_kernel"][0]
    assert len(kernel["positional"]) == 18 and kernel["keywords"] == ["grid", "block", "shared"]
    params = list(inspect.signature(hyperion.hyperion_apex_kernel).parameters)[:18]
    # argument meaning by position, as the reference's call site passes them (:1099-1114)
    assert params[0] == "worklist" and params[10] == "O" and params[17] == "causal"
    assert kernel["positional"][1] == "worklist.size(0)" and kernel["positional"][-1] == "True"


def test_glue_rebuilds_the_reference_work_item_fields():
    """For every recorded batch, glue.build_worklist with the scheduler's signature hash
    and engine.prefetch_hint gives the reference's (q_idx, kv_signature, prefetch_hint)
    for each request, once per query head, with the real (batch, head) row in field 1
    where the reference writes 0 (:926)."""
    fx = _fixture()
    reqs = {r["req_id"]: r for r in fx["requests"]}
    H = fx["model"]["num_heads"]
    for b in fx["batches"]:
        ref_wl = np.array(b["worklist"], dtype=np.int64)
        q_lens = [min(b["seq_q"], reqs[r]["seq_len"]) for r in b["req_ids"]]
        hints = [E.prefetch_hint(reqs[r]["block_table"], b["prefetch_blocks"]) for r in b["req_ids"]]
        wl = glue.build_worklist(torch.tensor(q_lens, dtype=torch.int32), H, kv_signatures=b["kv_signature_hash"],
                                 prefetch_hints=torch.tensor(hints, dtype=torch.int32)).numpy().astype(np.int64)
        assert wl.shape[0] == H * ref_wl.shape[0]
        pos = 0
        for i, n in enumerate(q_lens):
            ref_items = ref_wl[pos:pos + n]
            pos += n
            for h in range(H):
                mine = wl[wl[:, 1] == i * H + h]
                assert np.array_equal(mine[:, [0, 2, 3]], ref_items[:, [0, 2, 3]])
        assert (ref_wl[:, 1] == 0).all()


def test_launcher_splits_prompts_from_decode_steps():
    """Prompts run causal over their own keys, decode steps unmasked, in separate calls;
    a prompt whose ctx_len differs from its query rows is refused."""
    calls = []
    fake = types.SimpleNamespace(hyperion_reset_counter=lambda **k: calls.append(("reset", k)),
                                 hyperion_apex_kernel=lambda *a, **k: calls.append(("fwd", a, k)))
    pool = E.KVPool.allocate(2, 8, 16, 128, "cpu")
    launcher = E.BatchLauncher(fake, pool, num_heads=4)
    mk = lambda rid, L, ctx: types.SimpleNamespace(req_id=rid, kv_signature=(1, 2), block_table=[0, 1, 2], ctx_len=ctx)
    batch = [mk("a", 20, 20), mk("b", 1, 40), mk("c", 5, 5)]
    q = {"a": torch.zeros(4, 20, 4, dtype=torch.int32), "b": torch.zeros(4, 1, 4, dtype=torch.int32),
         "c": torch.zeros(4, 5, 4, dtype=torch.int32)}
    out = launcher.launch(batch, [], q)
    assert [lb.causal for lb in out] == [True, False]
    assert [sorted(lb.rows) for lb in out] == [["a", "c"], ["b"]]
    fwd = [c for c in calls if c[0] == "fwd"]
    assert [c[1][17] for c in fwd] == [True, False] and fwd[0][1][11] == 20 and fwd[1][1][11] == 1
    assert all(c[2]["kv_group"] == 2 for c in fwd)
    # per-KV-head rows: request b's KV head 1 reads pages 1*8 + [0, 1, 2]
    assert out[1].block_tables[1].tolist() == [8, 9, 10] and out[1].ctx_lens.tolist() == [40, 40]
    with pytest.raises(ValueError):
        launcher.launch([mk("d", 5, 9)], [], {"d": torch.zeros(4, 5, 4, dtype=torch.int32)})


def test_rerecording_matches_the_committed_batches():
    ref_dir = os.environ.get("HYPERION_REFERENCE_DIR")
    if not ref_dir or not os.path.exists(os.path.join(ref_dir, "hyperion_fa3_production_final.py")):
        pytest.skip("reference checkout not available (HYPERION_REFERENCE_DIR)")
    rec_mod = _recorder()
    rec = rec_mod.record(rec_mod.load_reference(ref_dir))
    rec["call_sites"] = rec_mod.call_sites(os.path.join(ref_dir, rec_mod.REF_MODULE))
    fx = _fixture()
    for key in ("model", "requests", "launch_config", "call_sites"):
        assert rec[key] == fx[key], key
    assert [b["req_ids"] for b in rec["batches"]] == [b["req_ids"] for b in fx["batches"]]
    assert [b["worklist"] for b in rec["batches"]] == [b["worklist"] for b in fx["batches"]]
