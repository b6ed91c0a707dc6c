"""Records what the reference's own engine code does with a seeded set of requests.

    HYPERION_REFERENCE_DIR=<reference checkout> python tests/golden/make_engine_batches.py

Writes tests/golden/engine_batches.json: the batches KVAwareSchedulerV2.get_next_batch
returns (hyperion_fa3_production_final.py:793-823) for requests submitted with
submit (:774-784), the work items PersistentKernelManager.prepare_worklist builds
for each batch (:914-929), and get_launch_config's triple (:907-912).  The
reference module is imported unmodified, with torch's load_inline replaced by a
function that raises, so its CUDA source is never compiled (it does not build
anyway; the module then runs with HYPERION_LOADED = False).  prepare_worklist puts
its tensor on 'cuda'; here it is made on the host.

The GPU test (tests/test_engine_gpu.py) replays these batches through the drop-in
forward with real Q, O and per-KV-head tables; the CPU test
(tests/test_engine_cpu.py) re-runs this recording and compares.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "engine_batches.json")
REF_MODULE = "hyperion_fa3_production_final.py"

# The engine's model shape (hyperion_fa3_production_final.py:852-856).
NUM_HEADS, NUM_KV_HEADS, HEAD_DIM, BLOCK_SIZE, NUM_BLOCKS = 32, 8, 128, 64, 1024
MAX_BATCH = 8
SM_COUNT = 148


def load_reference(ref_dir: str):
    """The reference module, imported without compiling its kernel."""
    import torch.utils.cpp_extension as cpp_ext

    def _no_build(*a, **k):
        raise RuntimeError("kernel build disabled while recording the engine's host code")

    saved = cpp_ext.load_inline
    cpp_ext.load_inline = _no_build
    try:
        spec = importlib.util.spec_from_file_location("hyperion_reference_engine", os.path.join(ref_dir, REF_MODULE))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        cpp_ext.load_inline = saved
    return mod


class _HostTorch:
    """torch with tensor()/zeros() made on the host: prepare_worklist asks for 'cuda'."""

    def __getattr__(self, name):
        return getattr(torch, name)

    @staticmethod
    def tensor(data, dtype=None, device=None):
        return torch.tensor(data, dtype=dtype)

    @staticmethod
    def zeros(*size, dtype=None, device=None):
        return torch.zeros(*size, dtype=dtype)


def seeded_requests(seed: int = 11):
    """12 requests: 7 decode steps (1 query row, 64 .. 3000 cached tokens) and 5 prompts
    (48 .. 300 rows, ctx_len = prompt length); two pairs share their first pages (a
    shared prefix, so the scheduler's locality queues hold more than one request)."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(NUM_BLOCKS, generator=g).tolist()
    reqs = []
    spec = [(1, 300), (130, 130), (1, 2900), (1, 64), (48, 48), (1, 1500), (300, 300), (1, 700), (1, 2200),
            (70, 70), (1, 1000), (200, 200)]
    shared = {5: 2, 8: 2, 10: 0}  # request i reuses the first pages of request j (same prefix)
    for i, (seq, ctx) in enumerate(spec):
        n_pages = (ctx + BLOCK_SIZE - 1) // BLOCK_SIZE
        pages = [perm.pop() for _ in range(n_pages)]
        if i in shared:
            j = shared[i]
            k = min(8, len(reqs[j]["block_table"]), n_pages)
            pages[:k] = reqs[j]["block_table"][:k]
        reqs.append({"req_id": f"req{i:02d}", "priority": int(torch.randint(0, 4, (1,), generator=g)),
                     "arrival_offset_s": round(0.25 * (12 - i), 3), "seq_len": seq, "ctx_len": ctx,
                     "block_table": pages, "kv_head": 0})
    return reqs


def call_sites(ref_file: str) -> dict:
    """How the reference calls its module object `hyperion`: for every call
    hyperion.<name>(...), the source of each positional argument, the keyword names
    and the line (read from the source with ast; nothing is executed)."""
    import ast

    tree = ast.parse(open(ref_file, encoding="utf-8").read(), filename=ref_file)
    out = {}
    for node in ast.walk(tree):
        if (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
                and isinstance(node.func.value, ast.Name) and node.func.value.id == "hyperion"):
            out.setdefault(node.func.attr, []).append({
                "line": node.lineno, "positional": [ast.unparse(a) for a in node.args],
                "keywords": [k.arg for k in node.keywords]})
    return out


def record(ref) -> dict:
    """Runs the reference's scheduler and worklist code on seeded_requests()."""
    sched = ref.KVAwareSchedulerV2(max_batch_size=MAX_BATCH)
    now = time.time()
    reqs = seeded_requests()
    for r in reqs:
        pr = ref.PrioritizedRequest(priority=r["priority"], arrival_time=now - r["arrival_offset_s"],
                                    req_id=r["req_id"], input_ids=torch.zeros(1, r["seq_len"], dtype=torch.long),
                                    max_tokens=1, kv_head=r["kv_head"], ctx_len=r["ctx_len"],
                                    block_table=list(r["block_table"]))
        sched.submit(pr)
    mgr = ref.PersistentKernelManager(sm_count=SM_COUNT)
    cfg = ref.HyperionApexConfig(num_heads=NUM_HEADS, num_kv_heads=NUM_KV_HEADS, head_dim=HEAD_DIM,
                                 block_size=BLOCK_SIZE, num_blocks=NUM_BLOCKS, max_batch_size=MAX_BATCH)
    grid, block, smem = mgr.get_launch_config(cfg)
    batches = []
    saved_torch = ref.torch
    ref.torch = _HostTorch()
    try:
        for _ in range(8):
            time.sleep(0.02)  # past the scheduler's clustering window
            batch, prefetch = sched.get_next_batch()
            if not batch:
                if not sched.locality_queues:
                    break
                continue
            seq_q = max(r.input_ids.size(1) for r in batch)
            wl = mgr.prepare_worklist(batch, seq_q, prefetch)
            batches.append({"req_ids": [r.req_id for r in batch], "prefetch_blocks": list(prefetch),
                            "kv_signature_hash": [hash(r.kv_signature) & 0x7FFFFFFF for r in batch],
                            "seq_q": seq_q, "worklist": wl.tolist()})
            for r in batch:  # as the batch loop does after the launch (:1116-1117)
                sched.complete(r.req_id, tokens_generated=1)
    finally:
        ref.torch = saved_torch
    return {
        "generator": "tests/golden/make_engine_batches.py",
        "source": "hyperion_fa3_production_final.py: KVAwareSchedulerV2.submit/get_next_batch (:774-823), "
                  "PersistentKernelManager.prepare_worklist/get_launch_config (:907-929)",
        "model": {"num_heads": NUM_HEADS, "num_kv_heads": NUM_KV_HEADS, "head_dim": HEAD_DIM,
                  "block_size": BLOCK_SIZE, "num_blocks": NUM_BLOCKS, "max_batch_size": MAX_BATCH},
        "requests": reqs,
        "launch_config": {"grid": list(grid), "block": list(block), "shared": int(smem)},
        "batches": batches,
    }


def main():
    ref_dir = os.environ.get("HYPERION_REFERENCE_DIR")
    if not ref_dir or not os.path.exists(os.path.join(ref_dir, REF_MODULE)):
        raise SystemExit("reference checkout not found: set HYPERION_REFERENCE_DIR")
    rec = record(load_reference(ref_dir))
    rec["call_sites"] = call_sites(os.path.join(ref_dir, REF_MODULE))
    with open(OUT, "w") as f:
        json.dump(rec, f, indent=None, separators=(",", ":"))
        f.write("\n")
    print(OUT, len(rec["batches"]), "batches")


if __name__ == "__main__":
    sys.exit(main())
