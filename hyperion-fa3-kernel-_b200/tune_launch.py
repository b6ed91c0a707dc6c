"""Measures the KV-split count of the row kernels on this GPU and writes the launch table.

    python hyperion-fa3-kernel-_b200/tune_launch.py [--quick] [--out-md FILE]

For decode (one query row per (batch, head)) the forward splits each row's keys
into n pieces so that the persistent grid has enough units; the pieces are merged
by a second kernel.  Too few pieces leave SMs idle, too many pay for partials and
merges.  This script times every candidate split count on a grid of shapes --
query rows x keys, for the row kernel (no grouped-query heads) and the two grouped
kernels (4 query heads per KV head; the P.V products on the CUDA cores or on the
tensor core) -- with CUDA events on the launch stream, the L2 flushed before each
timed call, and keeps the fastest.  `--kernels 2` re-measures only the listed
kernels and keeps the table's other rows.  It writes

  csrc/launch_table.h   the table the library's split choice reads (rebuild after);
  --out-md FILE         a summary of the sweep (default: print to stdout).

The table records the SM count it was measured with; on another SM count the
library falls back to its occupancy-based rule.
"""
from __future__ import annotations

import argparse
import math
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import torch  # noqa: E402

CANDIDATES = (1, 2, 3, 4, 6, 8, 12, 16)
ITEMS = (32, 128, 512, 2048, 8192)
KEYS = (512, 2048, 8192, 32768)
MAX_KV_BYTES = 6e9  # shapes whose KV stream is larger than this are skipped


def make_decode(n_items: int, keys: int, kv_group: int, dev) -> dict:
    """Random sign bits and FP8 codes for n_items query rows over n_items / kv_group
    contiguous KV rows of `keys` keys (the values do not change the timing)."""
    n_kv = max(1, n_items // kv_group)
    g = torch.Generator(device=dev)
    g.manual_seed(n_items * 7 + keys)
    k = torch.randint(-2**31, 2**31 - 1, (n_kv * keys, 4), dtype=torch.int32, generator=g, device=dev)
    v = torch.randint(0, 0x7E, (n_kv * keys, 128), dtype=torch.uint8, generator=g, device=dev)
    q = torch.randint(-2**31, 2**31 - 1, (n_kv * kv_group, 4), dtype=torch.int32, generator=g, device=dev)
    wl = torch.zeros(n_kv * kv_group, 4, dtype=torch.int32, device=dev)
    wl[:, 1] = torch.arange(n_kv * kv_group, dtype=torch.int32, device=dev)
    return dict(worklist=wl, q=q, k=k, v=v, v_scale=torch.full((1,), 0.01, device=dev),
                ctx=torch.full((n_kv,), keys, dtype=torch.int32, device=dev),
                bt=torch.zeros(0, dtype=torch.int32, device=dev), keys=keys, kv_group=kv_group,
                o=torch.empty(n_kv * kv_group, 128, dtype=torch.bfloat16, device=dev))


# kernel id -> (query heads per KV head, the forward's group_kernel)
KERNELS = {0: (1, "auto"), 1: (4, "cuda"), 2: (4, "mma")}
KERNEL_NAMES = {0: "row", 1: "grouped, CUDA cores (4 heads / KV head)", 2: "grouped, tensor core (4 heads / KV head)"}


def time_call(hyperion, w: dict, splits: int, reps: int, flush: torch.Tensor, group_kernel: str = "auto") -> float:
    """Median ms of `reps` calls with `splits` pieces per row (0: the library's choice)."""
    st = torch.cuda.current_stream()

    def call():
        hyperion.hyperion_apex_kernel(w["worklist"], w["worklist"].shape[0], w["q"], None, w["k"], None, w["v"],
                                      w["v_scale"], w["ctx"], w["bt"], w["o"], 1, 128, 16, w["keys"], 1,
                                      0.088, False, path="row", num_splits=splits, kv_group=w["kv_group"],
                                      group_kernel=group_kernel)

    call()
    times = []
    for _ in range(reps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        call()
        e1.record(st)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


def sweep(hyperion, quick: bool, kernels=(0, 1, 2)):
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    reps = 3 if quick else 7
    rows = []
    for kernel in kernels:
        kv_group, group_kernel = KERNELS[kernel]
        for n in ITEMS:
            for keys in KEYS:
                if n * keys * 144 / kv_group > MAX_KV_BYTES:
                    continue
                w = make_decode(n, keys, kv_group, dev)
                auto = time_call(hyperion, w, 0, reps, flush, group_kernel)
                auto_splits = hyperion.last_call_info()["splits"]
                best = None
                for s in CANDIDATES:
                    if s > 1 and keys // s < 256:
                        continue
                    t = time_call(hyperion, w, s, reps, flush, group_kernel)
                    if best is None or t < best[1]:
                        best = (s, t)
                rows.append(dict(kernel=kernel, kv_group=kv_group, items=n, keys=keys, best=best[0], best_ms=best[1],
                                 rule=auto_splits, rule_ms=auto))
                del w
                torch.cuda.empty_cache()
    return rows


def read_header(path: str):
    """The rows of an existing table (with the timings its comments record)."""
    import re
    rows = []
    if not os.path.exists(path):
        return rows
    pat = re.compile(r"\{(\d+), (\d+), (\d+), (\d+)\},\s*// ([0-9.]+) ms; the rule's (\d+): ([0-9.]+) ms")
    for line in open(path):
        m = pat.search(line)
        if m:
            k, n, keys, best, best_ms, rule, rule_ms = m.groups()
            rows.append(dict(kernel=int(k), kv_group=KERNELS[int(k)][0], items=int(n), keys=int(keys),
                             best=int(best), best_ms=float(best_ms), rule=int(rule), rule_ms=float(rule_ms)))
    return rows


def write_header(rows, sm_count: int, path: str):
    lines = [
        "// launch_table.h -- KV pieces per work item of the row kernels, measured on B200.",
        "//",
        "// Generated by tune_launch.py, which timed every candidate split count on a grid",
        "// of decode shapes (query rows x keys per row; kernel 0: row kernel, 1: grouped",
        "// row kernel with 4 query heads per KV head, 2: the grouped kernel with the P.V",
        "// products on the tensor core; head_dim 128) and kept the fastest.",
        "// The library uses an entry for a call within a factor of 2 of its shape on a",
        "// device with kSplitTableSms SMs, and its occupancy-based rule otherwise.",
        "#pragma once",
        "",
        "namespace hyp {",
        "namespace table {",
        "",
        "struct SplitEntry {",
        "  int kernel;  // 0 row kernel, 1 grouped row kernel, 2 tensor-core grouped kernel",
        "  int items;   // work items (query rows) of the call",
        "  int keys;    // keys per row (block_size * num_blocks)",
        "  int splits;  // fastest KV pieces per work item",
        "};",
        "",
        f"constexpr int kSplitTableSms = {sm_count};",
        "constexpr SplitEntry kSplitTable[] = {",
    ]
    for r in rows:
        lines.append(f"    {{{r['kernel']}, {r['items']}, {r['keys']}, {r['best']}}},"
                     f"  // {r['best_ms']:.4f} ms; the rule's {r['rule']}: {r['rule_ms']:.4f} ms")
    lines += ["};", "", "}  // namespace table", "}  // namespace hyp", ""]
    with open(path, "w") as f:
        f.write("\n".join(lines))


def summary(rows, sm_count: int) -> str:
    out = [f"Split sweep on {torch.cuda.get_device_name(0)} ({sm_count} SMs), head_dim 128, bf16 O, "
           "L2 flushed before each timed call, median of the timed calls.", "",
           "| kernel | query rows | keys | best splits | best ms | rule splits | rule ms | rule / best |",
           "|---|---|---|---|---|---|---|---|"]
    for r in rows:
        out.append(f"| {KERNEL_NAMES[r['kernel']]} | {r['items']} | {r['keys']} | "
                   f"{r['best']} | {r['best_ms']:.4f} | {r['rule']} | {r['rule_ms']:.4f} | "
                   f"{r['rule_ms'] / r['best_ms']:.3f} |")
    return "\n".join(out) + "\n"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--out-md", default=None)
    ap.add_argument("--header", default=os.path.join(HERE, "csrc", "launch_table.h"))
    ap.add_argument("--kernels", default="0,1,2", help="kernel ids to measure; the table keeps the others' rows")
    a = ap.parse_args()
    import hyperion_b200 as hyperion

    sm_count = torch.cuda.get_device_properties(0).multi_processor_count
    kernels = tuple(int(k) for k in a.kernels.split(","))
    kept = [r for r in read_header(a.header) if r["kernel"] not in kernels]
    rows = sorted(kept + sweep(hyperion, a.quick, kernels), key=lambda r: (r["kernel"], r["items"], r["keys"]))
    write_header(rows, sm_count, a.header)
    text = summary(rows, sm_count)
    if a.out_md:
        with open(a.out_md, "w") as f:
            f.write(text)
    print(text)
    return 0


if __name__ == "__main__":
    sys.exit(main())
