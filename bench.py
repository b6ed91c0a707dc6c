"""Benchmark of the sign-bit / FP8 attention forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload prefill|decode|paged_decode|longctx|cpu_ref|decode_gqa|paged_decode_gqa]
                    [--impl ours|reference] [--path auto|row|tile] [--no-sub]

For N > 1 launch with torchrun (one rank per GPU, NCCL):
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

One step = one forward call (`hyperion_apex_kernel`) over one batch of the
workload, inputs already in HBM.  The headline workload is the causal prefill
B4 H32 S_q=S_kv=4096 D128, bf16 output, per GPU; at N GPUs each rank runs its own
(batch, head) shard of a global batch of 4*N sequences (weak scaling, no
data-path collective).  The same line carries sub-records, measured in the same
run with the same method, for the decode workloads (whose metric is HBM GB/s)
and the long-context prefill (B1 H64 S32768, heads split over the ranks:
strong scaling).  At N > 1 every record also carries `with_gather`: the same
steps with the whole O gathered on every rank inside each step, in three forms:
the forward then an NCCL all-gather (serial), the forward in chunks whose
all-gathers overlap the next chunk (overlapped), and the forward storing its O
rows into every rank's output buffer over NVLink itself (fused); the fastest one
is its value.

Timing: W untimed warm-up steps; L2 flushed (256 MiB write) before every timed
step unless the inputs are larger than twice the L2; each step bracketed by CUDA
events on the launch stream; the K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides; the max over ranks is reported.  `e2e`
repeats the step through the public Python API with pinned host inputs: H2D
copies, the forward and the D2H copy of O are inside the timed region (decode
keeps the KV cache resident and writes each step's new token into it; prefill
pipelines its copies over two streams).
`cpu_baseline` times the CPU oracle (the C restatement of the reference
algorithm) on a bounded sample on this host's cores.

`--impl reference` times the reference's own CPU path for this forward: the
reference's kernel does not build and has no CPU attention, so that is the C
restatement of its algorithm (oracle/), run on all host threads, rank 0 only.
Its inputs are built on the host and the CUDA library is never loaded; each
step runs the oracle over the same fixed sample of (batch, head) rows.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
import types

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "hyperion-fa3-kernel-_b200")
sys.path.insert(0, PKG_DIR)
sys.path.insert(0, REPO)

import torch  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# B200 datasheet figures: HGX HBM3e bandwidth and dense bf16 tensor throughput.
SPEC_PEAKS = {"hbm_gbs": 7700.0, "bf16_tflops": 2250.0}
METRIC = "attn Q·KV-token pairs/s"
L2_BYTES = 126 << 20
SUB_WORKLOADS = ("decode", "paged_decode", "decode_gqa", "longctx")
GATHER_CHUNKS = 4   # runs of (batch, head) rows whose O gathers overlap the next run's compute
GATHER_SMS = 16     # SMs the forward leaves to NCCL while a gather runs beside it
NVLINK_GBS = 770.0  # measured peer-copy bandwidth per direction per GPU on this machine type


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def host_only_package():
    """Makes `hyperion_b200.workloads` / `.sharding` importable without running the
    package's __init__, which loads the CUDA library: the reference arm builds its
    inputs with them and must not load any of this repository's device code."""
    if "hyperion_b200" not in sys.modules:
        pkg = types.ModuleType("hyperion_b200")
        pkg.__path__ = [os.path.join(PKG_DIR, "hyperion_b200")]
        sys.modules["hyperion_b200"] = pkg


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = set(gpu_indices)
        self.proc = None
        self.out = None

    def start(self):
        try:
            self.out = open(os.path.join("/tmp", f"hyperion_clocks_{os.getpid()}.csv"), "w+")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.seek(0)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if self.gpus and idx not in self.gpus:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        self.out.close()
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------- workloads
def build_workload(name, rank, world, device):
    """The workload of `name` on this rank, its description and its scaling mode."""
    from hyperion_b200 import workloads as W
    from hyperion_b200.sharding import head_range

    if name == "longctx":
        H = W.CONFIGS["longctx"]["H"]
        heads = head_range(H, world, rank)
        wk = W.make_config("longctx", device=device, exact=False, heads=heads, seed=rank)
        desc = f"longctx B1 H{H} S_q=S_kv=32768 D128 causal, heads {heads.start}-{heads.stop - 1} on this rank"
        return wk, desc, "strong"
    wk = W.make_config(name, device=device, exact=False, seed=rank)
    c = W.CONFIGS[name]
    heads = f"H{c['H']}" + (f" over {c['Hkv']} KV heads" if "Hkv" in c else "")
    if name.startswith("paged_decode"):
        desc = (f"{name} B{c['B']} {heads} D128 S_q=1, L~U[{c['lo']},{c['hi']}] seed 1, page {c['page']}, "
                "random page pool, per GPU")
    else:
        desc = (f"{name} B{c['B']} {heads} S_q={c['S_q']} S_kv={c['S_kv']} D128 "
                f"{'causal' if c['causal'] else 'non-causal'}, per GPU")
    return wk, desc, "weak"


def input_bytes(wk):
    return sum(t.numel() * t.element_size() for t in (wk.q, wk.k, wk.v, wk.block_tables))


def workload_config(wk, desc, world, scaling):
    """The `config` object of a JSON line: a function of the workload and the world
    size only, so both arms of the benchmark print the same one."""
    l2 = ("flushed before every timed step (256 MiB write)" if input_bytes(wk) <= 2 * L2_BYTES else
          f"not flushed: inputs of {input_bytes(wk) / 1e9:.2f} GB are larger than L2")
    return {
        "workload": desc,
        "global_batch": wk.batch * world if scaling == "weak" else wk.batch,
        "heads": wk.heads if scaling == "weak" else wk.heads * world,
        "seq_len": wk.seq_q if wk.seq_q > 1 else int(wk.ctx_lens.max()),
        "head_dim": wk.head_dim,
        "causal": wk.causal,
        "parallelism": f"(batch, head) shards x{world}, no data-path collective",
        "l2": l2,
    }


def call_forward(hyperion, wk, o, path="auto", **kw):
    hyperion.hyperion_apex_kernel(wk.worklist, wk.total_work, wk.q, None, wk.k, None, wk.v, wk.v_scale, wk.ctx_lens,
                                  wk.block_tables, o, wk.seq_q, wk.head_dim, wk.head_dim // 8, wk.block_size,
                                  wk.num_blocks, wk.inv_sqrt_d, wk.causal, path=path, kv_group=wk.kv_group, **kw)


def roofline_numbers(wk, pairs, kernel_ms, pk):
    """Dominant kernel: algorithmic work per launch / average launch time, as a
    fraction of the measured peak and of the datasheet peak."""
    if wk.seq_q == 1:
        # decode: K (D/8 B) + V (D B) per distinct (KV row, key) pair, plus Q rows and
        # O rows.  Without grouped-query heads every pair has its own KV row.
        nbytes = wk.kv_keys() * wk.kv_bytes_per_pair() + wk.total_work * (wk.head_dim // 8) \
            + wk.total_work * wk.head_dim * torch.tensor([], dtype=wk.o_dtype).element_size()
        achieved = nbytes / (kernel_ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "spec_peak": SPEC_PEAKS["hbm_gbs"],
                "frac_of_spec": achieved / SPEC_PEAKS["hbm_gbs"], "algorithmic_bytes_per_launch": nbytes}
    flops = 2.0 * 2.0 * wk.head_dim * pairs  # QK (2D) + PV (2D) per pair
    achieved = flops / (kernel_ms * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": achieved / pk["bf16_tflops"], "spec_peak": SPEC_PEAKS["bf16_tflops"],
            "frac_of_spec": achieved / SPEC_PEAKS["bf16_tflops"], "algorithmic_flops_per_launch": flops}


# The arithmetic each kernel computes the path in.
DTYPES = {
    "tile": "sign-bit QK (e4m3 +-1 MMA, exact int) / f16 PV",
    "row": "sign-bit QK (popc, exact int) / f16x2 PV products, f32 accumulation",
    "group": "sign-bit QK (popc, exact int) / f16x2 PV products, f32 accumulation",
    "group_mma": "sign-bit QK (popc, exact int) / e4m3 PV MMA (V codes x weights in 3 e4m3 pieces), f32 accumulation",
}


def read_traffic(kernel_tag):
    """DRAM bytes per launch from the committed ncu summary, if one exists:
    a line `traffic_bytes_per_launch: <int>` in profiles/<kernel_tag>.md."""
    path = os.path.join(REPO, "profiles", f"{kernel_tag}.md")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            if line.strip().startswith("traffic_bytes_per_launch:"):
                try:
                    return int(float(line.split(":", 1)[1].strip()))
                except ValueError:
                    return None
    return None


# ---------------------------------------------------------------------------- CPU baseline
def _sample_rows(wk, n_rows):
    """The first n_rows of a seeded permutation of the workload's (batch, head) rows."""
    order = torch.randperm(wk.n_bh, generator=torch.Generator().manual_seed(0)).tolist()
    return order[:max(1, min(n_rows, wk.n_bh))]


def _rows_per_call(wk, threads):
    """Rows per oracle call: enough work items to keep every host thread busy."""
    return max(1, (4 * threads + wk.seq_q - 1) // wk.seq_q)


def cpu_baseline(wk_gpu, budget_s=12.0):
    """Times the C oracle on a sample of this workload's (batch, head) rows on all host
    threads.  Returns (pairs/s, threads, description)."""
    from oracle import oracle as O

    threads = O.lib().oracle_max_threads()
    n_bh = wk_gpu.n_bh
    bh_order = torch.randperm(n_bh, generator=torch.Generator().manual_seed(0)).tolist()
    per_call = _rows_per_call(wk_gpu, threads)
    done_pairs, spent, used = 0, 0.0, 0
    pos = 0
    # A workload shorter than the budget is timed again from its first row.
    while spent < budget_s * 0.5:
        start = pos % n_bh
        rows = bh_order[start: start + per_call]
        pos += len(rows)
        nrows = len(rows)
        sub = _subset_rows(wk_gpu, rows)
        t0 = time.perf_counter()
        O.forward_workload_c(sub, nthreads=threads)
        spent += time.perf_counter() - t0
        done_pairs += sub.pairs()
        used += nrows
    passes = used / n_bh
    desc = (f"{min(used, n_bh)} of {n_bh} (batch, head) rows of this workload with all their query rows"
            + (f", {passes:.1f} passes over the workload" if passes > 1 else "")
            + f", {per_call} rows per call, {spent:.1f} s")
    return done_pairs / spent, threads, desc


def _subset_rows(wk, rows):
    """The listed (batch, head) rows of a workload, with every query row of each, as a
    contiguous CPU workload (their keys gathered from the pool where it lies)."""
    from hyperion_b200 import workloads as W

    cap = wk.num_blocks * wk.block_size
    g = wk.kv_group
    lens = [min(int(wk.ctx_lens[bh // g]), cap) for bh in rows]
    Lmax = max(max(lens), 1)
    W_ = wk.head_dim // 32
    kk = torch.zeros(len(rows) * Lmax, W_, dtype=torch.int32, device=wk.k.device)
    vv = torch.zeros(len(rows) * Lmax, wk.head_dim, dtype=torch.uint8, device=wk.k.device)
    qq, sc = [], []
    vs = wk.v_scale
    for i, (bh, L) in enumerate(zip(rows, lens)):
        t = torch.arange(L, device=wk.k.device)
        page = t // wk.block_size
        kv = bh // g
        ids = wk.block_tables[kv].to(torch.int64)[page] if wk.block_tables.numel() else kv * wk.num_blocks + page
        slots = ids * wk.block_size + t % wk.block_size
        kk[i * Lmax: i * Lmax + L] = wk.k[slots]
        vv[i * Lmax: i * Lmax + L] = wk.v[slots]
        qq.append(wk.q[bh * wk.seq_q:(bh + 1) * wk.seq_q])
        sc.append(vs.reshape(-1)[0] if vs.numel() == 1 else vs[kv % vs.numel()])
    scale = torch.stack(sc).float()
    if scale.numel() == kk.shape[0]:  # keep the per-row scale unambiguous
        scale = torch.cat([scale, scale[:1]])
    wl = W.dense_worklist(len(rows), wk.seq_q, "cpu")
    if wk.seq_q == 1:
        wl[:, 0] = 0
    return W.Workload(name=wk.name + "_sample", worklist=wl, q=torch.cat(qq).cpu(), k=kk.cpu(), v=vv.cpu(),
                      v_scale=scale.cpu(), ctx_lens=torch.tensor(lens, dtype=torch.int32),
                      block_tables=torch.zeros(0, dtype=torch.int32), seq_q=wk.seq_q, head_dim=wk.head_dim,
                      block_size=Lmax, num_blocks=1, causal=wk.causal, o_dtype=torch.float32, batch=1,
                      heads=len(rows), inv_sqrt_d=wk.inv_sqrt_d)


# ---------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's CPU path on this host's cores: rank 0 alone, no GPU.

    A step is one pass of the C restatement of the reference's per-item loop
    (hyperion_fa3_production_final.py:338-593, oracle/hyperion_oracle.c) over a fixed
    sample of the workload's (batch, head) rows with all their query rows, on all host
    threads.  The sample is sized in the first warm-up step so that W + K steps take
    about a minute and a half; every timed step runs the same sample, and the line's
    ms_per_step is the measured time of those steps."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    host_only_package()
    from oracle import oracle as O

    wk, desc, scaling = build_workload(args.workload, 0, world, torch.device("cpu"))
    config = workload_config(wk, desc, world, scaling)
    threads = O.lib().oracle_max_threads()
    per_call = _rows_per_call(wk, threads)
    target_s = min(3.0, max(0.3, 90.0 / (args.warmup + args.steps)))
    # Calibration: one call's worth of rows.
    probe = _subset_rows(wk, _sample_rows(wk, per_call))
    t0 = time.perf_counter()
    O.forward_workload_c(probe, nthreads=threads)
    t_probe = max(time.perf_counter() - t0, 1e-4)
    n_calls = max(1, min(int(target_s / t_probe), (wk.n_bh + per_call - 1) // per_call))
    rows = _sample_rows(wk, n_calls * per_call)
    calls = [_subset_rows(wk, rows[i:i + per_call]) for i in range(0, len(rows), per_call)]
    sample_pairs = sum(c.pairs() for c in calls)
    step_s = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for c in calls:
            O.forward_workload_c(c, nthreads=threads)
        if i >= args.warmup:
            step_s.append(time.perf_counter() - t0)
    total_s = sum(step_s)
    value = sample_pairs * len(step_s) / total_s
    sample = (f"{len(rows)} of {wk.n_bh} (batch, head) rows of this workload with all their query rows "
              f"({sample_pairs} pairs, seeded choice), {per_call} rows per oracle call, the same rows every step")
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "pairs/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_s / len(step_s) * 1e3,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded random sign bits for Q/K, N(0,1) V as FP8 e4m3 with per-head scale",
        "config": config, "pairs_per_step": sample_pairs,
        "cpu_baseline": {"value": value, "unit": "pairs/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "pairs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
        "note": "the reference's CUDA kernel does not build and it has no CPU attention path; this is the C "
                "restatement of its algorithm (oracle/hyperion_oracle.c) on all host threads, inputs built on "
                "the host",
    }
    print(json.dumps(out))
    return 0


# ---------------------------------------------------------------------------- our arm
def run_e2e(hyperion, wk, o, args, barrier):
    """Times args.steps steps through the public Python API with pinned host buffers;
    returns (total ms, H2D bytes per step, D2H bytes per step, description).

    Decode (one query row): the KV cache stays on the device, as the reference's
    engine keeps it (hyperion_fa3_production_final.py:1017-1032).  A step copies in
    the new token's Q rows, K and V (bf16 [batch, KV heads, D]), positions and context
    lengths, writes K and V into the cache (kv_cache_write), runs the forward and
    copies O out.
    Prefill: a step copies in all of the forward's inputs and copies O out.
    In both, steps are pipelined: the inputs of step i+1 go in and the O of step i-1
    comes out while step i computes (copy streams, double buffers; cache writes and
    forwards stay in order on one stream, since they share the workspace)."""
    dev = o.device
    main = torch.cuda.current_stream(dev)
    if wk.seq_q == 1:
        B, Hkv, D = wk.batch, wk.heads // wk.kv_group, wk.head_dim
        ctx = wk.ctx_lens.view(B, Hkv)[:, 0].to(torch.int32)
        g = torch.Generator().manual_seed(5)
        host = {
            "q": wk.q.cpu().pin_memory(),
            "k_new": torch.randn(B, Hkv, D, generator=g).to(torch.bfloat16).pin_memory(),
            "v_new": torch.randn(B, Hkv, D, generator=g).to(torch.bfloat16).pin_memory(),
            "seq_ids": torch.arange(B, dtype=torch.int32).pin_memory(),
            "positions": (ctx - 1).clamp_min(0).cpu().pin_memory(),
            "ctx_lens": wk.ctx_lens.cpu().pin_memory(),
        }
        # The step's inputs sit in one pinned staging buffer (each at a 256-byte
        # offset) and go over PCIe in one copy into a device buffer that the
        # kernels read through fixed views.  Two device buffers and two O buffers
        # pipeline the steps as the prefill case does: the inputs of step i+1 go in
        # and the O of step i-1 comes out while step i computes; the cache writes
        # and forwards stay in order on one stream.
        offs, total = {}, 0
        for k_, t in host.items():
            offs[k_] = total
            total += (t.numel() * t.element_size() + 255) // 256 * 256
        stage_h = torch.zeros(total, dtype=torch.uint8).pin_memory()
        for k_, t in host.items():
            n = t.numel() * t.element_size()
            stage_h[offs[k_]: offs[k_] + n].copy_(t.contiguous().view(torch.uint8).reshape(-1))
        stage_d = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(2)]
        dbufs = [{k_: stage_d[b][offs[k_]: offs[k_] + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                  for k_, t in host.items()} for b in range(2)]
        subs = [type(wk)(**{**wk.__dict__, "q": dbufs[b]["q"], "ctx_lens": dbufs[b]["ctx_lens"]}) for b in range(2)]
        outs = [o, torch.empty_like(o)]
        o_hosts = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_done = [torch.cuda.Event() for _ in range(2)]
        fwd_done = [torch.cuda.Event() for _ in range(2)]
        out_done = [torch.cuda.Event() for _ in range(2)]

        def issue(i):
            b = i % 2
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(fwd_done[b])
                stage_d[b].copy_(stage_h, non_blocking=True)
                in_done[b].record(s_in)
            main.wait_event(in_done[b])
            if i >= 2:
                main.wait_event(out_done[b])
            d = dbufs[b]
            hyperion.kv_cache_write(d["k_new"], d["v_new"], d["seq_ids"], d["positions"], wk.block_tables,
                                    wk.block_size, wk.num_blocks, wk.v_scale, wk.k, wk.v)
            call_forward(hyperion, subs[b], outs[b], path=args.path)
            fwd_done[b].record(main)
            with torch.cuda.stream(s_out):
                s_out.wait_event(fwd_done[b])
                o_hosts[b].copy_(outs[b], non_blocking=True)
                out_done[b].record(s_out)

        for i in range(2):
            issue(i)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(main)
        s_in.wait_event(e0)
        for i in range(args.steps):
            issue(i)
        main.wait_stream(s_out)
        e1.record(main)
        torch.cuda.synchronize()
        barrier()
        h2d = total
        mode = ("resident KV cache: per step one H2D copy of Q, the new token's K/V (bf16), positions and context "
                "lengths from a pinned staging buffer; kv_cache_write; forward; D2H of O; steps pipelined over two "
                "copy streams")
        return e0.elapsed_time(e1), h2d, o_hosts[0].numel() * o_hosts[0].element_size(), mode

    keys = ("worklist", "q", "k", "v", "v_scale", "ctx_lens", "block_tables")
    host = {k: getattr(wk, k).cpu().pin_memory() for k in keys}
    dbufs = [{k: torch.empty_like(getattr(wk, k)) for k in keys} for _ in range(2)]
    subs = [type(wk)(**{**wk.__dict__, **dbufs[b]}) for b in range(2)]
    outs = [o, torch.empty_like(o)]
    o_hosts = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_done = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer b are on the device
    fwd_done = [torch.cuda.Event() for _ in range(2)]   # the forward has read buffer b and written O b
    out_done = [torch.cuda.Event() for _ in range(2)]   # O b has reached the host

    def issue(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(fwd_done[b])
            for k_ in keys:
                dbufs[b][k_].copy_(host[k_], non_blocking=True)
            in_done[b].record(s_in)
        main.wait_event(in_done[b])
        if i >= 2:
            main.wait_event(out_done[b])
        call_forward(hyperion, subs[b], outs[b], path=args.path)
        fwd_done[b].record(main)
        with torch.cuda.stream(s_out):
            s_out.wait_event(fwd_done[b])
            o_hosts[b].copy_(outs[b], non_blocking=True)
            out_done[b].record(s_out)

    for i in range(2):
        issue(i)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    s_in.wait_event(e0)
    for i in range(args.steps):
        issue(i)
    main.wait_stream(s_out)
    e1.record(main)
    torch.cuda.synchronize()
    barrier()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    mode = "all inputs H2D and O D2H every step, pipelined over two copy streams"
    return e0.elapsed_time(e1), h2d, o_hosts[0].numel() * o_hosts[0].element_size(), mode


def measure(hyperion, name, args, rank, world, dev, pg, cpu_budget_s):
    """One workload on every rank: warm-up, a sustained run under the clock sampler,
    args.steps timed steps, the e2e steps and, at N > 1, the steps with the output
    gather.  Every rank takes the same collectives in the same order.  Returns the
    JSON record on rank 0 and None elsewhere."""
    wk, desc, scaling = build_workload(name, rank, world, dev)
    o = wk.new_output()
    pairs = wk.pairs()
    # Between timed steps: inputs larger than twice the L2 (126 MB) are streamed
    # from HBM anyway; smaller ones are evicted by a 256 MiB write before each step.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if input_bytes(wk) <= 2 * L2_BYTES else None
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if pg is not None:
            pg.barrier()

    for _ in range(args.warmup):
        call_forward(hyperion, wk, o, path=args.path)
    torch.cuda.synchronize()
    info = hyperion.last_call_info()
    errs = hyperion.read_device_errors(dev, clear=True)

    # nvidia-smi samples every 200 ms, longer than a short timed region: the sampler
    # starts before a >= 1.5 s sustained run of the same step that leads straight
    # into the timed steps, and stops after them.
    clocks = ClockSampler([dev.index] if world == 1 else list(range(world)))
    if rank == 0:
        clocks.start()
    t_end = time.perf_counter() + 1.5
    n_sus = 0
    while time.perf_counter() < t_end or n_sus < 2:
        if flush is not None:
            flush.fill_(n_sus & 0xFF)
        call_forward(hyperion, wk, o, path=args.path)
        n_sus += 1
        if n_sus % 4 == 0:
            torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        if flush is not None:
            flush.fill_(i & 0xFF)
        starts[i].record(stream)
        call_forward(hyperion, wk, o, path=args.path)
        ends[i].record(stream)
    torch.cuda.synchronize()
    barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    clk = clocks.stop() if rank == 0 else None

    # e2e through the public API with pinned host buffers.
    e2e_ms, h2d, d2h, e2e_mode = run_e2e(hyperion, wk, o, args, barrier)

    # N > 1: the same steps with the all-gather of O (NCCL) inside each step, for a
    # caller that wants the whole output on every rank.  Two forms: the forward then
    # one gather (serial), and the forward in GATHER_CHUNKS runs of (batch, head) rows
    # whose gathers (on a second stream) overlap the next run's compute, with the
    # forward's persistent grid kept off GATHER_SMS SMs so that NCCL's kernels find
    # room beside it.
    gather_total = serial_total = fused_total = pushed_total = 0.0
    fused_why = None
    gather_checks = None
    if world > 1:
        from hyperion_b200 import sharding as S

        out_all = torch.empty((world,) + tuple(o.shape), dtype=o.dtype, device=dev)
        chunks = S.row_chunks(wk, GATHER_CHUNKS)
        rows_c = chunks[0][1].stop - chunks[0][1].start
        out_chunks = torch.empty((len(chunks), world, rows_c) + tuple(o.shape[1:]), dtype=o.dtype, device=dev)
        comm = torch.cuda.Stream(dev)
        budget = max(1, torch.cuda.get_device_properties(dev).multi_processor_count - GATHER_SMS)

        def forward_chunk(items, out=o, sm_budget=budget):
            wl = wk.worklist[items]
            hyperion.hyperion_apex_kernel(wl, wl.shape[0], wk.q, None, wk.k, None, wk.v, wk.v_scale, wk.ctx_lens,
                                          wk.block_tables, out, wk.seq_q, wk.head_dim, wk.head_dim // 8,
                                          wk.block_size, wk.num_blocks, wk.inv_sqrt_d, wk.causal, path=args.path,
                                          kv_group=wk.kv_group, sm_budget=sm_budget)

        def serial_step():
            call_forward(hyperion, wk, o, path=args.path)
            pg.all_gather_into_tensor(out_all, o)

        def overlapped_step():
            S.forward_and_gather(forward_chunk, chunks, o, out_chunks, comm_stream=comm)

        # fused: the forward stores its O rows into this rank's slot of every rank's
        # gathered buffer (peer stores over NVLink, CUDA IPC mappings), then a 4-byte
        # all-reduce stands as the barrier after which every rank may read its copy.
        # PeerOutput fails on every rank together (an IPC mapping refused on one of
        # them), and the fused form is then left out of the record.
        try:
            peer = S.PeerOutput(o.shape[0], o.shape[1], o.dtype, dev)
            fused_why = None
        except RuntimeError as e:
            peer, fused_why = None, str(e)[:200]
        tick = torch.zeros(1, dtype=torch.int32, device=dev)

        def fused_step():
            call_forward(hyperion, wk, peer.local, path=args.path, o_peers=peer.o_peers)
            pg.all_reduce(tick)

        # pushed: the forward in GATHER_CHUNKS runs on every SM into this rank's slot,
        # each finished run's O rows copied into every peer's gathered buffer by the
        # copy engines (one stream per peer) while the next run computes, then the
        # 4-byte all-reduce as the barrier.
        push_streams = [torch.cuda.Stream(dev) for _ in range(world - 1)]

        def pushed_step():
            S.forward_and_push(lambda items: forward_chunk(items, out=peer.local, sm_budget=0), chunks, peer,
                               push_streams)
            pg.all_reduce(tick)

        totals = []
        steps = (serial_step, overlapped_step) + ((fused_step, pushed_step) if peer is not None else ())
        pushed_diff = None
        for step in steps:
            step()
            torch.cuda.synchronize()
            g_st = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            g_en = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            barrier()
            torch.cuda.synchronize()
            for i in range(args.steps):
                if flush is not None:
                    flush.fill_(i & 0xFF)
                g_st[i].record(stream)
                step()
                g_en[i].record(stream)
            torch.cuda.synchronize()
            barrier()
            totals.append(sum(s.elapsed_time(e) for s, e in zip(g_st, g_en)))
            if step is fused_step:
                fused_same = torch.equal(peer.out.view(torch.uint8), out_all.view(torch.uint8))
            if step is pushed_step:
                pushed_diff = (peer.out.float() - out_all.float()).abs().max().item()
        serial_total, gather_total = totals[:2]
        fused_total = totals[2] if peer is not None else float("inf")
        pushed_total = totals[3] if peer is not None else float("inf")
        # The overlapped output is the serial one, rank by rank (a chunked call may
        # choose other KV splits, so the two agree to rounding, not bit for bit); the
        # fused output is the serial one bit for bit (the same call, stored twice).
        # Both checks are taken over every rank (a max), so that all ranks agree on the
        # outcome and take the same collectives after it: a form that disagrees is
        # reported in the record and left out of its value, not raised on one rank.
        diff = (out_chunks.transpose(0, 1).reshape(out_all.shape).float() - out_all.float()).abs().max().item()
        if peer is None:
            fused_same, pushed_diff = True, 0.0
        else:
            peer.close()
        chk = torch.tensor([diff if diff == diff else float("inf"), 0.0 if fused_same else 1.0,
                            pushed_diff if pushed_diff == pushed_diff else float("inf")],
                           dtype=torch.float64, device=dev)
        pg.all_reduce(chk, op=pg.ReduceOp.MAX)
        gather_checks = {"overlapped_max_abs_diff": float(chk[0]), "fused_bit_exact": bool(chk[1] == 0.0),
                         "pushed_max_abs_diff": float(chk[2])}
        if not float(chk[0]) <= 2e-2:
            gather_total = float("inf")
        if float(chk[1]) != 0.0:
            fused_total = float("inf")
        if not float(chk[2]) <= 2e-2:
            pushed_total = float("inf")
        del out_all, out_chunks, peer

    vals = torch.tensor([total_ms, e2e_ms, float(pairs), gather_total, serial_total, fused_total, pushed_total],
                        dtype=torch.float64, device=dev)
    if pg is not None:
        mx = vals.clone()
        pg.all_reduce(mx, op=pg.ReduceOp.MAX)
        sm = vals.clone()
        pg.all_reduce(sm, op=pg.ReduceOp.SUM)
        total_ms_max, e2e_ms_max, gather_max, serial_max = float(mx[0]), float(mx[1]), float(mx[3]), float(mx[4])
        fused_max, pushed_max = float(mx[5]), float(mx[6])
        pairs_all = float(sm[2])
    else:
        total_ms_max, e2e_ms_max, gather_max, serial_max, fused_max = total_ms, e2e_ms, 0.0, 0.0, 0.0
        pushed_max = 0.0
        pairs_all = float(pairs)

    rec = None
    if rank == 0:
        pk, pk_src = peaks()
        kernel_ms = total_ms / args.steps
        roof = roofline_numbers(wk, pairs, kernel_ms, pk)
        roof["peak_source"] = pk_src
        kname = {"row": "row_kernel", "group": "row_group_kernel", "group_mma": "row_mma_kernel",
                 "tile": "tile_kernel"}.get(info.get("kernel"), f"{info['path'] or 'row'}_kernel")
        roof["kernel"] = kname
        kernel_tag = f"{kname}_{name}"
        roof["traffic"] = read_traffic(kernel_tag)
        roof["traffic_source"] = (f"carried over from one ncu capture (profiles/{kernel_tag}.md), not measured in "
                                  "this run" if roof["traffic"] is not None else None)
        if world == 1 and cpu_budget_s > 0:
            v_cpu, cores, sample = cpu_baseline(wk, budget_s=cpu_budget_s)
            cpu = {"value": v_cpu, "unit": "pairs/s", "cores": cores, "kind": "port", "sample": sample}
        else:
            cpu = None
        value = pairs_all * args.steps / (total_ms_max * 1e-3)
        e2e_val = pairs_all * args.steps / (e2e_ms_max * 1e-3)
        rec = {
            "metric": METRIC, "value": value, "unit": "pairs/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms_max / args.steps, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None,
            "dtype": DTYPES.get(info.get("kernel"), DTYPES["row"]),
            "data": "synthetic: seeded random sign bits for Q/K, N(0,1) V as FP8 e4m3 with per-head scale",
            "config": workload_config(wk, desc, world, scaling),
            "launch": {"path": info["path"], "kv_splits": info["splits"], "grid": info["grid"]},
            "pairs_per_step": pairs_all,
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "pairs/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world, "mode": e2e_mode},
            "gpu_launches": info["kernels"] * args.steps,
            "clocks": clk, "device_errors": errs,
            "step_ms_min": min(step_ms), "step_ms_max": max(step_ms),
        }
        if roof["bound"] == "hbm":
            rec["hbm_gbs"] = roof["achieved"]
        if world > 1:
            o_bytes = o.numel() * o.element_size()
            forms = {"serial": serial_max}
            if gather_max != float("inf"):
                forms["overlapped"] = gather_max
            if fused_max != float("inf"):
                forms["fused"] = fused_max
            if pushed_max != float("inf"):
                forms["pushed"] = pushed_max
            form = min(forms, key=forms.get)
            best = forms[form]
            rec["with_gather"] = {
                "value": pairs_all * args.steps / (best * 1e-3), "unit": "pairs/s",
                "ms_per_step": best / args.steps,
                "form": form,
                "fused_ms_per_step": fused_max / args.steps if "fused" in forms else None,
                "fused_unavailable": fused_why,
                "pushed_ms_per_step": pushed_max / args.steps if "pushed" in forms else None,
                "checks_against_serial": gather_checks,
                "overlapped_ms_per_step": gather_max / args.steps if "overlapped" in forms else None,
                "serial_ms_per_step": serial_max / args.steps,
                "gather_bytes_received_per_rank": o_bytes * (world - 1),
                "nvlink_floor_ms": o_bytes * (world - 1) / NVLINK_GBS / 1e6,
                "mode": ("the fastest of four forms, max over ranks: fused = the forward storing each O row into "
                         "every rank's gathered buffer as well (peer stores over NVLink into CUDA IPC mappings), then "
                         "a 4-byte NCCL all-reduce as the barrier; pushed = the forward in "
                         f"{GATHER_CHUNKS} runs of (batch, head) rows on every SM, each finished run's O rows copied "
                         "into every peer's gathered buffer by the copy engines (cudaMemcpyAsync over the IPC "
                         "mappings, one stream per peer) while the next run computes, then the same barrier; "
                         f"overlapped = the forward in {GATHER_CHUNKS} runs of (batch, head) rows on {GATHER_SMS} "
                         "fewer SMs, each run's O all-gathered (NCCL all_gather_into_tensor, second stream) while the "
                         "next computes; serial = the forward, then one all-gather"),
                "limiter": ("NVLink: each rank receives (world-1) x its O bytes; the floor is that over the measured "
                            f"{NVLINK_GBS:.0f} GB/s peer-copy bandwidth per direction"),
            }
    del wk, o, flush
    torch.cuda.empty_cache()
    return rec


def run_ours(args):
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    import hyperion_b200 as hyperion

    out = measure(hyperion, args.workload, args, rank, world, dev, pg, 12.0 if not args.no_cpu_baseline else 0)
    if args.workload == "prefill" and not args.no_sub:
        subs = {}
        for name in SUB_WORKLOADS:
            rec = measure(hyperion, name, args, rank, world, dev, pg, 6.0 if not args.no_cpu_baseline else 0)
            if rank == 0:
                subs[name] = rec
        if rank == 0:
            out["sub"] = subs
    if rank == 0:
        print(json.dumps(out))
    if pg is not None:
        pg.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="prefill",
                    choices=["prefill", "decode", "paged_decode", "longctx", "cpu_ref", "decode_gqa",
                             "paged_decode_gqa"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--path", default="auto", choices=["auto", "row", "tile"])
    ap.add_argument("--no-sub", action="store_true", help="the headline workload only, without sub-records")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
