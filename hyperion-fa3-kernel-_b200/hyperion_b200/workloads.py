"""Seeded synthetic inputs in the reference's layouts (no dataset is involved).

The five workloads the path is measured and tested on:

  cpu_ref       B1  H8  S_q=S_kv=512,   non-causal, per-tensor V scale, fp32 O
  prefill       B4  H32 S_q=S_kv=4096,  causal,     per-head V scale,   bf16 O
  decode        B64 H32 S_q=1, S_kv=8192 contiguous, per-head V scale,   bf16 O
  longctx       B1  H64 S_q=S_kv=32768, causal (head-sharded over ranks), bf16 O
  paged_decode  B256 H32 S_q=1, L_b ~ U[512, 32768] (seed 1), 16-token pages in a
                shared pool behind a random permutation, per-head V scale, bf16 O

and the decode pair again with the reference engine's grouped-query head layout
(32 query heads over 8 KV heads): decode_gqa and paged_decode_gqa.

Encoding (identical for every workload and size):
  * Q, K ~ N(0, 1) in fp32; the sign bit (1 where x >= 0) of dim d goes to bit
    d % 32 of uint32 word d // 32 (LSB first), stored as int32;
  * V ~ N(0, 1); scale = max|V| / 448 per head (per tensor for cpu_ref);
    code = clamp(V / scale, -448, 448).to(float8_e4m3fn) viewed as uint8
    (clamping first: torch maps values above 448 to NaN);
  * work items are int32 rows {q_idx, bh, 0, 0} in (bh, q_idx) order, as the
    reference's prepare_worklist builds them (hyperion_fa3_production_final.py:914-929);
  * contiguous KV: slot of key t of bh = bh * S_kv + t, expressed as
    block_size = S_kv, num_blocks = 1 and an empty block table;
  * paged KV: global page g of sequence b is pool page perm[g]; the block of head h
    is perm[g] * H + h, so block_tables[b*H + h, j] = perm[page_j(b)] * H + h;
  * grouped-query attention (kv_heads = Hkv < H): K, V, context_lens, block-table
    rows and per-head V scales exist per KV head (the layouts above with Hkv for
    H); query head h of batch b reads KV row (b*H + h) // (H / Hkv).

`exact=True` draws Q, K, V with torch.manual_seed(seed) on the CPU in the order
Q, K, V (the recipe of the parity tests).  `exact=False` draws on `device` with a
seeded device generator, in chunks, for workloads too large for the CPU (same
encoding and distributions, different random stream).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch

FP8_MAX = 448.0


@dataclass
class Workload:
    name: str
    worklist: torch.Tensor  # int32 [n, 4]
    q: torch.Tensor  # int32 [n_bh * seq_q, W]
    k: torch.Tensor  # int32 [pool_rows, W]
    v: torch.Tensor  # uint8 [pool_rows, D]
    v_scale: torch.Tensor  # float32
    ctx_lens: torch.Tensor  # int32 [n_bh]
    block_tables: torch.Tensor  # int32 [n_bh, num_blocks] or empty
    seq_q: int
    head_dim: int
    block_size: int
    num_blocks: int
    causal: bool
    o_dtype: torch.dtype
    batch: int
    heads: int
    inv_sqrt_d: Optional[float] = None  # None: 1 / sqrt(head_dim); 0 gives flat weights
    meta: dict = field(default_factory=dict)
    kv_group: int = 1  # query heads per KV head; KV-side arrays are indexed by bh // kv_group

    def __post_init__(self):
        if self.inv_sqrt_d is None:
            self.inv_sqrt_d = 1.0 / math.sqrt(self.head_dim)

    @property
    def total_work(self) -> int:
        return self.worklist.size(0)

    @property
    def n_bh(self) -> int:
        """Query (batch, head) rows."""
        return self.ctx_lens.numel() * self.kv_group

    @property
    def n_kv_bh(self) -> int:
        """KV (batch, head) rows: numel of context_lens."""
        return self.ctx_lens.numel()

    def pairs(self) -> int:
        """Q.KV-token pairs attended (causal counts include the diagonal)."""
        ctx = self.ctx_lens.to(torch.int64).cpu()
        if self.seq_q == 1 and not self.causal and self.total_work == self.n_bh:
            return int(ctx.sum()) * self.kv_group
        q_idx = self.worklist[:, 0].to(torch.int64).cpu()
        bh = self.worklist[:, 1].to(torch.int64).cpu()
        lens = ctx[bh // self.kv_group]
        if self.causal:
            lens = torch.minimum(lens, q_idx + 1)
        return int(lens.clamp_min(0).sum())

    def kv_bytes_per_pair(self) -> int:
        return self.head_dim // 8 + self.head_dim

    def kv_keys(self) -> int:
        """Distinct (KV row, key) pairs the items attend: each is read once when the
        query heads of a KV head share its stream."""
        ctx = self.ctx_lens.to(torch.int64).cpu().clamp_min(0)
        if self.seq_q == 1 and not self.causal and self.total_work == self.n_bh:
            return int(ctx.sum())
        q_idx = self.worklist[:, 0].to(torch.int64).cpu()
        kv = self.worklist[:, 1].to(torch.int64).cpu() // self.kv_group
        lens = ctx[kv]
        if self.causal:
            lens = torch.minimum(lens, q_idx + 1)
        longest = torch.zeros(self.n_kv_bh, dtype=torch.int64).scatter_reduce(0, kv, lens, reduce="amax")
        return int(longest.sum())

    def to(self, device) -> "Workload":
        d = dict(self.__dict__)
        for k_ in ("worklist", "q", "k", "v", "v_scale", "ctx_lens", "block_tables"):
            d[k_] = getattr(self, k_).to(device)
        return Workload(**d)

    def new_output(self, device=None) -> torch.Tensor:
        dev = device if device is not None else self.q.device
        return torch.zeros(self.n_bh * self.seq_q, self.head_dim, dtype=self.o_dtype, device=dev)


# ---------------------------------------------------------------------------- encoding
def sign_pack(x: torch.Tensor) -> torch.Tensor:
    """[..., D] float -> int32 [..., D/32]: bit d%32 of word d/32 is (x[d] >= 0)."""
    d = x.shape[-1]
    assert d % 32 == 0
    bits = (x >= 0).reshape(*x.shape[:-1], d // 32, 32).to(torch.int64)
    weights = torch.bitwise_left_shift(torch.ones(32, dtype=torch.int64, device=x.device),
                                       torch.arange(32, device=x.device))
    words = (bits * weights).sum(-1)
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32)


def fp8_quantize(v: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp32 values and a broadcastable scale -> uint8 FP8 e4m3 codes of clamp(v/scale, +-448)."""
    return (v / scale).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def dense_worklist(n_bh: int, seq_q: int, device) -> torch.Tensor:
    bh = torch.arange(n_bh, dtype=torch.int32, device=device).repeat_interleave(seq_q)
    qi = torch.arange(seq_q, dtype=torch.int32, device=device).repeat(n_bh)
    wl = torch.zeros(n_bh * seq_q, 4, dtype=torch.int32, device=device)
    wl[:, 0] = qi
    wl[:, 1] = bh
    return wl


# ---------------------------------------------------------------------------- builders
def make_dense(name: str, B: int, H: int, S_q: int, S_kv: int, D: int = 128, causal: bool = False,
               scale_mode: str = "head", o_dtype=torch.bfloat16, seed: int = 0, exact: bool = True,
               device="cpu", gen_device=None, kv_heads: Optional[int] = None) -> Workload:
    """Contiguous KV: Q [B,H,S_q,D], K/V [B,Hkv,S_kv,D] with Hkv = kv_heads (default H);
    query head h reads KV head h // (H / Hkv)."""
    Hkv = kv_heads or H
    assert H % Hkv == 0, "H must be a multiple of kv_heads"
    n_bh = B * H
    n_kv = B * Hkv
    W = D // 32
    if exact:
        torch.manual_seed(seed)
        Qf = torch.randn(B, H, S_q, D)
        Kf = torch.randn(B, Hkv, S_kv, D)
        Vf = torch.randn(B, Hkv, S_kv, D)
        q = sign_pack(Qf).reshape(n_bh * S_q, W)
        k = sign_pack(Kf).reshape(n_kv * S_kv, W)
        if scale_mode == "tensor":
            vs = (Vf.abs().amax() / FP8_MAX).reshape(1)
            v8 = fp8_quantize(Vf, vs)
        else:
            vs_h = Vf.abs().amax(dim=(0, 2, 3)) / FP8_MAX  # [Hkv]
            v8 = fp8_quantize(Vf, vs_h.view(1, Hkv, 1, 1))
            vs = vs_h if scale_mode == "head" else vs_h.repeat(B)
        v = v8.reshape(n_kv * S_kv, D)
        q, k, v, vs = q.to(device), k.to(device), v.to(device), vs.to(torch.float32).to(device)
    else:
        gdev = torch.device(gen_device or device)
        g = torch.Generator(device=gdev)
        g.manual_seed(seed)
        q = torch.randint(-2**31, 2**31 - 1, (n_bh * S_q, W), dtype=torch.int32, generator=g, device=gdev)
        k = torch.randint(-2**31, 2**31 - 1, (n_kv * S_kv, W), dtype=torch.int32, generator=g, device=gdev)
        v = torch.empty(n_kv * S_kv, D, dtype=torch.uint8, device=gdev)
        amax = torch.zeros(Hkv, dtype=torch.float32, device=gdev)
        # Two passes over the same seeded chunks: per-head max, then quantise.
        rows_per_bh = S_kv
        for pass_ in (0, 1):
            for bh in range(n_kv):
                gc = torch.Generator(device=gdev)
                gc.manual_seed(seed * 1000003 + bh + 1)
                chunk = torch.randn(rows_per_bh, D, generator=gc, device=gdev)
                h = bh % Hkv
                if pass_ == 0:
                    amax[h] = torch.maximum(amax[h], chunk.abs().amax())
                else:
                    sc = amax[h] / FP8_MAX if scale_mode != "tensor" else amax.max() / FP8_MAX
                    v[bh * S_kv:(bh + 1) * S_kv] = fp8_quantize(chunk, sc)
        if scale_mode == "tensor":
            vs = (amax.max() / FP8_MAX).reshape(1)
        elif scale_mode == "head":
            vs = amax / FP8_MAX
        else:
            vs = (amax / FP8_MAX).repeat(B)
        q, k, v, vs = q.to(device), k.to(device), v.to(device), vs.to(torch.float32).to(device)
    ctx = torch.full((n_kv,), S_kv, dtype=torch.int32, device=device)
    wl = dense_worklist(n_bh, S_q, device)
    if S_q == 1:
        wl[:, 0] = 0
    return Workload(name=name, worklist=wl, q=q, k=k, v=v, v_scale=vs, ctx_lens=ctx,
                    block_tables=torch.zeros(0, dtype=torch.int32, device=device), seq_q=S_q, head_dim=D,
                    block_size=S_kv, num_blocks=1, causal=causal, o_dtype=o_dtype, batch=B, heads=H,
                    kv_group=H // Hkv)


def make_paged(name: str, B: int, H: int, lens: list, D: int = 128, page: int = 16, num_blocks: Optional[int] = None,
               seed: int = 0, perm_seed: int = 1, o_dtype=torch.bfloat16, device="cpu", exact: bool = True,
               gen_device=None, kv_heads: Optional[int] = None) -> Workload:
    """Paged decode (S_q = 1): per-sequence lengths `lens`, a shared pool of pages in a
    random order.  Pool rows = total_pages * Hkv * page, Hkv = kv_heads (default H);
    query head h reads KV head h // (H / Hkv)."""
    Hkv = kv_heads or H
    assert H % Hkv == 0, "H must be a multiple of kv_heads"
    lens_t = torch.tensor(lens, dtype=torch.int64)
    pages_b = (lens_t + page - 1) // page
    total_pages = int(pages_b.sum())
    if num_blocks is None:
        num_blocks = int(pages_b.max())
    gp = torch.Generator()
    gp.manual_seed(perm_seed)
    perm = torch.randperm(total_pages, generator=gp)
    offs = torch.cumsum(pages_b, 0) - pages_b
    n_bh = B * H
    n_kv = B * Hkv
    bt = torch.zeros(n_kv, num_blocks, dtype=torch.int64)
    for b in range(B):
        pg = perm[offs[b]: offs[b] + pages_b[b]]
        for h in range(Hkv):
            bt[b * Hkv + h, : pages_b[b]] = pg * Hkv + h
    pool_rows = total_pages * Hkv * page
    W = D // 32
    gdev = torch.device(gen_device or device)
    if exact:
        torch.manual_seed(seed)
        q = sign_pack(torch.randn(n_bh, D))
        k = sign_pack(torch.randn(pool_rows, D))
        Vf = torch.randn(pool_rows, D)
        head_of_row = (torch.arange(pool_rows) // page) % Hkv
        amax = torch.zeros(Hkv).scatter_reduce(0, head_of_row, Vf.abs().amax(1), reduce="amax")
        vs = amax / FP8_MAX
        v = fp8_quantize(Vf, vs[head_of_row].unsqueeze(1))
    else:
        g = torch.Generator(device=gdev)
        g.manual_seed(seed)
        q = torch.randint(-2**31, 2**31 - 1, (n_bh, W), dtype=torch.int32, generator=g, device=gdev)
        k = torch.randint(-2**31, 2**31 - 1, (pool_rows, W), dtype=torch.int32, generator=g, device=gdev)
        v = torch.empty(pool_rows, D, dtype=torch.uint8, device=gdev)
        chunk_rows = 1 << 22
        amax = torch.zeros(Hkv, dtype=torch.float32, device=gdev)
        for pass_ in (0, 1):
            for c0 in range(0, pool_rows, chunk_rows):
                c1 = min(pool_rows, c0 + chunk_rows)
                gc = torch.Generator(device=gdev)
                gc.manual_seed(seed * 1000003 + c0 // chunk_rows + 1)
                chunk = torch.randn(c1 - c0, D, generator=gc, device=gdev)
                head_of_row = (torch.arange(c0, c1, device=gdev) // page) % Hkv
                if pass_ == 0:
                    amax = amax.scatter_reduce(0, head_of_row, chunk.abs().amax(1), reduce="amax")
                else:
                    v[c0:c1] = fp8_quantize(chunk, (amax / FP8_MAX)[head_of_row].unsqueeze(1))
        vs = amax / FP8_MAX
    ctx = lens_t.repeat_interleave(Hkv).to(torch.int32)
    wl = dense_worklist(n_bh, 1, "cpu")
    wl[:, 0] = 0
    wk = Workload(name=name, worklist=wl.to(device), q=q.to(device), k=k.to(device), v=v.to(device),
                  v_scale=vs.to(torch.float32).to(device), ctx_lens=ctx.to(device),
                  block_tables=bt.to(torch.int32).to(device), seq_q=1, head_dim=D, block_size=page,
                  num_blocks=num_blocks, causal=False, o_dtype=o_dtype, batch=B, heads=H, kv_group=H // Hkv)
    wk.meta["total_pages"] = total_pages
    return wk


def paged_lengths(B: int, lo: int = 512, hi: int = 32768, seed: int = 1) -> list:
    g = torch.Generator()
    g.manual_seed(seed)
    return torch.randint(lo, hi + 1, (B,), generator=g).tolist()


# ---------------------------------------------------------------------------- named configs
CONFIGS = {
    "cpu_ref": dict(B=1, H=8, S_q=512, S_kv=512, causal=False, scale_mode="tensor", o_dtype=torch.float32),
    "prefill": dict(B=4, H=32, S_q=4096, S_kv=4096, causal=True, scale_mode="head", o_dtype=torch.bfloat16),
    "decode": dict(B=64, H=32, S_q=1, S_kv=8192, causal=False, scale_mode="head", o_dtype=torch.bfloat16),
    "longctx": dict(B=1, H=64, S_q=32768, S_kv=32768, causal=True, scale_mode="head", o_dtype=torch.bfloat16),
    "paged_decode": dict(B=256, H=32, page=16, lo=512, hi=32768),
    # The reference engine's head layout (num_heads 32, num_kv_heads 8) on the decode shapes.
    "decode_gqa": dict(B=64, H=32, Hkv=8, S_q=1, S_kv=8192, causal=False, scale_mode="head",
                       o_dtype=torch.bfloat16),
    "paged_decode_gqa": dict(B=256, H=32, Hkv=8, page=16, lo=512, hi=32768),
}


def make_config(name: str, device="cuda", exact: bool = False, heads: Optional[range] = None,
                batch: Optional[int] = None, seed: int = 0) -> Workload:
    """Builds one of CONFIGS.  `heads`/`batch` shrink it (a shard or a sample)."""
    c = dict(CONFIGS[name])
    H = len(heads) if heads is not None else c["H"]
    Hkv = None
    if "Hkv" in c:
        g = c["H"] // c["Hkv"]
        assert H % g == 0, "a head shard must hold whole KV groups"
        Hkv = H // g
    if name.startswith("paged_decode"):
        B = batch or c["B"]
        lens = paged_lengths(c["B"], c["lo"], c["hi"])[:B]
        return make_paged(name, B, H, lens, page=c["page"], num_blocks=c["hi"] // c["page"], seed=seed,
                          device=device, exact=exact, gen_device=device, kv_heads=Hkv)
    B = batch or c["B"]
    return make_dense(name, B, H, c["S_q"], c["S_kv"], causal=c["causal"], scale_mode=c["scale_mode"],
                      o_dtype=c["o_dtype"], seed=seed, exact=exact, device=device, gen_device=device,
                      kv_heads=Hkv)
