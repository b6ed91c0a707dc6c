// tile_kernel.cuh -- 128-row tcgen05 tile kernel: the prefill path.
//
// One CTA per SM, persistent.  A unit of work is a chunk of 256 consecutive work
// items (two 128-row Q tiles) of one (batch, head) row `bh`; chunks are taken
// with an atomic ticket in the caller's workspace (the reference's g_work_counter
// work stealing, hyperion_fa3_production_final.py:236-243, :332-336), longest
// causal rows first.  The unit's keys are walked in 128-key tiles:
//
//   scheduler warp takes the tickets and prepares each unit (segments of the chunk,
//                  context length, tile count; all dependent global reads) one
//                  unit ahead of the other roles, in a 2-slot ring;
//   loader warp    cp.async.bulk of the raw page pieces (sign bits 16 B/key, FP8
//                  codes 128 B/key) into a 2-stage ring, with the key-valid mask
//                  (context length, page ids inside the pool; :402-411, :479-486);
//   converters     (4 warps) sign bits -> e4m3 +-1 bytes in the 128B-swizzled
//                  K-major layout; FP8 codes -> f16 (the reference's decode,
//                  :122-141, divided by 256, exact) in the 128B-swizzled MN-major
//                  layout; Q rows of the unit likewise, once per unit;
//   MMA warps      (one per Q tile) S_t = Q_t K^T as kind::f8f6f4 tcgen05.mmas
//                  (the +-1 products sum to D - 2*popcount(q XOR k) exactly in the
//                  f32 accumulator, README.md:22), then O_t += P_t V, kind::f16
//                  MMAs with P read from TMEM; tcgen05.commit hands each result on;
//   softmax WG t   (4 warps per Q tile, one thread per row = TMEM lane) reads S,
//                  applies the masks (causal: key > q_idx, :483-486), keeps the
//                  running max with the reference's online update (:544-572),
//                  writes P as f16 over S, and at the end of the unit finalises
//                  O = acc * (l > 1e-6 ? 1/l : 1) (:582-593).
//
// Each 128-key tile is handled in two 64-key halves.  TMEM (512 columns): Q tile t
// owns S at [256t, 256t+128) -- half A (keys 0-63) in the first 64 columns, half B
// in the next 64 -- and O at [256t+128, 256t+256); P of a half is written over the
// first 32 columns of that half's S.  The QK of half A of tile g+1 only has to wait
// for the PV of half A of tile g, so it runs on the tensor core while the softmax
// is still on half B of tile g: the next scores are ready when the softmax wants
// them, and the two Q tiles' softmax passes overlap each other.  Every mbarrier
// wait is bounded; on a timeout the CTA raises HYPERION_DEVERR_WAIT_TIMEOUT, lets
// in-flight copies and MMAs land, frees TMEM and exits.
#pragma once

#include "common.cuh"
#include "tcgen05.cuh"

namespace hyp {
namespace tile {

constexpr int kRows = 128;
constexpr int kQTiles = 2;
constexpr int kChunk = kRows * kQTiles;
constexpr int kKeys = 128;  // keys per KV tile
constexpr int kRawStages = 2;
constexpr int kKvStages = 3;
constexpr int kMmaWarp = 8;  // warps 8 and 9: the MMA issuers of Q tiles 0 and 1
constexpr int kLoadWarp = 10;
constexpr int kConvWarp0 = 11;
constexpr int kConvWarps = 4;
constexpr int kSchedWarp = kConvWarp0 + kConvWarps;  // 15
constexpr int kThreads = 32 * (kSchedWarp + 1);        // 512
constexpr int kSchedConsumers = 4 * kQTiles + kQTiles + kConvWarps + 1;  // warps that read each unit
constexpr uint32_t kTmemCols = 512;
constexpr int kKTileBytes = kKeys * 128;      // e4m3 +-1, K-major SW128
constexpr int kVTileBytes = kKeys * 256;      // f16, MN-major SW128: two 64-dim blocks
constexpr int kVBlockBytes = kKeys * 128;     // one 64-dim block (LBO of the V descriptor)
// Lazy rescale threshold: P = exp(s - m) may grow to 2^8 before the running max
// is moved (8 / log2(e) in score units), well inside the f16 range of P.
constexpr float kTauS = 5.545177444479562f;

struct UnitInfo {
  int kind;     // 0 stop, 1 work
  int entry0;   // first work item of the chunk
  int n_entries;
  int seg_lo;   // rows [seg_lo, seg_hi) of the chunk belong to this unit
  int seg_hi;
  int bh;
  int ctx;      // clamped context length of bh
  int kv_len;   // keys [0, kv_len) are loaded
  int n_tiles;
  int kv;       // KV row of bh (bh / kv_group), resolved once per unit
  float vs;     // V scale of the unit
  int pad;
};

struct Smem {
  alignas(1024) uint8_t q[kQTiles][kRows * 128];
  alignas(1024) uint8_t kt[kKvStages][kKTileBytes];
  alignas(1024) uint8_t vt[kKvStages][kVTileBytes];
  alignas(128) uint8_t raw_k[kRawStages][kKeys * 16];
  alignas(128) uint8_t raw_v[kRawStages][kKeys * 128];
  uint32_t raw_mask[kRawStages][4];
  uint32_t kv_mask[kKvStages][4];
  UnitInfo unit[2];
  alignas(8) uint64_t sched_full[2];
  alignas(8) uint64_t sched_empty[2];
  alignas(8) uint64_t raw_full[kRawStages];
  alignas(8) uint64_t raw_empty[kRawStages];
  alignas(8) uint64_t kv_full[kKvStages];
  alignas(8) uint64_t kv_empty[kKvStages];
  alignas(8) uint64_t q_full;
  alignas(8) uint64_t q_empty;
  alignas(8) uint64_t s_full[kQTiles][2];  // [tile][half]: S of that half of the next KV tile
  alignas(8) uint64_t p_full[kQTiles][2];  // [tile][half]: P of that half written
  alignas(8) uint64_t o_full[kQTiles];
  alignas(8) uint64_t o_empty[kQTiles];
  alignas(8) uint64_t drain[kQTiles];
  uint32_t tmem_base;
  WaitCtl ctl;  // abort flag and wait bound of the CTA
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + alignment slack of the dynamic base

// 16 sign bits -> 16 e4m3 bytes: bit 1 -> +1.0 (0x38), bit 0 -> -1.0 (0xB8).  The
// multiply spreads the 4 bits of a nibble to bit 7 of 4 bytes (no carries: the
// partial products are 7 bits apart).
__device__ __forceinline__ uint4 expand16(uint32_t b) {
  uint4 o;
  o.x = (((b & 0xFu) * 0x10204080u) & 0x80808080u) ^ 0xB8B8B8B8u;
  o.y = ((((b >> 4) & 0xFu) * 0x10204080u) & 0x80808080u) ^ 0xB8B8B8B8u;
  o.z = ((((b >> 8) & 0xFu) * 0x10204080u) & 0x80808080u) ^ 0xB8B8B8B8u;
  o.w = ((((b >> 12) & 0xFu) * 0x10204080u) & 0x80808080u) ^ 0xB8B8B8B8u;
  return o;
}

// Four FP8 codes (dims d .. d+3) -> two f16x2 words, each value the reference's
// decode / 256, in the order {d, d+2}, {d+1, d+3}: V tiles hold every group of 4
// dims as d, d+2, d+1, d+3, so O's TMEM columns come out in that order too and the
// epilogue swaps them back (register renaming, no instruction).
__device__ __forceinline__ void fp8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = fp8x2_even_to_f16x2_div256(w);  // {b0, b2}
  hi = fp8x2_odd_to_f16x2_div256(w);   // {b1, b3}
}

// O columns of one 16-column chunk in dim order: columns hold dims d, d+2, d+1, d+3.
__device__ __forceinline__ void dims_in_order(float (&f)[16]) {
#pragma unroll
  for (int g = 0; g < 16; g += 4) {
    const float t = f[g + 1];
    f[g + 1] = f[g + 2];
    f[g + 2] = t;
  }
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Byte offset of 16-byte chunk `c` of row `r` in a 128B-swizzled tile of 128-byte rows.
__device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t c) {
  return (r >> 3) * 1024u + (r & 7u) * 128u + ((c ^ (r & 7u)) << 4);
}

// One 32-byte store (8 words), dst 32-byte aligned: a whole L2 sector per lane.
__device__ __forceinline__ void st_global_v8(void* dst, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// Stores 16 consecutive output values of one row (f32, bf16 or f16).  With a
// 32-byte aligned O (`sectors`) each 32 bytes go out as one store.
template <int kDtype>
__device__ __forceinline__ void store_row16(void* o, long long base, const float (&v)[16], bool sectors) {
  uint32_t w[16];
  constexpr int kWords = (kDtype == HYPERION_DTYPE_F32) ? 16 : 8;
  if constexpr (kDtype == HYPERION_DTYPE_F32) {
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if constexpr (kDtype == HYPERION_DTYPE_BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        w[i] = pack_f16x2(v[2 * i], v[2 * i + 1]);
      }
    }
  }
  uint32_t* dst = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(o) + base * (kDtype == HYPERION_DTYPE_F32 ? 4 : 2));
  if (sectors) {
#pragma unroll
    for (int j = 0; j < kWords; j += 8) {
      const uint32_t piece[8] = {w[j], w[j + 1], w[j + 2], w[j + 3], w[j + 4], w[j + 5], w[j + 6], w[j + 7]};
      st_global_v8(dst + j, piece);
    }
  } else {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < kWords; j += 4) d4[j / 4] = make_uint4(w[j], w[j + 1], w[j + 2], w[j + 3]);
  }
}

// Epilogue of one row: O = acc * scale from TMEM to global memory (and to every peer
// copy of O, same index), 16 columns at a time.
template <int kDtype>
__device__ __forceinline__ void store_o_row(const FwdParams& p, long long o_base, uint32_t o_col, float scale,
                                            bool row_ok) {
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    uint32_t v[16];
    tc::ld16(o_col + 16 * c, v);
    tc::ld_wait();
    if (row_ok) {
      float f[16];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const float2 t = __fmul2_rn(make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])),
                                    make_float2(scale, scale));
        f[i] = t.x;
        f[i + 1] = t.y;
      }
      dims_in_order(f);
      store_row16<kDtype>(p.o, o_base + 16 * c, f, p.o_align32);
      for (int k = 0; k < p.n_o_peers; ++k) store_row16<kDtype>(p.o_peers[k], o_base + 16 * c, f, p.o_align32);
    }
  }
}

__device__ __forceinline__ void store_zero_row(const FwdParams& p, long long o_base) {
  float z[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) z[i] = 0.f;
#pragma unroll 1
  for (int k = -1; k < p.n_o_peers; ++k) {
    void* o = k < 0 ? p.o : p.o_peers[k];
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      if (p.o_dtype == HYPERION_DTYPE_F32) {
        store_row16<HYPERION_DTYPE_F32>(o, o_base + 16 * c, z, p.o_align32);
      } else if (p.o_dtype == HYPERION_DTYPE_BF16) {
        store_row16<HYPERION_DTYPE_BF16>(o, o_base + 16 * c, z, p.o_align32);
      } else {
        store_row16<HYPERION_DTYPE_F16>(o, o_base + 16 * c, z, p.o_align32);
      }
    }
  }
}

// Valid-key bits of 16-key chunk h (keys kbase + 16h ..) for a row whose keys end at row_end.
__device__ __forceinline__ uint32_t chunk_bits(const uint32_t (&mk)[4], int h, int kbase, int row_end) {
  const int lim = row_end - kbase - 16 * h;
  const uint32_t lm = lim >= 16 ? 0xFFFFu : (lim <= 0 ? 0u : ((1u << lim) - 1u));
  return (mk[h >> 1] >> (16 * (h & 1))) & lm;
}

// Max of this thread's row over the 128 S columns of the tile (raw integer scores),
// two 16-column loads in flight per wait.
template <bool kMasked>
__device__ __forceinline__ float row_tile_max(uint32_t s_col, const uint32_t (&mk)[4], int kbase, int row_end) {
  float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll 1
  for (int h = 0; h < 8; h += 2) {
    uint32_t va[16], vb[16];
    tc::ld16(s_col + 16 * h, va);
    tc::ld16(s_col + 16 * (h + 1), vb);
    tc::ld_wait_regs(va);
    tc::ld_wait_regs(vb);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint32_t(&v)[16] = q ? vb : va;
      const uint32_t bits = kMasked ? chunk_bits(mk, h + q, kbase, row_end) : 0xFFFFu;
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        float x0 = __uint_as_float(v[i]), x1 = __uint_as_float(v[i + 1]);
        float x2 = __uint_as_float(v[i + 2]), x3 = __uint_as_float(v[i + 3]);
        if (kMasked) {
          x0 = ((bits >> i) & 1u) ? x0 : -INFINITY;
          x1 = ((bits >> (i + 1)) & 1u) ? x1 : -INFINITY;
          x2 = ((bits >> (i + 2)) & 1u) ? x2 : -INFINITY;
          x3 = ((bits >> (i + 3)) & 1u) ? x3 : -INFINITY;
        }
        a0 = fmaxf(a0, x0);
        a1 = fmaxf(a1, x1);
        a2 = fmaxf(a2, x2);
        a3 = fmaxf(a3, x3);
      }
    }
  }
  return fmaxf(fmaxf(a0, a1), fmaxf(a2, a3));
}

// The weight exp(|c| (S - S_m)) of an integer score S (exact in f32) relative to the
// row's integer maximum S_m, on the exponential unit as 2^(S*k2 + bias) with
// bias = -S_m*k2.
struct PExp {
  float k2, bias;
};

__device__ __forceinline__ float pexp_mufu(uint32_t s, const PExp& x) {
  return ex2_approx(fmaf(__uint_as_float(s), x.k2, x.bias));
}

// Two weights from two scores with one packed f32x2 FMA (half the FMA-pipe
// instructions of the softmax's exponent arguments) and two exponentials.
__device__ __forceinline__ void pexp2(uint32_t s0, uint32_t s1, const PExp& x, float& e0, float& e1) {
  const float2 t = __ffma2_rn(make_float2(__uint_as_float(s0), __uint_as_float(s1)), make_float2(x.k2, x.k2),
                              make_float2(x.bias, x.bias));
  e0 = ex2_approx(t.x);
  e1 = ex2_approx(t.y);
}

// Weights of one 16-column chunk.
__device__ __forceinline__ void p_exp16(const uint32_t (&v)[16], const PExp& x, float (&e)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i += 2) pexp2(v[i], v[i + 1], x, e[i], e[i + 1]);
}

// Finishes chunk h (exponentials in `e`: mask, add to l[], pack to f16 pairs, store
// over columns [8h, 8h+8) of S) while computing the exponentials of the next chunk
// (`vn` -> `en`) pair by pair: the exponential unit takes one warp instruction per
// 8 cycles, and the finishing work of chunk h fills the issue slots in between.
template <bool kMasked, bool kNext>
__device__ __forceinline__ void p_step(uint32_t s_col, int h, float (&e)[16], uint32_t bits, const uint32_t (&vn)[16],
                                       float (&en)[16], const PExp& x, float2& l) {
  uint32_t pk[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (kNext) pexp2(vn[2 * i], vn[2 * i + 1], x, en[2 * i], en[2 * i + 1]);
    float e0 = e[2 * i], e1 = e[2 * i + 1];
    if (kMasked) {
      e0 = ((bits >> (2 * i)) & 1u) ? e0 : 0.f;
      e1 = ((bits >> (2 * i + 1)) & 1u) ? e1 : 0.f;
    }
    l = __fadd2_rn(l, make_float2(e0, e1));
    pk[i] = pack_f16x2(e0, e1);
  }
  tc::st8(s_col + 8 * h, pk);
}

// P = exp(|c| (S - S_m)) for this thread's row over one 64-key half of the tile (S
// at s_col, 16-key chunks c0 .. c0+3 of the tile); returns sum(P).  While chunk h is
// finished, the exponentials of chunk h+1 run and the TMEM load of chunk h+2 is in
// flight.  P of chunk h goes to columns [8h, 8h+8) of the half, over S already read.
template <bool kMasked>
__device__ __forceinline__ float row_half_p(uint32_t s_col, const uint32_t (&mk)[4], int c0, int kbase, int row_end,
                                           const PExp& x) {
  float2 l = make_float2(0.f, 0.f);
  uint32_t va[16], vb[16];
  float ea[16], eb[16];
  tc::ld16(s_col, va);
  tc::ld16(s_col + 16, vb);
  tc::ld_wait_regs(va);
  tc::ld_wait_regs(vb);
  p_exp16(va, x, ea);
  tc::ld16(s_col + 32, va);
  p_step<kMasked, true>(s_col, 0, ea, kMasked ? chunk_bits(mk, c0, kbase, row_end) : 0xFFFFu, vb, eb, x, l);
  tc::ld_wait_regs(va);
  tc::ld16(s_col + 48, vb);
  p_step<kMasked, true>(s_col, 1, eb, kMasked ? chunk_bits(mk, c0 + 1, kbase, row_end) : 0xFFFFu, va, ea, x, l);
  tc::ld_wait_regs(vb);
  p_step<kMasked, true>(s_col, 2, ea, kMasked ? chunk_bits(mk, c0 + 2, kbase, row_end) : 0xFFFFu, vb, eb, x, l);
  p_step<kMasked, false>(s_col, 3, eb, kMasked ? chunk_bits(mk, c0 + 3, kbase, row_end) : 0xFFFFu, va, ea, x, l);
  return l.x + l.y;
}

// Chunks of a masked 64-key half that the warp computes: one past the last 16-key
// chunk in which any of its 32 rows attends a key (a warp-uniform count, 0-4).  On
// the causal diagonal the later chunks are masked for every row of a warp: for the
// first Q tile of a unit the whole last tile, and three chunks in eight of its
// diagonal tile on average.
__device__ __forceinline__ int half_chunks(const uint32_t (&mk)[4], int c0, int kbase, int row_end) {
  int n = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    if (__any_sync(0xffffffffu, chunk_bits(mk, c0 + c, kbase, row_end) != 0u)) n = c + 1;
  return n;
}

// The masked half with only its first `nch` chunks computed (nch < 4), one chunk
// after the other; the weights of the other chunks are zero, stored over their S
// columns.  Returns sum(P).
__device__ __noinline__ float row_half_p_prefix(uint32_t s_col, const uint32_t (&mk)[4], int c0, int kbase,
                                               int row_end, const PExp& x, int nch) {
  float2 l = make_float2(0.f, 0.f);
#pragma unroll 1
  for (int h = 0; h < nch; ++h) {
    uint32_t v[16];
    float e[16];
    tc::ld16(s_col + 16 * h, v);
    tc::ld_wait_regs(v);
    p_exp16(v, x, e);
    p_step<true, false>(s_col, h, e, chunk_bits(mk, c0 + h, kbase, row_end), v, e, x, l);
  }
  const uint32_t z[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll 1
  for (int h = nch; h < 4; ++h) tc::st8(s_col + 8 * h, z);
  return l.x + l.y;
}

// O row *= alpha (lanes that need no rescale pass alpha = 1).
__device__ __forceinline__ void rescale_row(uint32_t o_col, float alpha) {
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    uint32_t v[16];
    tc::ld16(o_col + 16 * c, v);
    tc::ld_wait_regs(v);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
    tc::st16(o_col + 16 * c, v);
  }
  tc::st_wait();
}

// Debug export: the integer score of every key this row attends in the tile.
__device__ __noinline__ void debug_row_scores(const FwdParams& p, uint32_t s_col, const uint32_t (&mk)[4], int kbase,
                                              int row_end, int item) {
  const bool flip = p.inv_sqrt_d < 0.f;
#pragma unroll 1
  for (int h = 0; h < 8; ++h) {
    uint32_t v[16];
    tc::ld16(s_col + 16 * h, v);
    tc::ld_wait_regs(v);
    const uint32_t bits = chunk_bits(mk, h, kbase, row_end);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if ((bits >> i) & 1u) {
        const int x = (int)__uint_as_float(v[i]);
        p.debug_scores[(long long)item * p.debug_ld + kbase + 16 * h + i] = flip ? -x : x;
      }
    }
  }
}

template <bool kDebug>
__global__ void __launch_bounds__(kThreads, 1) tile_fwd_kernel(FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_chunks = (p.total_work + kChunk - 1) / kChunk;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.sched_full[i], 1);
      mbar_init(&sm.sched_empty[i], kSchedConsumers);
    }
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(&sm.raw_full[i], 1);
      mbar_init(&sm.raw_empty[i], kConvWarps);
    }
    for (int i = 0; i < kKvStages; ++i) {
      mbar_init(&sm.kv_full[i], kConvWarps);
      mbar_init(&sm.kv_empty[i], kQTiles);  // a commit from each MMA issuer
    }
    mbar_init(&sm.q_full, kConvWarps);
    mbar_init(&sm.q_empty, kQTiles);
    for (int t = 0; t < kQTiles; ++t) {
      for (int h = 0; h < 2; ++h) {
        mbar_init(&sm.s_full[t][h], 1);
        mbar_init(&sm.p_full[t][h], 4);
      }
      mbar_init(&sm.o_full[t], 1);
      mbar_init(&sm.o_empty[t], 4);
      mbar_init(&sm.drain[t], 1);
    }
    sm.ctl.flag = 0;
    sm.ctl.limit = p.wait_cycles;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  volatile WaitCtl* abort = &sm.ctl;

  if (warp == kSchedWarp) {
    // ================================================================ scheduler
    uint32_t uc = 0;
    const long long cap = (long long)p.num_blocks * p.block_size;
    // Ticket order: in a (bh, q_idx)-ordered worklist chunk c holds q rows
    // [256*(c % cpb), ...) of its bh, and causal cost grows with that position.
    // Tickets walk the positions from the last to the first, all bh at each
    // position, so the most expensive chunks go first and the cheap ones fill
    // the tail.  When the KV of all bh rows would not stay in L2, the bh rows are
    // taken in groups of p.ticket_group, one group after the other, each walked
    // that way: the units running at any time then read the KV of one group, which
    // L2 holds, and the tail still ends on the cheapest chunks.  Any worklist
    // order stays correct; only the balance and the L2 reuse depend on it.
    const int cpb = max(1, (p.seq_q + kChunk - 1) / kChunk);
    const int groups = (n_chunks + cpb - 1) / cpb;
    const int n_tickets = groups * cpb;
    const int tg = (p.ticket_group > 0 && p.ticket_group < groups) ? p.ticket_group : groups;
    bool stop = false;
    while (!stop) {
      // Take the next ticket only once every role has started the previous unit:
      // the metadata of unit uc is then ready one unit ahead, and no CTA holds a
      // ticket it will not start soon (the tail stays balanced).
      if (uc >= 1 && !mbar_wait_warp(&sm.sched_empty[(uc - 1) & 1], ((uc - 1) >> 1) & 1, abort, p.err)) break;
      int c = -1;
      for (;;) {
        int t = 0;
        if (lane == 0) t = (int)atomicAdd(&p.counters[1], 1u);
        t = __shfl_sync(0xffffffffu, t, 0);
        if (t >= n_tickets) break;
        const int hg = t / (tg * cpb);                 // group of bh rows
        const int u = t - hg * (tg * cpb);             // ticket inside the group
        const int gs = min(tg, groups - hg * tg);      // rows in this group (the last may be short)
        const int qr = u / gs;
        const int g = hg * tg + (u - qr * gs);
        const int cand = g * cpb + (cpb - 1 - qr);
        if (cand < n_chunks) {
          c = cand;
          break;
        }
      }
      if (c < 0) {
        if (!mbar_wait_warp(&sm.sched_empty[uc & 1], ((uc >> 1) & 1) ^ 1, abort, p.err)) break;
        if (lane == 0) {
          sm.unit[uc & 1].kind = 0;
          mbar_arrive(&sm.sched_full[uc & 1]);
        }
        ++uc;
        break;
      }
      const int e0 = c * kChunk;
      const int ne = min(kChunk, p.total_work - e0);
      int seg_lo = 0;
      while (seg_lo < ne) {
        const int bh0 = __ldg(&p.worklist[e0 + seg_lo].y);
        int seg_hi = ne;
        for (int base = seg_lo + 1; base < ne; base += 32) {
          const int r = base + lane;
          const bool diff = (r < ne) && (__ldg(&p.worklist[e0 + r].y) != bh0);
          const unsigned b = __ballot_sync(0xffffffffu, diff);
          if (b) {
            seg_hi = base + __ffs(b) - 1;
            break;
          }
        }
        const bool bh_ok = bh0 >= 0 && bh0 < p.n_bh;
        int maxq = -1;
        for (int r = seg_lo + lane; r < seg_hi; r += 32) {
          const int qi = __ldg(&p.worklist[e0 + r].x);
          if (bh_ok && qi >= 0 && qi < p.seq_q) {
            maxq = max(maxq, qi);
          } else {
            raise_error(p.err, HYPERION_DEVERR_BAD_ITEM);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) maxq = max(maxq, __shfl_xor_sync(0xffffffffu, maxq, o));
        if (!bh_ok || maxq < 0) {
          seg_lo = seg_hi;
          continue;
        }
        const int kv0 = kv_of(p, bh0);
        int ctx = __ldg(p.ctx_lens + kv0);
        if (ctx < 0) {
          if (lane == 0) raise_error(p.err, HYPERION_DEVERR_NEG_CTX);
          ctx = 0;
        }
        if ((long long)ctx > cap) {
          if (lane == 0) raise_error(p.err, HYPERION_DEVERR_CTX_OVERFLOW);
          ctx = (int)cap;
        }
        const int kv_len = p.causal ? min(ctx, maxq + 1) : ctx;
        const int n_tiles = (kv_len + kKeys - 1) / kKeys;
        if (!mbar_wait_warp(&sm.sched_empty[uc & 1], ((uc >> 1) & 1) ^ 1, abort, p.err)) {
          stop = true;
          break;
        }
        if (lane == 0) {
          UnitInfo& u = sm.unit[uc & 1];
          u.kind = 1;
          u.entry0 = e0;
          u.n_entries = ne;
          u.seg_lo = seg_lo;
          u.seg_hi = seg_hi;
          u.bh = bh0;
          u.kv = kv0;
          u.vs = (p.v_scale_mode == 0) ? __ldg(p.v_scale) : __ldg(p.v_scale + (kv0 % p.v_scale_numel));
          u.ctx = ctx;
          u.kv_len = kv_len;
          u.n_tiles = n_tiles;
          mbar_arrive(&sm.sched_full[uc & 1]);
        }
        ++uc;
        seg_lo = seg_hi;
      }
    }
  } else if (warp == kLoadWarp) {
    // ================================================================ loader
    const uint64_t pol = policy_evict_last();
    // Pages of a tile by shifts when the page size is a power of two (every paged
    // pool in practice, and the contiguous layout of a power-of-two context): an
    // integer division by a run-time value costs this warp's per-tile chain, which
    // bounds the kernel, a few dozen cycles.
    const int bs = p.block_size;
    const bool bs_pow2 = (bs & (bs - 1)) == 0;
    const int bs_shift = __ffs(bs) - 1;
    uint32_t uc = 0, rit = 0;
    bool stop = false;
    while (!stop) {
      if (!mbar_wait_warp(&sm.sched_full[uc & 1], (uc >> 1) & 1, abort, p.err)) break;
      const UnitInfo u = sm.unit[uc & 1];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.sched_empty[uc & 1]);
      ++uc;
      if (u.kind == 0) break;
      {
        const int kv0 = u.kv;
        const int kv_len = u.kv_len;
        const int n_tiles = u.n_tiles;
        for (int j = 0; j < n_tiles; ++j) {
          const int r = rit % kRawStages;
          if (!mbar_wait_warp(&sm.raw_empty[r], ((rit / kRawStages) & 1) ^ 1, abort, p.err)) {
            stop = true;
            break;
          }
          const int k0 = j * kKeys;
          const int n = min(kKeys, kv_len - k0);
          const int p0 = bs_pow2 ? (k0 >> bs_shift) : k0 / bs;
          const int np = (bs_pow2 ? ((k0 + n - 1) >> bs_shift) : (k0 + n - 1) / bs) - p0 + 1;
          uint32_t bytes = 0;
          uint32_t mk[4] = {0u, 0u, 0u, 0u};
          for (int i = lane; i < np; i += 32) {
            const int page = p0 + i;
            const int lo = max(k0, page * bs) - k0;
            const int hi = min(k0 + n, (page + 1) * bs) - k0;
            if (page_block_id_kv(p, kv0, page) >= 0) {
              bytes += (uint32_t)(hi - lo) * (16u + 128u);
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                const int a = max(lo, 32 * w), b = min(hi, 32 * w + 32);
                if (a < b) mk[w] |= ((b - a == 32) ? 0xFFFFFFFFu : ((1u << (b - a)) - 1u)) << (a - 32 * w);
              }
            } else {
              raise_error(p.err, HYPERION_DEVERR_BAD_BLOCK);
            }
          }
          // One warp reduction per word (redux.sync), not a chain of shuffles: this
          // warp's per-tile latency lies on the kernel's critical path.
          bytes = __reduce_add_sync(0xffffffffu, bytes);
#pragma unroll
          for (int w = 0; w < 4; ++w) mk[w] = __reduce_or_sync(0xffffffffu, mk[w]);
          // Test hook: the raw stage numbered fault_stage is left unarmed, with no
          // copy in flight on it, so the converters' wait for it runs out.
          const bool armed = (int)rit != p.fault_stage;
          if (lane == 0 && armed) {
#pragma unroll
            for (int w = 0; w < 4; ++w) sm.raw_mask[r][w] = mk[w];
            if (bytes) {
              mbar_arrive_expect_tx(&sm.raw_full[r], bytes);
            } else {
              mbar_arrive(&sm.raw_full[r]);
            }
          }
          __syncwarp();
          for (int i = lane; armed && i < np; i += 32) {
            const int page = p0 + i;
            const int lo = max(k0, page * bs);
            const int hi = min(k0 + n, (page + 1) * bs);
            const long long id = page_block_id_kv(p, kv0, page);
            if (id >= 0) {
              const long long slot0 = id * bs + (lo - page * bs);
              const uint32_t cnt = (uint32_t)(hi - lo);
              bulk_g2s_stream(&sm.raw_k[r][(lo - k0) * 16], p.k + slot0 * 4, cnt * 16u, &sm.raw_full[r], pol);
              bulk_g2s_stream(&sm.raw_v[r][(lo - k0) * 128], p.v + slot0 * 128, cnt * 128u, &sm.raw_full[r], pol);
            }
          }
          ++rit;
        }
      }
    }
    if (abort->flag && lane == 0) {
      for (uint32_t i = (rit > (uint32_t)kRawStages ? rit - kRawStages : 0u); i < rit; ++i)
        mbar_drain(&sm.raw_full[i % kRawStages], (i / kRawStages) & 1, p.wait_cycles);
    }
  } else if (warp >= kConvWarp0 && warp < kConvWarp0 + kConvWarps) {
    // ================================================================ converters
    const int ct = threadIdx.x - 32 * kConvWarp0;  // 0..127
    uint32_t uc = 0, rit = 0, kvit = 0, uq = 0;
    const uint32_t q_base = smem_u32(&sm.q[0][0]);
    for (;;) {
      if (!mbar_wait_warp(&sm.sched_full[uc & 1], (uc >> 1) & 1, abort, p.err)) break;
      const UnitInfo u = sm.unit[uc & 1];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.sched_empty[uc & 1]);
      ++uc;
      if (u.kind == 0) break;
      if (u.n_tiles == 0) continue;
      // ---- Q rows of the unit -> e4m3 +-1, K-major SW128 (a negative inv_sqrt_d is
      // folded in by flipping every bit: the scores change sign).  The work items and
      // the sign bits are loaded before the wait for the Q buffer: the converters
      // reach this point tiles before the last QK of the previous unit frees it, so
      // the two dependent global reads are done by then instead of delaying the
      // next unit's first QK.
      uint4 qbits[kQTiles];
#pragma unroll
      for (int i = 0; i < kQTiles; ++i) {
        const int r = i * kRows + ct;
        qbits[i] = make_uint4(0u, 0u, 0u, 0u);
        if (r >= u.seg_lo && r < u.seg_hi) {
          const int qi = __ldg(&p.worklist[u.entry0 + r].x);
          if (qi >= 0 && qi < p.seq_q)
            qbits[i] = __ldg(reinterpret_cast<const uint4*>(p.q + ((long long)u.bh * p.seq_q + qi) * 4));
        }
      }
      if (!mbar_wait_warp(&sm.q_empty, (uq & 1) ^ 1, abort, p.err)) break;
#pragma unroll
      for (int i = 0; i < kQTiles; ++i) {
        uint4 bits = qbits[i];
        if (p.inv_sqrt_d < 0.f) bits = make_uint4(~bits.x, ~bits.y, ~bits.z, ~bits.w);
        const uint32_t words[4] = {bits.x, bits.y, bits.z, bits.w};
        const uint32_t tb = q_base + i * (kRows * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_shared_v4(tb + sw128_off(ct, c), expand16((words[c >> 1] >> (16 * (c & 1))) & 0xFFFFu));
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.q_full);
      ++uq;
      // ---- KV tiles
      bool ab = false;
      for (int j = 0; j < u.n_tiles; ++j) {
        const int r = rit % kRawStages;
        const int s = kvit % kKvStages;
        if (!mbar_wait_warp(&sm.raw_full[r], (rit / kRawStages) & 1, abort, p.err) ||
            !mbar_wait_warp(&sm.kv_empty[s], ((kvit / kKvStages) & 1) ^ 1, abort, p.err)) {
          ab = true;
          break;
        }
        // K: thread ct owns key ct (16 bytes of sign bits -> 128 e4m3 bytes).
        {
          const uint4 kb = *reinterpret_cast<const uint4*>(&sm.raw_k[r][ct * 16]);
          const uint32_t words[4] = {kb.x, kb.y, kb.z, kb.w};
          const uint32_t tb = smem_u32(&sm.kt[s][0]);
#pragma unroll
          for (int c = 0; c < 8; ++c)
            st_shared_v4(tb + sw128_off(ct, c), expand16((words[c >> 1] >> (16 * (c & 1))) & 0xFFFFu));
        }
        // V: 2048 (key, 8-dim chunk) tasks, 16 per thread in two batches of 8 loads;
        // 16 lanes cover one key row.
        {
          const uint32_t vb = smem_u32(&sm.vt[s][0]);
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {
            uint2 w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int task = ct + 128 * (8 * half + i);
              w[i] = *reinterpret_cast<const uint2*>(&sm.raw_v[r][(task >> 4) * 128 + (task & 15) * 8]);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int task = ct + 128 * (8 * half + i);
              const int key = task >> 4;
              const int c8 = task & 15;
              uint4 o;
              fp8x4_to_f16x4(w[i].x, o.x, o.y);
              fp8x4_to_f16x4(w[i].y, o.z, o.w);
              st_shared_v4(vb + (c8 >> 3) * (uint32_t)kVBlockBytes + sw128_off(key, c8 & 7), o);
            }
          }
        }
        if (ct < 4) sm.kv_mask[s][ct] = sm.raw_mask[r][ct];
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.kv_full[s]);
          mbar_arrive(&sm.raw_empty[r]);
        }
        ++rit;
        ++kvit;
      }
      if (ab) break;
    }
  } else if (warp >= kMmaWarp && warp < kMmaWarp + kQTiles) {
    // ================================================================ MMA issuers
    // Warp kMmaWarp + t issues every MMA and commit of Q tile t from one thread (a
    // tcgen05.commit tracks the MMAs of the thread that issues it, and the MMAs of
    // one thread run in order).  Per KV tile g and half h: PV(g, h) as soon as the
    // softmax has written P of that half, then QK(g+1, h) into the same S columns.
    const int t = warp - kMmaWarp;
    if (lane == 0) {
      uint32_t uc = 0, kvit = 0, uq = 0, uo = 0;
      const uint32_t q_base = smem_u32(&sm.q[0][0]);
      const uint32_t k_base = smem_u32(&sm.kt[0][0]);
      const uint32_t v_base = smem_u32(&sm.vt[0][0]);
      const uint64_t q_desc = tc::sw128_desc(q_base, 16, 1024);
      const uint64_t k_desc = tc::sw128_desc(k_base, 16, 1024);
      const uint64_t v_desc = tc::sw128_desc(v_base, kVBlockBytes, 1024);
      const uint32_t s_tm = tmem + (uint32_t)(t * 256);
      const uint32_t o_tm = s_tm + 128;
      const uint64_t ad = q_desc + (uint64_t)(t * (kRows * 128) / 16);
      bool ab = false;
      // S half h = Q_t K(stage s, keys 64h .. 64h+63)^T  (M 128, N 64, K 128 in 4 steps)
      auto qk = [&](int s, int h) {
        const uint64_t bd = k_desc + (uint64_t)((s * kKTileBytes + h * 64 * 128) / 16);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_f8f6f4_ss(s_tm + 64u * h, ad + 2 * kk, bd + 2 * kk, tc::kIdescQK64, kk > 0 ? 1u : 0u);
      };
      // O_t (+)= P(half h) V(stage s, keys 64h .. 64h+63)  (M 128, N 128, K 64 keys in 4 steps)
      auto pv = [&](int s, int h, bool acc) {
        const uint64_t bd = v_desc + (uint64_t)(s * kVTileBytes / 16) + 128u * 4u * h;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_f16_ts(o_tm, s_tm + 64u * h + 8u * kk, bd + 128 * kk, tc::kIdescPV, (acc || kk > 0) ? 1u : 0u);
      };
      for (;;) {
        if (!mbar_wait(&sm.sched_full[uc & 1], (uc >> 1) & 1, abort, p.err)) break;
        const UnitInfo u = sm.unit[uc & 1];
        mbar_arrive(&sm.sched_empty[uc & 1]);
        ++uc;
        if (u.kind == 0) break;
        const int n = u.n_tiles;
        if (n == 0) continue;
        if (!mbar_wait(&sm.q_full, uq & 1, abort, p.err)) break;
        ++uq;
        int s = kvit % kKvStages;
        if (!mbar_wait(&sm.kv_full[s], (kvit / kKvStages) & 1, abort, p.err)) break;
        tc::fence_after_sync();
        qk(s, 0);
        tc::commit(&sm.s_full[t][0]);
        qk(s, 1);
        tc::commit(&sm.s_full[t][1]);
        if (n == 1) tc::commit(&sm.q_empty);
        for (int j = 0; j < n; ++j) {
          const uint32_t g = kvit + j;
          s = g % kKvStages;
          const uint32_t nxt = g + 1;
          const int s2 = nxt % kKvStages;
          // ---- half A
          if (!mbar_wait(&sm.p_full[t][0], g & 1, abort, p.err) ||
              (j == 0 && !mbar_wait(&sm.o_empty[t], (uo & 1) ^ 1, abort, p.err))) {
            ab = true;
            break;
          }
          tc::fence_after_sync();
          pv(s, 0, j > 0);
          if (j + 1 < n) {
            if (!mbar_wait(&sm.kv_full[s2], (nxt / kKvStages) & 1, abort, p.err)) {
              ab = true;
              break;
            }
            tc::fence_after_sync();
            qk(s2, 0);
            tc::commit(&sm.s_full[t][0]);
          }
          // ---- half B
          if (!mbar_wait(&sm.p_full[t][1], g & 1, abort, p.err)) {
            ab = true;
            break;
          }
          tc::fence_after_sync();
          pv(s, 1, true);
          if (j == n - 1) tc::commit(&sm.o_full[t]);
          tc::commit(&sm.kv_empty[s]);
          if (j + 1 < n) {
            qk(s2, 1);
            tc::commit(&sm.s_full[t][1]);
            if (j + 2 == n) tc::commit(&sm.q_empty);
          }
        }
        if (ab) break;
        kvit += n;
        ++uo;
      }
      // Every MMA issued must land before TMEM is released.
      tc::commit(&sm.drain[t]);
      mbar_drain(&sm.drain[t], 0, p.wait_cycles);
    }
    __syncwarp();
  } else {
    // ================================================================ softmax (warps 0-7)
    const int t = warp >> 2;         // Q tile
    const int wq = warp & 3;         // TMEM lane quarter
    const int row = wq * 32 + lane;  // row of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t s_col = tmem + lane_off + (uint32_t)(t * 256);
    const uint32_t o_col = s_col + 128;
    // A negative inv_sqrt_d is folded into Q (the converters flip its bits), so the
    // tile scores here are always multiplied by |inv_sqrt_d| and their max is a max.
    const float cabs = fabsf(p.inv_sqrt_d);
    const float k2 = cabs * kLog2e;
    // Running max from which on a row needs no max pass: (head_dim * |inv_sqrt_d|)
    // minus 11, so exp(s - m) <= e^11 < 2^15.9 for every possible score s.
    const float m_safe = 128.f * cabs - 11.0f;
    uint32_t uc = 0, kvit = 0, oc = 0;
    // The next unit is taken from its slot, and the global load of this row's q_idx
    // issued, before the current unit's epilogue (the scheduler publishes units one
    // ahead): the load's latency then hides behind the epilogue's stores.
    UnitInfo nu;
    int n_qi = -1;
    auto fetch = [&]() -> bool {
      if (!mbar_wait_warp(&sm.sched_full[uc & 1], (uc >> 1) & 1, abort, p.err)) return false;
      nu = sm.unit[uc & 1];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.sched_empty[uc & 1]);
      ++uc;
      const int r = t * kRows + row;
      n_qi = (nu.kind != 0 && r >= nu.seg_lo && r < nu.seg_hi) ? __ldg(&p.worklist[nu.entry0 + r].x) : -1;
      return true;
    };
    bool have = fetch();
    while (have) {
      const UnitInfo u = nu;
      if (u.kind == 0) break;
      const int r = t * kRows + row;
      const int q_idx = (n_qi >= 0 && n_qi < p.seq_q) ? n_qi : -1;
      const bool row_ok = q_idx >= 0;
      const int n_tiles = u.n_tiles;
      const int item = u.entry0 + r;
      const long long o_base = row_ok ? ((long long)u.bh * p.seq_q + q_idx) * 128 : 0;
      const int row_end = row_ok ? (p.causal ? min(u.ctx, q_idx + 1) : u.ctx) : 0;
      if (n_tiles == 0) {
        if (row_ok) store_zero_row(p, o_base);
        have = fetch();
        continue;
      }
      float m = -INFINITY, l = 0.f;
      int s_m = 0;  // integer score whose scaled value is m (0 while m = -inf)
      bool ab = false;
      for (int j = 0; j < n_tiles; ++j) {
        const uint32_t g = kvit;
        const int s = g % kKvStages;
        if (!mbar_wait_warp(&sm.s_full[t][0], g & 1, abort, p.err)) {
          ab = true;
          break;
        }
        uint32_t mk[4] = {0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu};
        if (!p.pages_all_valid) {
          // Page ids can fall outside the pool: read the tile's key mask (the
          // converters copied it before completing this phase of kv_full).
          if (!mbar_wait_warp(&sm.kv_full[s], (g / kKvStages) & 1, abort, p.err)) {
            ab = true;
            break;
          }
#pragma unroll
          for (int w = 0; w < 4; ++w) mk[w] = sm.kv_mask[s][w];
        }
        tc::fence_after_sync();
        const int k0 = j * kKeys;
        const bool full_a = (mk[0] & mk[1]) == 0xFFFFFFFFu && k0 + 64 <= row_end;
        const bool full_b = (mk[2] & mk[3]) == 0xFFFFFFFFu && k0 + kKeys <= row_end;
        const bool wfa = __all_sync(0xffffffffu, full_a);
        const bool wfb = __all_sync(0xffffffffu, full_b);
        const bool max_pass = !__all_sync(0xffffffffu, m >= m_safe);
        bool have_b = false;
        if (kDebug || max_pass) {
          // Both halves' scores are needed first.  S of half B ready also means the
          // PV of tile g-1 is done (it was issued before that QK), so O may be
          // rescaled here.
          if (!mbar_wait_warp(&sm.s_full[t][1], g & 1, abort, p.err)) {
            ab = true;
            break;
          }
          tc::fence_after_sync();
          have_b = true;
          if (kDebug) debug_row_scores(p, s_col, mk, k0, row_end, item);
        }
        if (max_pass) {
          // ---- max pass (first tiles of a row, or scores too large for a fixed m)
          const float mx = (wfa && wfb) ? row_tile_max<false>(s_col, mk, k0, row_end)
                                        : row_tile_max<true>(s_col, mk, k0, row_end);
          const float mt = (mx == -INFINITY) ? -INFINITY : mx * cabs;
          const bool need = mt > m + kTauS;
          const bool resc = need && (m != -INFINITY);
          const float alpha = resc ? ex2_approx((m - mt) * kLog2e) : 1.f;
          if (need) {
            m = mt;
            s_m = (int)mx;
          }
          l *= alpha;
          if (__any_sync(0xffffffffu, resc)) rescale_row(o_col, alpha);
        }
        // Once m >= m_safe every score is <= head_dim * |inv_sqrt_d| <= m + 11, so
        // P <= 2^15.9 fits f16 and the running max never has to move again.
        PExp x;
        x.k2 = k2;
        x.bias = -(float)s_m * k2;
        // ---- half A: keys 0-63, P over S columns 0-31
        if (wfa) {
          l += row_half_p<false>(s_col, mk, 0, k0, row_end, x);
        } else {
          const int nch = half_chunks(mk, 0, k0, row_end);
          l += nch == 4 ? row_half_p<true>(s_col, mk, 0, k0, row_end, x)
                        : row_half_p_prefix(s_col, mk, 0, k0, row_end, x, nch);
        }
        tc::st_wait();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[t][0]);
        // ---- half B: keys 64-127, P over S columns 64-95
        if (!have_b) {
          if (!mbar_wait_warp(&sm.s_full[t][1], g & 1, abort, p.err)) {
            ab = true;
            break;
          }
          tc::fence_after_sync();
        }
        if (wfb) {
          l += row_half_p<false>(s_col + 64, mk, 4, k0, row_end, x);
        } else {
          const int nch = half_chunks(mk, 4, k0, row_end);
          l += nch == 4 ? row_half_p<true>(s_col + 64, mk, 4, k0, row_end, x)
                        : row_half_p_prefix(s_col + 64, mk, 4, k0, row_end, x, nch);
        }
        tc::st_wait();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[t][1]);
        ++kvit;
      }
      if (ab) break;
      have = fetch();
      // ---- epilogue: O row = acc * 256 * vscale / l
      if (!mbar_wait_warp(&sm.o_full[t], oc & 1, abort, p.err)) break;
      ++oc;
      tc::fence_after_sync();
      const float vs = u.vs;
      const float scale = 256.f * vs * ((l > 1e-6f) ? 1.f / l : 1.f);
      if (p.o_dtype == HYPERION_DTYPE_BF16) {
        store_o_row<HYPERION_DTYPE_BF16>(p, o_base, o_col, scale, row_ok);
      } else if (p.o_dtype == HYPERION_DTYPE_F32) {
        store_o_row<HYPERION_DTYPE_F32>(p, o_base, o_col, scale, row_ok);
      } else {
        store_o_row<HYPERION_DTYPE_F16>(p, o_base, o_col, scale, row_ok);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.o_empty[t]);
    }
  }

  fence_out_peers(p);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// Sets the kernel's shared-memory limit and checks that one CTA fits on an SM.
// On failure `why` names the step.
inline int setup(int& ctas, int& smem, const char** why) {
  smem = (int)kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(tile_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tile_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return HYPERION_ERR_CUDA;
  }
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas, tile_fwd_kernel<false>, kThreads, smem);
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return HYPERION_ERR_CUDA;
  }
  if (ctas < 1) {
    *why = "occupancy calculator: no CTA of the tile kernel fits on an SM";
    return HYPERION_ERR_UNSUPPORTED;
  }
  ctas = 1;  // one CTA per SM: the kernel allocates all 512 TMEM columns
  return HYPERION_OK;
}

// KV bytes of all bh rows up to which the ticket order keeps every row in one
// group, and the KV bytes of one group beyond that: both well inside the 126 MB L2,
// which the Q rows and the O stores pass through as well.
constexpr double kTicketAllBytes = 96.0 * (1 << 20);
constexpr double kTicketGroupBytes = 48.0 * (1 << 20);

// bh rows per group of the tile kernel's ticket order (0: one group of all rows),
// from the KV capacity of a row (its keys at most block_size * num_blocks, K and V
// bytes per key, shared by kv_group query rows).
inline int ticket_group(const FwdParams& p) {
  const int n_chunks = (p.total_work + kChunk - 1) / kChunk;
  const int cpb = std::max(1, (p.seq_q + kChunk - 1) / kChunk);
  const int rows = (n_chunks + cpb - 1) / cpb;
  const double per_row = (double)p.block_size * p.num_blocks * (p.head_dim / 8 + p.head_dim) / std::max(p.kv_group, 1);
  if (per_row <= 0.0 || rows * per_row <= kTicketAllBytes) return 0;
  return std::max(1, (int)(kTicketGroupBytes / per_row));
}

inline int launch(const FwdParams& p0, int n_sm, int ctas, int smem, cudaStream_t st, int* grid_out) {
  const int n_chunks = (p0.total_work + kChunk - 1) / kChunk;
  const int grid = std::min(n_chunks, n_sm * std::max(ctas, 1));
  if (grid <= 0) return HYPERION_OK;
  FwdParams p = p0;
  p.ticket_group = ticket_group(p0);
  if (p.debug_scores) {
    tile_fwd_kernel<true><<<grid, kThreads, smem, st>>>(p);
  } else {
    tile_fwd_kernel<false><<<grid, kThreads, smem, st>>>(p);
  }
  if (grid_out) *grid_out = grid;
  return HYPERION_OK;
}

}  // namespace tile
}  // namespace hyp
