// row_mma_kernel.cuh -- grouped-query decode with the P.V products on the tensor core.
//
// The grouped row kernel (row_group_kernel.cuh) streams a KV split once for the
// run of up to 4 query heads that share it, but does every w * v product on the
// CUDA cores (8 HFMA2 per key and lane for 4 queries), which leaves it issue-bound
// below the HBM roofline.  This kernel keeps its units, runs and producer and
// moves the products to tcgen05, reading the FP8 codes as they are:
//
//   O^T[d][n] += sum_k V^T[d][k] * P^T[n][k]     kind::f8f6f4, M = 128 dims,
//                                                 N = 48, K = 32 keys per MMA
//
//   A = V^T  the stage's FP8 codes, e4m3, straight from HBM: a tensor-map copy
//            with the 128-byte swizzle lays each 128-key stage out as the
//            MN-major operand (dims contiguous), with no pass over it;
//   B = P^T  the softmax weights, each split into three e4m3 pieces
//            x = h + m/16 + l/256 (x = 64 w <= 256), one 128-key row per
//            accumulator column n = 12 e + 3 j + piece (query j, epoch e), K-major;
//   D        f32 in TMEM, 128 lanes (dims) x 48 columns, two buffers, so the MMAs
//            of the next run start while the last one is read out.
//
// A stage is 128 keys: 16 KB of codes (the A operand itself), 2 KB of sign bits and
// the 6 KB P^T the consumers write; the MMAs' commit hands the stage back to the
// producer.  Roles (6 warps, 3 CTAs per SM):
//   warp 0    producer: the grouped kernels' tickets and runs, then per stage a
//             tensor-map copy per page piece of the codes and a bulk copy of the
//             sign bits (hyperion_fa3_production_final.py:402-411 for the pages);
//   warps 1-4 consumers; warp 1 + j owns query j of the run.  Per stage it scores
//             its query against the 128 keys (D - 2 popcount(q XOR k),
//             README.md:22), takes the softmax step and writes its three P^T rows.
//             At the end of a run the four read the accumulator, each its TMEM
//             lane quarter (32 dims of every query), and write the split's
//             (m, l, acc) or the finished row;
//   warp 5    lane 0 issues each stage's 4 MMAs and the commits.
//
// Softmax: the reference's online update (:544-572) with a lazy running max.  A
// query's m is set by its first stage with a valid key and moves only when a
// stage's max exceeds it by more than kTau = ln 4; the query then starts a new
// epoch, whose weights go to fresh accumulator columns, and the end of the run
// merges the columns with their factors exp(m_e - m).  No accumulator is rescaled
// in TMEM.  Every weight is then at most 4, so x = 64 w <= 256 fits e4m3 (448).
// The three pieces carry about 12 bits of a weight in e4m3's normal range and an
// absolute error below 2^-18 x (6e-8 w) under it, as an f16 weight would.  A
// query that would need a fifth epoch marks its run for the exact redo below.
// EXP_CLAMP (-80) never applies: with |inv_sqrt_d| <= 0.117 (the host's condition;
// the reference's 1/sqrt(128) is 0.088) every exponent is above -(2 D |c| + kTau).
//
// FP8 codes 0x7F / 0xFF: the tensor core reads them as NaN where the reference
// decodes +-480 (:122-141).  A NaN makes the query's accumulator columns
// non-finite; the run's split is then redone on the CUDA cores with the exact
// decode, keys read from global memory.  The rows of keys no query of the run may
// read (past the stage's last key, on a page outside the pool) are zeroed in
// shared memory before the MMAs, so only codes the reference reads can cause it.
#pragma once

#include <algorithm>
#include <climits>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "row_group_kernel.cuh"
#include "tcgen05.cuh"

namespace hyp {
namespace rmma {

constexpr int kD = 128;
constexpr int kW = kD / 32;                 // sign-bit words per row
constexpr int kKeys = 128;                  // keys per stage
constexpr int kStages = 3;
constexpr int kQ = row::kGroupMax;          // 4 queries per run
constexpr int kPieces = 3;                  // e4m3 pieces of a weight
constexpr int kEpochs = 4;
constexpr int kN = kQ * kPieces * kEpochs;  // 48 accumulator columns: n = 12 e + 3 j + piece
constexpr float kTau = 1.3862943611198906f;  // ln 4: weights <= 4
constexpr float kLog2XScale = 6.0f;         // x = 64 w <= 256 < 448 (e4m3 max)
constexpr int kConsumers = kQ;
constexpr int kMmaWarp = 1 + kConsumers;    // 5
constexpr int kThreads = 32 * (kMmaWarp + 1);
constexpr int kCtasPerSm = 3;
constexpr uint32_t kTmemCols = 128;         // two run buffers of kN columns
constexpr int kVBytes = kKeys * kD;         // codes of a stage: the A operand
constexpr int kKBytes = kKeys * kW * 4;
constexpr int kPBytes = kN * kKeys;         // P^T rows of a stage: the B operand
static_assert(kKeys == 128 && kD == 128, "a stage row of codes and a P^T row are one 128-byte swizzle row");

// Whether a call may take this kernel: head_dim 128, a per-tensor or per-head V
// scale, |inv_sqrt_d| small enough that random scores rarely need more epochs,
// pages the tensor-map boxes tile (one page per row, as in the contiguous layout;
// or 8 to 128 keys dividing 128; or a multiple of 128), a 16-byte aligned V pool
// of fewer than 2^32 rows.
inline bool fits(int head_dim, int v_scale_mode, float inv_sqrt_d, int block_size, int num_blocks, const void* v,
                 long long pool_rows) {
  const float c = inv_sqrt_d < 0.f ? -inv_sqrt_d : inv_sqrt_d;
  const bool pages =
      num_blocks == 1 || (block_size % kKeys == 0) || (block_size >= 8 && kKeys % block_size == 0);
  return head_dim == kD && v_scale_mode != 2 && 2.f * kD * c <= 30.f && pages &&
         (reinterpret_cast<uintptr_t>(v) & 15u) == 0 && pool_rows > 0 && pool_rows < (1LL << 32);
}

// Rows of one tensor-map box: a page, or a whole stage when pages are longer.
inline int box_rows(int block_size) { return block_size >= kKeys ? kKeys : block_size; }

struct StageHdr {
  int nkeys;         // keys of the stage (the last stage of a split may be shorter)
  int pad[3];
  uint32_t mask[4];  // bit k: key k of the stage is on a page inside the pool
};

struct Smem {
  alignas(1024) uint8_t v[kStages][kVBytes];   // A: codes, 128B-swizzled by the copy
  alignas(1024) uint8_t pt[kStages][kPBytes];  // B: weight pieces, 128B-swizzled
  alignas(128) uint8_t k[kStages][kKBytes];
  StageHdr hdr[kStages];
  row::RunSlot<kW> slot[2];
  float ep_m[2][kQ][kEpochs];  // [run parity][query][epoch]: m of the epoch, -inf unused
  float run_l[2][kQ];          // [run parity][query]: sum of x relative to the last m
  int run_bad;                 // number (1-based) of the last run to redo exactly
  alignas(8) uint64_t full[kStages];   // codes and sign bits landed (transaction bytes)
  alignas(8) uint64_t ready[kStages];  // P^T written, dead rows zeroed (4 consumer warps)
  alignas(8) uint64_t empty[kStages];  // the stage's MMAs done (commit)
  alignas(8) uint64_t run_full[2];
  alignas(8) uint64_t run_empty[2];
  alignas(8) uint64_t o_full[2];       // the run buffer's last MMA done (commit)
  alignas(8) uint64_t o_empty[2];      // the run buffer read out (4 consumer warps)
  alignas(8) uint64_t drain;
  alignas(8) uint64_t cbar;            // the consumer warps' end-of-run hand-off
  uint32_t tmem_base;
  WaitCtl ctl;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + alignment slack of the dynamic base

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// D - 2 popcount(q XOR k) of one 128-bit key row.
__device__ __forceinline__ int score16(const uint32_t (&q)[kW], uint4 k) {
  return kD - 2 * (__popc(q[0] ^ k.x) + __popc(q[1] ^ k.y) + __popc(q[2] ^ k.z) + __popc(q[3] ^ k.w));
}

// {a, b} -> two e4m3 codes (a in the low byte), round to nearest even, saturating.
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(a), "f"(b));
  return r;
}
// Two e4m3 codes (low 16 bits) -> their values as f32.
__device__ __forceinline__ void e4m3x2_to_f32(uint32_t c, float& a, float& b) {
  const uint32_t h = e4m3x2_to_f16x2_hw(c);
  a = f16_lo_to_f32(h);
  b = f16_hi_to_f32(h);
}

// Splits x0 .. x3 (each in [0, 256]) into three e4m3 pieces, x = h + m/16 + l/256,
// packed four keys to a word (key 0 in the low byte).
__device__ __forceinline__ void split4(const float (&x)[4], uint32_t& wh, uint32_t& wm, uint32_t& wl) {
  const uint32_t h01 = e4m3x2(x[0], x[1]), h23 = e4m3x2(x[2], x[3]);
  float a0, a1, a2, a3;
  e4m3x2_to_f32(h01, a0, a1);
  e4m3x2_to_f32(h23, a2, a3);
  const float r0 = (x[0] - a0) * 16.f, r1 = (x[1] - a1) * 16.f, r2 = (x[2] - a2) * 16.f, r3 = (x[3] - a3) * 16.f;
  const uint32_t m01 = e4m3x2(r0, r1), m23 = e4m3x2(r2, r3);
  e4m3x2_to_f32(m01, a0, a1);
  e4m3x2_to_f32(m23, a2, a3);
  const uint32_t l01 = e4m3x2((r0 - a0) * 16.f, (r1 - a1) * 16.f), l23 = e4m3x2((r2 - a2) * 16.f, (r3 - a3) * 16.f);
  wh = h01 | (h23 << 16);
  wm = m01 | (m23 << 16);
  wl = l01 | (l23 << 16);
}

// The tensor-map copy of one box of codes (pool rows [row, row + box)) into shared
// memory, completing on `bar`, with an L2 eviction hint.
__device__ __forceinline__ void tma_load_rows(uint32_t dst, const CUtensorMap* map, int row, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(row), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// One query's split recomputed on the CUDA cores with the reference's exact FP8
// decode, keys read from global memory: the path of a run whose accumulator met a
// 0x7F / 0xFF code or that ran out of epochs.  A warp; lane l owns dims 4l .. 4l+3.
// The first pass finds the exact max score, so every weight is at most 1.  Writes
// the partial (m, l, acc) or, unsplit, the finished row.
__device__ __noinline__ void redo_query(const FwdParams& p, const row::RunSlot<kW>& sl, int j, float vs) {
  const int lane = threadIdx.x & 31;
  const int bs = p.block_size;
  const int kend = min(sl.k_hi, sl.kv_end[j]);
  const float cabs = fabsf(p.inv_sqrt_d);
  const int sgn = p.inv_sqrt_d < 0.f ? -1 : 1;
  uint32_t qw[kW];
#pragma unroll
  for (int i = 0; i < kW; ++i) qw[i] = sl.q[j][i];
  int mx = INT_MIN;
  for (int key = sl.k_lo + lane; key < kend; key += 32) {
    const int page = key / bs;
    const long long id = page_block_id_kv(p, sl.kv, page);
    if (id < 0) continue;
    const uint32_t* kp = p.k + (id * bs + (key - page * bs)) * kW;
    mx = max(mx, sgn * sign_score<kW>(qw, kp));
  }
  mx = __reduce_max_sync(0xffffffffu, mx);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float l = 0.f;
  float m = -INFINITY;
  if (mx != INT_MIN) {
    m = (float)mx * cabs;
    for (int key = sl.k_lo; key < kend; ++key) {
      const int page = key / bs;
      const long long id = page_block_id_kv(p, sl.kv, page);
      if (id < 0) continue;
      const long long slot = id * bs + (key - page * bs);
      const float w = exp_clamped((float)(sgn * sign_score<kW>(qw, p.k + slot * kW)) * cabs - m);
      l += w;
      const uint32_t vb = __ldg(reinterpret_cast<const uint32_t*>(p.v + slot * kD) + lane);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = fmaf(w, fp8_bits_to_f32_scaled(vb >> (8 * i)) * kTwoPow120, acc[i]);
    }
  }
  if (p.n_split == 1) {
    const float inv_l = (l > 1e-6f) ? 1.f / l : 1.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      store_out_all(p, (long long)sl.orow[j] * kD + 4 * lane + i, acc[i] * vs * inv_l);
  } else {
    float* part = p.partials + ((long long)sl.item[j] * p.n_split + sl.split) * (2 + kD);
#pragma unroll
    for (int i = 0; i < 4; ++i) part[2 + 4 * lane + i] = acc[i] * vs;
    if (lane == 0) {
      part[0] = m;
      part[1] = l;
    }
  }
}

// The stages of one run: per 128 keys, a tensor-map copy of the codes per page
// piece (a box of box_rows keys; the whole stage when pages are longer) and a bulk
// copy of the sign bits, through the kStages ring full / empty.  Lane b handles box
// b of the stage.  `it` counts the stages armed.
__device__ __forceinline__ bool mma_stream(const FwdParams& p, Smem& sm, const CUtensorMap* vmap, uint32_t& it,
                                           int kv_r, int k_lo, int k_hi, uint64_t pol, volatile WaitCtl* abort) {
  const int lane = threadIdx.x & 31;
  const int bs = p.block_size;
  const int rows = bs >= kKeys ? kKeys : bs;  // keys of one box
  for (int k0 = k_lo; k0 < k_hi; k0 += kKeys) {
    const int s = it % kStages;
    if (!mbar_wait_warp(&sm.empty[s], ((it / kStages) & 1) ^ 1, abort, p.err)) return false;
    const int nk = min(kKeys, k_hi - k0);
    const int nbox = (nk + rows - 1) / rows;
    uint32_t bytes = 0;
    uint32_t mk[4] = {0u, 0u, 0u, 0u};
    long long src = -1;  // first pool row of this lane's box
    int cnt = 0;         // its keys inside the stage
    if (lane < nbox) {
      const int kb = k0 + rows * lane;
      const int page = kb / bs;
      const long long id = page_block_id_kv(p, kv_r, page);
      cnt = min(rows, k0 + nk - kb);
      if (id >= 0) {
        src = id * bs + (kb - page * bs);
        bytes = (uint32_t)rows * kD + (uint32_t)cnt * kW * 4;
        const int a = rows * lane, b = a + cnt;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int lo = max(a, 32 * w), hi = min(b, 32 * w + 32);
          if (lo < hi) mk[w] |= ((hi - lo == 32) ? 0xFFFFFFFFu : ((1u << (hi - lo)) - 1u)) << (lo - 32 * w);
        }
      } else {
        raise_error(p.err, HYPERION_DEVERR_BAD_BLOCK);
      }
    }
    bytes = __reduce_add_sync(0xffffffffu, bytes);
#pragma unroll
    for (int w = 0; w < 4; ++w) mk[w] = __reduce_or_sync(0xffffffffu, mk[w]);
    // Test hook: the stage numbered fault_stage is left unarmed, with no copy in
    // flight on it, so the consumers' wait for it runs out.
    const bool armed = (int)it != p.fault_stage;
    if (lane == 0 && armed) {
      sm.hdr[s].nkeys = nk;
#pragma unroll
      for (int w = 0; w < 4; ++w) sm.hdr[s].mask[w] = mk[w];
      if (bytes) {
        mbar_arrive_expect_tx(&sm.full[s], bytes);
      } else {
        mbar_arrive(&sm.full[s]);
      }
    }
    __syncwarp();
    if (armed && src >= 0) {
      tma_load_rows(smem_u32(&sm.v[s][rows * lane * kD]), vmap, (int)src, &sm.full[s], pol);
      bulk_g2s_stream(&sm.k[s][rows * lane * kW * 4], p.k + src * kW, (uint32_t)cnt * kW * 4, &sm.full[s], pol);
    }
    ++it;
  }
  return true;
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    row_mma_kernel(FwdParams p, int total_units, const __grid_constant__ CUtensorMap vmap) {
  // The split combine kernel is launched as a programmatic dependent of this one:
  // it may be scheduled now and waits in griddepcontrol.wait until this grid has
  // finished and its partials are visible, so its launch overlaps this kernel.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // The P^T stages start zeroed: a consumer warp clears only rows it wrote itself.
  for (int i = threadIdx.x; i < kStages * kPBytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(&sm.pt[0][0])[i] = make_uint4(0u, 0u, 0u, 0u);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.ready[s], kConsumers);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.run_full[s], 1);
      mbar_init(&sm.run_empty[s], kConsumers + 1);
      mbar_init(&sm.o_full[s], 1);
      mbar_init(&sm.o_empty[s], kConsumers);
    }
    mbar_init(&sm.drain, 1);
    mbar_init(&sm.cbar, kConsumers);
    sm.run_bad = 0;
    sm.ctl.flag = 0;
    sm.ctl.limit = p.wait_cycles;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  volatile WaitCtl* abort = &sm.ctl;

  if (warp == 0) {
    // ================================================================ producer
    const uint64_t pol = policy_evict_first();
    uint32_t it = 0;  // stages armed
    row::group_producer<kW>(p, sm, total_units, kKeys, abort, [&](int kv_r, int k_lo, int k_hi) {
      return mma_stream(p, sm, &vmap, it, kv_r, k_lo, k_hi, pol, abort);
    });
    if (abort->flag && lane == 0) row::drain_stages<kStages>(sm.full, it, p.wait_cycles);
  } else if (warp == kMmaWarp) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      // A: V^T, e4m3, MN-major: the 128 dims of a key are one 128-byte swizzle
      // row, 8-key groups 1024 B apart.  B: P^T, e4m3, K-major: 8-row groups 1024 B
      // apart.  K = 32 keys per MMA: 4096 B of A rows, 32 B of each B row.
      const uint64_t a0 = tc::sw128_desc(smem_u32(&sm.v[0][0]), kVBytes, 1024);
      const uint64_t b0 = tc::sw128_desc(smem_u32(&sm.pt[0][0]), 16, 1024);
      uint32_t it = 0, rc = 0, oc = 0;
      for (;;) {
        const int us = rc & 1;
        if (!mbar_wait(&sm.run_full[us], (rc >> 1) & 1, abort, p.err)) break;
        const int unit = sm.slot[us].unit;
        const int n_st = (sm.slot[us].k_hi - sm.slot[us].k_lo + kKeys - 1) / kKeys;
        ++rc;
        if (unit < 0) break;
        mbar_arrive(&sm.run_empty[us]);
        if (n_st <= 0) continue;
        const int rb = oc & 1;
        if (!mbar_wait(&sm.o_empty[rb], ((oc >> 1) & 1) ^ 1, abort, p.err)) break;
        bool ab = false;
        for (int st = 0; st < n_st; ++st, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&sm.ready[s], (it / kStages) & 1, abort, p.err)) {
            ab = true;
            break;
          }
          tc::fence_after_sync();
          const uint64_t ad = a0 + (uint64_t)(s * kVBytes / 16);
          const uint64_t bd = b0 + (uint64_t)(s * kPBytes / 16);
#pragma unroll
          for (int kk = 0; kk < kKeys / 32; ++kk)
            tc::mma_f8f6f4_ss(tmem + (uint32_t)(rb * kN), ad + 256u * kk, bd + 2u * kk, tc::kIdescOT8,
                              (st > 0 || kk > 0) ? 1u : 0u);
          tc::commit(&sm.empty[s]);
        }
        if (ab) break;
        tc::commit(&sm.o_full[rb]);
        ++oc;
      }
      // Every MMA issued must land before TMEM is released.
      tc::commit(&sm.drain);
      mbar_drain(&sm.drain, 0, p.wait_cycles);
    }
    __syncwarp();
  } else {
    // ================================================================ consumers
    const int c = warp - 1;    // query slot of the run this warp owns
    const int qd = warp & 3;   // TMEM lane quarter it may read: dims [32 qd, 32 qd + 32)
    const uint32_t t_lane = tmem + ((uint32_t)(32 * qd) << 16);
    const float cabs = fabsf(p.inv_sqrt_d);
    const float k2 = cabs * kLog2e;
    const int sgn = p.inv_sqrt_d < 0.f ? -1 : 1;
    uint32_t it = 0, rc = 0, oc = 0, cb = 0;
    int prow[kStages];  // first of the P^T rows this warp last wrote in each stage (-1: none)
#pragma unroll
    for (int i = 0; i < kStages; ++i) prow[i] = -1;
    // The four consumer warps meet on an mbarrier with a bounded wait (a named
    // barrier could not give up if a warp never came).
    auto consumers_meet = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.cbar);
      const bool ok = mbar_wait_warp(&sm.cbar, cb & 1, abort, p.err);
      ++cb;
      return ok;
    };
    for (;;) {
      const int us = rc & 1;
      if (!mbar_wait_warp(&sm.run_full[us], (rc >> 1) & 1, abort, p.err)) break;
      const row::RunSlot<kW>& sl = sm.slot[us];
      if (sl.unit < 0) break;
      const int rp = rc & 1;   // parity of this run's ep_m / run_l buffers
      const int run_no = (int)rc + 1;
      ++rc;
      const int nq = sl.nq;
      const bool mine = c < nq;  // warp-uniform
      uint32_t qw[kW] = {0u, 0u, 0u, 0u};
      int kv_end = 0, item = 0;
      if (mine) {
#pragma unroll
        for (int i = 0; i < kW; ++i) qw[i] = sl.q[c][i];
        kv_end = sl.kv_end[c];
        item = sl.item[c];
      }
      const int k_lo = sl.k_lo;
      const int n_st = (sl.k_hi - k_lo + kKeys - 1) / kKeys;
      float m = -INFINITY, l = 0.f;
      float mep[kEpochs];
#pragma unroll
      for (int e = 0; e < kEpochs; ++e) mep[e] = -INFINITY;
      int ep = 0;
      bool out_of_epochs = false;
      bool stop = false;
      for (int st = 0; st < n_st; ++st, ++it) {
        const int s = it % kStages;
        if (!mbar_wait_warp(&sm.full[s], (it / kStages) & 1, abort, p.err)) {
          stop = true;
          break;
        }
        const int nk = sm.hdr[s].nkeys;
        uint32_t mk[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) mk[w] = sm.hdr[s].mask[w];
        const bool whole = nk == kKeys && (mk[0] & mk[1] & mk[2] & mk[3]) == 0xFFFFFFFFu;
        // ---- rows of keys 32c .. 32c+31 nobody may read: zeros (the copy may have
        // brought a neighbour's codes there, or left an older stage's).
        if (!whole) {
          const int key = 32 * c + lane;
          if (!(key < nk && ((mk[key >> 5] >> (key & 31)) & 1u))) {
            const uint32_t rb0 = smem_u32(&sm.v[s][key * kD]);
#pragma unroll
            for (int i = 0; i < 8; ++i) st_shared_v4(rb0 + 16 * i, make_uint4(0u, 0u, 0u, 0u));
          }
        }
        // ---- query c: scores of keys 4 lane .. 4 lane + 3, softmax step, P^T rows
        int row = -1;
        uint32_t wh = 0u, wm = 0u, wl = 0u;
        if (mine) {
          const int key0 = k_lo + st * kKeys + 4 * lane;  // absolute index of this lane's first key
          const uint32_t mbits = (mk[lane >> 3] >> ((4 * lane) & 31)) & 0xFu;
          int x[4];
          bool ok[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int sc = score16(qw, *reinterpret_cast<const uint4*>(&sm.k[s][(4 * lane + t) * 16]));
            ok[t] = key0 + t < kv_end && (whole || (4 * lane + t < nk && ((mbits >> t) & 1u)));
            if (p.debug_scores && ok[t]) p.debug_scores[(long long)item * p.debug_ld + key0 + t] = sc;
            x[t] = ok[t] ? sgn * sc : INT_MIN;
          }
          const int mx = __reduce_max_sync(0xffffffffu, max(max(x[0], x[1]), max(x[2], x[3])));
          if (mx != INT_MIN) {
            const float mt = (float)mx * cabs;
            if (m == -INFINITY) {
              m = mt;
              mep[0] = mt;
            } else if (mt > m + kTau) {
              if (ep + 1 < kEpochs) {
                l *= ex2_approx((m - mt) * kLog2e);
                m = mt;
                ++ep;
#pragma unroll
                for (int e = 1; e < kEpochs; ++e)
                  if (e == ep) mep[e] = mt;
              } else {
                out_of_epochs = true;  // the run is redone exactly; keep m
              }
            }
            const float bias = kLog2XScale - m * kLog2e;
            float xs[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              xs[t] = ok[t] ? ex2_approx(fmaf((float)x[t], k2, bias)) : 0.f;
              if (out_of_epochs) xs[t] = fminf(xs[t], 256.f);
            }
            l += (xs[0] + xs[1]) + (xs[2] + xs[3]);
            split4(xs, wh, wm, wl);
            row = 12 * ep + 3 * c;
          }
        }
        {
          const uint32_t pb = smem_u32(&sm.pt[s][0]);
          int old = -1;
#pragma unroll
          for (int i = 0; i < kStages; ++i)
            if (i == s) old = prow[i];
          if (old >= 0 && old != row) {
#pragma unroll
            for (int pc = 0; pc < kPieces; ++pc) {
              const int r = old + pc;
              st_shared_u32(pb + (uint32_t)(r >> 3) * 1024u + (r & 7) * 128u + lane * 4u, 0u);
            }
          }
          if (row >= 0) {
            // keys 4 lane .. 4 lane + 3 of row r: chunk (lane / 4) ^ (r % 8), bytes 4 (lane % 4) ..
            const uint32_t pw[kPieces] = {wh, wm, wl};
#pragma unroll
            for (int pc = 0; pc < kPieces; ++pc) {
              const int r = row + pc;
              st_shared_u32(pb + (uint32_t)(r >> 3) * 1024u + (r & 7) * 128u +
                                ((((uint32_t)lane >> 2) ^ (uint32_t)(r & 7)) << 4) + (lane & 3) * 4u,
                            pw[pc]);
            }
          }
#pragma unroll
          for (int i = 0; i < kStages; ++i)
            if (i == s) prow[i] = row;
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.ready[s]);
      }
      // ---- end of the run: merge the epochs, write (m, l, acc) or the row.  Every
      // consumer warp meets the others twice, also after a wait gave up.
      stop = stop || (abort->flag != 0);
      const float l_run = row::warp_sum(l);
      if (lane == 0) {
#pragma unroll
        for (int e = 0; e < kEpochs; ++e) sm.ep_m[rp][c][e] = mep[e];
        sm.run_l[rp][c] = l_run;
        if (out_of_epochs) sm.run_bad = run_no;
      }
      if (!consumers_meet()) stop = true;
      float o[kQ] = {0.f, 0.f, 0.f, 0.f};  // dim 32 qd + lane of each query, in x units
      if (n_st > 0 && !stop) {
        const int rb = oc & 1;
        if (mbar_wait_warp(&sm.o_full[rb], (oc >> 1) & 1, abort, p.err)) {
          tc::fence_after_sync();
          uint32_t v0[16], v1[16], v2[16];
          tc::ld16(t_lane + (uint32_t)(rb * kN), v0);
          tc::ld16(t_lane + (uint32_t)(rb * kN + 16), v1);
          tc::ld16(t_lane + (uint32_t)(rb * kN + 32), v2);
          tc::ld_wait_regs(v0);
          tc::ld_wait_regs(v1);
          tc::ld_wait_regs(v2);
          bool bad = false;
#pragma unroll
          for (int j = 0; j < kQ; ++j) {
            float mm = -INFINITY;
#pragma unroll
            for (int e = 0; e < kEpochs; ++e) mm = fmaxf(mm, sm.ep_m[rp][j][e]);
            float a = 0.f;
#pragma unroll
            for (int e = 0; e < kEpochs; ++e) {
              const float me = sm.ep_m[rp][j][e];
              if (me != -INFINITY) {
                float col = 0.f;
#pragma unroll
                for (int pc = 0; pc < kPieces; ++pc) {
                  const int n = 12 * e + 3 * j + pc;
                  const uint32_t bits = n < 16 ? v0[n & 15] : (n < 32 ? v1[n & 15] : v2[n & 15]);
                  col = fmaf(__uint_as_float(bits), pc == 0 ? 1.f : (pc == 1 ? 0.0625f : 0.00390625f), col);
                }
                a = fmaf(col, ex2_approx((me - mm) * kLog2e), a);
              }
            }
            o[j] = a;
            if (j < nq) bad |= !isfinite(a);
          }
          if (__any_sync(0xffffffffu, bad) && lane == 0) sm.run_bad = run_no;
        } else {
          stop = true;
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.o_empty[rb]);
        ++oc;
      }
      if (!consumers_meet()) stop = true;
      if (!stop) {
        const float vs = v_scale_for(p, sl.bh0, 0);
        if (sm.run_bad != run_no) {
          const int d = 32 * qd + lane;
#pragma unroll
          for (int j = 0; j < kQ; ++j) {
            if (j < nq) {
              float mm = -INFINITY;
#pragma unroll
              for (int e = 0; e < kEpochs; ++e) mm = fmaxf(mm, sm.ep_m[rp][j][e]);
              const float L = sm.run_l[rp][j];
              if (p.n_split == 1) {
                const float inv_l = (L > 1e-6f) ? 1.f / L : 1.f;
                store_out_all(p, (long long)sl.orow[j] * kD + d, o[j] * vs * inv_l);
              } else {
                // x = 64 w: both sums back to weight units, exactly.
                float* part = p.partials + ((long long)sl.item[j] * p.n_split + sl.split) * (2 + kD);
                part[2 + d] = o[j] * vs * 0.015625f;
                if (d == 0) {
                  part[0] = mm;
                  part[1] = L * 0.015625f;
                }
              }
            }
          }
        } else if (mine) {
          redo_query(p, sl, c, vs);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.run_empty[us]);
      if (stop) break;
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

// Sets the kernel's shared-memory limit and works out its resident CTAs per SM from
// the shared memory, registers and tensor memory one CTA takes.  (The occupancy
// calculator answers 1 for any kernel that uses tensor memory, whatever it
// allocates; this one takes kTmemCols of an SM's 512 columns.)
inline cudaError_t setup(int& ctas, int& smem) {
  smem = (int)kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(row_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, row_mma_kernel);
  if (e != cudaSuccess) return e;
  int dev = 0, smem_sm = 0, reserved = 0, regs_sm = 0, threads_sm = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev)) != cudaSuccess) return e;
  const int regs_cta = ((fa.numRegs * 32 + 255) / 256 * 256) * (kThreads / 32);  // 256-register warp granules
  int n = kCtasPerSm;
  n = std::min(n, smem_sm / (smem + reserved));
  n = std::min(n, regs_sm / std::max(regs_cta, 1));
  n = std::min(n, threads_sm / kThreads);
  n = std::min(n, (int)(512 / kTmemCols));
  ctas = std::max(n, 0);
  return cudaSuccess;
}

// The tensor map of the V pool for this kernel: pool_rows rows of 128 bytes, boxes
// of box_rows(block_size) rows copied with the 128-byte swizzle.  Returns false
// when the driver's encoder is unavailable or refuses the map.
inline bool encode_vmap(CUtensorMap* map, const void* v, long long pool_rows, int block_size) {
  static const PFN_cuTensorMapEncodeTiled_v12000 encode = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)pool_rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kD};
  const cuuint32_t box[2] = {(cuuint32_t)kD, (cuuint32_t)box_rows(block_size)};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(v), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace rmma
}  // namespace hyp
