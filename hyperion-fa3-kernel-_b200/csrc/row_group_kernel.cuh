// row_group_kernel.cuh -- the split-KV row kernel for grouped-query attention.
//
// With kv_group > 1, several query heads read the same KV head.  The reference
// engine is configured that way (num_heads 32, num_kv_heads 8:
// hyperion_fa3_production_final.py:852-853), but its kernel has no notion of it:
// every (batch, head) row streams its own keys.  Here a unit is up to kGroupMax
// consecutive work items and one KV split.  The producer cuts the unit into runs
// of consecutive items on the same KV row and streams each run's keys once; every
// consumer warp scores and accumulates all queries of the run against each stage.
// HBM traffic per query falls by the run length.  The per-(query, key) arithmetic
// is the row kernel's (popcount score, the reference's clamped online softmax per
// 32-key group, f16x2 products of the hardware FP8 decode with the exact redo for
// codes 0x7F / 0xFF), with the FP8 decode of a key shared by the run's queries,
// and the running max moved only when a group exceeds it by more than ln 4.
//
// Each query keeps its own key range [0, kv_end), so a run may also hold rows of
// one (batch, head) at different causal positions; the run streams the longest.
#pragma once

#include <type_traits>

#include "row_kernel.cuh"

namespace hyp {
namespace row {

constexpr int kGroupMax = 4;  // queries per run
// Warp layout: a producer warp and 2 consumer warps, each consumer owning 32 keys
// of every 64-key stage (every lane scores one key against all queries of the run).
// Against 4 consumer warps of 16 keys, this keeps whole warps on the scores and
// pays each group's softmax step per 32 keys: decode with 32 query heads over 8 KV
// heads went from 0.232 to 0.179 ms.
constexpr int kGWarps = 2;
constexpr int kGKeysPerWarp = kKeysPerStage / kGWarps;  // 32
constexpr int kGThreads = 32 * (1 + kGWarps);
// KV ring depth: 2 stages, so that 10 CTAs (head_dim 128) or 5 (head_dim 256) fit
// an SM's shared memory.
constexpr int kGroupStages = 2;
// A query's running max is moved only when a 32-key group's max exceeds it by more
// than ln 4: the weights exp(s - m) then stay at most 4, so a group's f16 sums of
// w * v stay below 32 * 4 * 448 = 57344, inside the f16 range.
constexpr float kGroupTau = 1.3862943611198906f;

template <int W>
struct RunSlot {
  int unit;   // -1: no more work
  int split;
  int nq;     // queries of the run, 1..kGroupMax
  int bh0;    // query row of the run's first item
  int kv;     // the run's KV row
  int k_lo;
  int k_hi;
  int item[kGroupMax];
  int orow[kGroupMax];    // O row: bh * seq_q + q_idx
  int kv_end[kGroupMax];  // the query attends keys [0, kv_end)
  alignas(16) uint32_t q[kGroupMax][W];
};

template <int D>
struct GroupSmem {
  static constexpr int W = D / 32;
  static constexpr int kKBytes = kKeysPerStage * W * 4;
  static constexpr int kVBytes = kKeysPerStage * D;
  static constexpr int NS = kGroupStages;
  alignas(128) uint8_t k[NS][kKBytes];
  alignas(128) uint8_t v[NS][kVBytes];
  StageHeader hdr[NS];
  RunSlot<W> slot[2];
  float merge_m[kGWarps][2];  // two queries of the run per merge round
  float merge_l[kGWarps][2];
  float merge_acc[kGWarps][2][D];
  alignas(16) uint32_t wbuf[kGWarps][kGKeysPerWarp][kGroupMax];  // f16x2 {w, w} per key and query
  alignas(8) uint64_t full[NS];
  alignas(8) uint64_t empty[NS];
  alignas(8) uint64_t run_full[2];
  alignas(8) uint64_t run_empty[2];
  WaitCtl ctl;  // abort flag and wait bound of the CTA
};

// Resident CTAs per SM the register budget is set for.  The kernel is bound by
// instruction issue and latency rather than HBM, so resident warps pay: head_dim
// 128 runs 10 CTAs at 64 registers (a few bytes spilled), head_dim 256 runs 5.
template <int D>
constexpr int group_ctas() { return D == 128 ? 10 : 5; }

// The producer warp of the grouped kernels.  It takes unit tickets, cuts each
// unit (up to kGroupMax work items, one KV split) into runs of consecutive items on
// one KV row, publishes each run in a 2-slot ring (run_full / run_empty) and hands
// the run's key range of its split, [k_lo, k_hi) on KV row kv, to
// stream(kv, k_lo, k_hi), which loads its stages and returns false when a wait gave
// up.  A split starts at a multiple of key_round keys.
template <int W, class SM, class Stream>
__device__ __forceinline__ void group_producer(const FwdParams& p, SM& sm, int total_units, int key_round,
                                               volatile WaitCtl* abort, Stream&& stream) {
  const int lane = threadIdx.x & 31;
  uint32_t rc = 0;  // run slots published
  bool aborted = false;
  for (;;) {
    int t = 0;
    if (lane == 0) t = (int)atomicAdd(&p.counters[0], 1u);
    t = __shfl_sync(0xffffffffu, t, 0);
    if (t >= total_units) {
      const int us = rc & 1;
      if (!mbar_wait_warp(&sm.run_empty[us], ((rc >> 1) & 1) ^ 1, abort, p.err)) break;
      if (lane == 0) {
        sm.slot[us].unit = -1;
        mbar_arrive(&sm.run_full[us]);
      }
      ++rc;
      break;
    }
    const int unit = t;
    const int chunk = unit / p.n_split;
    const int split = unit - chunk * p.n_split;
    const int i0 = chunk * p.group_items;
    const int n = min(p.group_items, p.total_work - i0);
    // Lane j < n resolves item i0 + j.
    ItemInfo inf;
    inf.bh = 0;
    inf.q_idx = 0;
    inf.kv_end = 0;
    inf.valid = false;
    if (lane < n) {
      inf = resolve_item(p, i0 + lane);
      if (split == 0) check_item_errors(p, i0 + lane);
    }
    const int kvb = (lane < n && inf.valid) ? kv_of(p, inf.bh) : -1;
    int r = 0;
    while (r < n) {
      const int kv_r = __shfl_sync(0xffffffffu, kvb, r);
      if (kv_r < 0) {  // a bad item: flagged above, not written
        ++r;
        continue;
      }
      const unsigned diff = __ballot_sync(0xffffffffu, lane > r && lane < n && kvb != kv_r);
      const int e = diff ? (__ffs(diff) - 1) : n;
      const bool in_run = lane >= r && lane < e;
      const int maxend = __reduce_max_sync(0xffffffffu, in_run ? inf.kv_end : 0);
      int chunk_k = (maxend + p.n_split - 1) / p.n_split;
      chunk_k = (chunk_k + key_round - 1) / key_round * key_round;
      const int k_lo = min(split * chunk_k, maxend);
      const int k_hi = min(k_lo + chunk_k, maxend);
      const int bh_r = __shfl_sync(0xffffffffu, inf.bh, r);

      const int us = rc & 1;
      if (!mbar_wait_warp(&sm.run_empty[us], ((rc >> 1) & 1) ^ 1, abort, p.err)) {
        aborted = true;
        break;
      }
      RunSlot<W>& sl = sm.slot[us];
      if (in_run) {
        const int j = lane - r;
        sl.item[j] = i0 + lane;
        sl.orow[j] = inf.bh * p.seq_q + inf.q_idx;
        sl.kv_end[j] = inf.kv_end;
        const uint32_t* qrow = p.q + ((long long)inf.bh * p.seq_q + inf.q_idx) * W;
#pragma unroll
        for (int i = 0; i < W; ++i) sl.q[j][i] = __ldg(qrow + i);
      }
      if (lane == 0) {
        sl.unit = unit;
        sl.split = split;
        sl.nq = e - r;
        sl.bh0 = bh_r;
        sl.kv = kv_r;
        sl.k_lo = k_lo;
        sl.k_hi = k_hi;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.run_full[us]);
      ++rc;

      if (!stream(kv_r, k_lo, k_hi)) {
        aborted = true;
        break;
      }
      r = e;
    }
    if (aborted) break;
  }
}

// The grouped row kernel's stages: 64 keys each, sign bits to sm.k and FP8 codes to
// sm.v by bulk copies per page piece, the key count and valid-key mask to sm.hdr,
// through the NS-stage ring full / empty.  `it` counts the stages armed.
template <int D, int NS, class SM>
__device__ __forceinline__ bool group_stream(const FwdParams& p, SM& sm, uint32_t& it, int kv_r, int k_lo, int k_hi,
                                             uint64_t pol, volatile WaitCtl* abort) {
  constexpr int W = D / 32;
  const int lane = threadIdx.x & 31;
  for (int k0 = k_lo; k0 < k_hi; k0 += kKeysPerStage) {
    const int s = it % NS;
    if (!mbar_wait_warp(&sm.empty[s], ((it / NS) & 1) ^ 1, abort, p.err)) return false;
    const int nk = min(kKeysPerStage, k_hi - k0);
    const int bs = p.block_size;
    const int p0 = k0 / bs;
    const int np = (k0 + nk - 1) / bs - p0 + 1;
    uint32_t bytes = 0;
    unsigned long long mask = 0ull;
    for (int i = lane; i < np; i += 32) {
      const int page = p0 + i;
      const int lo = max(k0, page * bs);
      const int hi = min(k0 + nk, (page + 1) * bs);
      const long long id = page_block_id_kv(p, kv_r, page);
      if (id >= 0) {
        bytes += (uint32_t)(hi - lo) * (uint32_t)(W * 4 + D);
        const int a = lo - k0, b = hi - k0;
        const unsigned long long bits = (b - a >= 64) ? ~0ull : ((1ull << (b - a)) - 1ull);
        mask |= bits << a;
      } else {
        raise_error(p.err, HYPERION_DEVERR_BAD_BLOCK);
      }
    }
    bytes = __reduce_add_sync(0xffffffffu, bytes);
    mask = ((unsigned long long)__reduce_or_sync(0xffffffffu, (uint32_t)(mask >> 32)) << 32) |
           __reduce_or_sync(0xffffffffu, (uint32_t)mask);
    // Test hook: the stage numbered fault_stage is left unarmed, with no copy
    // in flight on it, so the consumers' wait for it runs out.
    const bool armed = (int)it != p.fault_stage;
    if (lane == 0 && armed) {
      sm.hdr[s].nkeys = nk;
      sm.hdr[s].mask = mask;
      if (bytes) {
        mbar_arrive_expect_tx(&sm.full[s], bytes);
      } else {
        mbar_arrive(&sm.full[s]);
      }
    }
    __syncwarp();
    for (int i = lane; armed && i < np; i += 32) {
      const int page = p0 + i;
      const int lo = max(k0, page * bs);
      const int hi = min(k0 + nk, (page + 1) * bs);
      const long long id = page_block_id_kv(p, kv_r, page);
      if (id >= 0) {
        const long long slot0 = id * bs + (lo - page * bs);
        const uint32_t cnt = (uint32_t)(hi - lo);
        bulk_g2s_stream(&sm.k[s][(lo - k0) * W * 4], p.k + slot0 * W, cnt * W * 4, &sm.full[s], pol);
        bulk_g2s_stream(&sm.v[s][(lo - k0) * D], p.v + slot0 * D, cnt * D, &sm.full[s], pol);
      }
    }
    ++it;
  }
  return true;
}

// On the way out of an aborted CTA: let the copies of the last (up to NS) armed
// stages land before the CTA's shared memory is released.
template <int NS>
__device__ __forceinline__ void drain_stages(uint64_t* full, uint32_t it, long long limit) {
  for (uint32_t i = (it > (uint32_t)NS ? it - NS : 0u); i < it; ++i) mbar_drain(&full[i % NS], (i / NS) & 1, limit);
}

template <int D>
__global__ void __launch_bounds__(kGThreads, group_ctas<D>()) row_group_kernel(FwdParams p, int total_units) {
  // The split combine kernel is launched as a programmatic dependent of this one:
  // it may be scheduled now and waits in griddepcontrol.wait until this grid has
  // finished and its partials are visible, so its launch overlaps this kernel.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int W = D / 32;
  constexpr int DPL = D / 32;  // dims per lane
  constexpr int NW = DPL / 4;  // 32-bit words of V bytes per lane and key
  constexpr int G = kGroupMax;
  constexpr int kGStages = GroupSmem<D>::NS;
  static_assert(D == 128 || D == 256, "row kernel: head_dim 128 or 256");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  GroupSmem<D>& sm = *reinterpret_cast<GroupSmem<D>*>(smem_raw);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Zeros in the V stages, so that a slot no load ever fills decodes to 0; the
  // fence orders these stores before the bulk copies that overwrite them.
  {
    uint4* v4 = reinterpret_cast<uint4*>(&sm.v[0][0]);
    for (int i = threadIdx.x; i < kGStages * GroupSmem<D>::kVBytes / 16; i += kGThreads)
      v4[i] = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kGWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.run_full[s], 1);
      mbar_init(&sm.run_empty[s], kGWarps);
    }
    sm.ctl.flag = 0;
    sm.ctl.limit = p.wait_cycles;
    fence_mbar_init();
  }
  __syncthreads();

  volatile WaitCtl* abort = &sm.ctl;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = policy_evict_first();
    uint32_t it = 0;  // stages armed
    group_producer<W>(p, sm, total_units, 16, abort, [&](int kv_r, int k_lo, int k_hi) {
      return group_stream<D, kGStages>(p, sm, it, kv_r, k_lo, k_hi, pol, abort);
    });
    if (abort->flag && lane == 0) drain_stages<kGStages>(sm.full, it, p.wait_cycles);
  } else {
    // ------------------------------------------------------------ consumers
    const int cw = warp - 1;
    uint32_t it = 0;
    uint32_t rc = 0;
    for (;;) {
      const int us = rc & 1;
      if (!mbar_wait_warp(&sm.run_full[us], (rc >> 1) & 1, abort, p.err)) break;
      ++rc;
      const RunSlot<W>& sl = sm.slot[us];
      if (sl.unit < 0) break;
      // The slot stays this run's until the warps release it after the merge.
      const int nq = sl.nq;

      float m[G], l[G], acc[G][DPL];
#pragma unroll
      for (int j = 0; j < G; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[j][i] = 0.f;
      }

      bool aborted = false;
      for (int k0 = sl.k_lo; k0 < sl.k_hi; k0 += kKeysPerStage) {
        const int s = it % kGStages;
        if (!mbar_wait_warp(&sm.full[s], (it / kGStages) & 1, abort, p.err)) {
          aborted = true;
          break;
        }
        // One stage for a run of NQ queries: NQ = 1 and NQ = G are compiled with
        // constant trip counts, NQ = 0 takes the run's length at run time.
        auto stage = [&](auto nqc) {
          constexpr int NQ = decltype(nqc)::value;
          constexpr int JN = (NQ == 0) ? G : NQ;  // query slots the loops visit
          const int nk = sm.hdr[s].nkeys;
          const unsigned long long mask = sm.hdr[s].mask;
          const int jl = cw * kGKeysPerWarp + (lane % kGKeysPerWarp);
          const int key = k0 + jl;
          const bool okk = (lane < kGKeysPerWarp) && (jl < nk) && ((mask >> jl) & 1ull);
          uint32_t kr[W];
#pragma unroll
          for (int i = 0; i < W; ++i) kr[i] = 0u;
          if (okk) {
            const uint4* kp = reinterpret_cast<const uint4*>(&sm.k[s][jl * W * 4]);
#pragma unroll
            for (int i = 0; i < W / 4; ++i) {
              const uint4 t4 = kp[i];
              kr[4 * i + 0] = t4.x;
              kr[4 * i + 1] = t4.y;
              kr[4 * i + 2] = t4.z;
              kr[4 * i + 3] = t4.w;
            }
          }
          // Scores and the online-softmax step of every query of the run.  A query
          // slot past the run's end (j >= nq) scores nothing, keeps w = 0 and is
          // never merged, so the product loop below needs no test on it.
          float w[JN];
          int si_all[JN];
          bool ok_all[JN];
          bool any_all = false;
#pragma unroll
          for (int j = 0; j < JN; ++j) {
            w[j] = 0.f;
            const bool ok = okk && (NQ != 0 || j < nq) && key < sl.kv_end[j];
            ok_all[j] = ok;
            int si = 0;
            if (ok) {
              const uint4* qp = reinterpret_cast<const uint4*>(&sl.q[j][0]);
              int pc = 0;
#pragma unroll
              for (int i = 0; i < W / 4; ++i) {
                const uint4 q4 = qp[i];
                pc += __popc(q4.x ^ kr[4 * i + 0]) + __popc(q4.y ^ kr[4 * i + 1]) +
                      __popc(q4.z ^ kr[4 * i + 2]) + __popc(q4.w ^ kr[4 * i + 3]);
              }
              si = D - 2 * pc;
            }
            si_all[j] = si;
            int ext;
            bool any;
            if (p.inv_sqrt_d >= 0.f) {
              ext = __reduce_max_sync(0xffffffffu, ok ? si : INT_MIN);
              any = ext != INT_MIN;
            } else {
              ext = __reduce_min_sync(0xffffffffu, ok ? si : INT_MAX);
              any = ext != INT_MAX;
            }
            if (any) {
              // The running max moves only when the group's max exceeds it by more
              // than kGroupTau (every first group does: m = -inf); otherwise the
              // weights exp(s - m) stay below 4 and the rescale is skipped.  The
              // normalised result is the same: m cancels between acc and l.
              const float mt = (float)ext * p.inv_sqrt_d;
              const float sc = (float)si * p.inv_sqrt_d;
              if (mt > m[j] + kGroupTau) {
                const float alpha = (m[j] == -INFINITY) ? 0.f : exp_clamped(m[j] - mt);
                l[j] *= alpha;
#pragma unroll
                for (int i = 0; i < DPL; ++i) acc[j][i] *= alpha;
                m[j] = mt;
              }
              w[j] = ok ? exp_clamped(sc - m[j]) : 0.f;
              l[j] += w[j];
              any_all = true;
            }
          }
          if (p.debug_scores) {
#pragma unroll
            for (int j = 0; j < JN; ++j)
              if (ok_all[j]) p.debug_scores[(long long)sl.item[j] * p.debug_ld + key] = si_all[j];
          }
          if (!any_all) return;
          const uint8_t* vbase = &sm.v[s][(cw * kGKeysPerWarp) * D];
          bool exact = p.v_scale_mode == 2;
          if (!exact) {
            // f16x2 products of the hardware decode, shared by the run's queries;
            // see row_fwd_kernel for the ranges and the NaN rule.
            // A lane's weights of every query go to one 16-byte row of wbuf, so the
            // product loop reads all of a key's weights with one broadcast load.
            if (lane < kGKeysPerWarp) {
#pragma unroll
              for (int j = 0; j < JN; ++j) sm.wbuf[cw][lane][j] = pack_f16x2(w[j], w[j]);
            }
            __syncwarp();
            uint32_t plo[JN][NW], phi[JN][NW];
#pragma unroll
            for (int j = 0; j < JN; ++j) {
#pragma unroll
              for (int i = 0; i < NW; ++i) plo[j][i] = phi[j][i] = 0u;
            }
#pragma unroll
            for (int jk = 0; jk < kGKeysPerWarp; ++jk) {
              uint32_t wk[JN];
              if constexpr (JN == G) {
                const uint4 t4 = *reinterpret_cast<const uint4*>(&sm.wbuf[cw][jk][0]);
                wk[0] = t4.x;
                wk[1] = t4.y;
                wk[2] = t4.z;
                wk[3] = t4.w;
              } else {
#pragma unroll
                for (int j = 0; j < JN; ++j) wk[j] = sm.wbuf[cw][jk][j];
              }
              uint32_t vw[NW];
              load_v_lane<D>(vbase + jk * D, lane, vw);
              uint32_t c0[NW], c1[NW];
#pragma unroll
              for (int i = 0; i < NW; ++i) {
                c0[i] = e4m3x2_to_f16x2_hw(vw[i]);
                c1[i] = e4m3x2_to_f16x2_hw(vw[i] >> 16);
              }
#pragma unroll
              for (int j = 0; j < JN; ++j) {
                if (NQ != 0 || j < nq) {
#pragma unroll
                  for (int i = 0; i < NW; ++i) {
                    plo[j][i] = hfma2(wk[j], c0[i], plo[j][i]);
                    phi[j][i] = hfma2(wk[j], c1[i], phi[j][i]);
                  }
                }
              }
            }
            // A code the hardware decodes to NaN poisons the sums of every query of
            // the lane (0 * NaN is NaN), so the first query's sums tell for all.
            uint32_t nan = 0u;
#pragma unroll
            for (int i = 0; i < NW; ++i) nan |= f16x2_nan_bits(plo[0][i]) | f16x2_nan_bits(phi[0][i]);
            if (!__any_sync(0xffffffffu, nan != 0u)) {
              // plo[j][i] holds dims 4i and 4i+1 of this lane, phi[j][i] dims 4i+2 and 4i+3.
#pragma unroll
              for (int j = 0; j < JN; ++j) {
#pragma unroll
                for (int i = 0; i < NW; ++i) {
                  acc[j][4 * i + 0] += f16_lo_to_f32(plo[j][i]);
                  acc[j][4 * i + 1] += f16_hi_to_f32(plo[j][i]);
                  acc[j][4 * i + 2] += f16_lo_to_f32(phi[j][i]);
                  acc[j][4 * i + 3] += f16_hi_to_f32(phi[j][i]);
                }
              }
            } else {
              exact = true;
            }
          }
          if (exact) {
            // Products in f32, one key at a time, with the exact bit-level decode:
            // the path for a per-slot V scale, and the redo of a group whose fast
            // decode met a NaN code.
            float vsl = 1.f;
            if (p.v_scale_mode == 2 && okk) {
              const int page = key / p.block_size;
              const long long id = page_block_id_kv(p, sl.kv, page);
              vsl = __ldg(p.v_scale + id * p.block_size + (key - page * p.block_size));
            }
            float ws[JN];
#pragma unroll
            for (int j = 0; j < JN; ++j) ws[j] = w[j] * vsl * kTwoPow120;
#pragma unroll 2
            for (int jj = 0; jj < kGKeysPerWarp; ++jj) {
              float wk[JN];
              bool nz = false;
#pragma unroll
              for (int j = 0; j < JN; ++j) {
                wk[j] = __shfl_sync(0xffffffffu, ws[j], jj);
                nz |= wk[j] != 0.f;
              }
              if (nz) {
                uint32_t vw[NW];
                load_v_lane<D>(vbase + jj * D, lane, vw);
#pragma unroll
                for (int i = 0; i < DPL; ++i) {
                  const float vd = fp8_bits_to_f32_scaled(vw[i >> 2] >> (8 * (i & 3)));
#pragma unroll
                  for (int j = 0; j < JN; ++j) acc[j][i] = fmaf(wk[j], vd, acc[j][i]);
                }
              }
            }
          }
        };
        if (nq == G) {
          stage(std::integral_constant<int, G>{});
        } else if (nq == 1) {
          stage(std::integral_constant<int, 1>{});
        } else {
          stage(std::integral_constant<int, 0>{});
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
        ++it;
      }
      // Every consumer warp reaches the named barriers below for every query of the
      // run, also when it gave up on a wait: the barriers have no timeout of their own.
      const bool stop = aborted || (abort->flag != 0);
      const float vs_run = (p.v_scale_mode == 2) ? 1.f : v_scale_for(p, sl.bh0, 0);

      // ---- merge the consumer warps' (m, l, acc), two queries per round ----
#pragma unroll
      for (int j0 = 0; j0 < G; j0 += 2) {
        if (j0 < nq) {
          const bool two = j0 + 1 < nq;  // the same in every thread
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            if (q == 0 || two) {
              const float l_warp = warp_sum(l[j0 + q]);
              if (lane == 0) {
                sm.merge_m[cw][q] = m[j0 + q];
                sm.merge_l[cw][q] = l_warp;
              }
#pragma unroll
              for (int i = 0; i < DPL; ++i) sm.merge_acc[cw][q][lane * DPL + i] = acc[j0 + q][i];
            }
          }
          named_bar_sync(1, 32 * kGWarps);
          for (int q = 0; q < (two ? 2 : 1); ++q) {
            const int j = j0 + q;
            float M = -INFINITY;
#pragma unroll
            for (int w2 = 0; w2 < kGWarps; ++w2) M = fmaxf(M, sm.merge_m[w2][q]);
            float f[kGWarps];
            float L = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < kGWarps; ++w2) {
              const float mw = sm.merge_m[w2][q];
              f[w2] = (mw == -INFINITY) ? 0.f : exp_clamped(mw - M);
              L += sm.merge_l[w2][q] * f[w2];
            }
            for (int d = cw * 32 + lane; d < D; d += 32 * kGWarps) {
              float a = 0.f;
#pragma unroll
              for (int w2 = 0; w2 < kGWarps; ++w2) a += sm.merge_acc[w2][q][d] * f[w2];
              a *= vs_run;
              if (stop) continue;
              if (p.n_split == 1) {
                const float inv_l = (L > 1e-6f) ? 1.f / L : 1.f;
                store_out_all(p, (long long)sl.orow[j] * D + d, a * inv_l);
              } else {
                float* part = p.partials + ((long long)sl.item[j] * p.n_split + sl.split) * (2 + D);
                part[2 + d] = a;
                if (d == 0) {
                  part[0] = M;
                  part[1] = L;
                }
              }
            }
          }
          named_bar_sync(1, 32 * kGWarps);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.run_empty[us]);
      if (stop) break;
    }
  }
  fence_out_peers(p);
}

}  // namespace row
}  // namespace hyp
