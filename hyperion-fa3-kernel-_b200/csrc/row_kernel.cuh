// row_kernel.cuh -- split-KV row kernel: one work item (one query row of one
// (batch, head)) against a contiguous or paged KV cache, on CUDA cores.
//
// This is the decode path (S_q = 1, the HBM-bound case) and the general path for
// any worklist.  It replaces the reference's persistent kernel
// (hyperion_fa3_production_final.py:268-596):
//   * work stealing: a per-call ticket in the caller's workspace instead of the
//     __device__ g_work_counter (:71, :236-243); one ticket is one (item, KV split)
//     unit, so a long context is spread over several CTAs and merged afterwards;
//   * loads: one producer warp streams K (16 B/key) and V (D B/key) pages through
//     the TMA engine (cp.async.bulk + mbarrier complete_tx) into an NS-stage ring,
//     replacing the cp.async 16 B copies and the 6-stage ring (:377-452);
//   * per page, the block table gives the pool block (:402-411); a page id outside
//     the pool raises HYPERION_DEVERR_BAD_BLOCK and its keys are skipped;
//   * consumers: 2 warps, each owning half of every stage's keys with its own
//     running (m, l, acc); the score is D - 2*popcount(q XOR k) (README.md:22),
//     the softmax the reference's clamped online update (:544-572) applied per
//     32-key group, and the FP8 decode the hardware e4m3 conversion, which agrees
//     with the reference's rule (:122-141) on every code but 0x7F / 0xFF; a group
//     that holds one of those is redone with the rule itself, as bit moves;
//   * the four per-warp states are merged through shared memory, then either
//     finalised (:582-593) or written as a split-KV partial for the combine kernel.
#pragma once

#include <climits>

#include "common.cuh"

namespace hyp {
namespace row {

constexpr int kKeysPerStage = 64;
// Two 64-key stages per CTA and 11 CTAs per SM: on B200 more resident CTAs with a
// shallow ring hide the HBM latency better than fewer CTAs with a deep one
// (decode B64 H32 S_kv 8192, 4 consumer warps: 2 stages x 8 CTAs reached 84 % of
// the measured copy bandwidth, 4 x 5 reached 76 %).  Two consumer warps of 32 keys
// each, rather than four of 16, put all 32 lanes on the scores and spread each
// group's softmax step over twice the keys; under the sustained power cap that
// took the same decode from 0.42 to 0.37 ms (0.87 to 0.99 of the copy bandwidth).
constexpr int kStages = 2;
constexpr int kConsumerWarps = 2;
constexpr int kThreads = 32 * (1 + kConsumerWarps);
constexpr int kKeysPerWarp = kKeysPerStage / kConsumerWarps;  // 32
constexpr int kRowCtasPerSm = 11;  // the register budget; shared memory allows 11

struct StageHeader {
  int nkeys;
  int pad;
  unsigned long long mask;  // bit j: key j of the stage is present
};

struct UnitSlot {
  int unit;   // -1: no more work
  int item;
  int orow;   // Q and O row: bh * seq_q + q_idx
  int k_lo;
  int k_hi;
  int valid;
  int kv;     // KV row of bh
};

template <int D>
struct Smem {
  static constexpr int W = D / 32;
  static constexpr int kKBytes = kKeysPerStage * W * 4;
  static constexpr int kVBytes = kKeysPerStage * D;
  alignas(128) uint8_t k[kStages][kKBytes];
  alignas(128) uint8_t v[kStages][kVBytes];
  StageHeader hdr[kStages];
  UnitSlot slot[2];
  float merge_m[kConsumerWarps];
  float merge_l[kConsumerWarps];
  float merge_acc[kConsumerWarps][D];
  alignas(16) uint32_t wbuf[kConsumerWarps][kKeysPerWarp];  // f16x2 {w, w} of each warp's keys
  alignas(8) uint64_t full[kStages];
  alignas(8) uint64_t empty[kStages];
  alignas(8) uint64_t unit_full[2];
  alignas(8) uint64_t unit_empty[2];
  WaitCtl ctl;  // abort flag and wait bound of the CTA
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Loads this lane's D/32 V bytes of one stage row (lane owns dims [lane*D/32, +D/32)).
template <int D>
__device__ __forceinline__ void load_v_lane(const uint8_t* row, int lane, uint32_t (&w)[(D / 32 + 3) / 4]) {
  if constexpr (D == 64) {
    w[0] = *reinterpret_cast<const uint16_t*>(row + lane * 2);
  } else if constexpr (D == 128) {
    w[0] = *reinterpret_cast<const uint32_t*>(row + lane * 4);
  } else {
    const uint2 t = *reinterpret_cast<const uint2*>(row + lane * 8);
    w[0] = t.x;
    w[1] = t.y;
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads, kRowCtasPerSm) row_fwd_kernel(FwdParams p, int total_units) {
  // The split combine kernel is launched as a programmatic dependent of this one:
  // it may be scheduled now and waits in griddepcontrol.wait until this grid has
  // finished and its partials are visible, so its launch overlaps this kernel.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int W = D / 32;
  constexpr int DPL = D / 32;  // dims per lane
  constexpr int NW = DPL / 4;  // 32-bit words of V bytes per lane and key
  static_assert(D == 128 || D == 256, "row kernel: head_dim 128 or 256");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>(smem_raw);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Zeros in the V stages, so that a slot no load ever fills decodes to 0 rather
  // than to whatever an earlier kernel left in shared memory; the fence orders
  // these stores before the bulk copies that later overwrite them.
  {
    uint4* v4 = reinterpret_cast<uint4*>(&sm.v[0][0]);
    for (int i = threadIdx.x; i < kStages * Smem<D>::kVBytes / 16; i += kThreads) v4[i] = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.unit_full[s], 1);
      mbar_init(&sm.unit_empty[s], kConsumerWarps);
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
    uint32_t it = 0;
    uint32_t ucount = 0;
    for (;;) {
      int t = 0;
      if (lane == 0) t = (int)atomicAdd(&p.counters[0], 1u);
      t = __shfl_sync(0xffffffffu, t, 0);
      const int unit = (t < total_units) ? t : -1;
      const int us = ucount & 1;
      if (!mbar_wait_warp(&sm.unit_empty[us], ((ucount >> 1) & 1) ^ 1, abort, p.err)) break;
      int item = 0, split = 0, k_lo = 0, k_hi = 0, bh = 0, q_idx = 0;
      bool valid = false;
      if (unit >= 0) {
        item = unit / p.n_split;
        split = unit - item * p.n_split;
        const ItemInfo inf = resolve_item(p, item);
        bh = inf.bh;
        q_idx = inf.q_idx;
        valid = inf.valid;
        if (valid) {
          int chunk = (inf.kv_end + p.n_split - 1) / p.n_split;
          chunk = (chunk + 15) & ~15;
          k_lo = min(split * chunk, inf.kv_end);
          k_hi = min(k_lo + chunk, inf.kv_end);
        }
        if (lane == 0 && split == 0) check_item_errors(p, item);
      }
      if (lane == 0) {
        UnitSlot& sl = sm.slot[us];
        sl.unit = unit;
        sl.item = item;
        sl.orow = bh * p.seq_q + q_idx;
        sl.k_lo = k_lo;
        sl.k_hi = k_hi;
        sl.valid = valid ? 1 : 0;
        sl.kv = kv_of(p, bh);
        mbar_arrive(&sm.unit_full[us]);
      }
      ++ucount;
      if (unit < 0) break;

      bool aborted = false;
      const int kv = kv_of(p, bh);
      for (int k0 = k_lo; k0 < k_hi; k0 += kKeysPerStage) {
        const int s = it % kStages;
        if (!mbar_wait_warp(&sm.empty[s], ((it / kStages) & 1) ^ 1, abort, p.err)) {
          aborted = true;
          break;
        }
        const int n = min(kKeysPerStage, k_hi - k0);
        const int bs = p.block_size;
        const int p0 = k0 / bs;
        const int np = (k0 + n - 1) / bs - p0 + 1;
        uint32_t bytes = 0;
        unsigned long long mask = 0ull;
        for (int i = lane; i < np; i += 32) {
          const int page = p0 + i;
          const int lo = max(k0, page * bs);
          const int hi = min(k0 + n, (page + 1) * bs);
          const long long id = page_block_id_kv(p, kv, page);
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
        // Test hook: the stage numbered fault_stage is left unarmed, with no copy in
        // flight on it, so the consumers' wait for it runs out.
        const bool armed = (int)it != p.fault_stage;
        if (lane == 0 && armed) {
          sm.hdr[s].nkeys = n;
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
          const int hi = min(k0 + n, (page + 1) * bs);
          const long long id = page_block_id_kv(p, kv, page);
          if (id >= 0) {
            const long long slot0 = id * bs + (lo - page * bs);
            const uint32_t cnt = (uint32_t)(hi - lo);
            bulk_g2s_stream(&sm.k[s][(lo - k0) * W * 4], p.k + slot0 * W, cnt * W * 4, &sm.full[s], pol);
            bulk_g2s_stream(&sm.v[s][(lo - k0) * D], p.v + slot0 * D, cnt * D, &sm.full[s], pol);
          }
        }
        ++it;
      }
      if (aborted) break;
    }
    if (abort->flag && lane == 0) {
      // Let the copies of the last (up to kStages) armed stages land before exit.
      for (uint32_t i = (it > (uint32_t)kStages ? it - kStages : 0u); i < it; ++i)
        mbar_drain(&sm.full[i % kStages], (i / kStages) & 1, p.wait_cycles);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int cw = warp - 1;
    uint32_t it = 0;
    uint32_t ucount = 0;
    for (;;) {
      const int us = ucount & 1;
      if (!mbar_wait_warp(&sm.unit_full[us], (ucount >> 1) & 1, abort, p.err)) break;
      const UnitSlot sl = sm.slot[us];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.unit_empty[us]);
      ++ucount;
      if (sl.unit < 0) break;

      uint32_t q[W];
      if (sl.valid) {
        const uint32_t* qrow = p.q + (long long)sl.orow * W;
#pragma unroll
        for (int i = 0; i < W; ++i) q[i] = __ldg(qrow + i);
      } else {
#pragma unroll
        for (int i = 0; i < W; ++i) q[i] = 0u;
      }
      float m = -INFINITY, l = 0.f;
      float acc[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] = 0.f;

      bool aborted = false;
      for (int k0 = sl.k_lo; k0 < sl.k_hi; k0 += kKeysPerStage) {
        const int s = it % kStages;
        if (!mbar_wait_warp(&sm.full[s], (it / kStages) & 1, abort, p.err)) {
          aborted = true;
          break;
        }
        const int n = sm.hdr[s].nkeys;
        const unsigned long long mask = sm.hdr[s].mask;
        const int jl = cw * kKeysPerWarp + (lane % kKeysPerWarp);
        const bool ok = (lane < kKeysPerWarp) && (jl < n) && ((mask >> jl) & 1ull);
        int si = 0;
        if (ok) {
          const uint32_t* kr = reinterpret_cast<const uint32_t*>(&sm.k[s][jl * W * 4]);
          si = sign_score<W>(q, kr);
          if (p.debug_scores) p.debug_scores[(long long)sl.item * p.debug_ld + (k0 + jl)] = si;
        }
        // The largest score of the group is the extreme integer score times
        // inv_sqrt_d (the product is monotonic): one warp reduction on integers.
        // Scores lie in [-D, D], so the sentinels mark a group with no key.
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
          const float mt = (float)ext * p.inv_sqrt_d;
          const float sc = (float)si * p.inv_sqrt_d;
          const float m_new = fmaxf(m, mt);
          const float alpha = (m == -INFINITY) ? 0.f : exp_clamped(m - m_new);
          float w = ok ? exp_clamped(sc - m_new) : 0.f;
          l = l * alpha + w;  // per lane; summed over the warp once per unit
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[i] *= alpha;
          const uint8_t* vbase = &sm.v[s][(cw * kKeysPerWarp) * D];
          bool exact = p.v_scale_mode == 2;
          if (!exact) {
            // Products on f16x2: w in [0, 1] and |V| <= 448, so the sums over this
            // warp's 32 keys stay below 32 * 448 = 14336, inside the f16 range; they
            // are added to the f32 accumulators once per stage.  A key that is
            // absent has w = 0, so its products are 0 unless its bytes decode to NaN.
            if (lane < kKeysPerWarp) sm.wbuf[cw][lane] = pack_f16x2(w, w);
            __syncwarp();
            // The decode is the hardware e4m3 -> f16x2 conversion, 2 instructions
            // per 4 bytes.  It reads codes 0x7F / 0xFF as NaN where the reference
            // reads +-480, and a NaN poisons the sums of the lane that met it; the
            // warp then redoes the group on the exact per-key path below.  The cache
            // writer saturates to +-448 and never writes those codes, and the V
            // slots a stage leaves unused hold zeros or earlier V rows, so the redo
            // runs only for a cache written elsewhere that holds them.
            uint32_t plo[NW], phi[NW];
#pragma unroll
            for (int i = 0; i < NW; ++i) plo[i] = phi[i] = 0u;
#pragma unroll
            for (int j4 = 0; j4 < kKeysPerWarp; j4 += 4) {
              const uint4 w4 = *reinterpret_cast<const uint4*>(&sm.wbuf[cw][j4]);
              const uint32_t wq[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                uint32_t vw[NW];
                load_v_lane<D>(vbase + (j4 + u) * D, lane, vw);
#pragma unroll
                for (int i = 0; i < NW; ++i) {
                  plo[i] = hfma2(wq[u], e4m3x2_to_f16x2_hw(vw[i]), plo[i]);
                  phi[i] = hfma2(wq[u], e4m3x2_to_f16x2_hw(vw[i] >> 16), phi[i]);
                }
              }
            }
            uint32_t nan = 0u;
#pragma unroll
            for (int i = 0; i < NW; ++i) nan |= f16x2_nan_bits(plo[i]) | f16x2_nan_bits(phi[i]);
            if (!__any_sync(0xffffffffu, nan != 0u)) {
              // plo[i] holds dims 4i and 4i+1 of this lane, phi[i] dims 4i+2 and 4i+3.
#pragma unroll
              for (int i = 0; i < NW; ++i) {
                acc[4 * i + 0] += f16_lo_to_f32(plo[i]);
                acc[4 * i + 1] += f16_hi_to_f32(plo[i]);
                acc[4 * i + 2] += f16_lo_to_f32(phi[i]);
                acc[4 * i + 3] += f16_hi_to_f32(phi[i]);
              }
            } else {
              exact = true;
            }
          }
          if (exact) {
            // Products in f32, one key at a time, with the exact bit-level decode:
            // the path for a per-slot V scale (w times the key's own scale), and the
            // redo of a group whose fast decode met a NaN code.
            if (p.v_scale_mode == 2 && ok) {
              const int key = k0 + jl;
              const int page = key / p.block_size;
              const long long id = page_block_id_kv(p, sl.kv, page);
              w *= __ldg(p.v_scale + id * p.block_size + (key - page * p.block_size));
            }
            w *= kTwoPow120;
#pragma unroll 4
            for (int jj = 0; jj < kKeysPerWarp; ++jj) {
              const float wj = __shfl_sync(0xffffffffu, w, jj);
              if (wj != 0.f) {
                uint32_t vw[NW];
                load_v_lane<D>(vbase + jj * D, lane, vw);
#pragma unroll
                for (int i = 0; i < DPL; ++i) {
                  acc[i] = fmaf(wj, fp8_bits_to_f32_scaled(vw[i >> 2] >> (8 * (i & 3))), acc[i]);
                }
              }
            }
          }
          m = m_new;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
        ++it;
      }
      // Every consumer warp reaches both named barriers below once per unit, also
      // when it gave up on a wait: the barriers have no timeout of their own.
      const bool stop = aborted || (abort->flag != 0);

      // ---- merge the consumer warps' (m, l, acc) ----
      const float l_warp = warp_sum(l);
      if (lane == 0) {
        sm.merge_m[cw] = m;
        sm.merge_l[cw] = l_warp;
      }
#pragma unroll
      for (int i = 0; i < DPL; ++i) sm.merge_acc[cw][lane * DPL + i] = acc[i];
      named_bar_sync(1, 32 * kConsumerWarps);
      float M = -INFINITY;
#pragma unroll
      for (int w2 = 0; w2 < kConsumerWarps; ++w2) M = fmaxf(M, sm.merge_m[w2]);
      float f[kConsumerWarps];
      float L = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < kConsumerWarps; ++w2) {
        const float mw = sm.merge_m[w2];
        f[w2] = (mw == -INFINITY) ? 0.f : exp_clamped(mw - M);
        L += sm.merge_l[w2] * f[w2];
      }
      const float vs_unit = (p.v_scale_mode == 0)   ? __ldg(p.v_scale)
                            : (p.v_scale_mode == 1) ? __ldg(p.v_scale + (sl.kv % p.v_scale_numel))
                                                    : 1.f;
      for (int d = cw * 32 + lane; d < D; d += 32 * kConsumerWarps) {
        float a = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < kConsumerWarps; ++w2) a += sm.merge_acc[w2][d] * f[w2];
        a *= vs_unit;
        if (stop) continue;
        if (p.n_split == 1) {
          if (sl.valid) {
            const float inv_l = (L > 1e-6f) ? 1.f / L : 1.f;
            store_out_all(p, (long long)sl.orow * D + d, a * inv_l);
          }
        } else {
          float* part = p.partials + (long long)sl.unit * (2 + D);
          part[2 + d] = a;
          if (d == 0) {
            part[0] = M;
            part[1] = L;
          }
        }
      }
      named_bar_sync(1, 32 * kConsumerWarps);
      if (stop) break;
    }
  }
  fence_out_peers(p);
}

// Merges the n_split partials (m, l, acc[D]) of every item and writes O.
template <int D>
__global__ void __launch_bounds__(128) row_combine_kernel(FwdParams p) {
  // Launched as a programmatic dependent of the split kernel: wait for that grid
  // to finish and its partials to be visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int item = blockIdx.x;
  const ItemInfo inf = resolve_item(p, item);
  if (!inf.valid) return;
  const float* base = p.partials + (long long)item * p.n_split * (2 + D);
  float M = -INFINITY;
  for (int s = 0; s < p.n_split; ++s) M = fmaxf(M, base[s * (2 + D)]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, a = 0.f;
    for (int s = 0; s < p.n_split; ++s) {
      const float* part = base + s * (2 + D);
      const float ms = part[0];
      const float f = (ms == -INFINITY) ? 0.f : exp_clamped(ms - M);
      L += part[1] * f;
      a += part[2 + d] * f;
    }
    const float inv_l = (L > 1e-6f) ? 1.f / L : 1.f;
    store_out_all(p, ((long long)inf.bh * p.seq_q + inf.q_idx) * D + d, a * inv_l);
  }
  fence_out_peers(p);
}

}  // namespace row
}  // namespace hyp
