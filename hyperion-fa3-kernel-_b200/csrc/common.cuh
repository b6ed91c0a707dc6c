// common.cuh -- device helpers shared by the row (split-KV) and tile (tcgen05) kernels.
//
// Everything here is sm_100a PTX or plain CUDA: mbarrier phase waits with a clock
// bound, bulk (TMA engine) global->shared copies, the reference's FP8 e4m3 decode
// as integer bit moves, and the sign-bit score.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "hyperion_b200.h"

namespace hyp {

// EXP_CLAMP of the reference (hyperion_fa3_production_final.py:59): every softmax
// exponent is max(x, -80) before exp.
constexpr float kExpClamp = -80.0f;
constexpr float kLog2e = 1.4426950408889634f;

// A bounded wait gives up after this many SM clock cycles (about 1 s at 1.9 GHz),
// raises HYPERION_DEVERR_WAIT_TIMEOUT and lets the CTA unwind.
constexpr long long kWaitCycles = 2000000000LL;

// Workspace layout (byte offsets).  The counters block is zeroed on the stream at
// the start of every forward; the error word is sticky until read and cleared.
constexpr size_t kWsCounters = 0;     // uint32[16]: [0] row-kernel ticket, [1] tile-kernel ticket
constexpr size_t kWsError = 64;       // uint32 error flags
constexpr size_t kWsPartials = 256;   // float partials of the split-KV row kernel

// Copies of the output a forward may write besides O: the gathered output buffers of
// the other ranks of a head-sharded forward, mapped into this process.
constexpr int kMaxOutPeers = 7;

struct FwdParams {
  const int4* worklist;
  int total_work;
  const uint32_t* q;      // [n_bh*seq_q, W]
  const uint32_t* k;      // [pool_rows, W]
  const uint8_t* v;       // [pool_rows, D]
  const float* v_scale;
  int v_scale_mode;       // 0 per tensor, 1 index kv_of(bh) % numel, 2 per slot
  long long v_scale_numel;
  const int* ctx_lens;     // [n_bh / kv_group]: per KV (batch, head)
  int n_bh;                // query (batch, head) rows: numel(ctx_lens) * kv_group
  int kv_group;            // query heads per KV head (1: none); KV row of bh is bh / kv_group
  int group_items;         // grouped row kernel: work items per unit (1..4)
  const int* block_tables;  // nullptr -> contiguous
  long long pool_rows;
  long long pool_blocks;    // pool_rows / block_size
  void* o;
  int o_dtype;
  int seq_q, head_dim, block_size, num_blocks;
  float inv_sqrt_d;
  int causal;
  uint32_t* counters;
  uint32_t* err;
  float* partials;
  int n_split;
  int* debug_scores;
  long long debug_ld;
  int pages_all_valid;  // 1: every page id the kernels can read is inside the pool (host-checked)
  int o_align32;        // 1: O is 32-byte aligned, so a 16-value row piece is whole 32-byte sectors
  long long wait_cycles;  // bound of every device wait: kWaitCycles, shorter only under a test hook
  int fault_stage;        // test hook: index of the KV stage the loading warp leaves unarmed (-1: none)
  int ticket_group;       // tile kernel: (batch, head) rows per group of its ticket order (0: all rows)
  int n_o_peers;          // copies of O written beside it (0: none)
  void* o_peers[kMaxOutPeers];  // each receives every output element at O's own index
};

// KV-side (batch, head) row of query row `bh`: grouped-query attention maps
// kv_group consecutive query heads onto one KV head.  Context lengths, block-table
// rows, the contiguous layout and a per-head V scale are all indexed by it.
__device__ __forceinline__ int kv_of(const FwdParams& p, int bh) {
  return p.kv_group == 1 ? bh : bh / p.kv_group;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void raise_error(uint32_t* err, uint32_t flag) {
  atomicOr(err, flag);
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps
// in the barrier unit until it completes or about `ns` nanoseconds pass, instead
// of returning at once and spinning in the issue slots the working warps need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Longest sleep of one try in a bounded wait: well under the shortest bound a
// test sets (about a millisecond), so a wait that runs out still ends promptly.
constexpr uint32_t kWaitSleepNs = 100000;

// Abort flag and wait bound of a CTA, kept in its shared memory: the flag is set
// by the first wait that runs out, and every other wait then gives up.
struct WaitCtl {
  int flag;
  int pad;
  long long limit;  // SM clock cycles a wait may take: kWaitCycles unless a test shortened it
};

// The spinning part of mbar_wait, kept out of line: the kernels have a few dozen
// wait sites, and one shared copy of the loop keeps their code small.
__device__ __noinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, volatile WaitCtl* ctl, uint32_t* err) {
  const long long t0 = clock64();
  const long long limit = ctl->limit;
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, kWaitSleepNs)) return true;
    if (ctl->flag) return false;
    if (clock64() - t0 > limit) {
      raise_error(err, HYPERION_DEVERR_WAIT_TIMEOUT);
      ctl->flag = 1;
      return false;
    }
  }
}

// Waits for the phase with parity `parity` to complete.  Returns false (and sets
// the CTA's abort flag) when the CTA is aborting or the wait exceeded ctl->limit SM
// clock cycles; the first waiter that times out records HYPERION_DEVERR_WAIT_TIMEOUT.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile WaitCtl* ctl, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_spin(bar, parity, ctl, err);
}

// mbar_wait for a whole warp: every lane waits, and the outcome is the same in all
// 32 lanes (a timeout in one lane fails the wait for the warp), so a warp never
// splits across a __syncwarp or a .sync.aligned instruction after a timeout.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile WaitCtl* ctl,
                                               uint32_t* err) {
  const bool ok = mbar_wait(bar, parity, ctl, err);
  return __all_sync(0xffffffffu, ok);
}

// Bounded wait that ignores the abort flag: used on the way out of an aborted CTA
// to let copies already in flight land before the CTA's shared memory is released.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, long long limit) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return;
  }
}

// ---------------------------------------------------------------------------
// Bulk copy global -> shared through the TMA engine (no tensor map: plain bytes).
// Both addresses 16-byte aligned, size a multiple of 16.
// ---------------------------------------------------------------------------
// The copy takes an L2 eviction-priority hint (evict-first for data read once,
// the KV streams; evict-last for data read again).
__device__ __forceinline__ void bulk_g2s_stream(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                                uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// Arithmetic
// ---------------------------------------------------------------------------
// 2^x with the hardware approximation (MUFU.EX2).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp(max(x, EXP_CLAMP)) as the reference writes it (__expf(fmaxf(x, EXP_CLAMP))).
__device__ __forceinline__ float exp_clamped(float x) {
  return ex2_approx(fmaxf(x, kExpClamp) * kLog2e);
}

// FP8 e4m3 -> f32 bit pattern scaled by 2^-120: sign to bit 31, the 7 exponent and
// mantissa bits to bits 26..20.  For every code this is exactly
// fp8_e4m3_to_fp32(code) * 2^-120 of the reference (hyperion_fa3_production_final.py:122-141),
// including subnormals (exponent field 0 -> f32 denormals) and the exponent-15
// codes 0x7F / 0xFF, which the reference decodes as +-480.
__device__ __forceinline__ float fp8_bits_to_f32_scaled(uint32_t byte_in_low_bits) {
  const uint32_t b = byte_in_low_bits & 0xFFu;
  return __uint_as_float(((b & 0x80u) << 24) | ((b & 0x7Fu) << 20));
}
constexpr float kTwoPow120 = 1.329227995784916e+36f;  // 2^120

// Two FP8 e4m3 codes held in bytes 1 and 3 of `v` -> f16x2 {byte1, byte3}, each
// equal to the reference decode divided by 256 (exact: f16 covers e4m3 / 256).
__device__ __forceinline__ uint32_t fp8x2_odd_to_f16x2_div256(uint32_t v) {
  return ((v >> 1) & 0x3F803F80u) | (v & 0x80008000u);
}
// Bytes 0 and 2 of `v` -> f16x2 {byte0, byte2}, decode / 256.
__device__ __forceinline__ uint32_t fp8x2_even_to_f16x2_div256(uint32_t v) {
  return ((v << 7) & 0x3F803F80u) | ((v << 8) & 0x80008000u);
}

// Two FP8 e4m3 codes in the low 16 bits of `v` -> f16x2 (byte 0 in the low half)
// by the hardware conversion: exact for every code except 0x7F and 0xFF, which it
// turns into NaN where the reference decodes them to +-480.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2_hw(uint32_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((unsigned short)(v & 0xFFFFu)));
  return r;
}
// Non-zero iff either half of the f16x2 `v` is a NaN (|bits| above 0x7C00): the
// add carries into bit 15 of a half exactly then, and never across halves.
__device__ __forceinline__ uint32_t f16x2_nan_bits(uint32_t v) {
  return ((v & 0x7FFF7FFFu) + 0x03FF03FFu) & 0x80008000u;
}

// {a, b} -> f16x2 (a in the low half), round to nearest even.
__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
  return r;
}
// a * b + c on f16x2 operands, round to nearest even.
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ float f16_lo_to_f32(uint32_t v) {
  float r;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; cvt.f32.f16 %0, l;}" : "=f"(r) : "r"(v));
  return r;
}
__device__ __forceinline__ float f16_hi_to_f32(uint32_t v) {
  float r;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %1; cvt.f32.f16 %0, h;}" : "=f"(r) : "r"(v));
  return r;
}

// Integer score D - 2*popcount(q XOR k) over W 32-bit words.
template <int W>
__device__ __forceinline__ int sign_score(const uint32_t (&q)[W], const uint32_t* k) {
  int p = 0;
#pragma unroll
  for (int i = 0; i < W; ++i) p += __popc(q[i] ^ k[i]);
  return W * 32 - 2 * p;
}

__device__ __forceinline__ float v_scale_for(const FwdParams& p, int bh, long long slot) {
  switch (p.v_scale_mode) {
    case 0: return __ldg(p.v_scale);
    case 1: return __ldg(p.v_scale + (kv_of(p, bh) % p.v_scale_numel));
    default: return __ldg(p.v_scale + slot);
  }
}

// Page id of page `page` of KV row `kv`, or -1 when it lies outside the pool.
__device__ __forceinline__ long long page_block_id_kv(const FwdParams& p, int kv, int page) {
  long long id;
  if (p.block_tables == nullptr) {
    id = (long long)kv * p.num_blocks + page;
  } else {
    id = __ldg(p.block_tables + (long long)kv * p.num_blocks + page);
  }
  if (id < 0 || id >= p.pool_blocks) return -1;
  return id;
}

// Page id of page `page` of query (batch, head) row `bh`, or -1 outside the pool.
__device__ __forceinline__ long long page_block_id(const FwdParams& p, int bh, int page) {
  return page_block_id_kv(p, kv_of(p, bh), page);
}

template <typename T>
__device__ __forceinline__ T to_out(float x);
template <>
__device__ __forceinline__ float to_out<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half to_out<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ void store_out(void* o, int dtype, long long idx, float x) {
  if (dtype == HYPERION_DTYPE_F32) {
    static_cast<float*>(o)[idx] = x;
  } else if (dtype == HYPERION_DTYPE_BF16) {
    static_cast<__nv_bfloat16*>(o)[idx] = __float2bfloat16_rn(x);
  } else {
    static_cast<__half*>(o)[idx] = __float2half_rn(x);
  }
}

// Final store of output element idx: to O and to every peer copy, same index.
__device__ __forceinline__ void store_out_all(const FwdParams& p, long long idx, float x) {
  store_out(p.o, p.o_dtype, idx, x);
  for (int k = 0; k < p.n_o_peers; ++k) store_out(p.o_peers[k], p.o_dtype, idx, x);
}

// A CTA that wrote into peer copies makes its stores visible system-wide before it
// exits; the caller's synchronisation after the forward then orders the readers.
__device__ __forceinline__ void fence_out_peers(const FwdParams& p) {
  if (p.n_o_peers > 0) __threadfence_system();
}

// Resolved key range of one work item: keys [0, kv_end) after the context length,
// the block-table width and the causal bound; `valid` false when the item itself
// is out of range (its output row is then not written).
struct ItemInfo {
  int bh;
  int q_idx;
  int kv_end;
  bool valid;
};

__device__ __forceinline__ ItemInfo resolve_item(const FwdParams& p, int item) {
  ItemInfo r;
  const int4 wl = __ldg(p.worklist + item);
  r.q_idx = wl.x;
  r.bh = wl.y;
  r.valid = (r.bh >= 0 && r.bh < p.n_bh && r.q_idx >= 0 && r.q_idx < p.seq_q);
  r.kv_end = 0;
  if (!r.valid) return r;
  int ctx = __ldg(p.ctx_lens + kv_of(p, r.bh));
  const long long cap = (long long)p.num_blocks * p.block_size;
  if (ctx < 0) ctx = 0;
  if ((long long)ctx > cap) ctx = (int)cap;
  if (p.causal && ctx > r.q_idx + 1) ctx = r.q_idx + 1;
  r.kv_end = ctx;
  return r;
}

// Raises the item-level error flags once per item (called by one thread).
__device__ __forceinline__ void check_item_errors(const FwdParams& p, int item) {
  const int4 wl = __ldg(p.worklist + item);
  const int q_idx = wl.x, bh = wl.y;
  if (!(bh >= 0 && bh < p.n_bh && q_idx >= 0 && q_idx < p.seq_q)) {
    raise_error(p.err, HYPERION_DEVERR_BAD_ITEM);
    return;
  }
  const int ctx = __ldg(p.ctx_lens + kv_of(p, bh));
  if (ctx < 0) raise_error(p.err, HYPERION_DEVERR_NEG_CTX);
  if ((long long)ctx > (long long)p.num_blocks * p.block_size) raise_error(p.err, HYPERION_DEVERR_CTX_OVERFLOW);
}

}  // namespace hyp
