// kv_write.cuh -- the cache writer: new keys and values in f16 / bf16 / f32 -> the
// forward's cache format (sign-bit K words, FP8 e4m3 V codes) at their paged slots.
//
// This is the step before the forward: the reference's engine allocates the paged
// pool (hyperion_fa3_production_final.py:1017-1032) but has no kernel that fills it.
// The format is the one the forward reads (README.md:18-23):
//   K: bit d%32 of word d/32 of the key's row is 1 where k[d] >= 0;
//   V: code = e4m3(clamp(v / scale, -448, 448)), rounded to nearest even, where the
//      scale is V_scale[0] (numel 1), V_scale[slot] (numel == pool rows, the
//      reference's per-slot layout) or V_scale[bh % numel] (per head / per (b, h)).
// Slot of token t of sequence b, head h (bh = b*H + h): page = t / block_size,
// id = block_tables[bh, page] (or bh*num_blocks + page with no table), slot =
// id*block_size + t%block_size -- the same addressing as the forward
// (hyperion_fa3_production_final.py:402-411).  Out-of-range ids or positions set an
// error flag and the row is skipped.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace hyp {
namespace kvw {

constexpr int kWarpsPerBlock = 8;

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// e4m3 code of y: round to nearest even, saturated to +-448 (y is already clamped,
// so saturation never changes a finite value; NaN stays NaN).
__device__ __forceinline__ uint32_t e4m3_code(float y) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.f), "f"(y));
  return r & 0xFFu;  // the second source lands in the low byte
}

struct Args {
  const void* k_new;  // [n_tokens, n_heads, D]
  const void* v_new;
  int n_tokens, n_heads;
  const int32_t* seq_ids;    // [n_tokens]
  const int32_t* positions;  // [n_tokens]
  const int32_t* block_tables;  // [batch*n_heads, num_blocks] or nullptr (contiguous)
  long long bt_rows;            // rows of block_tables (batch * n_heads)
  int block_size, num_blocks;
  const float* v_scale;
  long long v_scale_numel;
  uint32_t* k_cache;  // [pool_rows, D/32]
  uint8_t* v_cache;   // [pool_rows, D]
  long long pool_rows;
  uint32_t* err;
};

// One warp per (token, head).  Lane l reads dims l, l+32, ... so a ballot over the
// warp is one sign word, and each group of 32 V codes is one 32-byte store.
template <int D, typename T>
__global__ void __launch_bounds__(32 * kWarpsPerBlock) kv_write_kernel(Args a) {
  constexpr int W = D / 32;
  const int lane = threadIdx.x & 31;
  const long long wid = (long long)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (wid >= (long long)a.n_tokens * a.n_heads) return;
  const int tok = (int)(wid / a.n_heads);
  const int h = (int)(wid - (long long)tok * a.n_heads);
  const int b = __ldg(a.seq_ids + tok);
  const int t = __ldg(a.positions + tok);
  const long long bh = (long long)b * a.n_heads + h;
  const long long cap = (long long)a.num_blocks * a.block_size;
  if (b < 0 || t < 0 || (long long)t >= cap || (a.block_tables && bh >= a.bt_rows)) {
    if (lane == 0) raise_error(a.err, HYPERION_DEVERR_BAD_ITEM);
    return;
  }
  const int page = t / a.block_size;
  const long long id = a.block_tables ? (long long)__ldg(a.block_tables + bh * a.num_blocks + page)
                                      : bh * a.num_blocks + page;
  const long long slot = id * a.block_size + (t - page * a.block_size);
  if (id < 0 || slot >= a.pool_rows) {
    if (lane == 0) raise_error(a.err, HYPERION_DEVERR_BAD_BLOCK);
    return;
  }
  // The forward's rule for the scale a code is decoded with: per tensor (numel 1),
  // per slot (numel == pool rows), else per head / per (batch, head).
  const long long si = a.v_scale_numel == 1 ? 0 : (a.v_scale_numel == a.pool_rows ? slot : bh % a.v_scale_numel);
  const float scale = __ldg(a.v_scale + si);
  const T* kr = static_cast<const T*>(a.k_new) + wid * D;
  const T* vr = static_cast<const T*>(a.v_new) + wid * D;
  uint32_t word = 0;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const uint32_t bits = __ballot_sync(0xffffffffu, to_f32<T>(kr[32 * w + lane]) >= 0.f);
    if (lane == w) word = bits;
  }
  if (lane < W) a.k_cache[slot * W + lane] = word;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    float y = __fdiv_rn(to_f32<T>(vr[32 * w + lane]), scale);
    if (y == y) y = fminf(fmaxf(y, -448.f), 448.f);
    a.v_cache[slot * D + 32 * w + lane] = (uint8_t)e4m3_code(y);
  }
}

template <int D>
inline cudaError_t launch_d(const Args& a, int in_dtype, cudaStream_t st) {
  const long long warps = (long long)a.n_tokens * a.n_heads;
  const unsigned grid = (unsigned)((warps + kWarpsPerBlock - 1) / kWarpsPerBlock);
  if (grid == 0) return cudaSuccess;
  if (in_dtype == HYPERION_DTYPE_F32) {
    kv_write_kernel<D, float><<<grid, 32 * kWarpsPerBlock, 0, st>>>(a);
  } else if (in_dtype == HYPERION_DTYPE_BF16) {
    kv_write_kernel<D, __nv_bfloat16><<<grid, 32 * kWarpsPerBlock, 0, st>>>(a);
  } else {
    kv_write_kernel<D, __half><<<grid, 32 * kWarpsPerBlock, 0, st>>>(a);
  }
  return cudaGetLastError();
}

inline cudaError_t launch(const Args& a, int head_dim, int in_dtype, cudaStream_t st) {
  return head_dim == 256 ? launch_d<256>(a, in_dtype, st) : launch_d<128>(a, in_dtype, st);
}

}  // namespace kvw
}  // namespace hyp
