// capi.cu -- the C ABI declared in include/hyperion_b200.h.
//
// Host side of the forward: validates every pointer and size the reference's
// pybind boundary would have taken on trust (hyperion_fa3_production_final.py:598-601),
// derives the launch from the device (the reference hard-codes grid = min(2*SM, 256),
// block 256, :907-912), zeroes the per-call work counter on the caller's stream
// (the reference needs a separate reset launch, :73-77 / :905) and enqueues the
// row kernel or the tcgen05 tile kernel.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "row_kernel.cuh"
#include "row_group_kernel.cuh"
#include "row_mma_kernel.cuh"
#include "tile_kernel.cuh"
#include "kv_write.cuh"
#include "launch_table.h"

namespace {

// Main kernel of a call, out[4] of hyperion_last_call_info.
enum KernelId { kKernelNone = 0, kKernelRow = 1, kKernelGroup = 2, kKernelGroupMma = 3, kKernelTile = 4 };

thread_local std::string g_last_error;
thread_local int32_t g_last_call[5] = {0, 0, 0, 0, 0};
// Split count and workspace bytes of the last row-path call, for the message of a
// workspace refusal.
thread_local int g_last_splits = 1;
thread_local size_t g_last_need = 0;

void clear_last_call() {
  for (int32_t& v : g_last_call) v = 0;
}

// A fault armed by hyperion_debug_fault for the next forward of this thread.
struct FaultHook {
  bool armed = false;
  long long wait_cycles = 0;
  int stage = -1;
};
thread_local FaultHook g_fault;

int fail(int code, const char* msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return HYPERION_ERR_CUDA;
}

struct DevInfo {
  bool ready = false;
  int n_sm = 0;
  int row_ctas_128 = 1, row_ctas_256 = 1;
  int row_smem_128 = 0, row_smem_256 = 0;
  int group_ctas_128 = 1, group_ctas_256 = 1;  // grouped-query row kernel
  int group_smem_128 = 0, group_smem_256 = 0;
  int tile_ctas = 0, tile_smem = 0;
  bool tile_ok = false;
  std::string tile_why;  // why the tile kernel is unavailable ("" when it is)
  int mma_ctas = 0, mma_smem = 0;  // grouped-query kernel with the products on the tensor core
  bool mma_ok = false;
};

constexpr int kMaxDevices = 64;
DevInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

template <int D>
int setup_row(int& ctas, int& smem) {
  smem = (int)sizeof(hyp::row::Smem<D>);
  cudaError_t e = cudaFuncSetAttribute(hyp::row::row_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(row)");
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas, hyp::row::row_fwd_kernel<D>, hyp::row::kThreads, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(row)");
  if (ctas < 1) ctas = 1;
  return HYPERION_OK;
}

template <int D>
int setup_group(int& ctas, int& smem) {
  smem = (int)sizeof(hyp::row::GroupSmem<D>);
  cudaError_t e =
      cudaFuncSetAttribute(hyp::row::row_group_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(row group)");
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas, hyp::row::row_group_kernel<D>, hyp::row::kGThreads, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(row group)");
  if (ctas < 1) ctas = 1;
  return HYPERION_OK;
}

int get_dev(const DevInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(HYPERION_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DevInfo& di = g_dev[dev];
  if (!di.ready) {
    e = cudaDeviceGetAttribute(&di.n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    int rc = setup_row<128>(di.row_ctas_128, di.row_smem_128);
    if (rc) return rc;
    rc = setup_row<256>(di.row_ctas_256, di.row_smem_256);
    if (rc) return rc;
    rc = setup_group<128>(di.group_ctas_128, di.group_smem_128);
    if (rc) return rc;
    rc = setup_group<256>(di.group_ctas_256, di.group_smem_256);
    if (rc) return rc;
    const char* why = "";
    rc = hyp::tile::setup(di.tile_ctas, di.tile_smem, &why);
    di.tile_ok = (rc == HYPERION_OK);
    if (!di.tile_ok) {
      di.tile_ctas = 0;
      di.tile_why = why;
      cudaGetLastError();
    }
    di.mma_ok = hyp::rmma::setup(di.mma_ctas, di.mma_smem) == cudaSuccess && di.mma_ctas > 0;
    if (!di.mma_ok) {
      di.mma_ctas = 0;
      cudaGetLastError();
    }
    di.ready = true;
  }
  *out = &di;
  return HYPERION_OK;
}

// The measured split count for a call of `kernel` (0 row kernel, 1 grouped row
// kernel with 4 query heads per KV head, 2 the same on the tensor-core grouped
// kernel) with `items` work items of up to `keys`
// keys, or 0 when the launch table (launch_table.h, written by tune_launch.py from a
// sweep on B200) has no entry within a factor of 2 of both, or was measured on
// another SM count or head_dim.
int table_splits(const DevInfo& di, int kernel, int D, long long items, long long keys) {
  if (D != 128 || di.n_sm != hyp::table::kSplitTableSms || items <= 0 || keys <= 0) return 0;
  int best = 0;
  double best_d = 1e30;
  for (const hyp::table::SplitEntry& e : hyp::table::kSplitTable) {
    if (e.kernel != kernel) continue;
    const double di_ = std::fabs(std::log2((double)items / e.items));
    const double dk = std::fabs(std::log2((double)keys / e.keys));
    if (di_ > 1.0 || dk > 1.0) continue;
    if (di_ + dk < best_d) {
      best_d = di_ + dk;
      best = e.splits;
    }
  }
  return best;
}

// KV splits per item of the row kernel: the launch table's measured count near the
// call's shape, else this rule.  A worklist that alone gives every CTA slot about
// 16 units is not split.  A shorter one is split until it does, and at least into
// pieces of at most 8192 keys of the table; no piece is shorter than 512 keys, and
// an item has at most 16 pieces.
int choose_splits(const DevInfo& di, int D, int total_work, long long max_keys) {
  if (total_work <= 0) return 1;
  const int measured = table_splits(di, 0, D, total_work, max_keys);
  if (measured > 0) return measured;
  const int ctas = (D == 256) ? di.row_ctas_256 : di.row_ctas_128;
  const long long target = (long long)di.n_sm * ctas * 16;
  if (total_work >= target) return 1;
  long long ns = (target + total_work - 1) / total_work;
  ns = std::max<long long>(ns, (max_keys + 8191) / 8192);
  ns = std::min<long long>(ns, std::max<long long>(1, max_keys / 512));
  ns = std::min<long long>(ns, 16);
  return (int)std::max<long long>(ns, 1);
}

// KV splits per unit of a grouped kernel (`mma`: the one with the products on the
// tensor core), whose unit holds up to group_items (at most 4) work items.  Decode
// with 4 query heads per KV head takes the launch table's measured count near its
// shape for that kernel; otherwise the rule: enough
// units for 4 per CTA slot and, while units are scarce (fewer than 16 per slot),
// pieces of at most 2048 keys (8192 on the tensor-core kernel) so that ragged
// contexts balance; no piece shorter
// than 512 keys, at most 16 pieces.  (Paged decode with 32 query heads over 8 KV
// heads, contexts U[512, 32768]: 1.21 ms at 13-16 pieces against 1.27 ms at the row
// kernel's choice of 4 in isolated calls; the same 1.26 ms under the sustained
// power cap, where the whole step with host copies gains 4 %.)
int choose_group_splits(const DevInfo& di, int D, long long items, int group_items, bool decode,
                        long long max_keys, bool mma) {
  if (items <= 0) return 1;
  if (decode && group_items == 4) {
    const int measured = table_splits(di, mma ? 2 : 1, D, items, max_keys);
    if (measured > 0) return measured;
  }
  const long long chunks = (items + group_items - 1) / group_items;
  const long long slots =
      (long long)di.n_sm * (mma ? di.mma_ctas : (D == 256) ? di.group_ctas_256 : di.group_ctas_128);
  if (chunks >= 16 * slots) return 1;
  long long ns = (4 * slots + chunks - 1) / chunks;
  // The tensor-core kernel pays more per piece (a TMEM read-out) and less per key.
  const long long piece = mma ? 8192 : 2048;
  ns = std::max(ns, (max_keys + piece - 1) / piece);
  ns = std::min(ns, std::max<long long>(1, max_keys / 512));
  ns = std::min<long long>(ns, 16);
  return (int)std::max<long long>(ns, 1);
}

size_t partial_bytes(int total_work, int n_split, int D) {
  if (n_split <= 1) return 0;
  return (size_t)total_work * n_split * (2 + D) * sizeof(float);
}

// Workspace of the automatic split choice, for either row kernel (a forced
// num_splits needs 256 + total_work * num_splits * (2 + head_dim) * 4 bytes).
// The grouped kernels' choice is bounded by their smallest unit count, 4 items a unit.
size_t workspace_needed(const DevInfo& di, int total_work, int D, int block_size, int num_blocks) {
  const long long max_keys = (long long)std::max(block_size, 1) * std::max(num_blocks, 1);
  int ns = std::max({choose_splits(di, D, total_work, max_keys),
                     choose_group_splits(di, D, total_work, 4, true, max_keys, false),
                     choose_group_splits(di, D, total_work, 4, false, max_keys, false)});
  if (di.mma_ok)
    ns = std::max({ns, choose_group_splits(di, D, total_work, 4, true, max_keys, true),
                   choose_group_splits(di, D, total_work, 4, false, max_keys, true)});
  return hyp::kWsPartials + partial_bytes(total_work, ns, D);
}

}  // namespace

extern "C" {

int32_t hyperion_version(void) { return 1 * 10000 + 4 * 100 + 0; }

const char* hyperion_last_error_string(void) { return g_last_error.c_str(); }

int hyperion_last_call_info(int32_t* out, int32_t n) {
  if (out == nullptr) return fail(HYPERION_ERR_INVALID_ARG, "out is NULL");
  for (int i = 0; i < n && i < 5; ++i) out[i] = g_last_call[i];
  return HYPERION_OK;
}

size_t hyperion_workspace_bytes(int32_t total_work, int32_t head_dim, int32_t block_size, int32_t num_blocks) {
  const DevInfo* di = nullptr;
  if (get_dev(&di) != HYPERION_OK) return 0;
  if (total_work < 0) total_work = 0;
  return workspace_needed(*di, total_work, head_dim == 256 ? 256 : 128, block_size, num_blocks);
}

int hyperion_launch_info(int32_t* out, int32_t n) {
  const DevInfo* di = nullptr;
  const int rc = get_dev(&di);
  if (rc) return rc;
  const int32_t v[15] = {di->n_sm,           di->row_ctas_128,      di->row_smem_128,  di->tile_ctas,
                         di->tile_smem,       di->row_ctas_256,      di->tile_ok ? 1 : 0, hyp::row::kThreads,
                         hyp::row::kGThreads, di->group_ctas_128,    di->group_smem_128, hyp::tile::kThreads,
                         di->mma_ok ? hyp::rmma::kThreads : 0, di->mma_ctas, di->mma_ok ? di->mma_smem : 0};
  for (int i = 0; i < n && i < 15; ++i) out[i] = v[i];
  if (!di->tile_ok) g_last_error = "tile kernel unavailable: " + di->tile_why;
  return HYPERION_OK;
}

int hyperion_apex_kernel_ex(const int32_t* worklist, int32_t total_work, const uint32_t* Q, const float* Q_scale,
                            const uint32_t* K_cache, const float* K_scale, const uint8_t* V_cache,
                            const float* V_scale, const int32_t* context_lens, const int32_t* block_tables,
                            void* O, int32_t seq_q, int32_t head_dim, int32_t k_packed_bytes, int32_t block_size,
                            int32_t num_blocks, float inv_sqrt_d, int32_t causal, const hyperion_extents* ext,
                            const hyperion_options* opt, void* workspace, size_t workspace_bytes, void* stream) {
  (void)Q_scale;
  (void)K_scale;
  if (ext == nullptr) return fail(HYPERION_ERR_INVALID_ARG, "ext (sizes) is NULL");
  if (total_work < 0) return fail(HYPERION_ERR_INVALID_ARG, "total_work < 0");
  if (head_dim != 128 && head_dim != 256)
    return fail(HYPERION_ERR_UNSUPPORTED, "head_dim must be 128 or 256");
  if (k_packed_bytes != head_dim / 8)
    return fail(HYPERION_ERR_INVALID_ARG, "k_packed_bytes must be head_dim/8 (sign-bit K)");
  if (seq_q < 1) return fail(HYPERION_ERR_INVALID_ARG, "seq_q < 1");
  if (block_size < 1) return fail(HYPERION_ERR_INVALID_ARG, "block_size < 1");
  if (num_blocks < 1) return fail(HYPERION_ERR_INVALID_ARG, "num_blocks < 1");
  if (!std::isfinite(inv_sqrt_d)) return fail(HYPERION_ERR_INVALID_ARG, "inv_sqrt_d is not finite");
  if (total_work == 0) {
    // Nothing to do, whatever the tensors hold: a rank that owns no (batch, head)
    // row passes empty ones.
    clear_last_call();
    return HYPERION_OK;
  }
  if (ext->n_bh < 1) return fail(HYPERION_ERR_INVALID_ARG, "n_bh (context_lens numel) < 1");
  if (ext->pool_rows < 1) return fail(HYPERION_ERR_INVALID_ARG, "pool_rows < 1");
  if (ext->v_scale_numel < 1) return fail(HYPERION_ERR_INVALID_ARG, "V_scale is empty");
  if (ext->o_dtype != HYPERION_DTYPE_F16 && ext->o_dtype != HYPERION_DTYPE_BF16 && ext->o_dtype != HYPERION_DTYPE_F32)
    return fail(HYPERION_ERR_INVALID_ARG, "o_dtype is not F16, BF16 or F32");
  if (opt && opt->kv_group < 0) return fail(HYPERION_ERR_INVALID_ARG, "kv_group < 0");
  if (opt && opt->sm_budget < 0) return fail(HYPERION_ERR_INVALID_ARG, "sm_budget < 0");
  const int kv_group = (opt && opt->kv_group > 1) ? opt->kv_group : 1;
  if ((long long)ext->n_bh * kv_group > 0x7fffffffLL)
    return fail(HYPERION_ERR_INVALID_ARG, "n_bh * kv_group exceeds int32");
  const bool paged = ext->block_tables_numel != 0;
  if (paged) {
    if (block_tables == nullptr) return fail(HYPERION_ERR_INVALID_ARG, "block_tables is NULL but numel > 0");
    if (ext->block_tables_numel < (int64_t)ext->n_bh * num_blocks)
      return fail(HYPERION_ERR_INVALID_ARG, "block_tables numel < n_bh * num_blocks");
  }
  if (workspace == nullptr) return fail(HYPERION_ERR_WORKSPACE, "workspace is NULL");
  if (workspace_bytes < hyp::kWsPartials)
    return fail(HYPERION_ERR_WORKSPACE, "workspace smaller than hyperion_workspace_bytes()");
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(HYPERION_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  if (!worklist || !Q || !K_cache || !V_cache || !V_scale || !context_lens || !O)
    return fail(HYPERION_ERR_INVALID_ARG, "a tensor pointer is NULL");
  if (reinterpret_cast<uintptr_t>(worklist) % 16 != 0)
    return fail(HYPERION_ERR_INVALID_ARG, "worklist must be 16-byte aligned (int4 rows)");
  if (reinterpret_cast<uintptr_t>(K_cache) % 16 != 0 || reinterpret_cast<uintptr_t>(V_cache) % 16 != 0)
    return fail(HYPERION_ERR_INVALID_ARG, "K_cache and V_cache must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(Q) % 16 != 0) return fail(HYPERION_ERR_INVALID_ARG, "Q must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(O) % 16 != 0) return fail(HYPERION_ERR_INVALID_ARG, "O must be 16-byte aligned");

  const DevInfo* di = nullptr;
  int rc = get_dev(&di);
  if (rc) return rc;

  const int path_req = opt ? opt->path : HYPERION_PATH_AUTO;
  // SMs the persistent grids are sized for: all of them, or the caller's budget.
  const int sm_use = (opt && opt->sm_budget > 0) ? std::min<int>(opt->sm_budget, di->n_sm) : di->n_sm;
  if (path_req != HYPERION_PATH_AUTO && path_req != HYPERION_PATH_ROW && path_req != HYPERION_PATH_TILE)
    return fail(HYPERION_ERR_INVALID_ARG, "unknown path");

  hyp::FwdParams p;
  std::memset(&p, 0, sizeof(p));
  p.worklist = reinterpret_cast<const int4*>(worklist);
  p.total_work = total_work;
  p.q = Q;
  p.k = K_cache;
  p.v = V_cache;
  p.v_scale = V_scale;
  p.v_scale_numel = ext->v_scale_numel;
  p.v_scale_mode = (ext->v_scale_numel == 1) ? 0 : (ext->v_scale_numel == ext->pool_rows ? 2 : 1);
  p.ctx_lens = context_lens;
  p.n_bh = ext->n_bh * kv_group;
  p.kv_group = kv_group;
  p.group_items = 1;
  p.block_tables = paged ? block_tables : nullptr;
  p.pool_rows = ext->pool_rows;
  p.pool_blocks = ext->pool_rows / block_size;
  p.o = O;
  p.o_dtype = ext->o_dtype;
  p.seq_q = seq_q;
  p.head_dim = head_dim;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.inv_sqrt_d = inv_sqrt_d;
  p.causal = causal ? 1 : 0;
  // Contiguous layout: page ids are bh * num_blocks + page; all of them are in the
  // pool when the pool holds n_bh * num_blocks pages.
  p.pages_all_valid = (!paged && (long long)ext->n_bh * num_blocks <= p.pool_blocks) ? 1 : 0;
  p.o_align32 = (reinterpret_cast<uintptr_t>(O) % 32 == 0) ? 1 : 0;
  // Peer copies of O: the same elements at the same indices, for a head-sharded
  // caller whose ranks all hold the gathered output.
  const int n_peers = opt ? opt->n_o_peers : 0;
  if (n_peers < 0 || n_peers > hyp::kMaxOutPeers)
    return fail(HYPERION_ERR_INVALID_ARG, "n_o_peers must be in [0, 7]");
  if (n_peers > 0 && opt->o_peers == nullptr) return fail(HYPERION_ERR_INVALID_ARG, "o_peers is NULL");
  p.n_o_peers = n_peers;
  for (int k = 0; k < n_peers; ++k) {
    void* q = opt->o_peers[k];
    if (q == nullptr) return fail(HYPERION_ERR_INVALID_ARG, "an o_peers entry is NULL");
    if (reinterpret_cast<uintptr_t>(q) % 16 != 0)
      return fail(HYPERION_ERR_INVALID_ARG, "o_peers entries must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(q) % 32 != 0) p.o_align32 = 0;
    p.o_peers[k] = q;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.counters = reinterpret_cast<uint32_t*>(ws + hyp::kWsCounters);
  p.err = reinterpret_cast<uint32_t*>(ws + hyp::kWsError);
  p.partials = reinterpret_cast<float*>(ws + hyp::kWsPartials);
  p.debug_scores = opt ? opt->debug_scores : nullptr;
  p.debug_ld = opt ? opt->debug_ld : 0;
  if (p.debug_scores && p.debug_ld < 1) return fail(HYPERION_ERR_INVALID_ARG, "debug_ld < 1");
  p.wait_cycles = hyp::kWaitCycles;
  p.fault_stage = -1;
  if (g_fault.armed) {  // consumed by this call
    p.wait_cycles = g_fault.wait_cycles;
    p.fault_stage = g_fault.stage;
    g_fault.armed = false;
  }

  clear_last_call();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long max_keys = (long long)block_size * num_blocks;

  // Kernel choice: the tile kernel needs head_dim 128, a per-tensor / per-head V
  // scale and enough query rows per (batch, head) to fill 128-row tiles.
  const bool tile_fits = di->tile_ok && head_dim == 128 && p.v_scale_mode != 2;
  int path = path_req;
  if (path == HYPERION_PATH_AUTO) path = (tile_fits && seq_q >= 64) ? HYPERION_PATH_TILE : HYPERION_PATH_ROW;
  if (path == HYPERION_PATH_TILE && !tile_fits)
    return fail(HYPERION_ERR_UNSUPPORTED,
                ("tile path needs head_dim 128, a per-tensor or per-head V scale and a device that loaded it" +
                 (di->tile_ok ? std::string() : "; " + di->tile_why)).c_str());

  // The work counters are zeroed on the stream just before the kernels, once every
  // check has passed: a refused call leaves the workspace untouched.
  cudaError_t e = cudaSuccess;
  if (path == HYPERION_PATH_TILE) {
    e = cudaMemsetAsync(ws + hyp::kWsCounters, 0, 64, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(counters)");
    int grid = 0;
    rc = hyp::tile::launch(p, sm_use, di->tile_ctas, di->tile_smem, st, &grid);
    if (rc) return rc;
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "tile kernel launch");
    g_last_call[0] = HYPERION_PATH_TILE;
    g_last_call[1] = 1;
    g_last_call[2] = 1;
    g_last_call[3] = grid;
    g_last_call[4] = kKernelTile;
    return HYPERION_OK;
  }

  // Grouped row kernel: a unit is up to 4 consecutive work items and one KV
  // split, and a run of them on one KV row streams its keys once: the query heads
  // of one KV head (grouped-query attention), or neighbouring query rows of one
  // (batch, head) in a prefill worklist.
  // At head_dim 128 with a per-tensor or per-head V scale the grouped runs take the
  // kernel with the P.V products on the tensor core (row_mma_kernel.cuh); otherwise,
  // or when the caller asks for it, the one with the products on the CUDA cores.
  const bool grouped = kv_group > 1 || seq_q > 1;
  p.group_items = !grouped ? 1 : (kv_group > 1) ? std::min(kv_group, hyp::row::kGroupMax) : hyp::row::kGroupMax;
  const int group_req = opt ? opt->group_kernel : HYPERION_GROUP_AUTO;
  if (group_req != HYPERION_GROUP_AUTO && group_req != HYPERION_GROUP_CUDA && group_req != HYPERION_GROUP_MMA)
    return fail(HYPERION_ERR_INVALID_ARG, "group_kernel must be HYPERION_GROUP_AUTO, _CUDA or _MMA");
  CUtensorMap vmap;
  const bool mma_fits = grouped && group_req != HYPERION_GROUP_CUDA && di->mma_ok &&
                        hyp::rmma::fits(head_dim, p.v_scale_mode, inv_sqrt_d, block_size, num_blocks, V_cache,
                                        ext->pool_rows) &&
                        hyp::rmma::encode_vmap(&vmap, V_cache, ext->pool_rows, block_size);
  if (grouped && group_req == HYPERION_GROUP_MMA && !mma_fits)
    return fail(HYPERION_ERR_UNSUPPORTED,
                "the tensor-core grouped kernel needs head_dim 128, a per-tensor or per-head V scale, "
                "|inv_sqrt_d| <= 0.117, one page per row or pages of 8 to 128 keys dividing 128 or of a multiple of "
                "128 keys, a "
                "16-byte aligned V_cache of fewer than 2^32 rows, and a device that loaded it");
  const bool use_mma = mma_fits;
  const long long chunks = ((long long)total_work + p.group_items - 1) / p.group_items;
  int ns = (opt && opt->num_splits > 0) ? std::min(opt->num_splits, 16)
           : grouped                    ? choose_group_splits(*di, head_dim, total_work, p.group_items, seq_q == 1,
                                                                  max_keys, use_mma)
                                        : choose_splits(*di, head_dim, total_work, max_keys);
  const size_t need = hyp::kWsPartials + partial_bytes(total_work, ns, head_dim);
  g_last_splits = ns;
  g_last_need = need;
  if (workspace_bytes < need) return fail(HYPERION_ERR_WORKSPACE, "workspace smaller than hyperion_workspace_bytes()");
  p.n_split = ns;
  const long long units = (long long)total_work * ns;
  if (units > 0x7fffffffLL) return fail(HYPERION_ERR_UNSUPPORTED, "too many work units");
  if (grouped && chunks * ns > 0x7fffffffLL) return fail(HYPERION_ERR_UNSUPPORTED, "too many work units");
  e = cudaMemsetAsync(ws + hyp::kWsCounters, 0, 64, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(counters)");
  int grid = 0;
  int kernel = kKernelRow;
  if (use_mma) {
    const long long gunits = chunks * ns;
    grid = (int)std::min<long long>(gunits, (long long)sm_use * di->mma_ctas);
    hyp::rmma::row_mma_kernel<<<grid, hyp::rmma::kThreads, di->mma_smem, st>>>(p, (int)gunits, vmap);
    kernel = kKernelGroupMma;
  } else if (grouped) {
    kernel = kKernelGroup;
    const long long gunits = chunks * ns;
    const int ctas = (head_dim == 256) ? di->group_ctas_256 : di->group_ctas_128;
    const int smem = (head_dim == 256) ? di->group_smem_256 : di->group_smem_128;
    grid = (int)std::min<long long>(gunits, (long long)sm_use * ctas);
    if (head_dim == 256) {
      hyp::row::row_group_kernel<256><<<grid, hyp::row::kGThreads, smem, st>>>(p, (int)gunits);
    } else {
      hyp::row::row_group_kernel<128><<<grid, hyp::row::kGThreads, smem, st>>>(p, (int)gunits);
    }
  } else {
    const int ctas = (head_dim == 256) ? di->row_ctas_256 : di->row_ctas_128;
    const int smem = (head_dim == 256) ? di->row_smem_256 : di->row_smem_128;
    grid = (int)std::min<long long>(units, (long long)sm_use * ctas);
    if (head_dim == 256) {
      hyp::row::row_fwd_kernel<256><<<grid, hyp::row::kThreads, smem, st>>>(p, (int)units);
    } else {
      hyp::row::row_fwd_kernel<128><<<grid, hyp::row::kThreads, smem, st>>>(p, (int)units);
    }
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "row kernel launch");
  if (ns > 1) {
    // Programmatic dependent launch: the combine is scheduled while the split kernel
    // runs (which allows it at its start) and waits on the device for that grid to
    // finish, instead of the launch starting only after it.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)total_work);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (head_dim == 256) {
      e = cudaLaunchKernelEx(&cfg, hyp::row::row_combine_kernel<256>, p);
    } else {
      e = cudaLaunchKernelEx(&cfg, hyp::row::row_combine_kernel<128>, p);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "combine kernel launch");
  }
  g_last_call[0] = HYPERION_PATH_ROW;
  g_last_call[1] = ns;
  g_last_call[2] = ns > 1 ? 2 : 1;
  g_last_call[3] = grid;
  g_last_call[4] = kernel;
  return HYPERION_OK;
}

int hyperion_apex_kernel(const int32_t* worklist, int32_t total_work, const uint32_t* Q, const float* Q_scale,
                         const uint32_t* K_cache, const float* K_scale, const uint8_t* V_cache, const float* V_scale,
                         const int32_t* context_lens, const int32_t* block_tables, void* O, int32_t seq_q,
                         int32_t head_dim, int32_t k_packed_bytes, int32_t block_size, int32_t num_blocks,
                         float inv_sqrt_d, int32_t causal, const hyperion_extents* ext, void* workspace,
                         size_t workspace_bytes, void* stream) {
  return hyperion_apex_kernel_ex(worklist, total_work, Q, Q_scale, K_cache, K_scale, V_cache, V_scale, context_lens,
                                 block_tables, O, seq_q, head_dim, k_packed_bytes, block_size, num_blocks, inv_sqrt_d,
                                 causal, ext, nullptr, workspace, workspace_bytes, stream);
}

int hyperion_debug_fault(int64_t wait_cycles, int32_t stage) {
  if (wait_cycles <= 0) return fail(HYPERION_ERR_INVALID_ARG, "wait_cycles must be > 0");
  g_fault.armed = true;
  g_fault.wait_cycles = wait_cycles;
  g_fault.stage = stage < 0 ? -1 : stage;
  return HYPERION_OK;
}

int hyperion_reset_counter(void* workspace, size_t workspace_bytes, void* stream) {
  if (workspace == nullptr || workspace_bytes < hyp::kWsPartials)
    return fail(HYPERION_ERR_WORKSPACE, "workspace missing or too small");
  cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(workspace) + hyp::kWsCounters, 0, 64,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(counters)");
  return HYPERION_OK;
}

int hyperion_read_device_errors(void* workspace, size_t workspace_bytes, void* stream, uint32_t* flags,
                                int32_t clear) {
  if (workspace == nullptr || workspace_bytes < hyp::kWsPartials || flags == nullptr)
    return fail(HYPERION_ERR_INVALID_ARG, "workspace or flags missing");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaError_t e = cudaMemcpyAsync(&v, ws + hyp::kWsError, sizeof(v), cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(error word)");
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  *flags = v;
  if (clear) {
    e = cudaMemsetAsync(ws + hyp::kWsError, 0, sizeof(uint32_t), st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(error word)");
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  }
  return HYPERION_OK;
}

}  // extern "C"

extern "C" int hyperion_kv_cache_write(const void* K_new, const void* V_new, int32_t in_dtype, int32_t n_tokens,
                                       int32_t n_heads, int32_t head_dim, const int32_t* seq_ids,
                                       const int32_t* positions, const int32_t* block_tables,
                                       int64_t block_tables_numel, int32_t block_size, int32_t num_blocks,
                                       const float* V_scale, int64_t v_scale_numel, uint32_t* K_cache,
                                       uint8_t* V_cache, int64_t pool_rows, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  if (in_dtype != HYPERION_DTYPE_F16 && in_dtype != HYPERION_DTYPE_BF16 && in_dtype != HYPERION_DTYPE_F32)
    return fail(HYPERION_ERR_INVALID_ARG, "in_dtype is not F16, BF16 or F32");
  if (head_dim != 128 && head_dim != 256) return fail(HYPERION_ERR_UNSUPPORTED, "head_dim must be 128 or 256");
  if (n_tokens < 0) return fail(HYPERION_ERR_INVALID_ARG, "n_tokens < 0");
  if (n_heads < 1) return fail(HYPERION_ERR_INVALID_ARG, "n_heads < 1");
  if (block_size < 1 || num_blocks < 1) return fail(HYPERION_ERR_INVALID_ARG, "block_size and num_blocks must be >= 1");
  if (v_scale_numel < 1) return fail(HYPERION_ERR_INVALID_ARG, "V_scale is empty");
  if (pool_rows < 1) return fail(HYPERION_ERR_INVALID_ARG, "pool_rows < 1");
  if (block_tables_numel < 0 || (block_tables_numel > 0 && block_tables == nullptr))
    return fail(HYPERION_ERR_INVALID_ARG, "block_tables is NULL but numel > 0");
  if (workspace == nullptr || workspace_bytes < hyp::kWsPartials ||
      reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(HYPERION_ERR_WORKSPACE, "workspace missing, smaller than 256 bytes or not 256-byte aligned");
  if (n_tokens == 0) return HYPERION_OK;
  if (!K_new || !V_new || !seq_ids || !positions || !V_scale || !K_cache || !V_cache)
    return fail(HYPERION_ERR_INVALID_ARG, "a tensor pointer is NULL");
  if (reinterpret_cast<uintptr_t>(K_cache) % 16 != 0) return fail(HYPERION_ERR_INVALID_ARG, "K_cache must be 16-byte aligned");
  const size_t esz = in_dtype == HYPERION_DTYPE_F32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(K_new) % esz != 0 || reinterpret_cast<uintptr_t>(V_new) % esz != 0)
    return fail(HYPERION_ERR_INVALID_ARG, "K_new / V_new are not aligned to their element size");
  hyp::kvw::Args a;
  a.k_new = K_new;
  a.v_new = V_new;
  a.n_tokens = n_tokens;
  a.n_heads = n_heads;
  a.seq_ids = seq_ids;
  a.positions = positions;
  a.block_tables = block_tables_numel > 0 ? block_tables : nullptr;
  a.bt_rows = block_tables_numel / num_blocks;
  a.block_size = block_size;
  a.num_blocks = num_blocks;
  a.v_scale = V_scale;
  a.v_scale_numel = v_scale_numel;
  a.k_cache = K_cache;
  a.v_cache = V_cache;
  a.pool_rows = pool_rows;
  a.err = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + hyp::kWsError);
  const cudaError_t e = hyp::kvw::launch(a, head_dim, in_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cache writer launch");
  return HYPERION_OK;
}

// ---------------------------------------------------------------------------
// The forward for callers that cannot allocate device memory.
//
// Its scratch (work counter at +0, error word at +64, split-KV partials from +256,
// the same layout as a caller workspace) is this file-scope array: one copy per
// device, created when the library's device code is loaded there and kept until
// the process exits.  Host code may not use the array's name as a device address
// (on the host it names a stand-in object), so each device's address is looked up
// once with cudaGetSymbolAddress and cached.
static __device__ __align__(256) uint8_t g_noalloc_scratch[HYPERION_NOALLOC_SCRATCH_BYTES];

namespace {

void* g_noalloc_addr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of the current device's copy of g_noalloc_scratch.
int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(HYPERION_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    if (ptr == nullptr || reinterpret_cast<uintptr_t>(ptr) % 256 != 0)
      return fail(HYPERION_ERR_CUDA, "scratch array has no 256-byte aligned device address");
    g_noalloc_addr[dev] = ptr;
  }
  *out = static_cast<uint8_t*>(g_noalloc_addr[dev]);
  return HYPERION_OK;
}

}  // namespace

extern "C" {

int hyperion_ipc_alloc(size_t bytes, void** ptr, uint8_t* handle) {
  if (ptr == nullptr || handle == nullptr) return fail(HYPERION_ERR_INVALID_ARG, "ptr or handle is NULL");
  if (bytes == 0) return fail(HYPERION_ERR_INVALID_ARG, "bytes is 0");
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, d);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "cudaIpcGetMemHandle");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == HYPERION_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = d;
  return HYPERION_OK;
}

int hyperion_ipc_open(const uint8_t* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return fail(HYPERION_ERR_INVALID_ARG, "ptr or handle is NULL");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* d = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&d, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *ptr = d;
  return HYPERION_OK;
}

int hyperion_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? HYPERION_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int hyperion_ipc_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? HYPERION_OK : cuda_fail(e, "cudaFree");
}

int hyperion_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return HYPERION_OK;
  if (dst == nullptr || src == nullptr) return fail(HYPERION_ERR_INVALID_ARG, "dst or src is NULL");
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HYPERION_OK : cuda_fail(e, "cudaMemcpyAsync");
}

}  // extern "C"

extern "C" int hyperion_apex_kernel_noalloc(const int32_t* worklist, int32_t total_work, const uint32_t* Q,
                                            const float* Q_scale, const uint32_t* K_cache, const float* K_scale,
                                            const uint8_t* V_cache, const float* V_scale,
                                            const int32_t* context_lens, const int32_t* block_tables, void* O,
                                            int32_t seq_q, int32_t head_dim, int32_t k_packed_bytes,
                                            int32_t block_size, int32_t num_blocks, float inv_sqrt_d,
                                            int32_t causal, const hyperion_extents* ext, void* stream) {
  uint8_t* scratch = nullptr;
  const int rc0 = noalloc_scratch(&scratch);
  if (rc0) return rc0;
  // The forward zeroes the work counter on `stream` before its kernels, and
  // rejects a call whose split-KV partials exceed the bytes it is given.
  const int rc = hyperion_apex_kernel_ex(worklist, total_work, Q, Q_scale, K_cache, K_scale, V_cache, V_scale,
                                         context_lens, block_tables, O, seq_q, head_dim, k_packed_bytes, block_size,
                                         num_blocks, inv_sqrt_d, causal, ext, nullptr, scratch,
                                         HYPERION_NOALLOC_SCRATCH_BYTES, stream);
  if (rc == HYPERION_ERR_WORKSPACE) {
    // The split count and scratch the forward worked out before it refused.
    const int ns = g_last_splits;
    char msg[320];
    std::snprintf(msg, sizeof(msg),
                  "hyperion_apex_kernel_noalloc: this call needs %zu bytes of scratch (%d work items x %d KV splits "
                  "of %d floats), more than its fixed %zu bytes; pass fewer work items per call or use "
                  "hyperion_apex_kernel with a workspace",
                  g_last_need, (int)total_work, ns,
                  2 + (int)head_dim, (size_t)HYPERION_NOALLOC_SCRATCH_BYTES);
    g_last_error = msg;
  }
  return rc;
}
