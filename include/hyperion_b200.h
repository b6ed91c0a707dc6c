/*
 * hyperion_b200.h -- C ABI of the B200 (sm_100a) sign-bit / FP8 attention forward.
 *
 * The reference project exposes its forward as a torch extension built by
 * `load_inline` (hyperion_fa3_production_final.py:613-628) whose module object
 * `hyperion` has two entry points:
 *
 *   hyperion.hyperion_apex_kernel(worklist, total_work, Q, Q_scale, K_cache, K_scale,
 *        V_cache, V_scale, context_lens, block_tables, O, seq_q, head_dim,
 *        k_packed_bytes, block_size, num_blocks, inv_sqrt_d, causal,
 *        grid=, block=, shared=)          -- call site hyperion_fa3_production_final.py:1099-1114
 *   hyperion.hyperion_reset_counter(grid=, block=)
 *                                          -- call site hyperion_fa3_production_final.py:905
 *
 * The functions below are what an FFI (ctypes / cffi / pybind) binds in place of
 * that module.  The positional arguments keep the reference's order and meaning;
 * the sizes a raw pointer does not carry travel in `hyperion_extents`.  No torch
 * type appears in any signature: tensors are plain device pointers, the stream is
 * a cudaStream_t passed as void*.
 *
 * Data layout (device memory, caller-owned):
 *   worklist      int32 [total_work, 4]  {q_idx, bh, kv_signature, prefetch_hint};
 *                 only q_idx and bh are read (hyperion_fa3_production_final.py:248-253).
 *   Q             uint32 [n_bh * seq_q, head_dim/32]  sign bits, bit d%32 of word d/32,
 *                 bit = 1 where the value is >= 0.  Row (bh*seq_q + q_idx).
 *   K_cache       uint32 [pool_rows, head_dim/32]  sign bits, same packing.
 *   V_cache       uint8  [pool_rows, head_dim]     FP8 e4m3 codes, decoded with the
 *                 reference's rule (bias 7, subnormals, exponent 15 finite:
 *                 hyperion_fa3_production_final.py:122-141).
 *   V_scale       float32, per tensor (numel 1), per slot (numel == pool_rows) or
 *                 per head / per (batch, head) (index bh % numel).
 *   context_lens  int32 [n_bh]   number of keys of each (batch, head).
 *   block_tables  int32 [n_bh, num_blocks]  page ids; key t of bh lives in slot
 *                 block_tables[bh*num_blocks + t/block_size]*block_size + t%block_size
 *                 (hyperion_fa3_production_final.py:402-411).  A NULL table (or
 *                 block_tables_numel == 0) means the contiguous layout
 *                 slot = bh*num_blocks*block_size + t.
 *   O             [n_bh * seq_q, head_dim] of f16, bf16 or f32 (ext->o_dtype).
 *   Q_scale, K_scale are accepted and ignored: the reference ignores Q_scale, and
 *   a sign-bit K has no magnitude.
 *
 * Math (per work item, q = Q row, keys t < context_lens[bh], and t <= q_idx when causal):
 *   s_t = (head_dim - 2*popcount(q XOR k_t)) * inv_sqrt_d       (README.md:22)
 *   online softmax with EXP_CLAMP = -80 (hyperion_fa3_production_final.py:544-547),
 *   acc = sum_t w_t * fp8(v_t) * vscale, O = acc * (l > 1e-6 ? 1/l : 1)  (:582-593).
 */
#ifndef HYPERION_B200_H
#define HYPERION_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Host-side status codes returned by every entry point. */
#define HYPERION_OK                 0
#define HYPERION_ERR_INVALID_ARG    1  /* a pointer, size or alignment check failed */
#define HYPERION_ERR_UNSUPPORTED    2  /* a valid request this build does not implement */
#define HYPERION_ERR_WORKSPACE      3  /* workspace missing or too small */
#define HYPERION_ERR_CUDA           4  /* a CUDA runtime call failed */

/* Device-side error flags, accumulated in the workspace error word and read back
 * with hyperion_read_device_errors().  The kernels never trap: a bad input sets a
 * flag and the offending key / item is skipped. */
#define HYPERION_DEVERR_BAD_ITEM      0x1u  /* worklist bh or q_idx out of range: row not written */
#define HYPERION_DEVERR_BAD_BLOCK     0x2u  /* block-table page id outside the page pool: keys skipped */
#define HYPERION_DEVERR_CTX_OVERFLOW  0x4u  /* context_lens beyond num_blocks*block_size: tail skipped */
#define HYPERION_DEVERR_NEG_CTX       0x8u  /* negative context length, treated as 0 */
#define HYPERION_DEVERR_WAIT_TIMEOUT  0x10u /* a bounded device wait expired; output incomplete */

/* Output element types for hyperion_extents.o_dtype. */
#define HYPERION_DTYPE_F16   0
#define HYPERION_DTYPE_BF16  1
#define HYPERION_DTYPE_F32   2

/* Kernel selection for hyperion_options.path. */
#define HYPERION_PATH_AUTO   0  /* tile path when seq_q >= 64 and the inputs allow it, else row path */
#define HYPERION_PATH_ROW    1  /* split-KV row kernel (CUDA cores, HBM streaming): any input */
#define HYPERION_PATH_TILE   2  /* 128-row tcgen05 tile kernel: head_dim 128, non per-slot V scale */

/* Kernel of the row path's grouped runs (kv_group > 1, or seq_q > 1): */
#define HYPERION_GROUP_AUTO  0  /* the tensor-core kernel where it applies, else the CUDA-core one */
#define HYPERION_GROUP_CUDA  1  /* products w * v on the CUDA cores: any input */
#define HYPERION_GROUP_MMA   2  /* products on tcgen05 (O^T = V^T P^T): head_dim 128, a per-tensor or
                                   per-head V scale, |inv_sqrt_d| <= 0.117, num_blocks 1 or a
                                   block_size of 8..128 dividing 128 or a multiple of 128, and a
                                   16-byte aligned V_cache */

typedef struct hyperion_extents {
  int32_t n_bh;               /* numel of context_lens: number of (batch, head) rows (KV rows under kv_group) */
  int64_t pool_rows;          /* rows of K_cache and of V_cache */
  int64_t v_scale_numel;      /* numel of V_scale */
  int64_t block_tables_numel; /* numel of block_tables; 0 selects the contiguous layout */
  int32_t o_dtype;            /* HYPERION_DTYPE_* of O */
  int32_t grid_hint;          /* the reference's grid= x (advisory, may be 0) */
  int32_t block_hint;         /* the reference's block= x (advisory, may be 0) */
  int32_t shared_hint;        /* the reference's shared= bytes (advisory, may be 0) */
} hyperion_extents;

typedef struct hyperion_options {
  int32_t path;          /* HYPERION_PATH_* */
  int32_t num_splits;    /* row path: KV splits per item, 0 = automatic */
  int32_t* debug_scores; /* optional: int32 [total_work, debug_ld] receives the integer
                            scores head_dim - 2*popcount for every key the item attends
                            (masked keys are left untouched); NULL in production */
  int64_t debug_ld;      /* row stride of debug_scores in elements */
  int32_t kv_group;      /* grouped-query attention: query heads per KV head; 0 or 1 = none.
                            Work items, Q and O stay indexed by the query row bh, in
                            [0, n_bh * kv_group); context_lens, the block-table rows, the
                            contiguous layout and a per-head V_scale are indexed by the KV
                            row bh / kv_group, so ext->n_bh counts KV rows.  The row path
                            then streams each KV stage once for up to 4 consecutive work
                            items on the same KV row.  No counterpart in the reference,
                            whose engine config has num_kv_heads (hyperion_fa3_production_final.py:853)
                            but whose kernel reads one KV row per (batch, head). */
  int32_t sm_budget;     /* SMs the forward's persistent kernels may occupy; 0 = all of them.
                            A caller that runs a collective (an NCCL all-gather of O, say)
                            on another stream during the forward leaves the rest to it: the
                            kernels size their grids to sm_budget SMs.  No counterpart in
                            the reference.  Added in version 1.1.0. */
  int32_t group_kernel;  /* HYPERION_GROUP_*: the kernel of the grouped runs of the row path.
                            No counterpart in the reference.  Added in version 1.2.0. */
  void* const* o_peers;  /* n_o_peers device pointers (at most 7), each written with every output
                            element at O's own index, beside O.  A head-sharded caller passes the
                            other ranks' gathered outputs, offset to this rank's rows and mapped
                            into this process (hyperion_ipc_open): the forward then is also the
                            all-gather of O, by peer stores over NVLink while it computes.  The
                            caller synchronises the ranks before reading.  NULL / 0: none.
                            No counterpart in the reference.  Added in version 1.3.0. */
  int32_t n_o_peers;
} hyperion_options;

/* Bytes of device workspace the forward needs for these sizes with the automatic
 * KV-split choice.  A call that forces hyperion_options.num_splits = n > 1 needs
 * 256 + total_work * n * (2 + head_dim) * 4 bytes. */
size_t hyperion_workspace_bytes(int32_t total_work, int32_t head_dim,
                                int32_t block_size, int32_t num_blocks);

/* Replaces hyperion.hyperion_apex_kernel (hyperion_fa3_production_final.py:268-288
 * signature, call site :1099-1114).  Asynchronous on `stream`; returns a host
 * status after validating every size and pointer and enqueueing the kernels.
 * `workspace` must be device memory of at least hyperion_workspace_bytes() bytes,
 * 256-byte aligned; it holds the work counter, the error word and split-KV partials. */
int hyperion_apex_kernel(const int32_t* worklist, int32_t total_work,
                         const uint32_t* Q, const float* Q_scale,
                         const uint32_t* K_cache, const float* K_scale,
                         const uint8_t* V_cache, const float* V_scale,
                         const int32_t* context_lens, const int32_t* block_tables,
                         void* O, int32_t seq_q, int32_t head_dim, int32_t k_packed_bytes,
                         int32_t block_size, int32_t num_blocks, float inv_sqrt_d,
                         int32_t causal, const hyperion_extents* ext,
                         void* workspace, size_t workspace_bytes, void* stream);

/* The same forward with kernel selection and the debug score export. */
int hyperion_apex_kernel_ex(const int32_t* worklist, int32_t total_work,
                            const uint32_t* Q, const float* Q_scale,
                            const uint32_t* K_cache, const float* K_scale,
                            const uint8_t* V_cache, const float* V_scale,
                            const int32_t* context_lens, const int32_t* block_tables,
                            void* O, int32_t seq_q, int32_t head_dim, int32_t k_packed_bytes,
                            int32_t block_size, int32_t num_blocks, float inv_sqrt_d,
                            int32_t causal, const hyperion_extents* ext,
                            const hyperion_options* opt,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Replaces hyperion.hyperion_reset_counter (hyperion_fa3_production_final.py:73-77,
 * call site :905).  The work counter lives in the caller's workspace instead of a
 * __device__ global, so two streams never share it; the forward zeroes it itself
 * on its own stream, and this call zeroes it explicitly (asynchronous on `stream`). */
int hyperion_reset_counter(void* workspace, size_t workspace_bytes, void* stream);

/* Test hook for the bounded device waits; it has no counterpart in the reference,
 * whose kernel waits without a bound.  Arms a fault for the next forward issued on
 * this host thread (hyperion_apex_kernel, _ex or _noalloc), then disarms:
 *   - every device wait of that call gives up after `wait_cycles` SM clock cycles
 *     instead of about one second;
 *   - when `stage` >= 0, the warp that streams the keys leaves the stage-th KV stage
 *     it would load unarmed, with no copy in flight on it, so the first wait on it
 *     runs out.
 * The call still returns HYPERION_OK; on the device the wait that runs out raises
 * HYPERION_DEVERR_WAIT_TIMEOUT, the kernel unwinds (copies and MMAs in flight land,
 * tensor memory is freed) and returns with its output incomplete, and the device
 * and the workspace stay usable for the next call.  wait_cycles must be > 0. */
int hyperion_debug_fault(int64_t wait_cycles, int32_t stage);

/* Synchronises `stream`, returns the accumulated HYPERION_DEVERR_* flags of this
 * workspace in *flags and clears them when `clear` is non-zero. */
int hyperion_read_device_errors(void* workspace, size_t workspace_bytes, void* stream,
                                uint32_t* flags, int32_t clear);

/* Launch facts the library derived from the device.  Fills up to `n` int32 values of
 * `out` (returns HYPERION_OK):
 *   [0] SM count            [1] row kernel CTAs per SM   [2] row kernel shared bytes
 *   [3] tile kernel CTAs/SM [4] tile kernel shared bytes [5] row kernel CTAs per SM, head_dim 256
 *   [6] tile kernel loaded  [7] row kernel threads       [8] grouped row kernel threads
 *   [9] grouped row kernel CTAs per SM  [10] its shared bytes  [11] tile kernel threads
 *   [12] tensor-core grouped kernel threads (0 when it did not load)
 *   [13] its CTAs per SM    [14] its shared bytes */
int hyperion_launch_info(int32_t* out, int32_t n);

/* What the last forward on this thread did: out[0] = path (HYPERION_PATH_ROW or
 * _TILE, 0 when nothing was launched), out[1] = KV splits per item, out[2] = kernels
 * launched, out[3] = grid size of the main kernel, out[4] = the main kernel: 1 row
 * kernel, 2 grouped kernel on the CUDA cores, 3 grouped kernel on the tensor core,
 * 4 tile kernel (0 when nothing was launched).  Fills up to `n` values. */
int hyperion_last_call_info(int32_t* out, int32_t n);

/* Device memory that other processes may map: `bytes` from cudaMalloc (CUDA IPC needs an
 * allocation's base), and its HYPERION_IPC_HANDLE_BYTES-byte handle for them.  With
 * hyperion_ipc_open another process maps it (peer access enabled as needed); release with
 * hyperion_ipc_close there and hyperion_ipc_free here.  The gathered output of a head-sharded
 * forward (hyperion_options.o_peers) lives in such buffers.  No counterpart in the reference. */
#define HYPERION_IPC_HANDLE_BYTES 64
int hyperion_ipc_alloc(size_t bytes, void** ptr, uint8_t* handle);
int hyperion_ipc_open(const uint8_t* handle, void** ptr);
int hyperion_ipc_close(void* ptr);
int hyperion_ipc_free(void* ptr);

/* Copies `bytes` from src to dst on the copy engines, asynchronously on `stream`
 * (cudaMemcpyAsync, either address this device's memory or a peer mapping from
 * hyperion_ipc_open).  It moves the rows of a finished piece of a head-sharded
 * forward into every rank's gathered output while the next piece computes, with no
 * kernel of its own and no SM taken from the forward.  No counterpart in the
 * reference.  Added in version 1.4.0. */
int hyperion_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/* Last CUDA error string seen by the library on this thread ("" if none). */
const char* hyperion_last_error_string(void);

/* Library version as major*10000 + minor*100 + patch. */
int32_t hyperion_version(void);

/* Writes new keys and values into the cache format the forward reads.  It has no
 * counterpart in the reference, whose engine allocates the paged pool
 * (hyperion_fa3_production_final.py:1017-1032) but has no kernel that fills it.
 * K_new, V_new: [n_tokens, n_heads, head_dim] of in_dtype (HYPERION_DTYPE_*).
 * Token i belongs to sequence seq_ids[i] at position positions[i]; its row for head
 * h (bh = seq_ids[i]*n_heads + h) goes to the slot the forward reads it from:
 * block_tables[bh*num_blocks + pos/block_size]*block_size + pos%block_size (or the
 * contiguous slot bh*num_blocks*block_size + pos when block_tables_numel is 0).
 * K: sign bits (1 where k >= 0) into K_cache [pool_rows, head_dim/32] uint32;
 * V: e4m3 codes of clamp(v / scale, -448, 448), round to nearest even, into V_cache
 * [pool_rows, head_dim] uint8, with the scale the forward decodes that slot with:
 * V_scale[0] (numel 1), V_scale[slot] (numel == pool_rows) or V_scale[bh % numel].
 * Positions or page ids outside the pool set HYPERION_DEVERR_BAD_ITEM / _BAD_BLOCK in
 * the workspace error word and that row is skipped.  Asynchronous on `stream`. */
int hyperion_kv_cache_write(const void* K_new, const void* V_new, int32_t in_dtype,
                            int32_t n_tokens, int32_t n_heads, int32_t head_dim,
                            const int32_t* seq_ids, const int32_t* positions,
                            const int32_t* block_tables, int64_t block_tables_numel,
                            int32_t block_size, int32_t num_blocks,
                            const float* V_scale, int64_t v_scale_numel,
                            uint32_t* K_cache, uint8_t* V_cache, int64_t pool_rows,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Fixed scratch of hyperion_apex_kernel_noalloc, per device, in bytes. */
#define HYPERION_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)

/* The forward without a caller workspace.  It has no counterpart in the reference.
 *
 * Some callers cannot allocate device memory.  Examples are a plugin whose host
 * framework owns the device allocator, an engine that reserves all memory at start-up,
 * and a binding with no allocator of its own.  For them, this entry point keeps the
 * forward's scratch (work counter, error word and split-KV partials) in a fixed array
 * of HYPERION_NOALLOC_SCRATCH_BYTES that the library holds on every device where its
 * device code is loaded, until the process exits.  It calls no cudaMalloc or cudaFree.
 * The caller passes the inputs and O exactly as for hyperion_apex_kernel.
 *
 * - The first call on a device looks up that device's copy of the array, with the
 *   device current.  Make that first call before any stream capture.
 * - A call whose split-KV partials do not fit in the array returns
 *   HYPERION_ERR_WORKSPACE, with the bytes it needed in hyperion_last_error_string().
 *   Smaller worklists per call, or hyperion_apex_kernel, avoid that.
 * - Every call on a device shares the one array.  The work counter is zeroed on
 *   `stream` at the start of each call.  Two calls that overlap on the same GPU (two
 *   streams, or two host threads) race on the array: order them on one stream.
 * - Device-side error flags are kept in the array and are not readable through
 *   this entry point. */
int hyperion_apex_kernel_noalloc(const int32_t* worklist, int32_t total_work,
                                 const uint32_t* Q, const float* Q_scale,
                                 const uint32_t* K_cache, const float* K_scale,
                                 const uint8_t* V_cache, const float* V_scale,
                                 const int32_t* context_lens, const int32_t* block_tables,
                                 void* O, int32_t seq_q, int32_t head_dim, int32_t k_packed_bytes,
                                 int32_t block_size, int32_t num_blocks, float inv_sqrt_d,
                                 int32_t causal, const hyperion_extents* ext, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HYPERION_B200_H */
