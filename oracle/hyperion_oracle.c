/*
 * hyperion_oracle.c -- CPU restatement of the Hyperion sign-bit / FP8 attention
 * forward.  TEST INFRASTRUCTURE: only the tests, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py may load this library, and only as the checker or
 * the timed CPU baseline.  The product path never calls it.
 *
 * Parity status: partially pinned.  The FP8 decode is checked code-for-code
 * against the reference's own fp8_e4m3_to_fp32 compiled from its source
 * (oracle/build.py, build_ref() -> oracle/_ref); the reference ships no tests, golden
 * vectors or runnable attention kernel (its CUDA source does not compile), so the
 * scoring and softmax below are restated from its source and README and pinned
 * only by hand-built known-answer cases.
 *
 * What it restates, statement by statement, from hyperion_fa3_production_final.py
 * (REF) and README.md:
 *   work item {q_idx, bh}                         REF:248-253, REF:342-350
 *   keys t < context_lens[bh]                     REF:352-353, REF:479-482
 *   causal: key t masked when t > q_idx            REF:483-486
 *   paged slot = table[bh*nb + t/bs]*bs + t%bs     REF:402-411 (ids outside the pool are
 *                                                  skipped; the reference skips the load)
 *   score = (D - 2*popcount(q XOR k)) * inv_sqrt_d README.md:22 (v2 sign-bit Q and K),
 *                                                  scale as REF:519 without K_scale
 *   fp8 e4m3 decode                                REF:122-141
 *   online softmax, EXP_CLAMP = -80               REF:59, REF:544-547, REF:571-572
 *   acc = acc*alpha + w*fp8(v)*vscale             REF:556-568
 *   masked keys skipped                            REF:539
 *   O = acc * (l > 1e-6 ? 1/l : 1)                 REF:584-591
 * Keys are visited in increasing order, one at a time, as the reference's
 * accumulate warps do (REF:537).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <float.h>
#include <pthread.h>
#include <unistd.h>

#define ORACLE_EXP_CLAMP (-80.0f)

#define ORACLE_ERR_BAD_ITEM 0x1u
#define ORACLE_ERR_BAD_BLOCK 0x2u
#define ORACLE_ERR_CTX_OVERFLOW 0x4u
#define ORACLE_ERR_NEG_CTX 0x8u

/* REF:122-141 restated: bias 7, subnormals mant * 2^-9, exponent 15 finite. */
float oracle_fp8_e4m3_to_f32(uint8_t x) {
  if (x == 0) return 0.f;
  if (x == 0x80) return -0.f;
  const int sign_bit = (x >> 7) & 1;
  const float sign = sign_bit ? -1.f : 1.f;
  const int e = (x >> 3) & 0xF;
  const int mant = x & 0x7;
  if (e == 0) return sign * ldexpf((float)mant, -9);
  return sign * ldexpf(1.f + (float)mant / 8.f, e - 7);
}

static int popc32(uint32_t v) { return __builtin_popcount(v); }

/* The 256 decoded values of oracle_fp8_e4m3_to_f32, filled before any parallel use. */
static float g_fp8_lut[256];
static int g_fp8_lut_ready = 0;

static void fp8_lut_init(void) {
  if (g_fp8_lut_ready) return;
  for (int c = 0; c < 256; ++c) g_fp8_lut[c] = oracle_fp8_e4m3_to_f32((uint8_t)c);
  g_fp8_lut_ready = 1;
}

/* Integer score D - 2*popcount(q XOR k) over D/32 words (README.md:22). */
int oracle_sign_score(const uint32_t* q, const uint32_t* k, int head_dim) {
  int p = 0;
  for (int i = 0; i < head_dim / 32; ++i) p += popc32(q[i] ^ k[i]);
  return head_dim - 2 * p;
}

/* V scale of one key: per tensor (numel 1), per slot (numel == pool_rows), else bh % numel. */
static float vscale_of(const float* v_scale, int64_t numel, int64_t pool_rows, int bh, int64_t slot) {
  if (numel == 1) return v_scale[0];
  if (numel == pool_rows) return v_scale[slot];
  return v_scale[bh % numel];
}

typedef struct {
  const int32_t* worklist;
  int32_t total_work;
  const uint32_t* q;
  const uint32_t* k;
  const uint8_t* v;
  const float* v_scale;
  int64_t v_scale_numel;
  const int32_t* ctx_lens;
  int32_t n_bh;
  const int32_t* block_tables;
  int64_t bt_numel;
  int64_t pool_rows;
  float* o;
  uint8_t* o_written;
  int32_t seq_q, head_dim, block_size, num_blocks;
  float inv_sqrt_d;
  int32_t causal;
  int32_t* scores;
  int64_t ld;
  int32_t next_item; /* shared ticket, taken with __atomic_fetch_add */
  uint32_t errs;     /* accumulated with __atomic_fetch_or */
} oracle_job;

/* One work item, the reference's per-item loop (REF:338-593) for the sign-bit path. */
static uint32_t run_item(const oracle_job* j, int32_t item) {
  const int W = j->head_dim / 32;
  const int64_t pool_blocks = j->pool_rows / j->block_size;
  const int64_t cap = (int64_t)j->num_blocks * j->block_size;
  uint32_t errs = 0;
  const int q_idx = j->worklist[4 * (int64_t)item + 0];
  const int bh = j->worklist[4 * (int64_t)item + 1];
  if (bh < 0 || bh >= j->n_bh || q_idx < 0 || q_idx >= j->seq_q) return ORACLE_ERR_BAD_ITEM;
  int64_t ctx = j->ctx_lens[bh];
  if (ctx < 0) {
    errs |= ORACLE_ERR_NEG_CTX;
    ctx = 0;
  }
  if (ctx > cap) {
    errs |= ORACLE_ERR_CTX_OVERFLOW;
    ctx = cap;
  }
  const uint32_t* qrow = j->q + ((int64_t)bh * j->seq_q + q_idx) * W;
  float acc[1024];
  for (int d = 0; d < j->head_dim; ++d) acc[d] = 0.f;
  float m_i = -FLT_MAX;
  float l_i = 0.f;
  for (int64_t t = 0; t < ctx; ++t) {
    if (j->causal && t > q_idx) continue;
    const int64_t page = t / j->block_size;
    int64_t id;
    if (j->bt_numel == 0 || j->block_tables == NULL) {
      id = (int64_t)bh * j->num_blocks + page;
    } else {
      id = j->block_tables[(int64_t)bh * j->num_blocks + page];
    }
    if (id < 0 || id >= pool_blocks) {
      errs |= ORACLE_ERR_BAD_BLOCK;
      continue;
    }
    const int64_t slot = id * j->block_size + t % j->block_size;
    const int si = oracle_sign_score(qrow, j->k + slot * W, j->head_dim);
    if (j->scores) j->scores[(int64_t)item * j->ld + t] = si;
    const float s = (float)si * j->inv_sqrt_d;
    const float m_new = fmaxf(m_i, s);
    const float alpha = expf(fmaxf(m_i - m_new, ORACLE_EXP_CLAMP));
    const float w = expf(fmaxf(s - m_new, ORACLE_EXP_CLAMP));
    const float vs = vscale_of(j->v_scale, j->v_scale_numel, j->pool_rows, bh, slot);
    const uint8_t* vrow = j->v + slot * j->head_dim;
    for (int d = 0; d < j->head_dim; ++d) acc[d] = acc[d] * alpha + w * (g_fp8_lut[vrow[d]] * vs);
    l_i = l_i * alpha + w;
    m_i = m_new;
  }
  const float inv_l = (l_i > 1e-6f) ? 1.f / l_i : 1.f;
  float* orow = j->o + ((int64_t)bh * j->seq_q + q_idx) * j->head_dim;
  for (int d = 0; d < j->head_dim; ++d) orow[d] = acc[d] * inv_l;
  if (j->o_written) j->o_written[item] = 1;
  return errs;
}

static void* worker(void* arg) {
  oracle_job* j = (oracle_job*)arg;
  uint32_t errs = 0;
  for (;;) {
    const int32_t item = __atomic_fetch_add(&j->next_item, 1, __ATOMIC_RELAXED);
    if (item >= j->total_work) break;
    errs |= run_item(j, item);
  }
  __atomic_fetch_or(&j->errs, errs, __ATOMIC_RELAXED);
  return NULL;
}

/*
 * Forward over `total_work` items.  o is fp32 [n_bh*seq_q, head_dim]; rows of
 * invalid items are left untouched and o_written[item] (optional) is set to 1 for
 * every row written.  scores (optional, int32 [total_work, ld]) receives the
 * integer score of every attended key.  *err_flags accumulates ORACLE_ERR_*.
 * nthreads <= 0 uses every online CPU.  Returns 0, or -1 on bad arguments.
 */
int oracle_apex_forward(const int32_t* worklist, int32_t total_work, const uint32_t* q, const uint32_t* k,
                        const uint8_t* v, const float* v_scale, int64_t v_scale_numel, const int32_t* ctx_lens,
                        int32_t n_bh, const int32_t* block_tables, int64_t bt_numel, int64_t pool_rows, float* o,
                        uint8_t* o_written, int32_t seq_q, int32_t head_dim, int32_t block_size, int32_t num_blocks,
                        float inv_sqrt_d, int32_t causal, int32_t* scores, int64_t ld, uint32_t* err_flags,
                        int32_t nthreads) {
  if (head_dim <= 0 || head_dim % 32 != 0 || head_dim > 1024 || block_size <= 0 || num_blocks <= 0) return -1;
  fp8_lut_init();
  oracle_job j = {worklist, total_work, q, k, v, v_scale, v_scale_numel, ctx_lens, n_bh, block_tables, bt_numel,
                  pool_rows, o, o_written, seq_q, head_dim, block_size, num_blocks, inv_sqrt_d, causal, scores, ld,
                  0, 0u};
  int nt = nthreads > 0 ? nthreads : (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (nt < 1) nt = 1;
  if (nt > 1024) nt = 1024;
  if (nt > total_work) nt = total_work > 0 ? total_work : 1;
  pthread_t tids[1024];
  int started = 0;
  for (int i = 1; i < nt; ++i) {
    if (pthread_create(&tids[started], NULL, worker, &j) == 0) ++started;
  }
  worker(&j);
  for (int i = 0; i < started; ++i) pthread_join(tids[i], NULL);
  if (err_flags) *err_flags |= j.errs;
  return 0;
}

int oracle_max_threads(void) { return (int)sysconf(_SC_NPROCESSORS_ONLN); }
