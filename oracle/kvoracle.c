/*
 * kvoracle.c — CPU restatement of mobile-moe.zig's paged KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA product.  See
 * kvoracle.h for the list of reference functions restated here, the parity
 * pins, and the documented deviations.  Build with -ffp-contract=off so every
 * float operation rounds exactly as written (the seeded generator must be
 * bit-identical to the device one).
 */
#include "kvoracle.h"

#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ===================== f16 <-> f32 (src/dequant.zig:19-95) ===================== */

/* src/dequant.zig:19-47: exact widening, subnormals normalised, NaN payload kept. */
float kvo_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15);
  uint32_t exp_raw = (uint32_t)((h >> 10) & 0x1F);
  uint32_t mant = (uint32_t)(h & 0x3FF);
  if (exp_raw == 0) {
    if (mant == 0) return u2f(sign << 31);
    uint32_t m = mant, e = 0;
    while ((m & 0x400) == 0) {
      m <<= 1;
      e += 1;
    }
    m &= 0x3FF;
    return u2f((sign << 31) | ((127 - 14 - e) << 23) | (m << 13));
  }
  if (exp_raw == 31) {
    if (mant == 0) return u2f((sign << 31) | 0x7F800000u);
    return u2f((sign << 31) | 0x7F800000u | (mant << 13));
  }
  return u2f((sign << 31) | ((exp_raw - 15 + 127) << 23) | (mant << 13));
}

/* src/dequant.zig:50-95: f32 subnormals -> signed zero, overflow -> inf,
 * NaN keeps the top mantissa bits (forced non-zero), normals round to nearest
 * even.  The f16-subnormal branch (exp16 in [-10, 0]) is computed with correct
 * IEEE RNE (deviation 1 in kvoracle.h). */
uint16_t kvo_f32_to_f16(float v) {
  uint32_t bits = f2u(v);
  uint32_t sign = (bits >> 31) & 1u;
  uint32_t exp_raw = (bits >> 23) & 0xFFu;
  uint32_t mant = bits & 0x7FFFFFu;
  uint32_t e, m;
  if (exp_raw == 0) {
    e = 0;
    m = 0;
  } else if (exp_raw == 0xFF) {
    e = 0x1F;
    m = mant >> 13;
    if (mant != 0 && m == 0) m = 1;
  } else {
    int exp16 = (int)exp_raw - 127 + 15;
    if (exp16 >= 31) {
      e = 0x1F;
      m = 0;
    } else if (exp16 <= 0) {
      if (exp16 < -10) {
        e = 0;
        m = 0;
      } else {
        uint32_t full = mant | 0x800000u;
        uint32_t shift = (uint32_t)(14 - exp16); /* 14..24 */
        uint32_t q = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q += 1; /* may carry into e=1: correct */
        e = 0;
        m = q;
      }
    } else {
      e = (uint32_t)exp16;
      m = mant >> 13;
      uint32_t round_bits = mant & 0x1FFFu;
      if (round_bits > 0x1000u || (round_bits == 0x1000u && (m & 1u))) {
        m += 1;
        if (m == 0x400u) {
          m = 0;
          e += 1;
        }
      }
    }
  }
  return (uint16_t)((sign << 15) | (e << 10) | m);
}

/* ======================= Q8_0 (src/kv_cache.zig:294-349) ======================= */

static void quantize_block(const float* x, uint32_t cnt, kvo_block_q8* b) {
  float max_abs = 0.0f;
  for (uint32_t i = 0; i < cnt; ++i) {
    float av = fabsf(x[i]);
    if (av > max_abs) max_abs = av; /* NaN never compares greater: skipped */
  }
  float d = max_abs > 0.0f ? max_abs / 127.0f : 0.0f;
  b->d = kvo_f32_to_f16(d);
  if (d > 0.0f) {
    for (uint32_t i = 0; i < cnt; ++i) {
      float r = roundf(x[i] / d); /* @round: half away from zero */
      int32_t q;
      if (r != r) q = 0; /* deviation 2 */
      else if (r > 127.0f) q = 127;
      else if (r < -127.0f) q = -127;
      else q = (int32_t)r;
      b->qs[i] = (int8_t)q;
    }
  } else {
    for (uint32_t i = 0; i < cnt; ++i) b->qs[i] = 0;
  }
  for (uint32_t i = cnt; i < 32; ++i) b->qs[i] = 0;
}

void kvo_quantize_q8_0(const float* x, uint32_t n, kvo_block_q8* out) {
  uint32_t nb = (n + 31) / 32;
  for (uint32_t bi = 0; bi < nb; ++bi) {
    uint32_t start = bi * 32;
    uint32_t end = start + 32 < n ? start + 32 : n;
    quantize_block(x + start, end - start, out + bi);
  }
}

/* src/kv_cache.zig:236-244: f16ToF32(d) * f32(q). */
void kvo_dequantize_q8_0(const kvo_block_q8* b, uint32_t n, float* out) {
  for (uint32_t i = 0; i < n; ++i) {
    float d = kvo_f16_to_f32(b[i / 32].d);
    out[i] = d * (float)b[i / 32].qs[i % 32];
  }
}

/* ============================ pool (reference layout) ============================ */

static inline uint32_t nq8(uint32_t n) { return (n + 31) / 32; }

int kvo_pool_init(kvo_pool* p, uint32_t n_layers, uint32_t num_blocks, uint32_t block_size,
                  uint32_t kv_rank, uint32_t rope_dim, int quantized) {
  memset(p, 0, sizeof(*p));
  if (!n_layers || !num_blocks || !block_size || !kv_rank || !rope_dim) return KVO_ERR_INVALID_ARG;
  p->n_layers = n_layers;
  p->num_blocks = num_blocks;
  p->block_size = block_size;
  p->kv_rank = kv_rank;
  p->rope_dim = rope_dim;
  uint64_t rows = (uint64_t)n_layers * num_blocks * block_size;
  /* src/kv_cache.zig:72-78: zeroed f32 pools.  A pool created quantized has
   * no f32 pools (the single-sequence kvo_cache keeps both, as the reference). */
  if (!quantized) {
    p->kv = (float*)calloc(rows * kv_rank, sizeof(float));
    p->pe = (float*)calloc(rows * rope_dim, sizeof(float));
    if (!p->kv || !p->pe) {
      kvo_pool_free(p);
      return KVO_ERR_NO_MEMORY;
    }
  }
  if (quantized) {
    p->kv_q8 = (kvo_block_q8*)calloc(rows * nq8(kv_rank), sizeof(kvo_block_q8));
    p->pe_q8 = (kvo_block_q8*)calloc(rows * nq8(rope_dim), sizeof(kvo_block_q8));
    if (!p->kv_q8 || !p->pe_q8) {
      kvo_pool_free(p);
      return KVO_ERR_NO_MEMORY;
    }
    p->quantized = 1;
  }
  return KVO_OK;
}

void kvo_pool_free(kvo_pool* p) {
  free(p->kv);
  free(p->pe);
  free(p->kv_q8);
  free(p->pe_q8);
  p->kv = p->pe = NULL;
  p->kv_q8 = p->pe_q8 = NULL;
}

static inline uint64_t row_index(const kvo_pool* p, uint32_t layer, uint32_t block, uint32_t off) {
  return ((uint64_t)layer * p->num_blocks + block) * p->block_size + off;
}

/* src/kv_cache.zig:289-356 */
void kvo_pool_put(kvo_pool* p, uint32_t layer, uint32_t block, uint32_t offset,
                  const float* kv_comp, const float* k_pe) {
  uint64_t r = row_index(p, layer, block, offset);
  if (p->quantized) {
    kvo_quantize_q8_0(kv_comp, p->kv_rank, p->kv_q8 + r * nq8(p->kv_rank));
    kvo_quantize_q8_0(k_pe, p->rope_dim, p->pe_q8 + r * nq8(p->rope_dim));
  } else {
    memcpy(p->kv + r * p->kv_rank, kv_comp, sizeof(float) * p->kv_rank);
    memcpy(p->pe + r * p->rope_dim, k_pe, sizeof(float) * p->rope_dim);
  }
}

void kvo_pool_put_rows(kvo_pool* p, uint32_t layer, uint32_t n, const uint32_t* blocks,
                       const uint32_t* offsets, const float* rows) {
  const uint64_t w = p->kv_rank + p->rope_dim;
  for (uint32_t r = 0; r < n; ++r)
    kvo_pool_put(p, layer, blocks[r], offsets[r], rows + r * w, rows + r * w + p->kv_rank);
}

/* src/kv_cache.zig:225-277 */
void kvo_pool_get(const kvo_pool* p, uint32_t layer, uint32_t block, uint32_t offset,
                  float* kv_out, float* pe_out) {
  uint64_t r = row_index(p, layer, block, offset);
  if (p->quantized) {
    if (kv_out) kvo_dequantize_q8_0(p->kv_q8 + r * nq8(p->kv_rank), p->kv_rank, kv_out);
    if (pe_out) kvo_dequantize_q8_0(p->pe_q8 + r * nq8(p->rope_dim), p->rope_dim, pe_out);
  } else {
    if (kv_out) memcpy(kv_out, p->kv + r * p->kv_rank, sizeof(float) * p->kv_rank);
    if (pe_out) memcpy(pe_out, p->pe + r * p->rope_dim, sizeof(float) * p->rope_dim);
  }
}

void kvo_pool_gather(const kvo_pool* p, uint32_t layer, const uint32_t* table, uint32_t len,
                     float* out) {
  uint32_t w = p->kv_rank + p->rope_dim;
  for (uint32_t pos = 0; pos < len; ++pos) {
    uint32_t blk = table[pos / p->block_size];
    kvo_pool_get(p, layer, blk, pos % p->block_size, out + (uint64_t)pos * w,
                 out + (uint64_t)pos * w + p->kv_rank);
  }
}

uint64_t kvo_pool_bytes(const kvo_pool* p) {
  uint64_t rows = (uint64_t)p->n_layers * p->num_blocks * p->block_size;
  if (p->quantized) return rows * (nq8(p->kv_rank) + nq8(p->rope_dim)) * sizeof(kvo_block_q8);
  return rows * (p->kv_rank + p->rope_dim) * sizeof(float);
}

/* src/kv_cache.zig:484-492: Q8_0 kv pool then pe pool, else f32 kv then pe. */
void kvo_pool_serialize(const kvo_pool* p, uint8_t* dst) {
  uint64_t rows = (uint64_t)p->n_layers * p->num_blocks * p->block_size;
  if (p->quantized) {
    uint64_t a = rows * nq8(p->kv_rank) * sizeof(kvo_block_q8);
    memcpy(dst, p->kv_q8, a);
    memcpy(dst + a, p->pe_q8, rows * nq8(p->rope_dim) * sizeof(kvo_block_q8));
  } else {
    uint64_t a = rows * p->kv_rank * sizeof(float);
    memcpy(dst, p->kv, a);
    memcpy(dst + a, p->pe, rows * p->rope_dim * sizeof(float));
  }
}

void kvo_pool_deserialize(kvo_pool* p, const uint8_t* src) {
  uint64_t rows = (uint64_t)p->n_layers * p->num_blocks * p->block_size;
  if (p->quantized) {
    uint64_t a = rows * nq8(p->kv_rank) * sizeof(kvo_block_q8);
    memcpy(p->kv_q8, src, a);
    memcpy(p->pe_q8, src + a, rows * nq8(p->rope_dim) * sizeof(kvo_block_q8));
  } else {
    uint64_t a = rows * p->kv_rank * sizeof(float);
    memcpy(p->kv, src, a);
    memcpy(p->pe, src + a, rows * p->rope_dim * sizeof(float));
  }
}

/* ================== attention core (src/inference.zig:572-660) ================== */

#define KVO_CHUNK 64 /* src/inference.zig:572: BLOCK_SIZE = 64 */

static void attention_head(const kvo_pool* p, uint32_t layer, const uint32_t* table, uint32_t len,
                           const float* qh, float scale, float* outh, float* kv_row,
                           float* pe_row, float* o_vec) {
  const uint32_t R = p->kv_rank, P = p->rope_dim;
  float m_vec = -INFINITY, l_vec = 0.0f;
  float scores[KVO_CHUNK];
  memset(o_vec, 0, sizeof(float) * R);
  for (uint32_t b_start = 0; b_start < len; b_start += KVO_CHUNK) {
    uint32_t b_end = b_start + KVO_CHUNK < len ? b_start + KVO_CHUNK : len;
    uint32_t b_len = b_end - b_start;
    for (uint32_t pos = b_start; pos < b_end; ++pos) {
      kvo_pool_get(p, layer, table[pos / p->block_size], pos % p->block_size, kv_row, pe_row);
      float score = 0.0f;
      for (uint32_t i = 0; i < R; ++i) score += qh[i] * kv_row[i];
      for (uint32_t i = 0; i < P; ++i) score += qh[R + i] * pe_row[i];
      scores[pos - b_start] = score * scale;
    }
    float m_j = -INFINITY;
    for (uint32_t i = 0; i < b_len; ++i)
      if (scores[i] > m_j) m_j = scores[i];
    float l_j = 0.0f;
    for (uint32_t i = 0; i < b_len; ++i) {
      scores[i] = expf(scores[i] - m_j);
      l_j += scores[i];
    }
    float m_new = m_vec > m_j ? m_vec : m_j;
    float scale_o = expf(m_vec - m_new);
    float scale_s = expf(m_j - m_new);
    for (uint32_t i = 0; i < R; ++i) o_vec[i] = o_vec[i] * scale_o;
    for (uint32_t pos = b_start; pos < b_end; ++pos) {
      float w = scores[pos - b_start] * scale_s;
      /* V is the latent part of the same cached row (absorbed MLA). */
      kvo_pool_get(p, layer, table[pos / p->block_size], pos % p->block_size, kv_row, NULL);
      for (uint32_t i = 0; i < R; ++i) o_vec[i] += w * kv_row[i];
    }
    m_vec = m_new;
    l_vec = l_vec * scale_o + l_j * scale_s;
  }
  for (uint32_t i = 0; i < R; ++i) outh[i] = l_vec > 0.0f ? o_vec[i] / l_vec : 0.0f;
}

void kvo_attention(const kvo_pool* p, uint32_t layer, const uint32_t* table, uint32_t len,
                   const float* q, uint32_t n_heads, float scale, float* out) {
  const uint32_t R = p->kv_rank, W = p->kv_rank + p->rope_dim;
  float* kv_row = (float*)malloc(sizeof(float) * R);
  float* pe_row = (float*)malloc(sizeof(float) * p->rope_dim);
  float* o_vec = (float*)malloc(sizeof(float) * R);
  for (uint32_t h = 0; h < n_heads; ++h)
    attention_head(p, layer, table, len, q + (uint64_t)h * W, scale, out + (uint64_t)h * R, kv_row,
                   pe_row, o_vec);
  free(kv_row);
  free(pe_row);
  free(o_vec);
}

/* ---- pthread mutex/cond FIFO pool (src/thread_pool.zig:15-99) ---- */

typedef struct {
  void (*run)(void* ctx, int tid);
  void* ctx;
} kvo_task;

typedef struct {
  pthread_t* threads;
  int n_threads;
  kvo_task* queue; /* ring buffer */
  size_t cap, head, count;
  pthread_mutex_t mutex;
  pthread_cond_t cond;
  int shutdown;
  int running;
} kvo_tpool;

typedef struct {
  kvo_tpool* pool;
  int tid;
} kvo_worker_arg;

static void* worker_loop(void* arg) {
  kvo_worker_arg* wa = (kvo_worker_arg*)arg;
  kvo_tpool* pool = wa->pool;
  for (;;) {
    pthread_mutex_lock(&pool->mutex);
    while (pool->count == 0 && !pool->shutdown) pthread_cond_wait(&pool->cond, &pool->mutex);
    if (pool->shutdown && pool->count == 0) {
      pthread_mutex_unlock(&pool->mutex);
      break;
    }
    kvo_task t = pool->queue[pool->head];
    pool->head = (pool->head + 1) % pool->cap;
    pool->count -= 1;
    pool->running += 1;
    pthread_mutex_unlock(&pool->mutex);
    t.run(t.ctx, wa->tid);
    pthread_mutex_lock(&pool->mutex);
    pool->running -= 1;
    pthread_cond_broadcast(&pool->cond);
    pthread_mutex_unlock(&pool->mutex);
  }
  return NULL;
}

static int tpool_init(kvo_tpool* pool, int n_threads, size_t cap, kvo_worker_arg* args) {
  memset(pool, 0, sizeof(*pool));
  pool->threads = (pthread_t*)calloc((size_t)n_threads, sizeof(pthread_t));
  pool->queue = (kvo_task*)calloc(cap, sizeof(kvo_task));
  if (!pool->threads || !pool->queue) return KVO_ERR_NO_MEMORY;
  pool->cap = cap;
  pool->n_threads = n_threads;
  pthread_mutex_init(&pool->mutex, NULL);
  pthread_cond_init(&pool->cond, NULL);
  for (int i = 0; i < n_threads; ++i) {
    args[i].pool = pool;
    args[i].tid = i;
    pthread_create(&pool->threads[i], NULL, worker_loop, &args[i]);
  }
  return KVO_OK;
}

static void tpool_submit(kvo_tpool* pool, kvo_task t) {
  pthread_mutex_lock(&pool->mutex);
  pool->queue[(pool->head + pool->count) % pool->cap] = t;
  pool->count += 1;
  pthread_cond_signal(&pool->cond);
  pthread_mutex_unlock(&pool->mutex);
}

static void tpool_wait_all(kvo_tpool* pool) {
  pthread_mutex_lock(&pool->mutex);
  while (pool->count > 0 || pool->running > 0) pthread_cond_wait(&pool->cond, &pool->mutex);
  pthread_mutex_unlock(&pool->mutex);
}

static void tpool_deinit(kvo_tpool* pool) {
  pthread_mutex_lock(&pool->mutex);
  pool->shutdown = 1;
  pthread_cond_broadcast(&pool->cond);
  pthread_mutex_unlock(&pool->mutex);
  for (int i = 0; i < pool->n_threads; ++i) pthread_join(pool->threads[i], NULL);
  free(pool->threads);
  free(pool->queue);
  pthread_mutex_destroy(&pool->mutex);
  pthread_cond_destroy(&pool->cond);
}

typedef struct {
  const kvo_pool* p;
  uint32_t layer;
  const uint32_t* table;
  uint32_t len;
  const float* qh;
  float scale;
  float* outh;
  float** scratch; /* per-thread [3] buffers */
} attn_task_ctx;

static void attn_task_run(void* ctx, int tid) {
  attn_task_ctx* a = (attn_task_ctx*)ctx;
  float** s = a->scratch + 3 * tid;
  attention_head(a->p, a->layer, a->table, a->len, a->qh, a->scale, a->outh, s[0], s[1], s[2]);
}

void kvo_attention_batch(const kvo_pool* p, uint32_t layer, uint32_t n_seqs,
                         const uint32_t* table_offsets, const uint32_t* tables,
                         const uint32_t* lens, const float* q, uint32_t n_heads, float scale,
                         float* out, int n_threads) {
  const uint32_t R = p->kv_rank, W = p->kv_rank + p->rope_dim;
  if (n_threads <= 1) {
    for (uint32_t b = 0; b < n_seqs; ++b)
      kvo_attention(p, layer, tables + table_offsets[b], lens[b], q + (uint64_t)b * n_heads * W,
                    n_heads, scale, out + (uint64_t)b * n_heads * R);
    return;
  }
  size_t n_tasks = (size_t)n_seqs * n_heads;
  attn_task_ctx* ctxs = (attn_task_ctx*)calloc(n_tasks, sizeof(attn_task_ctx));
  float** scratch = (float**)calloc((size_t)n_threads * 3, sizeof(float*));
  for (int t = 0; t < n_threads; ++t) {
    scratch[3 * t + 0] = (float*)malloc(sizeof(float) * R);
    scratch[3 * t + 1] = (float*)malloc(sizeof(float) * p->rope_dim);
    scratch[3 * t + 2] = (float*)malloc(sizeof(float) * R);
  }
  kvo_worker_arg* args = (kvo_worker_arg*)calloc((size_t)n_threads, sizeof(kvo_worker_arg));
  kvo_tpool pool;
  tpool_init(&pool, n_threads, n_tasks + 1, args);
  for (uint32_t b = 0; b < n_seqs; ++b) {
    for (uint32_t h = 0; h < n_heads; ++h) {
      attn_task_ctx* c = &ctxs[(size_t)b * n_heads + h];
      c->p = p;
      c->layer = layer;
      c->table = tables + table_offsets[b];
      c->len = lens[b];
      c->qh = q + ((uint64_t)b * n_heads + h) * W;
      c->scale = scale;
      c->outh = out + ((uint64_t)b * n_heads + h) * R;
      c->scratch = scratch;
      kvo_task t = {attn_task_run, c};
      tpool_submit(&pool, t);
    }
  }
  tpool_wait_all(&pool);
  tpool_deinit(&pool);
  for (int t = 0; t < 3 * n_threads; ++t) free(scratch[t]);
  free(scratch);
  free(args);
  free(ctxs);
}

/* ======================= KVCache (src/kv_cache.zig:24-546) ======================= */

#define NO_HASH UINT64_MAX

typedef struct {
  uint64_t key;
  uint32_t value;
  int used;
} hm_entry;

struct kvo_cache {
  kvo_pool pool;
  uint32_t* ref_count;
  uint64_t* hash;
  uint32_t* free_list; /* stack; top = free_list[n_free-1] */
  uint32_t n_free;
  uint32_t* table;
  uint32_t table_len, table_cap;
  uint32_t len;
  /* prefix hash map: open addressing, capacity = 4 * num_blocks */
  hm_entry* hm;
  uint32_t hm_cap;
};

static hm_entry* hm_find(kvo_cache* c, uint64_t key) {
  uint32_t i = (uint32_t)(kvo_splitmix64(key) % c->hm_cap);
  for (uint32_t n = 0; n < c->hm_cap; ++n) {
    hm_entry* e = &c->hm[(i + n) % c->hm_cap];
    if (e->used == 0) return NULL;
    if (e->used == 1 && e->key == key) return e;
  }
  return NULL;
}
static void hm_put(kvo_cache* c, uint64_t key, uint32_t v) {
  hm_entry* e = hm_find(c, key);
  if (e) {
    e->value = v;
    return;
  }
  uint32_t i = (uint32_t)(kvo_splitmix64(key) % c->hm_cap);
  for (uint32_t n = 0; n < c->hm_cap; ++n) {
    hm_entry* s = &c->hm[(i + n) % c->hm_cap];
    if (s->used != 1) {
      s->used = 1;
      s->key = key;
      s->value = v;
      return;
    }
  }
}
static void hm_remove(kvo_cache* c, uint64_t key) {
  hm_entry* e = hm_find(c, key);
  if (e) e->used = 2; /* tombstone */
}

kvo_cache* kvo_cache_init(uint32_t n_layers, uint32_t kv_rank, uint32_t rope_dim,
                          uint32_t max_seq_len, uint32_t block_size) {
  if (block_size == 0) block_size = 16; /* src/kv_cache.zig:14 */
  uint32_t num_blocks = (max_seq_len + block_size - 1) / block_size; /* :69 */
  if (num_blocks == 0) return NULL;
  kvo_cache* c = (kvo_cache*)calloc(1, sizeof(kvo_cache));
  if (!c) return NULL;
  if (kvo_pool_init(&c->pool, n_layers, num_blocks, block_size, kv_rank, rope_dim, 0) != KVO_OK) {
    free(c);
    return NULL;
  }
  c->ref_count = (uint32_t*)calloc(num_blocks, sizeof(uint32_t));
  c->hash = (uint64_t*)malloc(sizeof(uint64_t) * num_blocks);
  c->free_list = (uint32_t*)malloc(sizeof(uint32_t) * num_blocks);
  c->table_cap = num_blocks;
  c->table = (uint32_t*)malloc(sizeof(uint32_t) * (c->table_cap ? c->table_cap : 1));
  c->hm_cap = 4 * num_blocks + 8;
  c->hm = (hm_entry*)calloc(c->hm_cap, sizeof(hm_entry));
  for (uint32_t i = 0; i < num_blocks; ++i) {
    c->hash[i] = NO_HASH;
    c->free_list[i] = num_blocks - 1 - i; /* :89-91: pops hand out 0,1,2,... */
  }
  c->n_free = num_blocks;
  return c;
}

void kvo_cache_deinit(kvo_cache* c) {
  if (!c) return;
  kvo_pool_free(&c->pool);
  free(c->ref_count);
  free(c->hash);
  free(c->free_list);
  free(c->table);
  free(c->hm);
  free(c);
}

/* src/kv_cache.zig:142-154 (pools zeroed: deviation 3). */
int kvo_cache_enable_quantization(kvo_cache* c) {
  if (c->pool.quantized) return KVO_OK;
  uint64_t rows = (uint64_t)c->pool.n_layers * c->pool.num_blocks * c->pool.block_size;
  c->pool.kv_q8 = (kvo_block_q8*)calloc(rows * nq8(c->pool.kv_rank), sizeof(kvo_block_q8));
  c->pool.pe_q8 = (kvo_block_q8*)calloc(rows * nq8(c->pool.rope_dim), sizeof(kvo_block_q8));
  if (!c->pool.kv_q8 || !c->pool.pe_q8) return KVO_ERR_NO_MEMORY;
  c->pool.quantized = 1;
  return KVO_OK;
}

/* :158-164 */
static int allocate_block(kvo_cache* c, uint32_t* out) {
  if (c->n_free == 0) return KVO_ERR_OUT_OF_BLOCKS;
  uint32_t id = c->free_list[--c->n_free];
  c->ref_count[id] = 1;
  c->hash[id] = NO_HASH;
  *out = id;
  return KVO_OK;
}

/* :166-178 */
static void release_block(kvo_cache* c, uint32_t id) {
  if (id >= c->pool.num_blocks || c->ref_count[id] == 0) return;
  c->ref_count[id] -= 1;
  if (c->ref_count[id] == 0) {
    if (c->hash[id] != NO_HASH) hm_remove(c, c->hash[id]);
    c->hash[id] = NO_HASH;
    c->free_list[c->n_free++] = id;
  }
}

/* :180-183 */
static void retain_block(kvo_cache* c, uint32_t id) { c->ref_count[id] += 1; }

static int table_push(kvo_cache* c, uint32_t id) {
  if (c->table_len == c->table_cap) {
    uint32_t nc = c->table_cap ? 2 * c->table_cap : 4;
    uint32_t* t = (uint32_t*)realloc(c->table, sizeof(uint32_t) * nc);
    if (!t) return KVO_ERR_NO_MEMORY;
    c->table = t;
    c->table_cap = nc;
  }
  c->table[c->table_len++] = id;
  return KVO_OK;
}

/* :188-194 */
int kvo_cache_ensure_capacity(kvo_cache* c, uint32_t n_tokens) {
  uint32_t needed = (n_tokens + c->pool.block_size - 1) / c->pool.block_size;
  while (c->table_len < needed) {
    uint32_t id;
    int rc = allocate_block(c, &id);
    if (rc) return rc;
    rc = table_push(c, id);
    if (rc) return rc;
  }
  return KVO_OK;
}

/* :197-206 */
void kvo_cache_truncate(kvo_cache* c, uint32_t n_tokens) {
  uint32_t needed = (n_tokens + c->pool.block_size - 1) / c->pool.block_size;
  while (c->table_len > needed) release_block(c, c->table[--c->table_len]);
  if (n_tokens < c->len) c->len = n_tokens;
}

/* :209-215 */
void kvo_cache_reset(kvo_cache* c) {
  for (uint32_t i = 0; i < c->table_len; ++i) release_block(c, c->table[i]);
  c->table_len = 0;
  c->len = 0;
}

/* :279-361 */
int kvo_cache_put(kvo_cache* c, uint32_t layer, uint32_t pos, const float* kv_comp,
                  const float* k_pe) {
  if (layer >= c->pool.n_layers) return KVO_ERR_LAYER_OOB;
  uint32_t bi = pos / c->pool.block_size;
  if (bi >= c->table_len) return KVO_ERR_POSITION_OOB;
  kvo_pool_put(&c->pool, layer, c->table[bi], pos % c->pool.block_size, kv_comp, k_pe);
  if (pos >= c->len) c->len = pos + 1;
  return KVO_OK;
}

/* :225-277 */
static int resolve_get(kvo_cache* c, uint32_t layer, uint32_t pos, uint32_t* blk) {
  if (layer >= c->pool.n_layers) return KVO_ERR_LAYER_OOB;
  if (pos >= c->len) return KVO_ERR_POSITION_NOT_WRITTEN;
  uint32_t bi = pos / c->pool.block_size;
  if (bi >= c->table_len) return KVO_ERR_POSITION_OOB;
  *blk = c->table[bi];
  return KVO_OK;
}

int kvo_cache_get_kv_compressed(kvo_cache* c, uint32_t layer, uint32_t pos, float* out) {
  uint32_t blk;
  int rc = resolve_get(c, layer, pos, &blk);
  if (rc) return rc;
  kvo_pool_get(&c->pool, layer, blk, pos % c->pool.block_size, out, NULL);
  return KVO_OK;
}

int kvo_cache_get_kpe(kvo_cache* c, uint32_t layer, uint32_t pos, float* out) {
  uint32_t blk;
  int rc = resolve_get(c, layer, pos, &blk);
  if (rc) return rc;
  kvo_pool_get(&c->pool, layer, blk, pos % c->pool.block_size, NULL, out);
  return KVO_OK;
}

uint32_t kvo_cache_len(const kvo_cache* c) { return c->len; }
uint32_t kvo_cache_num_blocks(const kvo_cache* c) { return c->pool.num_blocks; }
uint32_t kvo_cache_num_free_blocks(const kvo_cache* c) { return c->n_free; }
int kvo_cache_quantized(const kvo_cache* c) { return c->pool.quantized; }
uint32_t kvo_cache_block_table_len(const kvo_cache* c) { return c->table_len; }
const uint32_t* kvo_cache_block_table(const kvo_cache* c) { return c->table; }
uint32_t kvo_cache_refcount(const kvo_cache* c, uint32_t id) {
  return id < c->pool.num_blocks ? c->ref_count[id] : 0;
}
/* :439-443: f32 pool bytes only (as the reference reports). */
uint64_t kvo_cache_memory_usage(const kvo_cache* c) {
  uint64_t rows = (uint64_t)c->pool.n_layers * c->pool.num_blocks * c->pool.block_size;
  return rows * (c->pool.kv_rank + c->pool.rope_dim) * sizeof(float);
}
const kvo_pool* kvo_cache_pool(const kvo_cache* c) { return &c->pool; }

int kvo_cache_set_free_list(kvo_cache* c, const uint32_t* ids, uint32_t n) {
  if (n > c->pool.num_blocks) return KVO_ERR_INVALID_ARG;
  for (uint32_t i = 0; i < n; ++i)
    if (ids[i] >= c->pool.num_blocks) return KVO_ERR_INVALID_ARG;
  memcpy(c->free_list, ids, sizeof(uint32_t) * n);
  c->n_free = n;
  return KVO_OK;
}

/* ---- prefix caching (:367-436) ---- */
void kvo_cache_cache_block(kvo_cache* c, uint32_t block_idx, const uint32_t* token_ids,
                           uint32_t n_tokens, uint64_t prefix_hash) {
  if (block_idx >= c->table_len) return;
  if (n_tokens != c->pool.block_size) return;
  uint32_t id = c->table[block_idx];
  uint64_t h = kvo_compute_hash(token_ids, n_tokens, prefix_hash);
  hm_entry* e = hm_find(c, h);
  if (e && e->value != id) return; /* collision: skip */
  c->hash[id] = h;
  hm_put(c, h, id);
}

uint32_t kvo_cache_find_prefix_blocks(kvo_cache* c, const uint32_t* tokens, uint32_t n) {
  uint64_t prefix = NO_HASH;
  uint32_t reusable = 0;
  uint32_t bs = c->pool.block_size;
  uint32_t nb = (n + bs - 1) / bs;
  for (uint32_t bi = 0; bi < nb; ++bi) {
    uint32_t start = bi * bs;
    uint32_t end = start + bs < n ? start + bs : n;
    if (end - start != bs) break;
    uint64_t h = kvo_compute_hash(tokens + start, bs, prefix);
    if (hm_find(c, h)) {
      prefix = h;
      reusable += 1;
    } else {
      break;
    }
  }
  return reusable;
}

int kvo_cache_reuse_prefix_blocks(kvo_cache* c, const uint32_t* tokens, uint32_t n,
                                  uint32_t n_blocks) {
  if (n_blocks == 0) return KVO_OK;
  uint32_t bs = c->pool.block_size;
  if ((uint64_t)n_blocks * bs > n) return KVO_ERR_INVALID_ARG;
  uint64_t prefix = NO_HASH;
  for (uint32_t bi = 0; bi < n_blocks; ++bi) {
    uint64_t h = kvo_compute_hash(tokens + (uint64_t)bi * bs, bs, prefix);
    hm_entry* e = hm_find(c, h);
    if (!e) return KVO_ERR_PREFIX_MISS;
    uint32_t cached = e->value;
    /* retain before release so a block that is already in place survives */
    retain_block(c, cached);
    if (bi < c->table_len) {
      release_block(c, c->table[bi]);
      c->table[bi] = cached;
    } else {
      int rc = table_push(c, cached);
      if (rc) return rc;
    }
    prefix = h;
  }
  c->len = n_blocks * bs;
  return KVO_OK;
}

/* ---- checkpoint v1 (:453-591) ---- */

static int write_all(int fd, const void* buf, size_t n) {
  const uint8_t* p = (const uint8_t*)buf;
  while (n) {
    ssize_t rc = write(fd, p, n);
    if (rc < 0) {
      if (errno == EINTR) continue;
      return KVO_ERR_IO;
    }
    if (rc == 0) return KVO_ERR_IO;
    p += rc;
    n -= (size_t)rc;
  }
  return KVO_OK;
}

static int read_no_eof(int fd, void* buf, size_t n) {
  uint8_t* p = (uint8_t*)buf;
  while (n) {
    ssize_t rc = read(fd, p, n);
    if (rc < 0) {
      if (errno == EINTR) continue;
      return KVO_ERR_IO;
    }
    if (rc == 0) return KVO_ERR_EOF;
    p += rc;
    n -= (size_t)rc;
  }
  return KVO_OK;
}

static void put_u32(uint8_t* b, uint32_t v) {
  b[0] = (uint8_t)v;
  b[1] = (uint8_t)(v >> 8);
  b[2] = (uint8_t)(v >> 16);
  b[3] = (uint8_t)(v >> 24);
}
static uint32_t get_u32(const uint8_t* b) {
  return (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
}

/* CheckpointHeader, :549-560 (extern struct, 40 bytes). */
int kvo_cache_save(const kvo_cache* c, const char* path) {
  int fd = open(path, O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
  if (fd < 0) return KVO_ERR_IO;
  uint8_t h[40];
  memset(h, 0, sizeof(h));
  memcpy(h, "KVCK", 4);
  put_u32(h + 4, 1);
  put_u32(h + 8, c->len);
  h[12] = c->pool.quantized ? 1 : 0;
  put_u32(h + 16, c->table_len);
  put_u32(h + 20, c->pool.n_layers);
  put_u32(h + 24, c->pool.num_blocks);
  put_u32(h + 28, c->pool.block_size);
  put_u32(h + 32, c->pool.kv_rank);
  put_u32(h + 36, c->pool.rope_dim);
  int rc = write_all(fd, h, sizeof(h));
  for (uint32_t i = 0; rc == KVO_OK && i < c->table_len; ++i) {
    uint8_t b[4];
    put_u32(b, c->table[i]);
    rc = write_all(fd, b, 4);
  }
  if (rc == KVO_OK) {
    uint64_t nbytes = kvo_pool_bytes(&c->pool);
    uint8_t* buf = (uint8_t*)malloc(nbytes);
    if (!buf) rc = KVO_ERR_NO_MEMORY;
    else {
      kvo_pool_serialize(&c->pool, buf);
      rc = write_all(fd, buf, nbytes);
      free(buf);
    }
  }
  close(fd);
  return rc;
}

int kvo_cache_load(kvo_cache* c, const char* path) {
  int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return KVO_ERR_IO;
  uint8_t h[40];
  int rc = read_no_eof(fd, h, sizeof(h));
  if (rc) goto done;
  if (memcmp(h, "KVCK", 4) != 0) {
    rc = KVO_ERR_BAD_MAGIC;
    goto done;
  }
  if (get_u32(h + 4) != 1) {
    rc = KVO_ERR_BAD_VERSION;
    goto done;
  }
  if (get_u32(h + 20) != c->pool.n_layers || get_u32(h + 24) != c->pool.num_blocks ||
      get_u32(h + 28) != c->pool.block_size || get_u32(h + 32) != c->pool.kv_rank ||
      get_u32(h + 36) != c->pool.rope_dim) {
    rc = KVO_ERR_SHAPE_MISMATCH;
    goto done;
  }
  {
    uint32_t len = get_u32(h + 8);
    uint32_t tlen = get_u32(h + 16);
    int quant = h[12] == 1;
    if (tlen > c->pool.num_blocks || (uint64_t)len > (uint64_t)tlen * c->pool.block_size ||
        (!quant && c->pool.quantized)) {
      rc = KVO_ERR_SHAPE_MISMATCH;
      goto done;
    }
    uint32_t* ids = (uint32_t*)malloc(sizeof(uint32_t) * (tlen ? tlen : 1));
    for (uint32_t i = 0; i < tlen; ++i) {
      uint8_t b[4];
      rc = read_no_eof(fd, b, 4);
      if (rc) {
        free(ids);
        goto done;
      }
      ids[i] = get_u32(b);
      if (ids[i] >= c->pool.num_blocks) {
        free(ids);
        rc = KVO_ERR_BAD_BLOCK_ID; /* deviation 4 */
        goto done;
      }
    }
    if (quant && !c->pool.quantized) {
      rc = kvo_cache_enable_quantization(c);
      if (rc) {
        free(ids);
        goto done;
      }
    }
    uint64_t nbytes = kvo_pool_bytes(&c->pool);
    uint8_t* buf = (uint8_t*)malloc(nbytes);
    if (!buf) {
      free(ids);
      rc = KVO_ERR_NO_MEMORY;
      goto done;
    }
    rc = read_no_eof(fd, buf, nbytes);
    if (rc) {
      free(buf);
      free(ids);
      goto done;
    }
    /* Commit: release the old table, retain the loaded ids and take them off
     * the free list (deviation 4), then restore the pool bytes. */
    for (uint32_t i = 0; i < c->table_len; ++i) release_block(c, c->table[i]);
    c->table_len = 0;
    for (uint32_t i = 0; i < tlen; ++i) {
      uint32_t id = ids[i];
      if (c->ref_count[id] == 0) {
        for (uint32_t k = 0; k < c->n_free; ++k) {
          if (c->free_list[k] == id) {
            memmove(c->free_list + k, c->free_list + k + 1, sizeof(uint32_t) * (c->n_free - k - 1));
            c->n_free -= 1;
            break;
          }
        }
      }
      retain_block(c, id);
      table_push(c, id);
    }
    c->len = len;
    kvo_pool_deserialize(&c->pool, buf);
    free(buf);
    free(ids);
  }
done:
  close(fd);
  return rc;
}

/* ===================== XXH64 (published xxHash specification) ===================== */

#define XP1 0x9E3779B185EBCA87ull
#define XP2 0xC2B2AE3D27D4EB4Full
#define XP3 0x165667B19E3779F9ull
#define XP4 0x85EBCA77C2B2AE63ull
#define XP5 0x27D4EB2F165667C5ull

static inline uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
static inline uint64_t rd64(const uint8_t* p) {
  uint64_t v = 0;
  for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
  return v;
}
static inline uint64_t xround(uint64_t acc, uint64_t in) {
  acc += in * XP2;
  acc = rotl64(acc, 31);
  return acc * XP1;
}
static inline uint64_t xmerge(uint64_t acc, uint64_t v) {
  acc ^= xround(0, v);
  return acc * XP1 + XP4;
}

uint64_t kvo_xxh64(const void* data, size_t len, uint64_t seed) {
  const uint8_t* p = (const uint8_t*)data;
  const uint8_t* end = p + len;
  uint64_t h;
  if (len >= 32) {
    uint64_t v1 = seed + XP1 + XP2, v2 = seed + XP2, v3 = seed, v4 = seed - XP1;
    while (p + 32 <= end) {
      v1 = xround(v1, rd64(p));
      v2 = xround(v2, rd64(p + 8));
      v3 = xround(v3, rd64(p + 16));
      v4 = xround(v4, rd64(p + 24));
      p += 32;
    }
    h = rotl64(v1, 1) + rotl64(v2, 7) + rotl64(v3, 12) + rotl64(v4, 18);
    h = xmerge(h, v1);
    h = xmerge(h, v2);
    h = xmerge(h, v3);
    h = xmerge(h, v4);
  } else {
    h = seed + XP5;
  }
  h += (uint64_t)len;
  while (p + 8 <= end) {
    h ^= xround(0, rd64(p));
    h = rotl64(h, 27) * XP1 + XP4;
    p += 8;
  }
  if (p + 4 <= end) {
    h ^= (uint64_t)get_u32(p) * XP1;
    h = rotl64(h, 23) * XP2 + XP3;
    p += 4;
  }
  while (p < end) {
    h ^= (uint64_t)(*p) * XP5;
    h = rotl64(h, 11) * XP1;
    p += 1;
  }
  h ^= h >> 33;
  h *= XP2;
  h ^= h >> 29;
  h *= XP3;
  h ^= h >> 32;
  return h;
}

uint64_t kvo_compute_hash(const uint32_t* token_ids, uint32_t n, uint64_t prefix_hash) {
  size_t nbytes = (prefix_hash != NO_HASH ? 8 : 0) + 4 * (size_t)n;
  uint8_t stackbuf[1024] = {0};
  uint8_t* buf = nbytes <= sizeof(stackbuf) ? stackbuf : (uint8_t*)malloc(nbytes);
  size_t o = 0;
  if (prefix_hash != NO_HASH) {
    for (int i = 0; i < 8; ++i) buf[o++] = (uint8_t)(prefix_hash >> (8 * i));
  }
  for (uint32_t i = 0; i < n; ++i) {
    put_u32(buf + o, token_ids[i]);
    o += 4;
  }
  uint64_t h = kvo_xxh64(buf, nbytes, 0);
  if (buf != stackbuf) free(buf);
  return h;
}

/* ============================ seeded synthetic inputs ============================ */

/* SplitMix64 (Steele, Lea & Flood, "Fast splittable pseudorandom number
 * generators", OOPSLA 2014; finaliser constants as published by Vigna). */
uint64_t kvo_splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Natural log for s in (0, 1) from basic IEEE operations only, so the host
 * and the device agree to the bit: s = 2^e * m with m in [sqrt(1/2), sqrt(2)),
 * ln m = 2 atanh(t), t = (m-1)/(m+1), atanh as its Taylor series to t^13
 * (|t| <= 0.1716, truncation error below 3e-13). */
float kvo_log_det(float s) {
  uint32_t bits = f2u(s);
  int e = (int)((bits >> 23) & 0xFF) - 127;
  float m = u2f((bits & 0x7FFFFFu) | 0x3F800000u);
  if (m > 1.41421356f) {
    m = m * 0.5f;
    e += 1;
  }
  float t = (m - 1.0f) / (m + 1.0f);
  float t2 = t * t;
  float p = 0.0769230769f; /* 1/13 */
  p = p * t2;
  p = p + 0.0909090909f; /* 1/11 */
  p = p * t2;
  p = p + 0.111111111f; /* 1/9 */
  p = p * t2;
  p = p + 0.142857143f; /* 1/7 */
  p = p * t2;
  p = p + 0.2f; /* 1/5 */
  p = p * t2;
  p = p + 0.333333333f; /* 1/3 */
  p = p * t2;
  p = p + 1.0f;
  float tt = t + t;
  float lnm = tt * p;
  float el = (float)e * 0.693147181f;
  return el + lnm;
}

static inline uint64_t gen_key(uint64_t seed, uint64_t a, uint64_t b, uint64_t c) {
  uint64_t k = kvo_splitmix64(seed ^ kvo_splitmix64(a));
  k = kvo_splitmix64(k ^ b);
  return kvo_splitmix64(k ^ c);
}

/* Marsaglia polar method on 23-bit symmetric uniforms (never 0), at most 64
 * attempts (then 0), optional outlier: with probability outlier_p the value is
 * multiplied by 20. */
float kvo_gen_normal(uint64_t seed, uint64_t a, uint64_t b, uint64_t c, float outlier_p) {
  uint64_t key = gen_key(seed, a, b, c);
  float z = 0.0f;
  for (uint32_t j = 0; j < 64; ++j) {
    uint64_t r = kvo_splitmix64(key + j);
    uint32_t ux = (uint32_t)(r >> 41);
    uint32_t uy = (uint32_t)(r >> 18) & 0x7FFFFFu;
    float x = (float)(2u * ux + 1u) * 1.1920928955078125e-07f - 1.0f;
    float y = (float)(2u * uy + 1u) * 1.1920928955078125e-07f - 1.0f;
    float xx = x * x;
    float yy = y * y;
    float s = xx + yy;
    if (s >= 1.0f) continue;
    float ls = kvo_log_det(s);
    float num = -2.0f * ls;
    float ratio = num / s;
    float f = sqrtf(ratio);
    z = x * f;
    break;
  }
  if (outlier_p > 0.0f) {
    uint64_t r = kvo_splitmix64(key ^ 0xD1B54A32D192ED03ull);
    float u = (float)(uint32_t)(r >> 40) * 5.9604644775390625e-08f;
    if (u < outlier_p) z = z * 20.0f;
  }
  return z;
}

typedef struct {
  uint64_t seed, a;
  const uint32_t* b;
  const uint32_t* c;
  uint32_t width;
  float outlier_p;
  float* out;
  uint32_t r0, r1;
} gen_ctx;

static void* gen_worker(void* arg) {
  gen_ctx* g = (gen_ctx*)arg;
  for (uint32_t r = g->r0; r < g->r1; ++r)
    for (uint32_t i = 0; i < g->width; ++i)
      g->out[(uint64_t)r * g->width + i] =
          kvo_gen_normal(g->seed, g->a, g->b[r], (uint64_t)g->c[r] * 1024u + i, g->outlier_p);
  return NULL;
}

void kvo_gen_rows(uint64_t seed, uint64_t a, uint32_t n_rows, const uint32_t* b,
                  const uint32_t* c, uint32_t width, float outlier_p, float* out,
                  int n_threads) {
  if (n_threads < 1) n_threads = 1;
  if ((uint32_t)n_threads > n_rows) n_threads = n_rows ? (int)n_rows : 1;
  pthread_t th[256];
  gen_ctx ctx[256];
  if (n_threads > 256) n_threads = 256;
  uint32_t per = (n_rows + (uint32_t)n_threads - 1) / (uint32_t)n_threads;
  for (int t = 0; t < n_threads; ++t) {
    gen_ctx g = {seed, a, b, c, width, outlier_p, out, 0, 0};
    g.r0 = (uint32_t)t * per;
    g.r1 = g.r0 + per < n_rows ? g.r0 + per : n_rows;
    if (g.r0 > n_rows) g.r0 = n_rows;
    ctx[t] = g;
  }
  if (n_threads == 1) {
    gen_worker(&ctx[0]);
    return;
  }
  for (int t = 0; t < n_threads; ++t) pthread_create(&th[t], NULL, gen_worker, &ctx[t]);
  for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
}
