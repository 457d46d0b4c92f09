/*
 * kvoracle.h — CPU restatement of mobile-moe.zig's paged KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * product in `mobile-moe.zig_b200/`.  Only `tests/`, `__graft_entry__.smoke()`
 * and `bench.py`'s CPU-baseline leg may load it; the product never links it and
 * never falls back to it.
 *
 * What it restates (paths relative to the reference project root):
 *   - f16 <-> f32 bit conversion            src/dequant.zig:19-95
 *   - Q8_0 block quantize / dequantize      src/kv_cache.zig:289-349, :232-246,
 *                                           src/dequant.zig:98-142, :372-377
 *   - KVCache pool layout, LIFO free list,  src/kv_cache.zig:64-122, :158-215
 *     refcounts, block_table, put/get       src/kv_cache.zig:219-361
 *   - prefix-cache hash chain (XXH64)       src/kv_cache.zig:367-436, :596-609
 *   - v1 checkpoint (header/table/pool)     src/kv_cache.zig:453-591
 *   - MLA decode attention core, absorbed   src/inference.zig:572-660
 *     form, 64-token online-softmax chunks
 *   - threaded CPU baseline on a pthread    src/thread_pool.zig:15-99
 *     mutex/cond FIFO pool
 *
 * Parity pin: the Zig reference cannot be built here (no zig toolchain), so
 * this restatement is pinned against the reference's own known-answer tests
 * (src/kv_cache.zig:643-842, src/dequant.zig:663-707, src/root.zig:298-315)
 * and against independent numpy / python-xxhash fixtures in tests/golden/.
 *
 * Deliberate, documented deviations from the reference (shared with the
 * product so both sides agree):
 *   1. f32ToF16 for results in the f16-subnormal range uses correct IEEE
 *      round-to-nearest-even.  The reference shifts by (1-exp16) instead of
 *      (14-exp16) at src/dequant.zig:76-77 and overflows u16 there.
 *   2. A Q8_0 quotient x/d that is NaN (only reachable with inf/NaN inputs,
 *      undefined behaviour in the reference) quantizes to 0.
 *   3. Q8_0 pools are zero-initialised (the reference leaves them undefined,
 *      src/kv_cache.zig:151-152), and the checkpoint header's 3 padding bytes
 *      are written as zeros.
 *   4. loadFromFile bounds-checks loaded block ids and removes them from the
 *      free list (the reference only retains them, src/kv_cache.zig:527-533).
 *   5. The attention score is multiplied by `scale` (1/sqrt(head_dim)) where
 *      the reference divides by sqrt(head_dim) (src/inference.zig:613).
 *   6. reusePrefixBlocks retains the cached block before releasing the one it
 *      replaces, so re-syncing a sequence onto its own cached blocks keeps
 *      them off the free list (the reference releases first,
 *      src/kv_cache.zig:418-424, which frees a block that stays in the table).
 */
#ifndef KVORACLE_H
#define KVORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes: the same numbers as the product's KVCU_* codes. */
enum {
  KVO_OK = 0,
  KVO_ERR_OUT_OF_BLOCKS = -1,      /* error.OutOfKVCacheBlocks */
  KVO_ERR_POSITION_OOB = -2,       /* error.PositionOutOfBounds */
  KVO_ERR_LAYER_OOB = -3,          /* error.LayerOutOfBounds */
  KVO_ERR_POSITION_NOT_WRITTEN = -4, /* error.PositionNotWritten */
  KVO_ERR_PREFIX_MISS = -5,        /* error.PrefixCacheMiss */
  KVO_ERR_BAD_MAGIC = -6,          /* error.InvalidCheckpointMagic */
  KVO_ERR_BAD_VERSION = -7,        /* error.UnsupportedCheckpointVersion */
  KVO_ERR_SHAPE_MISMATCH = -8,     /* error.CheckpointShapeMismatch */
  KVO_ERR_EOF = -9,                /* error.EndOfStream */
  KVO_ERR_IO = -10,                /* POSIX open/read/write errors */
  KVO_ERR_INVALID_ARG = -11,
  KVO_ERR_NO_MEMORY = -14,
  KVO_ERR_BAD_BLOCK_ID = -15
};

/* BlockQ8_0, src/dequant.zig:372-377: 34 bytes, {f16 d; i8 qs[32]}. */
typedef struct {
  uint16_t d;
  int8_t qs[32];
} kvo_block_q8;

/* ---- numerics ---- */
float kvo_f16_to_f32(uint16_t h);
uint16_t kvo_f32_to_f16(float v);
/* Quantize n floats into ceil(n/32) blocks (tail zero-filled). */
void kvo_quantize_q8_0(const float* x, uint32_t n, kvo_block_q8* out);
/* Dequantize n floats out of ceil(n/32) blocks. */
void kvo_dequantize_q8_0(const kvo_block_q8* b, uint32_t n, float* out);

/* ---- pool (reference layout) ---- */
typedef struct {
  uint32_t n_layers, num_blocks, block_size, kv_rank, rope_dim;
  int quantized;
  float* kv;            /* [L][NB][BS][kv_rank]  (kv_compressed) */
  float* pe;            /* [L][NB][BS][rope_dim] (k_pe)          */
  kvo_block_q8* kv_q8;  /* [L][NB][BS][ceil(kv_rank/32)]         */
  kvo_block_q8* pe_q8;  /* [L][NB][BS][ceil(rope_dim/32)]        */
} kvo_pool;

int kvo_pool_init(kvo_pool* p, uint32_t n_layers, uint32_t num_blocks, uint32_t block_size,
                  uint32_t kv_rank, uint32_t rope_dim, int quantized);
void kvo_pool_free(kvo_pool* p);
/* Write one row (kv_comp[kv_rank], k_pe[rope_dim]) at (layer, block, offset). */
void kvo_pool_put(kvo_pool* p, uint32_t layer, uint32_t block, uint32_t offset,
                  const float* kv_comp, const float* k_pe);
/* Batched put: row r (rows[r][kv_rank+rope_dim]) goes to (blocks[r], offsets[r]). */
void kvo_pool_put_rows(kvo_pool* p, uint32_t layer, uint32_t n, const uint32_t* blocks,
                       const uint32_t* offsets, const float* rows);
/* Read (dequantize) one row. */
void kvo_pool_get(const kvo_pool* p, uint32_t layer, uint32_t block, uint32_t offset,
                  float* kv_out, float* pe_out);
/* Gather `len` rows of a sequence through its table into out[len][kv_rank+rope_dim]. */
void kvo_pool_gather(const kvo_pool* p, uint32_t layer, const uint32_t* table, uint32_t len,
                     float* out);
/* Bytes of the pool section of a checkpoint (kv then pe, reference order). */
uint64_t kvo_pool_bytes(const kvo_pool* p);
/* Copy the pool section out / in (reference byte layout). */
void kvo_pool_serialize(const kvo_pool* p, uint8_t* dst);
void kvo_pool_deserialize(kvo_pool* p, const uint8_t* src);

/* ---- MLA decode attention core (absorbed form) ----
 * q: [n_heads][kv_rank + rope_dim]; out: [n_heads][kv_rank]. */
void kvo_attention(const kvo_pool* p, uint32_t layer, const uint32_t* table, uint32_t len,
                   const float* q, uint32_t n_heads, float scale, float* out);
/* Batched: sequence b uses tables[table_offsets[b] ...], length lens[b].
 * q: [B][H][R+P], out: [B][H][R].  n_threads <= 1 runs inline; otherwise a
 * pthread mutex/cond FIFO pool runs one task per (sequence, head). */
void kvo_attention_batch(const kvo_pool* p, uint32_t layer, uint32_t n_seqs,
                         const uint32_t* table_offsets, const uint32_t* tables,
                         const uint32_t* lens, const float* q, uint32_t n_heads, float scale,
                         float* out, int n_threads);

/* ---- single-sequence KVCache (src/kv_cache.zig:24-546) ---- */
typedef struct kvo_cache kvo_cache;
kvo_cache* kvo_cache_init(uint32_t n_layers, uint32_t kv_rank, uint32_t rope_dim,
                          uint32_t max_seq_len, uint32_t block_size);
void kvo_cache_deinit(kvo_cache* c);
int kvo_cache_enable_quantization(kvo_cache* c);
int kvo_cache_ensure_capacity(kvo_cache* c, uint32_t n_tokens);
void kvo_cache_truncate(kvo_cache* c, uint32_t n_tokens);
void kvo_cache_reset(kvo_cache* c);
int kvo_cache_put(kvo_cache* c, uint32_t layer, uint32_t pos, const float* kv_comp,
                  const float* k_pe);
int kvo_cache_get_kv_compressed(kvo_cache* c, uint32_t layer, uint32_t pos, float* out);
int kvo_cache_get_kpe(kvo_cache* c, uint32_t layer, uint32_t pos, float* out);
uint32_t kvo_cache_len(const kvo_cache* c);
uint32_t kvo_cache_num_blocks(const kvo_cache* c);
uint32_t kvo_cache_num_free_blocks(const kvo_cache* c);
int kvo_cache_quantized(const kvo_cache* c);
uint32_t kvo_cache_block_table_len(const kvo_cache* c);
const uint32_t* kvo_cache_block_table(const kvo_cache* c);
uint32_t kvo_cache_refcount(const kvo_cache* c, uint32_t block_id);
uint64_t kvo_cache_memory_usage(const kvo_cache* c);
const kvo_pool* kvo_cache_pool(const kvo_cache* c);
/* Overwrite the free list (LIFO: the last entry is handed out first). */
int kvo_cache_set_free_list(kvo_cache* c, const uint32_t* ids, uint32_t n);
int kvo_cache_save(const kvo_cache* c, const char* path);
int kvo_cache_load(kvo_cache* c, const char* path);
void kvo_cache_cache_block(kvo_cache* c, uint32_t block_idx, const uint32_t* token_ids,
                           uint32_t n_tokens, uint64_t prefix_hash);
uint32_t kvo_cache_find_prefix_blocks(kvo_cache* c, const uint32_t* tokens, uint32_t n);
int kvo_cache_reuse_prefix_blocks(kvo_cache* c, const uint32_t* tokens, uint32_t n,
                                  uint32_t n_blocks);

/* ---- hashing ---- */
uint64_t kvo_xxh64(const void* data, size_t len, uint64_t seed);
/* src/kv_cache.zig:596-609: XXH64(seed 0) over [prefix LE u64 unless
 * prefix == UINT64_MAX] ++ [token ids LE u32]. */
uint64_t kvo_compute_hash(const uint32_t* token_ids, uint32_t n, uint64_t prefix_hash);

/* ---- seeded synthetic inputs (bit-identical to the product generator) ---- */
uint64_t kvo_splitmix64(uint64_t x);
float kvo_log_det(float s);
float kvo_gen_normal(uint64_t seed, uint64_t a, uint64_t b, uint64_t c, float outlier_p);
/* out[r][i] = gen_normal(seed, a, b[r], c[r]*1024 + i, outlier_p), i < width. */
void kvo_gen_rows(uint64_t seed, uint64_t a, uint32_t n_rows, const uint32_t* b,
                  const uint32_t* c, uint32_t width, float outlier_p, float* out,
                  int n_threads);

#ifdef __cplusplus
}
#endif
#endif
