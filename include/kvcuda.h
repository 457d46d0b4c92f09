/*
 * kvcuda.h — C-ABI of libkvcuda.so, the B200 (sm_100a) paged MLA KV-cache
 * library: Q8_0/f32 token append through a block table, block-table
 * gather/dequant, paged MLA decode attention, checkpoint I/O.
 *
 * It is the drop-in boundary for mobile-moe.zig's KV-cache hot path.  The
 * reference's host code (Zig) would bind these functions with `extern fn`
 * declarations exactly as src/metal_backend.zig:7-26 binds src/metal_bridge.c.
 * Conventions copied from
 * src/metal_bridge.c: a process-wide last-error string (:50-52), `int` return
 * codes (0 = success, negative = error, :54-87), opaque handles with explicit
 * release (:89-96).  No entry point ever falls back to the CPU: without a
 * usable CUDA device every call returns an error.
 *
 * Two layers:
 *   kvcu_*     device-level operations on device pointers (what a host
 *              allocator written in another language drives);
 *   kvcache_*  a C++ host mirror of src/kv_cache.zig's KVCache (block
 *              allocator, block_table, put/get, prefix cache, checkpoint)
 *              extended to many sequences on one pool, taking HOST buffers.
 *
 * Device pool layout (per GPU, all layers in one pool):
 *   f32 pools  : kv [L][NB][BS][kv_rank] f32 and pe [L][NB][BS][rope_dim] f32,
 *                identical to src/kv_cache.zig:34-37.
 *   Q8_0 pools : qs [L][NB][BS][nblk*32] int8 and sc [L][NB][BS][nblk] f16 bits,
 *                nblk = ceil(kv_rank/32) + ceil(rope_dim/32).  Same bytes as
 *                the reference's BlockQ8_0 pools (src/kv_cache.zig:55-57),
 *                split into payload and scales; checkpoints convert to the
 *                reference's 34-byte block order.
 *
 * Threading: handles are not re-entrant (as KVCache is not, because of its
 * shared dequant scratch, src/kv_cache.zig:59-60); use one host thread per GPU.
 *
 * Deliberate differences from the reference, where its behaviour is undefined
 * or wrong: f32->f16 in the f16-subnormal range rounds to nearest even (the
 * reference mis-shifts, src/dequant.zig:76-77); a NaN quotient x/d quantizes
 * to 0; Q8_0 pools start zeroed (src/kv_cache.zig:151-152 leaves them
 * undefined) and the checkpoint header's padding bytes are written as zeros;
 * loadFromFile bounds-checks block ids and takes them off the free list
 * (src/kv_cache.zig:527-533 only retains them); the attention score is
 * multiplied by `scale` rather than divided by sqrt(head_dim)
 * (src/inference.zig:613); reusePrefixBlocks retains the cached block before
 * releasing the one it replaces (src/kv_cache.zig:418-424 releases first).
 */
#ifndef KVCUDA_H
#define KVCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- errors */
/* The first eleven mirror the reference's error set (src/kv_cache.zig). */
#define KVCU_OK 0
#define KVCU_ERR_OUT_OF_BLOCKS (-1)        /* error.OutOfKVCacheBlocks   kv_cache.zig:159 */
#define KVCU_ERR_POSITION_OOB (-2)         /* error.PositionOutOfBounds  kv_cache.zig:221 */
#define KVCU_ERR_LAYER_OOB (-3)            /* error.LayerOutOfBounds     kv_cache.zig:226 */
#define KVCU_ERR_POSITION_NOT_WRITTEN (-4) /* error.PositionNotWritten   kv_cache.zig:227 */
#define KVCU_ERR_PREFIX_MISS (-5)          /* error.PrefixCacheMiss      kv_cache.zig:416 */
#define KVCU_ERR_BAD_MAGIC (-6)            /* error.InvalidCheckpointMagic kv_cache.zig:509 */
#define KVCU_ERR_BAD_VERSION (-7)          /* error.UnsupportedCheckpointVersion :510 */
#define KVCU_ERR_SHAPE_MISMATCH (-8)       /* error.CheckpointShapeMismatch :517 */
#define KVCU_ERR_EOF (-9)                  /* error.EndOfStream          kv_cache.zig:588 */
#define KVCU_ERR_IO (-10)                  /* POSIX errors of open/read/write */
#define KVCU_ERR_INVALID_ARG (-11)
#define KVCU_ERR_CUDA (-12)                /* a CUDA runtime call failed (see last error) */
#define KVCU_ERR_DEVICE (-13)              /* a kernel flagged a bad index (status word) */
#define KVCU_ERR_NO_MEMORY (-14)
#define KVCU_ERR_BAD_BLOCK_ID (-15)        /* checkpoint names a block id >= num_blocks */
#define KVCU_ERR_UNSUPPORTED (-16)         /* shape outside what the kernels implement */
#define KVCU_ERR_NO_DEVICE (-17)

/* Device status-word bits set by kernels instead of trapping. */
#define KVCU_STATUS_BAD_TABLE 0x1u   /* pos / block_size beyond the sequence's table */
#define KVCU_STATUS_BAD_BLOCK 0x2u   /* table entry >= num_blocks */
#define KVCU_STATUS_BAD_SEQ 0x4u     /* sequence id >= n_seqs */
#define KVCU_STATUS_BAD_LEN 0x8u     /* lens[s] > table length * block_size */
#define KVCU_STATUS_TIMEOUT 0x10u    /* a bounded device-side wait gave up */
#define KVCU_STATUS_MISALIGNED 0x20u /* a decode tile did not start on a block-row boundary */
#define KVCU_STATUS_BAD_PLAN 0x40u   /* the decode plan has more CTA ranges than the decode grid */

/* metal_get_last_error, src/metal_bridge.c:50-52.  Thread-local. */
const char* kvcu_get_last_error(void);
/* metal_init, src/metal_bridge.c:54-87: select a CUDA device, check it is
 * sm_100 (B200), create its context and reserve the fixed scratch of
 * kvcu_mla_decode_noalloc on it.  0 on success. */
int kvcu_init(int device);
/* Number of visible CUDA devices (0 without a driver/GPU). */
int kvcu_device_count(void);
/* Library version, for the binding to check. */
uint32_t kvcu_version(void);

/* ------------------------------------------------------------ block pool */
typedef struct kvcu_pool kvcu_pool;

typedef struct {
  uint32_t n_layers, num_blocks, block_size, kv_rank, rope_dim;
  uint32_t quantized;       /* 1: Q8_0 pools, 0: f32 pools */
  uint32_t nblk;            /* Q8_0 blocks per row */
  int32_t device;
  void* kv;                 /* f32 kv pool (NULL when quantized) */
  void* pe;                 /* f32 pe pool (NULL when quantized) */
  void* qs;                 /* Q8_0 payload pool (NULL when f32) */
  void* sc;                 /* Q8_0 scale pool (NULL when f32) */
  uint64_t pool_bytes;      /* device bytes of the data pools */
  uint64_t checkpoint_bytes;/* bytes of the pool section of a checkpoint */
} kvcu_pool_desc;

/* The pool half of KVCache.init + enableQuantization (src/kv_cache.zig:64-122,
 * :142-154): allocate and zero the physical block pool for all layers on
 * `device`.  block_size must be a multiple of 16 (the reference's 16, or 64
 * for long contexts).  NULL on failure. */
kvcu_pool* kvcu_pool_create(int device, uint32_t n_layers, uint32_t num_blocks,
                            uint32_t block_size, uint32_t kv_rank, uint32_t rope_dim,
                            int quantized);
/* metal_release analogue (src/metal_bridge.c:94-96); KVCache.deinit's frees
 * (src/kv_cache.zig:124-139). */
int kvcu_pool_destroy(kvcu_pool* pool);
int kvcu_pool_describe(const kvcu_pool* pool, kvcu_pool_desc* out);
/* Zero every pool byte (stream-ordered). */
int kvcu_pool_zero(kvcu_pool* pool, void* stream);
/* Read and clear the device status word (synchronises `stream`). */
int kvcu_pool_status(kvcu_pool* pool, uint32_t* status_out, void* stream);
/* Copy physical block `src` to `dst` in every layer, device to device
 * (stream-ordered): the copy of a copy-on-write of a shared prefix block. */
int kvcu_pool_copy_block(kvcu_pool* pool, uint32_t src, uint32_t dst, void* stream);

/* ------------------------------------------------------------ append / gather
 * Sequences are described by device arrays indexed by sequence id s:
 *   table_offsets[s] .. table_offsets[s+1]  its slice of `tables` (CSR),
 *   tables[...]                              physical block ids, logical order.
 */

/* KVCache.put batched (src/kv_cache.zig:279-361; callers inference.zig:516,733):
 * for every row r < n_rows, quantize (Q8_0 pool) or copy (f32 pool) the row
 * latent[r*latent_stride .. +kv_rank] ++ rope[r*rope_stride .. +rope_dim] into
 * (layer, tables[table_offsets[row_seq[r]] + row_pos[r]/BS], row_pos[r]%BS).
 * Q8_0 bytes equal the reference's bit for bit.  If `lens` is not NULL it is
 * updated as the reference updates `len` (src/kv_cache.zig:358-360):
 * lens[s] = max(lens[s], pos + 1).  All pointers are device pointers; bad ids
 * set the status word and skip the row.  Stream-ordered. */
int kvcu_append(kvcu_pool* pool, uint32_t layer, uint32_t n_rows, const float* latent,
                uint64_t latent_stride, const float* rope, uint64_t rope_stride,
                const uint32_t* row_seq, const uint32_t* row_pos, uint32_t n_seqs,
                const uint32_t* table_offsets, const uint32_t* tables, uint32_t* lens,
                void* stream);

/* kvcu_append for layers [layer, layer + n_layers) in one launch: the rows of
 * layer layer+i start at latent + i*latent_layer_stride and rope +
 * i*rope_layer_stride (floats), same row_seq / row_pos for every layer. */
int kvcu_append_layers(kvcu_pool* pool, uint32_t layer, uint32_t n_layers, uint32_t n_rows, const float* latent,
                       uint64_t latent_stride, uint64_t latent_layer_stride, const float* rope,
                       uint64_t rope_stride, uint64_t rope_layer_stride, const uint32_t* row_seq,
                       const uint32_t* row_pos, uint32_t n_seqs, const uint32_t* table_offsets,
                       const uint32_t* tables, uint32_t* lens, void* stream);

/* getKVCompressed + getKPe for every position of a sequence
 * (src/kv_cache.zig:225-277): out[len][kv_rank + rope_dim] f32, dequantized
 * exactly as f16ToF32(d) * q.  `table` is a device pointer to `table_len` ids. */
int kvcu_gather(kvcu_pool* pool, uint32_t layer, const uint32_t* table, uint32_t table_len,
                uint32_t len, float* out, void* stream);

/* Batched gather: rows r < n_rows, out[r][kv_rank + rope_dim] = row (row_seq[r], row_pos[r]). */
int kvcu_gather_rows(kvcu_pool* pool, uint32_t layer, uint32_t n_rows, const uint32_t* row_seq,
                     const uint32_t* row_pos, uint32_t n_seqs, const uint32_t* table_offsets,
                     const uint32_t* tables, float* out, void* stream);

/* ------------------------------------------------------------ MLA decode
 * The attention core of InferenceEngine.mlaAttention (src/inference.zig:518-660)
 * in absorbed form: for batch entry b (sequence s = seq_ids ? seq_ids[b] : b,
 * length lens[s]) and head h,
 *   score_p = scale * (q[b][h][0:R] . latent_p + q[b][h][R:R+P] . rope_p)
 *   out[b][h][0:R] = sum_p softmax(score)_p * latent_p   (0 when lens[s] == 0)
 * over positions p < lens[s] read through the block table.  R = kv_rank = 512,
 * P = rope_dim = 64, n_heads <= 32.  q: [n][n_heads][R+P] f32, out: [n][n_heads][R]
 * f32, device pointers.  Long sequences are split across CTAs (split-KV); the
 * partial results live in the workspace and are combined by a second kernel. */
typedef struct kvcu_decode_ws kvcu_decode_ws;

/* Workspace for up to max_batch entries of up to max_heads heads. */
kvcu_decode_ws* kvcu_decode_ws_create(int device, uint32_t max_batch, uint32_t max_heads);
int kvcu_decode_ws_destroy(kvcu_decode_ws* ws);
/* Split the batch into work items from the device lengths (one small kernel,
 * stream-ordered).  Each sequence's last item is open-ended, so a plan stays
 * valid while appends grow the sequences (re-plan when the batch changes or
 * sequences shrink); all layers of a step share it. */
int kvcu_decode_plan(kvcu_decode_ws* ws, const kvcu_pool* pool, uint32_t n, const uint32_t* seq_ids,
                     uint32_t n_seqs, const uint32_t* lens, void* stream);
/* The plan for causal multi-query attention, the loop of
 * InferenceEngine.mlaAttentionBatch (src/inference.zig:771-877): entry b
 * attends positions [0, min(entry_lens[b], lens[seq])) of its sequence, so the
 * n new positions p0..p0+n-1 of one prompt become n entries of the same
 * sequence with entry_lens = p0+1 .. p0+n (their rows appended first, as the
 * reference puts every position before attending, :733).  Entries of any
 * sequences may be mixed.  entry_lens is a device array that must stay
 * unchanged while decodes use this plan (kvcu_mla_decode / _layers read it);
 * the next kvcu_decode_plan drops it. */
int kvcu_decode_plan_causal(kvcu_decode_ws* ws, const kvcu_pool* pool, uint32_t n, const uint32_t* seq_ids,
                            uint32_t n_seqs, const uint32_t* lens, const uint32_t* entry_lens, void* stream);
/* Run decode for one layer with the last plan of `ws`.  The batch must be the
 * one planned (the plan's items index seq_ids, q and out): an n other than the
 * plan's returns KVCU_ERR_INVALID_ARG, as does a decode before any plan. */
int kvcu_mla_decode(kvcu_decode_ws* ws, kvcu_pool* pool, uint32_t layer, uint32_t n,
                    const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* table_offsets,
                    const uint32_t* tables, const uint32_t* lens, const float* q,
                    uint32_t n_heads, float scale, float* out, void* stream);
/* kvcu_mla_decode that also writes lse[b][h] = log(sum_p exp(s_p)) of the
 * scaled scores (natural log; -inf for an empty context), so that further
 * positions can be merged into out (kvcu_mla_finish does this for the newest
 * token of a step). */
int kvcu_mla_decode_lse(kvcu_decode_ws* ws, kvcu_pool* pool, uint32_t layer, uint32_t n,
                        const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* table_offsets,
                        const uint32_t* tables, const uint32_t* lens, const float* q,
                        uint32_t n_heads, float scale, float* out, float* lse, void* stream);
/* The MLA decode step around the cache, in absorbed form (src/inference.zig:
 * 492-513 and 518-660).  Step = kvcu_mla_prepare, kvcu_append(rows) at the
 * positions, kvcu_mla_decode_lse over the history (lens = positions), then
 * kvcu_mla_finish.  All pointers are device pointers; weights are row-major as
 * the reference's matVecMul reads them (src/math.zig:79-99).
 * prepare: q [n][H][qk_nope + P] (after q_b_proj), kv_a [n][R + P] (after
 *   kv_a_proj), positions [n], norm_w [R] (kv_a_norm), k_b [H*qk_nope][R] ->
 *   rows [n][R + P] = [RMSNorm(kv_a[0:R]) * norm_w, RoPE(kv_a[R:], pos)]
 *   (src/math.zig:7-35, 197-240) and q_abs [n][H][R + P] =
 *   [k_b_h^T q_nope_h, RoPE(q_rope_h, pos)].
 * finish: merges the newest token (its unquantized latent rows[b][0:R] and its
 *   k_pe as the cache stores it) into the history's out / lse (latent is the
 *   decode's out, updated in place), then attn [n][H][v_dim] = v_b_h latent_h
 *   with v_b [H*v_dim][R]. */
int kvcu_mla_prepare(kvcu_pool* pool, uint32_t n, uint32_t n_heads, uint32_t qk_nope, const float* q,
                     const float* kv_a, const uint32_t* positions, const float* norm_w, float eps,
                     float rope_base, const float* k_b, float* q_abs, float* rows, void* stream);
int kvcu_mla_finish(kvcu_pool* pool, uint32_t n, uint32_t n_heads, uint32_t v_dim, const float* q_abs,
                    const float* rows, float* latent, const float* lse, float scale, const float* v_b,
                    float* attn, void* stream);
/* Several layers in one call, all with the workspace's last plan (the batch and
 * lengths are the same for every layer of a step): layers [layer, layer +
 * n_layers) of the pool, layer+i reading q + i*q_layer_stride and writing
 * out + i*out_layer_stride (strides in floats).  The tensor-core path runs
 * them as ONE persistent launch plus one combine, so the per-launch fill and
 * drain are paid once per step instead of once per layer.  With a one-layer
 * plan (kvcu_decode_plan) every CTA takes its plan range once per layer; with
 * a plan from kvcu_decode_plan_layers for the same n_layers, every CTA takes
 * one range of the list of all (layer, entry) pairs.  It suits work whose
 * layers' queries are all known up front (a benchmark step, re-scoring a
 * cached context, layer-parallel checks); a model's decode, where layer l+1's
 * query depends on layer l's output (src/inference.zig:279-373), calls
 * kvcu_mla_decode per layer.  The workspace must come from
 * kvcu_decode_ws_create_layers with max_layers >= n_layers. */
kvcu_decode_ws* kvcu_decode_ws_create_layers(int device, uint32_t max_batch, uint32_t max_heads,
                                             uint32_t max_layers);
/* The plan for one kvcu_mla_decode_layers call of n_layers layers (no
 * counterpart in the reference, which decodes layer by layer): the n_layers x n
 * (layer, entry) pairs are laid end to end and cut into equal-cost CTA ranges
 * as one list, so the whole launch splits at most (CTAs - 1) of them, where a
 * one-layer plan repeated per layer splits up to (CTAs - 1) in every layer.
 * Fewer split entries mean fewer item set-ups per CTA and fewer outputs left
 * for the combine kernel after the decode (the ones that cross PCIe last when
 * `out` is host memory).  Valid only for kvcu_mla_decode_layers with the same
 * n_layers on the tensor-core path (Q8_0 pool, <= 24 heads); kvcu_mla_decode,
 * and a call with another layer count, return KVCU_ERR_INVALID_ARG until the
 * next one-layer plan.  n_layers = 1 gives the one-layer plan.  Needs
 * max_layers >= n_layers. */
int kvcu_decode_plan_layers(kvcu_decode_ws* ws, const kvcu_pool* pool, uint32_t n, const uint32_t* seq_ids,
                            uint32_t n_seqs, const uint32_t* lens, uint32_t n_layers, void* stream);
int kvcu_mla_decode_layers(kvcu_decode_ws* ws, kvcu_pool* pool, uint32_t layer, uint32_t n_layers, uint32_t n,
                           const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* table_offsets,
                           const uint32_t* tables, const uint32_t* lens, const float* q, uint64_t q_layer_stride,
                           uint32_t n_heads, float scale, float* out, uint64_t out_layer_stride, void* stream);
/* The step's per-head contractions as one call: for head z < heads,
 * C_z[m][n] = sum_k A_z[m][k] * B_z(k, n) with A_z = A + z*a_hs (row stride
 * lda), C_z = C + z*c_hs (ldc), B_z(k, n) = B[z*b_hs + (trans_b ? n*ldb + k :
 * k*ldb + n)], all f32 device arrays.  impl 0: the tcgen05 kernel (3xTF32:
 * hi/lo TF32 parts, three MMAs per K-step, f32 accumulation in TMEM) where the
 * shapes fit it (N % 128 == 0, K % 32 == 0, 16-byte aligned rows), else the
 * CUDA-core f32 kernel; 1: CUDA cores; 2: tensor cores or
 * KVCU_ERR_UNSUPPORTED.  kvcu_mla_prepare / kvcu_mla_finish use impl 0.
 * `pool` gives the device and the status word for a timed-out wait. */
int kvcu_head_gemm(int trans_b, uint32_t heads, uint32_t M, uint32_t N, uint32_t K, const float* A, uint32_t lda,
                   uint64_t a_hs, const float* B, uint32_t ldb, uint64_t b_hs, float* C, uint32_t ldc,
                   uint64_t c_hs, int impl, kvcu_pool* pool, void* stream);
/* Kernel launches the last kvcu_mla_decode issued (for launch accounting). */
uint32_t kvcu_decode_last_launches(const kvcu_decode_ws* ws);
/* Decode kernel selection.  AUTO uses the tcgen05 tensor-core kernel for Q8_0
 * pools with kv_rank 512 / rope_dim 64 / <= 24 heads / block sizes dividing or
 * multiples of 128, and the CUDA-core kernel otherwise (f32 pools, 25..32
 * heads).  Forcing TENSOR_CORE on an unsupported shape returns
 * KVCU_ERR_UNSUPPORTED.  kvcu_decode_last_impl reports the kernel used. */
#define KVCU_DECODE_AUTO 0
#define KVCU_DECODE_CUDA_CORE 1
#define KVCU_DECODE_TENSOR_CORE 2
int kvcu_decode_ws_set_impl(kvcu_decode_ws* ws, int impl);
/* Every wait of the tensor-core decode kernel is bounded: after `cycles` SM
 * clocks (0 = the default, 2^31, about a second at 1.9 GHz) the CTA records
 * KVCU_STATUS_TIMEOUT in the pool's status word, all its roles unwind, its
 * in-flight copies and MMAs are waited for (with the same bound) and its TMEM
 * is released, so the context stays usable and the host reads the error.  At
 * most 2^40. */
int kvcu_decode_ws_set_wait_limit(kvcu_decode_ws* ws, uint64_t cycles);
/* Test hook for that unwind, needing no GPU fault: in the tensor-core kernel,
 * every CTA's producer skips the copy and the arrival of the first slice of
 * its tile number `tile` (0-based, counted over the CTA's whole range), so the
 * waits on that tile run out.  0xFFFFFFFF turns it off (the default). */
int kvcu_decode_ws_test_withhold(kvcu_decode_ws* ws, uint32_t tile);
int kvcu_decode_last_impl(const kvcu_decode_ws* ws);

/* Decode without any allocation.  No counterpart in the reference: this is an
 * extra entry point of this library for callers that must not allocate device
 * memory at decode time -- a runtime that reserves all of its memory up front
 * (an allocator that owns the whole device, a hard memory budget), code running
 * where an allocation would stall or fail (a latency-critical serving loop),
 * or embedders with no workspace lifetime to manage.  It plans and decodes one
 * layer in a single call, with the same semantics and kernels as
 * kvcu_decode_plan + kvcu_mla_decode, but keeps the split-KV scratch (work
 * items, per-item partial outputs) in a fixed array compiled into the library
 * (KVCU_NOALLOC_SCRATCH_BYTES of device memory per device) instead of a
 * kvcu_decode_ws.  The array is reserved on a device by kvcu_init(device),
 * which kvcu_pool_create also calls, so a runtime that reserves the rest of
 * the device afterwards loses nothing at its first no-alloc decode.
 *   Limits: n <= KVCU_NOALLOC_MAX_BATCH, 1 <= n_heads <= KVCU_NOALLOC_MAX_HEADS;
 *   larger requests return KVCU_ERR_INVALID_ARG and change nothing.  Long
 *   sequences are split into at most KVCU_NOALLOC_MAX_ITEMS work items in all.
 *   The array's device address is looked up once per device, with that
 *   device current, by kvcu_init (or by the first call on a device that
 *   kvcu_init never saw); make that first call before capturing `stream`
 *   into a graph.  The scratch is one per device and is not guarded: calls that may
 *   overlap on the same device (other streams, other host threads) race on it
 *   and must be serialised by the caller. */
#define KVCU_NOALLOC_MAX_BATCH 64u
#define KVCU_NOALLOC_MAX_HEADS 32u
#define KVCU_NOALLOC_MAX_ITEMS 256u
#define KVCU_NOALLOC_SCRATCH_BYTES \
  (KVCU_NOALLOC_MAX_ITEMS * KVCU_NOALLOC_MAX_HEADS * (512u + 2u) * 4u + KVCU_NOALLOC_MAX_ITEMS * 16u + \
   16u + (KVCU_NOALLOC_MAX_ITEMS + 1u) * 4u + 2u * KVCU_NOALLOC_MAX_BATCH * 4u)
int kvcu_mla_decode_noalloc(kvcu_pool* pool, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                            uint32_t n_seqs, const uint32_t* table_offsets, const uint32_t* tables,
                            const uint32_t* lens, const float* q, uint32_t n_heads, float scale,
                            float* out, void* stream);

/* ------------------------------------------------------------ checkpoint I/O
 * Bytes of the pool section of a v1 checkpoint in the reference's order
 * (src/kv_cache.zig:484-492): Q8_0 -> all [rows][ceil(kv_rank/32)] 34-byte
 * blocks, then all [rows][ceil(rope_dim/32)]; f32 -> kv pool then pe pool.
 * Copy out / in the byte range [offset, offset+nbytes) of that section through
 * a host buffer (synchronous on `stream`). */
int kvcu_pool_read_checkpoint(kvcu_pool* pool, uint64_t offset, uint64_t nbytes, void* host_dst,
                              void* stream);
int kvcu_pool_write_checkpoint(kvcu_pool* pool, uint64_t offset, uint64_t nbytes,
                               const void* host_src, void* stream);

/* ------------------------------------------------------------ synthetic inputs
 * Seeded counter-based N(0,1) generator used by the benchmarks and tests:
 * out[r*width + i] = normal(seed, a, b[r], c[r]*1024 + i), with probability
 * outlier_p multiplied by 20.  b, c, out are device pointers. */
int kvcu_synth_rows(uint64_t seed, uint64_t a, uint32_t n_rows, const uint32_t* b,
                    const uint32_t* c, uint32_t width, float outlier_p, float* out, void* stream);

/* =============================================================== kvcache_*
 * Host mirror of src/kv_cache.zig's KVCache over one kvcu_pool, extended to
 * many sequences sharing the pool (sequence 0 is the reference's single
 * sequence).  Block allocator, refcounts, free list, block tables and the
 * prefix-cache hash map live on the host exactly as in the reference; data
 * lives on the device.  Buffers are HOST pointers unless a name ends in _dev.
 */
typedef struct kvcache kvcache;

/* KVCache.init (src/kv_cache.zig:64-122): num_blocks = ceil(max_seq_len/BS). */
kvcache* kvcache_init(int device, uint32_t n_layers, uint32_t kv_rank, uint32_t rope_dim,
                      uint32_t max_seq_len, uint32_t block_size);
/* Same with an explicit block count (a pool shared by many sequences). */
kvcache* kvcache_init_blocks(int device, uint32_t n_layers, uint32_t kv_rank, uint32_t rope_dim,
                             uint32_t num_blocks, uint32_t block_size, int quantized);
void kvcache_deinit(kvcache* c);                               /* :124-139 */
int kvcache_enable_quantization(kvcache* c);                   /* :142-154 */
int kvcache_ensure_capacity(kvcache* c, uint32_t n_tokens);    /* :188-194 */
void kvcache_truncate(kvcache* c, uint32_t n_tokens);          /* :197-206 */
void kvcache_reset(kvcache* c);                                /* :209-215 */
int kvcache_put(kvcache* c, uint32_t layer, uint32_t pos, const float* kv_comp,
                const float* k_pe);                            /* :279-361 */
int kvcache_get_kv_compressed(kvcache* c, uint32_t layer, uint32_t pos, float* out); /* :225-250 */
int kvcache_get_kpe(kvcache* c, uint32_t layer, uint32_t pos, float* out);           /* :252-277 */
uint32_t kvcache_len(const kvcache* c);
uint32_t kvcache_num_blocks(const kvcache* c);
uint32_t kvcache_block_size(const kvcache* c);
int kvcache_quantized(const kvcache* c);
uint32_t kvcache_num_free_blocks(const kvcache* c);            /* :446-448 */
uint64_t kvcache_memory_usage(const kvcache* c);               /* :439-443 */
uint32_t kvcache_block_table(const kvcache* c, uint32_t* out, uint32_t cap);
uint32_t kvcache_refcount(const kvcache* c, uint32_t block_id);
/* Overwrite the free list (LIFO: the last id is handed out first), e.g. to
 * shuffle the allocation order. */
int kvcache_set_free_list(kvcache* c, const uint32_t* ids, uint32_t n);
kvcu_pool* kvcache_pool(kvcache* c);
int kvcache_save_to_file(kvcache* c, const char* path);       /* :453-494 */
int kvcache_load_from_file(kvcache* c, const char* path);     /* :497-546 */
/* Prefix caching (src/kv_cache.zig:367-436, hash :596-609). */
void kvcache_cache_block(kvcache* c, uint32_t block_idx, const uint32_t* token_ids,
                         uint32_t n_tokens, uint64_t prefix_hash);
uint32_t kvcache_find_prefix_blocks(kvcache* c, const uint32_t* tokens, uint32_t n);
int kvcache_reuse_prefix_blocks(kvcache* c, const uint32_t* tokens, uint32_t n, uint32_t n_blocks);
uint64_t kvcache_compute_hash(const uint32_t* token_ids, uint32_t n, uint64_t prefix_hash);
/* The same for any sequence of the pool, so that sequences share cached prefix
 * blocks on the device (the hash map, and so kvcache_find_prefix_blocks, is
 * pool-wide).  reuse makes `seq`'s first n_blocks blocks the cached ones
 * (retained) and sets its len to n_blocks * block_size.  A shared block is never
 * written: every write path (put, append_batch(_dev), the MLA step) first copies
 * a block held by more than one owner to a fresh block for the writing sequence
 * (copy-on-write). */
int kvcache_seq_cache_block(kvcache* c, uint32_t seq, uint32_t block_idx, const uint32_t* token_ids,
                            uint32_t n_tokens, uint64_t prefix_hash);
int kvcache_seq_reuse_prefix_blocks(kvcache* c, uint32_t seq, const uint32_t* tokens, uint32_t n,
                                    uint32_t n_blocks);

/* ---- many sequences on one pool (sequence 0 always exists) ---- */
/* New empty sequence; returns its id or a negative error. */
int64_t kvcache_seq_create(kvcache* c);
uint32_t kvcache_num_seqs(const kvcache* c);
int kvcache_seq_ensure_capacity(kvcache* c, uint32_t seq, uint32_t n_tokens);
int kvcache_seq_truncate(kvcache* c, uint32_t seq, uint32_t n_tokens);
int kvcache_seq_reset(kvcache* c, uint32_t seq);
uint32_t kvcache_seq_len(const kvcache* c, uint32_t seq);
uint32_t kvcache_seq_block_table(const kvcache* c, uint32_t seq, uint32_t* out, uint32_t cap);
/* appendBatch: rows[r] = latent ++ rope ([n][kv_rank+rope_dim] f32) for
 * (seq_ids[r], positions[r]); the positions must lie inside each sequence's
 * capacity.  Sets len = max(len, pos+1).  `rows` is a HOST pointer; the
 * _dev variant takes device pointers for rows, seq_ids and positions (the
 * host copies of seq_ids/positions are still needed for the length update).
 * The _dev calls are stream-ordered: changed block tables and lengths are
 * uploaded on `stream` from pinned staging, and a later call on another
 * stream is ordered after that upload; the host does not wait. */
int kvcache_append_batch(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                         const uint32_t* positions, const float* rows);
int kvcache_append_batch_dev(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                             const uint32_t* positions, const uint32_t* seq_ids_dev,
                             const uint32_t* positions_dev, const float* rows_dev, void* stream);
/* Several layers per call, for work whose layers' rows and queries are all
 * known up front (see kvcu_mla_decode_layers; a model's decode goes layer by
 * layer).  Layer layer+i reads rows + i*rows_layer_stride (device, floats) and
 * the same seq_ids / positions; the decode uses q + i*q_layer_stride and
 * writes out + i*out_layer_stride, one multi-layer launch. */
int kvcache_append_layers_dev(kvcache* c, uint32_t layer, uint32_t n_layers, uint32_t n, const uint32_t* seq_ids,
                              const uint32_t* positions, const uint32_t* seq_ids_dev, const uint32_t* positions_dev,
                              const float* rows_dev, uint64_t rows_layer_stride, void* stream);
int kvcache_mla_decode_layers_dev(kvcache* c, uint32_t layer, uint32_t n_layers, uint32_t n,
                                  const uint32_t* seq_ids, const float* q_dev, uint64_t q_layer_stride,
                                  uint32_t n_heads, float scale, float* out_dev, uint64_t out_layer_stride,
                                  void* stream);
/* appendBatch + mlaDecode for layers [layer, layer + n_layers) in one call with
 * HOST buffers and one synchronise: rows [n_layers][n][kv_rank+rope_dim] are
 * appended at (seq_ids[b], positions[b]) in every layer, then each layer is
 * decoded, q [n_layers][n][n_heads][kv_rank+rope_dim] -> out
 * [n_layers][n][n_heads][kv_rank].  Pinned, mapped q / out are used in place
 * (as kvcache_mla_decode does). */
int kvcache_append_decode_layers(kvcache* c, uint32_t layer, uint32_t n_layers, uint32_t n, const uint32_t* seq_ids,
                                 const uint32_t* positions, const float* rows, const float* q, uint32_t n_heads,
                                 float scale, float* out);
/* gather(layer, seq): out[len][kv_rank + rope_dim] (HOST buffer). */
int kvcache_gather(kvcache* c, uint32_t layer, uint32_t seq, float* out);
/* mlaDecode (the call replacing src/inference.zig:518-660): HOST q
 * [n][n_heads][R+P] and out [n][n_heads][R]; returns when out is complete.
 * Pageable buffers are copied in and out around the kernels.  When both are
 * pinned and mapped (cudaHostAlloc / cudaHostRegister) and their allocations
 * hold the whole arrays, the kernels read q and write out in host memory
 * directly, so the transfers overlap the decode instead of preceding and
 * following it. */
int kvcache_mla_decode(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                       const float* q, uint32_t n_heads, float scale, float* out);
/* mlaAttentionBatch (src/inference.zig:670-883, its attention loop :771-877):
 * the n_pos prompt positions start_pos .. start_pos+n_pos-1 of sequence `seq`
 * (already appended, so len >= start_pos + n_pos, else
 * KVCU_ERR_POSITION_NOT_WRITTEN) attend causally: query i sees positions
 * [0, start_pos + i].  q [n_pos][n_heads][R+P] -> out [n_pos][n_heads][R], HOST
 * buffers (used in place when pinned and mapped); the _dev variant takes
 * device pointers and is stream-ordered.  One causal plan + one decode. */
int kvcache_mla_attention_batch(kvcache* c, uint32_t layer, uint32_t seq, uint32_t start_pos, uint32_t n_pos,
                                const float* q, uint32_t n_heads, float scale, float* out);
int kvcache_mla_attention_batch_dev(kvcache* c, uint32_t layer, uint32_t seq, uint32_t start_pos, uint32_t n_pos,
                                    const float* q_dev, uint32_t n_heads, float scale, float* out_dev,
                                    void* stream);
/* 1 when the last kvcache_mla_decode used its buffers in place (pinned,
 * mapped), 0 when it copied. */
int kvcache_last_decode_mapped(const kvcache* c);
/* How the host-buffer decode calls move q and out: KVCACHE_HOST_IO_AUTO (the
 * default) reads q and writes out in place over PCIe from the kernels when the
 * buffers are pinned and mapped, else copies; KVCACHE_HOST_IO_COPY always
 * copies them by DMA before and after the kernels; KVCACHE_HOST_IO_COPY_IN
 * makes kvcache_append_decode_layers copy q by DMA and let the kernels write
 * out in place (the other host-buffer calls copy both ways in this mode).  When many GPUs share the host's PCIe and memory, large DMA
 * transfers can move the bytes faster than the kernels' own reads. */
#define KVCACHE_HOST_IO_AUTO 0
#define KVCACHE_HOST_IO_COPY 1
#define KVCACHE_HOST_IO_COPY_IN 2
int kvcache_set_host_io(kvcache* c, int mode);
/* One MLA decode step of layer `layer` for a batch of sequences (the batched
 * form of src/inference.zig:492-660): each entry b appends its new token at
 * positions[b] (host array; each sequence at most once) and attends over
 * positions <= positions[b].  Device inputs as for kvcu_mla_prepare /
 * kvcu_mla_finish (q [n][H][qk_nope + rope_dim], kv_a [n][kv_rank + rope_dim],
 * norm_w [kv_rank], k_b [H*qk_nope][kv_rank], v_b [H*v_dim][kv_rank]); output
 * attn [n][H][v_dim] (before o_proj).  scale = 1/sqrt(qk_nope + rope_dim) as
 * in the reference.  Stream-ordered; the call returns before the kernels end. */
int kvcache_mla_step_dev(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                         const uint32_t* positions, const float* q_dev, const float* kv_a_dev,
                         const float* norm_w_dev, float eps, float rope_base, const float* k_b_dev,
                         const float* v_b_dev, uint32_t n_heads, uint32_t qk_nope, uint32_t v_dim,
                         float scale, float* attn_dev, void* stream);
/* Device variant: q/out device pointers, no host copies; plans once per step
 * (a plan is reused until a sequence length or the batch changes). */
int kvcache_mla_decode_dev(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                           const float* q_dev, uint32_t n_heads, float scale, float* out_dev,
                           void* stream);
/* Launches issued by the last kvcache_* data call (for launch accounting). */
uint32_t kvcache_last_launches(const kvcache* c);
/* Decode kernel selection for this cache (KVCU_DECODE_*), and the kernel the
 * last decode used. */
int kvcache_set_decode_impl(kvcache* c, int impl);
int kvcache_last_decode_impl(const kvcache* c);
/* Multi-sequence checkpoint (v2: header, per-sequence lengths and tables,
 * pool).  Single-sequence caches use kvcache_save_to_file (v1, byte-exact). */
int kvcache_save_to_file_v2(kvcache* c, const char* path);
int kvcache_load_from_file_v2(kvcache* c, const char* path);
/* The v2 save in the background, overlapped with serving (the asynchronous
 * checkpoint I/O around src/kv_cache.zig:453-591).  The call captures the
 * header, every sequence's length and block table, and retains each block of
 * those tables once more, so none returns to the free list and any later write
 * into one first copies it (copy-on-write): the file holds the cache exactly
 * as it was when the work queued on `stream` (may be NULL) and on the cache's
 * own stream had run.  A worker thread then copies the pool section device ->
 * pinned host -> file on its own CUDA stream while the caller keeps appending
 * and decoding.  kvcache_save_wait joins it, drops the snapshot's references
 * and returns its status; kvcache_save_done polls.  One save per cache at a
 * time; loadFromFile and enableQuantization are refused while it runs, and
 * kvcache_deinit waits for it. */
typedef struct kvcache_save kvcache_save;
int kvcache_save_to_file_v2_async(kvcache* c, const char* path, void* stream, kvcache_save** job);
int kvcache_save_done(const kvcache_save* job);
int kvcache_save_wait(kvcache_save* job);

/* ---- continuous batching over one pool (BatchScheduler, src/batch_queue.zig:75-232) ----
 * Each request is a sequence of the kvcache (instead of owning a KVCache,
 * src/batch_queue.zig:33-52); ids start at 1.  collect returns up to
 * max_batch_size requests that are running or waiting and not finished
 * (completed, max_tokens generated, or last token == eos), highest priority
 * first, then in arrival order, with their pool sequences.  reap_completed
 * drops completed requests and resets their sequences (blocks back to the
 * pool); the sequences are reused by later requests.  reclaim_blocks resets
 * the sequences of paused and completed requests and returns the blocks freed.
 * Host-only; not thread-safe (one scheduler per host thread, as in the
 * reference). */
#define KVCU_SEQ_WAITING 0
#define KVCU_SEQ_RUNNING 1
#define KVCU_SEQ_PAUSED 2
#define KVCU_SEQ_COMPLETED 3
#define KVCU_PRIORITY_LOW 0
#define KVCU_PRIORITY_NORMAL 1
#define KVCU_PRIORITY_HIGH 2
#define KVCU_PRIORITY_CRITICAL 3
typedef struct kvcu_batch kvcu_batch;
kvcu_batch* kvcu_batch_create(kvcache* c, uint32_t max_batch_size);
int kvcu_batch_destroy(kvcu_batch* b);
/* addRequest / addRequestWithPriority: the new id, or a negative error. */
int64_t kvcu_batch_add_request(kvcu_batch* b, uint32_t max_tokens, int priority);
/* collectBatchIndices: writes ids and pool sequences; returns how many. */
uint32_t kvcu_batch_collect(kvcu_batch* b, uint32_t eos_token, uint64_t* ids_out, uint32_t* seqs_out,
                            uint32_t cap);
int kvcu_batch_mark_running(kvcu_batch* b, const uint64_t* ids, uint32_t n);
int kvcu_batch_mark_completed(kvcu_batch* b, uint64_t id);
int kvcu_batch_set_status(kvcu_batch* b, uint64_t id, int status);
int kvcu_batch_status(const kvcu_batch* b, uint64_t id);
/* Record a generated token (Sequence.tokens); is_finished returns 1 / 0. */
int kvcu_batch_push_token(kvcu_batch* b, uint64_t id, uint32_t token);
int kvcu_batch_is_finished(kvcu_batch* b, uint64_t id, uint32_t eos_token);
uint32_t kvcu_batch_reap_completed(kvcu_batch* b);
uint32_t kvcu_batch_reclaim_blocks(kvcu_batch* b);
uint32_t kvcu_batch_running_count(const kvcu_batch* b);
uint32_t kvcu_batch_size(const kvcu_batch* b);
/* The request's pool sequence, or a negative error. */
int64_t kvcu_batch_seq(const kvcu_batch* b, uint64_t id);

#ifdef __cplusplus
}
#endif
#endif /* KVCUDA_H */
