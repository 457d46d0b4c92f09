// kvcu_internal.h — internal structures shared by the libkvcuda translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/kvcuda.h"

struct kvcu_pool {
  int device;
  uint32_t n_layers, num_blocks, block_size, kv_rank, rope_dim;
  uint32_t quantized;
  uint32_t nbk, nbp, nblk;   // Q8_0 blocks: latent, rope, total per row
  float* kv;                 // f32 [L][NB][BS][kv_rank]
  float* pe;                 // f32 [L][NB][BS][rope_dim]
  int8_t* qs;                // int8 [L][NB][BS][nblk*32]
  uint16_t* sc;              // f16 bits [L][NB][BS][nblk]
  uint32_t* status;          // device status word (KVCU_STATUS_* bits)
  uint32_t* status_host;     // pinned host word its reads land in (one synchronise per read)
  uint8_t* staging;          // device staging for checkpoint repacking
  uint64_t staging_bytes;
  uint64_t rows() const { return (uint64_t)n_layers * num_blocks * block_size; }
};

// Split-KV work item: batch entry b, tokens [start, end), of layer offset
// `layer` (always 0 in a one-layer plan; in a layered plan, the offset from the
// decode call's first layer).
struct kvcu_item {
  uint32_t b, start, end, layer;
};

struct kvcu_decode_ws {
  int device;
  uint32_t max_batch, max_heads, max_items, max_ranges;
  uint32_t max_layers;       // layers one multi-layer decode may cover (partials per layer)
  kvcu_item* items;          // [max_layers * max_items]
  uint32_t* meta;            // [0] n_items, [1] CTA ranges G
  uint32_t* ranges;          // [max_ranges + 1] first item of each CTA range
  uint32_t* seq_first;       // [max_layers * max_batch] first item of plan entry e
  uint32_t* seq_count;       // [max_layers * max_batch] items of plan entry e
  float* part_o;             // [max_layers][max_items][max_heads][512]
  float* part_ml;            // [max_layers][max_items][max_heads][2] (m, l)
  // Layers the last plan balances as one list (plan entry e = layer * n + b,
  // n the batch): 1 for a one-layer plan, which a multi-layer decode repeats
  // for every layer; L > 1 for kvcu_decode_plan_layers, valid only for a
  // multi-layer decode of exactly L layers.
  uint32_t plan_layers;
  // Entries per layer of the last plan: a decode must cover the same batch,
  // since the plan's items index its seq_ids, q and out (~0 after a failed plan).
  uint32_t plan_n;
  const uint32_t* entry_lens;  // per-entry lengths of the last plan (device; nullptr: whole sequences)
  uint64_t wait_limit;         // clocks a bounded device wait may take (0: the default, ~2^31)
  uint32_t withhold_plus1;     // test hook: 0, or 1 + the tile whose first slice the producer withholds
  uint32_t last_launches;
  int num_sms;
  int decode_ctas;           // resident decode CTAs (grid of the persistent kernel)
  int impl;                  // KVCU_DECODE_AUTO / _CUDA_CORE / _TENSOR_CORE
  int last_impl;             // the kernel the last decode used
};

// ---- programmatic dependent launch ----
// A kernel launched with kvcu_launch_pdl may start while its predecessor in the
// stream is still finishing (once every predecessor CTA has triggered or
// exited); it runs its independent prologue, then kvcu_pdl_wait() before it
// touches anything earlier work wrote.  Both device calls are no-ops for an
// ordinary launch.
#ifdef __CUDACC__
__device__ __forceinline__ void kvcu_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void kvcu_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t kvcu_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}
#endif

// ---- error plumbing (kvcu_api.cu) ----
void kvcu_set_error(const char* fmt, ...);
int kvcu_check_cuda(cudaError_t e, const char* what);
// One-time set-up of a kernel (function attributes such as its dynamic shared
// memory limit) for the CURRENT device: `setup(ctx)` runs the first time the
// pair (key, device) is seen, under a process-wide lock, and is recorded only
// when it returns KVCU_OK.  Function attributes are per device, so a process
// that drives several GPUs configures each one; host threads may race here.
int kvcu_configure_once(const void* key, int (*setup)(const void* ctx), const void* ctx);
// Multiprocessor count of the current device (cached per device).
int kvcu_current_sm_count();
#define KVCU_CUDA(call) \
  do { \
    int _rc = kvcu_check_cuda((call), #call); \
    if (_rc) return _rc; \
  } while (0)

// ---- kernel launchers (kvcu_kernels.cu) ----
int kvcu_launch_append(kvcu_pool* p, uint32_t layer, uint32_t n_rows, const float* latent,
                       uint64_t ls, const float* rope, uint64_t ps, const uint32_t* row_seq,
                       const uint32_t* row_pos, uint32_t n_seqs, const uint32_t* table_offsets,
                       const uint32_t* tables, uint32_t* lens, cudaStream_t st);
// Layers [layer, layer + n_layers_call): rows of layer layer+i at latent +
// i*llat and rope + i*lrope (floats); one launch on the fast path.
int kvcu_launch_append_layers(kvcu_pool* p, uint32_t layer, uint32_t n_layers_call, uint32_t n_rows,
                              const float* latent, uint64_t ls, uint64_t llat, const float* rope, uint64_t ps,
                              uint64_t lrope, const uint32_t* row_seq, const uint32_t* row_pos, uint32_t n_seqs,
                              const uint32_t* toff, const uint32_t* tables, uint32_t* lens, cudaStream_t st);
int kvcu_launch_gather_rows(kvcu_pool* p, uint32_t layer, uint32_t n_rows, const uint32_t* row_seq,
                            const uint32_t* row_pos, uint32_t n_seqs, const uint32_t* table_offsets,
                            const uint32_t* tables, const uint32_t* table, uint32_t table_len,
                            float* out, cudaStream_t st);
int kvcu_launch_pack_q8(kvcu_pool* p, int part, uint64_t blk0, uint64_t nblocks, uint8_t* dst,
                        cudaStream_t st);
int kvcu_launch_unpack_q8(kvcu_pool* p, int part, uint64_t blk0, uint64_t nblocks,
                          const uint8_t* src, cudaStream_t st);
int kvcu_launch_synth(uint64_t seed, uint64_t a, uint32_t n_rows, const uint32_t* b,
                      const uint32_t* c, uint32_t width, float outlier_p, float* out,
                      cudaStream_t st);

// ---- decode (kvcu_decode.cu) ----
int kvcu_decode_setup(kvcu_decode_ws* ws);
// entry_lens (nullable, device): entry b attends min(entry_lens[b], lens[seq])
// positions; recorded in the workspace for the decodes that use the plan.
int kvcu_launch_plan(kvcu_decode_ws* ws, const kvcu_pool* p, uint32_t n, const uint32_t* seq_ids,
                     uint32_t n_seqs, const uint32_t* lens, cudaStream_t st, const uint32_t* entry_lens = nullptr);
int kvcu_launch_plan_target(kvcu_decode_ws* ws, const kvcu_pool* p, uint32_t n,
                            const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* lens,
                            uint32_t target, cudaStream_t st, const uint32_t* entry_lens = nullptr,
                            uint32_t n_layers = 1);
// Whether a multi-layer decode of this batch runs as one tensor-core launch,
// the only form a layered plan (n_layers > 1) serves.
bool kvcu_decode_layers_fused(const kvcu_decode_ws* ws, const kvcu_pool* p, uint32_t n, uint32_t n_heads);
// ---- checkpoint bytes through a caller-owned device staging buffer (kvcu_api.cu) ----
int kvcu_pool_read_checkpoint_staged(kvcu_pool* p, uint64_t offset, uint64_t nbytes, void* host_dst,
                                     cudaStream_t st, uint8_t* staging, uint64_t staging_bytes);
// ---- per-head GEMM on the tensor cores, 3xTF32 (kvcu_gemm_tc.cu) ----
// KVCU_ERR_UNSUPPORTED (nothing launched) unless N % 128 == 0, K % 32 == 0 and
// every row and pointer is 16-byte aligned.
// With `mrg`, the A operand of head z is the log-sum-exp merge of the MLA
// step's newest token into the history output, formed while A is loaded:
// A'[m][k] = (A[m][k] * wh + rows[m * ldr + k] * wc) * inv, (wh, wc, inv) =
// w[(m * heads + z) * 3 ..]; the history term is dropped (not multiplied)
// where wh == 0, so a NaN there does not reach the product.
struct kvcu_gemm_merge {
  const float* rows;
  uint32_t ldr;
  const float* w;
};
int kvcu_launch_head_gemm_tc(bool trans_b, uint32_t heads, uint32_t M, uint32_t N, uint32_t K, const float* A,
                             uint32_t lda, uint64_t a_hs, const float* B, uint32_t ldb, uint64_t b_hs, float* C,
                             uint32_t ldc, uint64_t c_hs, uint32_t* status, cudaStream_t st,
                             const kvcu_gemm_merge* mrg = nullptr);
// kvcu_mla_finish with scratch w [n][n_heads][3] for the merge weights, so the
// v_b GEMM merges while it loads (kvcu_mla.cu); stream-ordered on st.
int kvcu_mla_finish_fused(kvcu_pool* pool, uint32_t n, uint32_t n_heads, uint32_t v_dim, const float* q_abs,
                          const float* rows, float* latent, const float* lse, float* w, float scale,
                          const float* v_b, float* attn, cudaStream_t st);
// ---- allocation-free decode (kvcu_noalloc.cu) ----
// Resolve (and so reserve) the fixed decode scratch on `device`, which must be
// current; kvcu_init calls it.
int kvcu_noalloc_prepare(int device);
// ---- tensor-core decode (kvcu_decode_tc.cu) ----
bool kvcu_decode_tc_supported(const kvcu_pool* p, uint32_t n_heads);
// Layers [layer, layer + n_layers_call) with one plan: q / out / lse of layer
// layer+i at + i * its stride (floats).  With a one-layer plan the partials of
// layer i sit at item index i * ws->max_items + item (ws->max_layers >=
// n_layers_call); a layered plan of n_layers_call layers numbers its items
// across all layers, and each item's partials sit at its own index.
int kvcu_launch_decode_tc(kvcu_decode_ws* ws, kvcu_pool* p, uint32_t layer, uint32_t n_layers_call, uint32_t n,
                          const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* toff,
                          const uint32_t* tables, const uint32_t* lens, const float* q, uint64_t q_lstride,
                          uint32_t n_heads, float scale, float* out, uint64_t out_lstride, float* lse,
                          uint64_t lse_lstride, cudaStream_t st);
// `lse` (nullable): [n][n_heads] log-sum-exp of the scaled scores, natural log
// (-inf for an empty context), for merging further terms into `out`.
int kvcu_launch_decode(kvcu_decode_ws* ws, kvcu_pool* p, uint32_t layer, uint32_t n,
                       const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* table_offsets,
                       const uint32_t* tables, const uint32_t* lens, const float* q,
                       uint32_t n_heads, float scale, float* out, float* lse, cudaStream_t st);
// Several layers with one plan (strides in floats between consecutive layers'
// q, out and lse); one decode launch and one combine launch on the tensor-core
// path, a launch pair per layer on the CUDA-core path (one-layer plans only).
int kvcu_launch_decode_layers(kvcu_decode_ws* ws, kvcu_pool* p, uint32_t layer, uint32_t n_layers_call,
                              uint32_t n, const uint32_t* seq_ids, uint32_t n_seqs,
                              const uint32_t* table_offsets, const uint32_t* tables, const uint32_t* lens,
                              const float* q, uint64_t q_lstride, uint32_t n_heads, float scale, float* out,
                              uint64_t out_lstride, float* lse, uint64_t lse_lstride, cudaStream_t st);
