// kvcu_api.cu — the kvcu_* C-ABI (include/kvcuda.h): device selection, pool
// lifetime, the append / gather / decode entry points and checkpoint
// repacking.  Modelled on src/metal_bridge.c: a last-error string, integer
// return codes, opaque handles with explicit release.  There is no CPU path:
// every entry point either runs CUDA work or returns an error.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <new>
#include <set>
#include <utility>

#include "kvcu_internal.h"

#define KVCU_VERSION 0x00010000u

static thread_local char g_last_error[512] = {0};

void kvcu_set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int kvcu_check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return KVCU_OK;
  kvcu_set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  if (e == cudaErrorMemoryAllocation) return KVCU_ERR_NO_MEMORY;
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return KVCU_ERR_NO_DEVICE;
  return KVCU_ERR_CUDA;
}

namespace {
std::mutex g_config_mutex;
std::set<std::pair<const void*, int>> g_configured;  // (kernel key, device) pairs set up
std::mutex g_sm_mutex;
std::map<int, int> g_sm_count;
}  // namespace

int kvcu_configure_once(const void* key, int (*setup)(const void* ctx), const void* ctx) {
  int dev = 0;
  KVCU_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_config_mutex);
  if (g_configured.count({key, dev})) return KVCU_OK;
  const int rc = setup(ctx);
  if (rc == KVCU_OK) g_configured.insert({key, dev});
  return rc;
}

int kvcu_current_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(g_sm_mutex);
  auto it = g_sm_count.find(dev);
  if (it != g_sm_count.end()) return it->second;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  g_sm_count[dev] = sms;
  return sms;
}

namespace {

// Make `device` current for the duration of a call, restoring the caller's.
struct DeviceGuard {
  int prev = -1;
  int rc = KVCU_OK;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) rc = kvcu_check_cuda(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

bool valid_pool(const kvcu_pool* p) { return p != nullptr && (p->kv || p->qs); }

uint64_t checkpoint_bytes(const kvcu_pool* p) {
  if (p->quantized) return p->rows() * (uint64_t)(p->nbk + p->nbp) * 34u;
  return p->rows() * (uint64_t)(p->kv_rank + p->rope_dim) * 4u;
}

constexpr uint64_t kStagingBytes = 64ull << 20;

}  // namespace

extern "C" {

const char* kvcu_get_last_error(void) { return g_last_error; }

uint32_t kvcu_version(void) { return KVCU_VERSION; }

int kvcu_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int kvcu_init(int device) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    kvcu_set_error("kvcu_init: no CUDA device (%s)", cudaGetErrorString(e));
    return KVCU_ERR_NO_DEVICE;
  }
  if (device < 0 || device >= n) {
    kvcu_set_error("kvcu_init: device %d out of range [0, %d)", device, n);
    return KVCU_ERR_INVALID_ARG;
  }
  cudaDeviceProp prop;
  KVCU_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) {
    kvcu_set_error("kvcu_init: device %d is sm_%d%d; this library is built for sm_100a (B200)",
                   device, prop.major, prop.minor);
    return KVCU_ERR_UNSUPPORTED;
  }
  DeviceGuard g(device);
  if (g.rc) return g.rc;
  KVCU_CUDA(cudaFree(nullptr));  // create the primary context
  // reserve the allocation-free decode's fixed scratch now, not at its first call
  return kvcu_noalloc_prepare(device);
}

kvcu_pool* kvcu_pool_create(int device, uint32_t n_layers, uint32_t num_blocks,
                            uint32_t block_size, uint32_t kv_rank, uint32_t rope_dim,
                            int quantized) {
  if (!n_layers || !num_blocks || !kv_rank || !rope_dim || block_size == 0 || block_size % 16 ||
      block_size > 1024) {
    kvcu_set_error("kvcu_pool_create: bad shape L=%u NB=%u BS=%u R=%u P=%u (BS must be a "
                   "multiple of 16, <= 1024)",
                   n_layers, num_blocks, block_size, kv_rank, rope_dim);
    return nullptr;
  }
  if (kvcu_init(device) != KVCU_OK) return nullptr;
  DeviceGuard g(device);
  if (g.rc) return nullptr;
  kvcu_pool* p = new (std::nothrow) kvcu_pool();
  if (!p) return nullptr;
  memset(p, 0, sizeof(*p));
  p->device = device;
  p->n_layers = n_layers;
  p->num_blocks = num_blocks;
  p->block_size = block_size;
  p->kv_rank = kv_rank;
  p->rope_dim = rope_dim;
  p->quantized = quantized ? 1u : 0u;
  p->nbk = (kv_rank + 31) / 32;
  p->nbp = (rope_dim + 31) / 32;
  p->nblk = p->nbk + p->nbp;
  const uint64_t rows = p->rows();
  int rc = KVCU_OK;
  if (p->quantized) {
    rc = kvcu_check_cuda(cudaMalloc(&p->qs, rows * 32ull * p->nblk), "cudaMalloc(qs)");
    if (!rc) rc = kvcu_check_cuda(cudaMalloc(&p->sc, rows * 2ull * p->nblk), "cudaMalloc(sc)");
  } else {
    rc = kvcu_check_cuda(cudaMalloc(&p->kv, rows * 4ull * kv_rank), "cudaMalloc(kv)");
    if (!rc) rc = kvcu_check_cuda(cudaMalloc(&p->pe, rows * 4ull * rope_dim), "cudaMalloc(pe)");
  }
  if (!rc) rc = kvcu_check_cuda(cudaMalloc(&p->status, sizeof(uint32_t)), "cudaMalloc(status)");
  if (!rc)
    rc = kvcu_check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&p->status_host), 64, cudaHostAllocDefault),
                         "cudaHostAlloc(status)");
  if (!rc) rc = kvcu_pool_zero(p, nullptr);
  if (!rc) rc = kvcu_check_cuda(cudaDeviceSynchronize(), "pool zeroing");
  if (rc) {
    kvcu_pool_destroy(p);
    return nullptr;
  }
  return p;
}

int kvcu_pool_destroy(kvcu_pool* p) {
  if (!p) return KVCU_OK;
  DeviceGuard g(p->device);
  cudaFree(p->kv);
  cudaFree(p->pe);
  cudaFree(p->qs);
  cudaFree(p->sc);
  cudaFree(p->status);
  if (p->status_host) cudaFreeHost(p->status_host);
  cudaFree(p->staging);
  delete p;
  return KVCU_OK;
}

int kvcu_pool_describe(const kvcu_pool* p, kvcu_pool_desc* out) {
  if (!valid_pool(p) || !out) return KVCU_ERR_INVALID_ARG;
  out->n_layers = p->n_layers;
  out->num_blocks = p->num_blocks;
  out->block_size = p->block_size;
  out->kv_rank = p->kv_rank;
  out->rope_dim = p->rope_dim;
  out->quantized = p->quantized;
  out->nblk = p->nblk;
  out->device = p->device;
  out->kv = p->kv;
  out->pe = p->pe;
  out->qs = p->qs;
  out->sc = p->sc;
  out->pool_bytes = p->quantized ? p->rows() * 34ull * p->nblk
                                 : p->rows() * 4ull * (p->kv_rank + p->rope_dim);
  out->checkpoint_bytes = checkpoint_bytes(p);
  return KVCU_OK;
}

int kvcu_pool_zero(kvcu_pool* p, void* stream) {
  if (!valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  cudaStream_t st = (cudaStream_t)stream;
  const uint64_t rows = p->rows();
  if (p->quantized) {
    KVCU_CUDA(cudaMemsetAsync(p->qs, 0, rows * 32ull * p->nblk, st));
    KVCU_CUDA(cudaMemsetAsync(p->sc, 0, rows * 2ull * p->nblk, st));
  } else {
    KVCU_CUDA(cudaMemsetAsync(p->kv, 0, rows * 4ull * p->kv_rank, st));
    KVCU_CUDA(cudaMemsetAsync(p->pe, 0, rows * 4ull * p->rope_dim, st));
  }
  KVCU_CUDA(cudaMemsetAsync(p->status, 0, sizeof(uint32_t), st));
  return KVCU_OK;
}

int kvcu_pool_status(kvcu_pool* p, uint32_t* status_out, void* stream) {
  if (!valid_pool(p) || !status_out) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  cudaStream_t st = (cudaStream_t)stream;
  // into pinned memory: the copy is asynchronous, and one synchronise covers
  // the read and the reset
  KVCU_CUDA(cudaMemcpyAsync(p->status_host, p->status, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  KVCU_CUDA(cudaMemsetAsync(p->status, 0, sizeof(uint32_t), st));
  KVCU_CUDA(cudaStreamSynchronize(st));
  *status_out = *p->status_host;
  return KVCU_OK;
}

int kvcu_pool_copy_block(kvcu_pool* p, uint32_t src, uint32_t dst, void* stream) {
  if (!valid_pool(p) || src >= p->num_blocks || dst >= p->num_blocks) return KVCU_ERR_INVALID_ARG;
  if (src == dst) return KVCU_OK;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  cudaStream_t st = (cudaStream_t)stream;
  // one block of one array is BS contiguous rows per layer; layers are NB*BS rows apart
  auto copy = [&](void* base, size_t row_bytes) -> int {
    if (!base) return KVCU_OK;
    char* b = static_cast<char*>(base);
    const size_t width = (size_t)p->block_size * row_bytes, pitch = (size_t)p->num_blocks * width;
    return kvcu_check_cuda(cudaMemcpy2DAsync(b + dst * width, pitch, b + src * width, pitch, width, p->n_layers,
                                             cudaMemcpyDeviceToDevice, st),
                           "cudaMemcpy2DAsync(block copy)");
  };
  int rc;
  if (p->quantized) {
    rc = copy(p->qs, 32ull * p->nblk);
    if (!rc) rc = copy(p->sc, 2ull * p->nblk);
  } else {
    rc = copy(p->kv, 4ull * p->kv_rank);
    if (!rc) rc = copy(p->pe, 4ull * p->rope_dim);
  }
  return rc;
}

int kvcu_append(kvcu_pool* p, uint32_t layer, uint32_t n_rows, const float* latent,
                uint64_t latent_stride, const float* rope, uint64_t rope_stride,
                const uint32_t* row_seq, const uint32_t* row_pos, uint32_t n_seqs,
                const uint32_t* table_offsets, const uint32_t* tables, uint32_t* lens,
                void* stream) {
  if (!valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (layer >= p->n_layers) {
    kvcu_set_error("kvcu_append: layer %u >= n_layers %u", layer, p->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if (n_rows && (!latent || !rope || !row_seq || !row_pos || !table_offsets || !tables)) {
    kvcu_set_error("kvcu_append: null pointer argument");
    return KVCU_ERR_INVALID_ARG;
  }
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_append(p, layer, n_rows, latent, latent_stride, rope, rope_stride, row_seq,
                            row_pos, n_seqs, table_offsets, tables, lens, (cudaStream_t)stream);
}

int kvcu_append_layers(kvcu_pool* p, uint32_t layer, uint32_t n_layers, uint32_t n_rows, const float* latent,
                       uint64_t latent_stride, uint64_t latent_layer_stride, const float* rope,
                       uint64_t rope_stride, uint64_t rope_layer_stride, const uint32_t* row_seq,
                       const uint32_t* row_pos, uint32_t n_seqs, const uint32_t* table_offsets,
                       const uint32_t* tables, uint32_t* lens, void* stream) {
  if (!valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (n_layers == 0 || layer >= p->n_layers || n_layers > p->n_layers - layer) {
    kvcu_set_error("kvcu_append_layers: layers [%u, %u + %u) outside the pool's %u", layer, layer, n_layers,
                   p->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if (n_rows && (!latent || !rope || !row_seq || !row_pos || !table_offsets || !tables)) {
    kvcu_set_error("kvcu_append_layers: null pointer argument");
    return KVCU_ERR_INVALID_ARG;
  }
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_append_layers(p, layer, n_layers, n_rows, latent, latent_stride, latent_layer_stride, rope,
                                   rope_stride, rope_layer_stride, row_seq, row_pos, n_seqs, table_offsets, tables,
                                   lens, (cudaStream_t)stream);
}

int kvcu_gather(kvcu_pool* p, uint32_t layer, const uint32_t* table, uint32_t table_len,
                uint32_t len, float* out, void* stream) {
  if (!valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (layer >= p->n_layers) {
    kvcu_set_error("kvcu_gather: layer %u >= n_layers %u", layer, p->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if ((uint64_t)len > (uint64_t)table_len * p->block_size) {
    kvcu_set_error("kvcu_gather: len %u exceeds table capacity %u*%u", len, table_len,
                   p->block_size);
    return KVCU_ERR_POSITION_OOB;
  }
  if (len && (!table || !out)) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_gather_rows(p, layer, len, nullptr, nullptr, 0, nullptr, nullptr, table,
                                 table_len, out, (cudaStream_t)stream);
}

int kvcu_gather_rows(kvcu_pool* p, uint32_t layer, uint32_t n_rows, const uint32_t* row_seq,
                     const uint32_t* row_pos, uint32_t n_seqs, const uint32_t* table_offsets,
                     const uint32_t* tables, float* out, void* stream) {
  if (!valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (layer >= p->n_layers) return KVCU_ERR_LAYER_OOB;
  if (n_rows && (!row_seq || !row_pos || !table_offsets || !tables || !out))
    return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_gather_rows(p, layer, n_rows, row_seq, row_pos, n_seqs, table_offsets,
                                 tables, nullptr, 0, out, (cudaStream_t)stream);
}

// ---------------------------------------------------------------- decode
kvcu_decode_ws* kvcu_decode_ws_create(int device, uint32_t max_batch, uint32_t max_heads) {
  return kvcu_decode_ws_create_layers(device, max_batch, max_heads, 1);
}

kvcu_decode_ws* kvcu_decode_ws_create_layers(int device, uint32_t max_batch, uint32_t max_heads,
                                             uint32_t max_layers) {
  if (!max_batch || !max_heads || max_heads > 32 || !max_layers) {
    kvcu_set_error("kvcu_decode_ws_create: max_batch=%u max_heads=%u max_layers=%u (heads must be 1..32, "
                   "layers >= 1)",
                   max_batch, max_heads, max_layers);
    return nullptr;
  }
  if (kvcu_init(device) != KVCU_OK) return nullptr;
  DeviceGuard g(device);
  if (g.rc) return nullptr;
  kvcu_decode_ws* ws = new (std::nothrow) kvcu_decode_ws();
  if (!ws) return nullptr;
  memset(ws, 0, sizeof(*ws));
  ws->device = device;
  ws->max_batch = max_batch;
  ws->max_heads = max_heads;
  ws->max_layers = max_layers;
  int rc = kvcu_decode_setup(ws);
  // items <= batch + ranges - 1 per layer (each cut between CTA ranges splits
  // at most one entry); a layered plan numbers up to max_layers layers' items
  ws->max_ranges = (uint32_t)ws->decode_ctas;
  ws->max_items = max_batch + ws->max_ranges + 1u;
  const uint64_t mi = ws->max_items, ml = (uint64_t)max_layers;
  if (!rc && ml * mi > 0x7FFFFFFFull) {
    kvcu_set_error("kvcu_decode_ws_create: %u layers x %u batch entries is too large", max_layers, max_batch);
    rc = KVCU_ERR_INVALID_ARG;
  }
  if (!rc) rc = kvcu_check_cuda(cudaMalloc(&ws->items, ml * mi * sizeof(kvcu_item)), "cudaMalloc(items)");
  if (!rc) rc = kvcu_check_cuda(cudaMalloc(&ws->meta, 4 * sizeof(uint32_t)), "cudaMalloc(meta)");
  if (!rc)
    rc = kvcu_check_cuda(cudaMalloc(&ws->ranges, (ws->max_ranges + 1ull) * sizeof(uint32_t)),
                         "cudaMalloc(ranges)");
  if (!rc) rc = kvcu_check_cuda(cudaMalloc(&ws->seq_first, ml * max_batch * 4ull), "cudaMalloc");
  if (!rc) rc = kvcu_check_cuda(cudaMalloc(&ws->seq_count, ml * max_batch * 4ull), "cudaMalloc");
  if (!rc) rc = kvcu_check_cuda(cudaMalloc(&ws->part_o, ml * mi * max_heads * 512ull * 4), "cudaMalloc");
  if (!rc) rc = kvcu_check_cuda(cudaMalloc(&ws->part_ml, ml * mi * max_heads * 2ull * 4), "cudaMalloc");
  if (!rc) rc = kvcu_check_cuda(cudaMemset(ws->meta, 0, 4 * sizeof(uint32_t)), "cudaMemset");
  if (rc) {
    kvcu_decode_ws_destroy(ws);
    return nullptr;
  }
  return ws;
}

int kvcu_decode_ws_destroy(kvcu_decode_ws* ws) {
  if (!ws) return KVCU_OK;
  DeviceGuard g(ws->device);
  cudaFree(ws->items);
  cudaFree(ws->meta);
  cudaFree(ws->ranges);
  cudaFree(ws->seq_first);
  cudaFree(ws->seq_count);
  cudaFree(ws->part_o);
  cudaFree(ws->part_ml);
  delete ws;
  return KVCU_OK;
}

int kvcu_decode_plan(kvcu_decode_ws* ws, const kvcu_pool* p, uint32_t n, const uint32_t* seq_ids,
                     uint32_t n_seqs, const uint32_t* lens, void* stream) {
  if (!ws || !valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (n > ws->max_batch) {
    kvcu_set_error("kvcu_decode_plan: batch %u exceeds workspace capacity %u", n, ws->max_batch);
    return KVCU_ERR_INVALID_ARG;
  }
  if (ws->device != p->device) return KVCU_ERR_INVALID_ARG;
  if (n && !lens) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_plan(ws, p, n, seq_ids, n_seqs, lens, (cudaStream_t)stream);
}

int kvcu_decode_plan_layers(kvcu_decode_ws* ws, const kvcu_pool* p, uint32_t n, const uint32_t* seq_ids,
                            uint32_t n_seqs, const uint32_t* lens, uint32_t n_layers, void* stream) {
  if (!ws || !valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (n > ws->max_batch) {
    kvcu_set_error("kvcu_decode_plan_layers: batch %u exceeds workspace capacity %u", n, ws->max_batch);
    return KVCU_ERR_INVALID_ARG;
  }
  if (n_layers == 0 || n_layers > ws->max_layers) {
    kvcu_set_error("kvcu_decode_plan_layers: %u layers, the workspace holds %u", n_layers, ws->max_layers);
    return KVCU_ERR_INVALID_ARG;
  }
  if (ws->device != p->device) return KVCU_ERR_INVALID_ARG;
  if (n && !lens) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_plan_target(ws, p, n, seq_ids, n_seqs, lens, (uint32_t)ws->decode_ctas, (cudaStream_t)stream,
                                 nullptr, n_layers);
}

int kvcu_mla_decode(kvcu_decode_ws* ws, kvcu_pool* p, uint32_t layer, uint32_t n,
                    const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* table_offsets,
                    const uint32_t* tables, const uint32_t* lens, const float* q,
                    uint32_t n_heads, float scale, float* out, void* stream) {
  if (!ws || !valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (ws->device != p->device) return KVCU_ERR_INVALID_ARG;
  if (layer >= p->n_layers) {
    kvcu_set_error("kvcu_mla_decode: layer %u >= n_layers %u", layer, p->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if (n && (!table_offsets || !tables || !lens || !q || !out)) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_decode(ws, p, layer, n, seq_ids, n_seqs, table_offsets, tables, lens, q,
                            n_heads, scale, out, nullptr, (cudaStream_t)stream);
}

int kvcu_decode_plan_causal(kvcu_decode_ws* ws, const kvcu_pool* p, uint32_t n, const uint32_t* seq_ids,
                            uint32_t n_seqs, const uint32_t* lens, const uint32_t* entry_lens, void* stream) {
  if (!ws || !valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (n > ws->max_batch) {
    kvcu_set_error("kvcu_decode_plan_causal: batch %u exceeds workspace capacity %u", n, ws->max_batch);
    return KVCU_ERR_INVALID_ARG;
  }
  if (ws->device != p->device) return KVCU_ERR_INVALID_ARG;
  if (n && (!lens || !entry_lens)) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_plan(ws, p, n, seq_ids, n_seqs, lens, (cudaStream_t)stream, entry_lens);
}

int kvcu_mla_decode_layers(kvcu_decode_ws* ws, kvcu_pool* p, uint32_t layer, uint32_t n_layers, uint32_t n,
                           const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* table_offsets,
                           const uint32_t* tables, const uint32_t* lens, const float* q, uint64_t q_layer_stride,
                           uint32_t n_heads, float scale, float* out, uint64_t out_layer_stride, void* stream) {
  if (!ws || !valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (ws->device != p->device) return KVCU_ERR_INVALID_ARG;
  if (n_layers == 0 || layer >= p->n_layers || n_layers > p->n_layers - layer) {
    kvcu_set_error("kvcu_mla_decode_layers: layers [%u, %u + %u) outside the pool's %u", layer, layer, n_layers,
                   p->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if (n_layers > ws->max_layers) {
    kvcu_set_error("kvcu_mla_decode_layers: %u layers, the workspace holds partials for %u", n_layers,
                   ws->max_layers);
    return KVCU_ERR_INVALID_ARG;
  }
  if (n && (!table_offsets || !tables || !lens || !q || !out)) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_decode_layers(ws, p, layer, n_layers, n, seq_ids, n_seqs, table_offsets, tables, lens, q,
                                   q_layer_stride, n_heads, scale, out, out_layer_stride, nullptr, 0,
                                   (cudaStream_t)stream);
}

int kvcu_mla_decode_lse(kvcu_decode_ws* ws, kvcu_pool* p, uint32_t layer, uint32_t n,
                        const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* table_offsets,
                        const uint32_t* tables, const uint32_t* lens, const float* q,
                        uint32_t n_heads, float scale, float* out, float* lse, void* stream) {
  if (!ws || !valid_pool(p)) return KVCU_ERR_INVALID_ARG;
  if (ws->device != p->device) return KVCU_ERR_INVALID_ARG;
  if (layer >= p->n_layers) {
    kvcu_set_error("kvcu_mla_decode_lse: layer %u >= n_layers %u", layer, p->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if (n && (!table_offsets || !tables || !lens || !q || !out || !lse)) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return kvcu_launch_decode(ws, p, layer, n, seq_ids, n_seqs, table_offsets, tables, lens, q,
                            n_heads, scale, out, lse, (cudaStream_t)stream);
}

uint32_t kvcu_decode_last_launches(const kvcu_decode_ws* ws) { return ws ? ws->last_launches : 0; }

int kvcu_decode_ws_set_impl(kvcu_decode_ws* ws, int impl) {
  if (!ws || impl < KVCU_DECODE_AUTO || impl > KVCU_DECODE_TENSOR_CORE) return KVCU_ERR_INVALID_ARG;
  ws->impl = impl;
  return KVCU_OK;
}

int kvcu_decode_last_impl(const kvcu_decode_ws* ws) { return ws ? ws->last_impl : 0; }

int kvcu_decode_ws_set_wait_limit(kvcu_decode_ws* ws, uint64_t cycles) {
  if (!ws || cycles > (1ull << 40)) return KVCU_ERR_INVALID_ARG;
  ws->wait_limit = cycles;
  return KVCU_OK;
}

int kvcu_decode_ws_test_withhold(kvcu_decode_ws* ws, uint32_t tile) {
  if (!ws) return KVCU_ERR_INVALID_ARG;
  ws->withhold_plus1 = tile == 0xFFFFFFFFu ? 0u : tile + 1u;
  return KVCU_OK;
}

// ---------------------------------------------------------------- checkpoint
static int ensure_staging(kvcu_pool* p) {
  if (p->staging) return KVCU_OK;
  KVCU_CUDA(cudaMalloc(&p->staging, kStagingBytes));
  p->staging_bytes = kStagingBytes;
  return KVCU_OK;
}

// Walk [offset, offset+nbytes) of the checkpoint pool section in chunks.
// f32: plain copies out of / into the kv and pe pools.  Q8_0: whole 34-byte
// blocks are (un)packed through the device staging buffer.
// Q8_0 pools repack through `stg` (stg_bytes of device memory); f32 pools need none.
static int checkpoint_io(kvcu_pool* p, uint64_t offset, uint64_t nbytes, uint8_t* host,
                         bool to_host, cudaStream_t st, uint8_t* stg, uint64_t stg_bytes) {
  const uint64_t total = checkpoint_bytes(p);
  if (offset > total || nbytes > total - offset) {
    kvcu_set_error("checkpoint range [%llu, +%llu) outside the %llu-byte pool section",
                   (unsigned long long)offset, (unsigned long long)nbytes,
                   (unsigned long long)total);
    return KVCU_ERR_INVALID_ARG;
  }
  if (!nbytes) return KVCU_OK;
  if (!p->quantized) {
    const uint64_t kv_bytes = p->rows() * 4ull * p->kv_rank;
    uint64_t done = 0;
    while (done < nbytes) {
      const uint64_t off = offset + done;
      uint8_t* dev;
      uint64_t avail;
      if (off < kv_bytes) {
        dev = reinterpret_cast<uint8_t*>(p->kv) + off;
        avail = kv_bytes - off;
      } else {
        dev = reinterpret_cast<uint8_t*>(p->pe) + (off - kv_bytes);
        avail = total - off;
      }
      const uint64_t n = std::min(avail, nbytes - done);
      if (to_host)
        KVCU_CUDA(cudaMemcpyAsync(host + done, dev, n, cudaMemcpyDeviceToHost, st));
      else
        KVCU_CUDA(cudaMemcpyAsync(dev, host + done, n, cudaMemcpyHostToDevice, st));
      done += n;
    }
    KVCU_CUDA(cudaStreamSynchronize(st));
    return KVCU_OK;
  }
  int rc = KVCU_OK;
  if (!stg || stg_bytes < 34u) {
    kvcu_set_error("checkpoint repacking needs a device staging buffer");
    return KVCU_ERR_INVALID_ARG;
  }
  const uint64_t part0_blocks = p->rows() * p->nbk;
  const uint64_t part0_bytes = part0_blocks * 34u;
  const uint64_t chunk_blocks = stg_bytes / 34u;
  uint64_t done = 0;
  while (done < nbytes) {
    const uint64_t off = offset + done;
    const int part = off < part0_bytes ? 0 : 1;
    const uint64_t part_off = part == 0 ? off : off - part0_bytes;
    const uint64_t part_blocks = part == 0 ? part0_blocks : p->rows() * p->nbp;
    const uint64_t blk0 = part_off / 34u;
    const uint64_t skip = part_off - blk0 * 34u;  // bytes into the first block
    const uint64_t part_end = part == 0 ? part0_bytes : total;
    const uint64_t want = std::min(nbytes - done, part_end - off);
    uint64_t nblk = std::min((skip + want + 33u) / 34u, chunk_blocks);
    nblk = std::min(nblk, part_blocks - blk0);
    const uint64_t n = std::min(want, nblk * 34u - skip);
    if (to_host) {
      rc = kvcu_launch_pack_q8(p, part, blk0, nblk, stg, st);
      if (rc) return rc;
      KVCU_CUDA(cudaMemcpyAsync(host + done, stg + skip, n, cudaMemcpyDeviceToHost, st));
      KVCU_CUDA(cudaStreamSynchronize(st));
    } else {
      // partial first/last blocks: read-modify-write through the staging buffer
      if (skip != 0 || n != nblk * 34u) {
        rc = kvcu_launch_pack_q8(p, part, blk0, nblk, stg, st);
        if (rc) return rc;
      }
      KVCU_CUDA(cudaMemcpyAsync(stg + skip, host + done, n, cudaMemcpyHostToDevice, st));
      rc = kvcu_launch_unpack_q8(p, part, blk0, nblk, stg, st);
      if (rc) return rc;
      KVCU_CUDA(cudaStreamSynchronize(st));
    }
    done += n;
  }
  return KVCU_OK;
}

int kvcu_pool_read_checkpoint(kvcu_pool* p, uint64_t offset, uint64_t nbytes, void* host_dst,
                              void* stream) {
  if (!valid_pool(p) || (nbytes && !host_dst)) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  if (p->quantized) {
    const int rc = ensure_staging(p);
    if (rc) return rc;
  }
  return checkpoint_io(p, offset, nbytes, static_cast<uint8_t*>(host_dst), true, (cudaStream_t)stream, p->staging,
                       p->staging_bytes);
}

int kvcu_pool_write_checkpoint(kvcu_pool* p, uint64_t offset, uint64_t nbytes,
                               const void* host_src, void* stream) {
  if (!valid_pool(p) || (nbytes && !host_src)) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  if (p->quantized) {
    const int rc = ensure_staging(p);
    if (rc) return rc;
  }
  return checkpoint_io(p, offset, nbytes, const_cast<uint8_t*>(static_cast<const uint8_t*>(host_src)), false,
                       (cudaStream_t)stream, p->staging, p->staging_bytes);
}

}  // extern "C"

// Read a checkpoint byte range through a caller-owned staging buffer (the
// background save uses its own, so the pool's stays free for other calls).
int kvcu_pool_read_checkpoint_staged(kvcu_pool* p, uint64_t offset, uint64_t nbytes, void* host_dst,
                                     cudaStream_t st, uint8_t* staging, uint64_t staging_bytes) {
  if (!valid_pool(p) || (nbytes && !host_dst)) return KVCU_ERR_INVALID_ARG;
  DeviceGuard g(p->device);
  if (g.rc) return g.rc;
  return checkpoint_io(p, offset, nbytes, static_cast<uint8_t*>(host_dst), true, st, staging, staging_bytes);
}

extern "C" {

int kvcu_synth_rows(uint64_t seed, uint64_t a, uint32_t n_rows, const uint32_t* b,
                    const uint32_t* c, uint32_t width, float outlier_p, float* out, void* stream) {
  if (n_rows && (!b || !c || !out)) return KVCU_ERR_INVALID_ARG;
  return kvcu_launch_synth(seed, a, n_rows, b, c, width, outlier_p, out, (cudaStream_t)stream);
}

}  // extern "C"
