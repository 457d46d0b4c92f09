// kvcache_host.cu — host mirror of src/kv_cache.zig's KVCache over a kvcu_pool.
//
// The reference keeps its allocator state on the host; so does this mirror:
//   block refcounts, hashes and the LIFO free list   src/kv_cache.zig:17-21, :86-91, :158-183
//   block_table / len per sequence                    src/kv_cache.zig:46-49, :188-215
//   prefix-cache hash map (chained XXH64)             src/kv_cache.zig:367-436, :596-609
//   v1 checkpoint (40-byte header, table, pool)       src/kv_cache.zig:453-591
// Data never touches the host except through the explicit host-buffer calls:
// put/get/gather/decode launch the CUDA kernels of kvcu_kernels.cu and
// kvcu_decode.cu.  Sequence 0 is the reference's single sequence; more
// sequences share the pool (the multi-sequence serving surface).
//
// Deviations from the reference (also listed in kvcuda.h): Q8_0 pools start
// zeroed; loadFromFile bounds-checks block ids and takes them off the free
// list; reusePrefixBlocks retains before it releases.
#include <cuda.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <errno.h>
#include <string>
#include <new>
#include <thread>
#include <unordered_map>
#include <vector>

#include "kvcu_internal.h"

namespace {

constexpr uint64_t kNoHash = ~0ull;

// ---- XXH64 (published xxHash specification), used by computeHash ----
constexpr uint64_t P1 = 0x9E3779B185EBCA87ull, P2 = 0xC2B2AE3D27D4EB4Full,
                   P3 = 0x165667B19E3779F9ull, P4 = 0x85EBCA77C2B2AE63ull,
                   P5 = 0x27D4EB2F165667C5ull;
inline uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
inline uint64_t le64(const uint8_t* p) {
  uint64_t v;
  memcpy(&v, p, 8);
  return v;
}
inline uint32_t le32(const uint8_t* p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}
inline uint64_t xx_round(uint64_t acc, uint64_t in) { return rotl(acc + in * P2, 31) * P1; }
inline uint64_t xx_merge(uint64_t h, uint64_t v) { return (h ^ xx_round(0, v)) * P1 + P4; }

uint64_t xxh64(const uint8_t* p, size_t len, uint64_t seed) {
  const uint8_t* const end = p + len;
  uint64_t h;
  if (len >= 32) {
    uint64_t v[4] = {seed + P1 + P2, seed + P2, seed, seed - P1};
    for (; p + 32 <= end; p += 32)
      for (int i = 0; i < 4; ++i) v[i] = xx_round(v[i], le64(p + 8 * i));
    h = rotl(v[0], 1) + rotl(v[1], 7) + rotl(v[2], 12) + rotl(v[3], 18);
    for (int i = 0; i < 4; ++i) h = xx_merge(h, v[i]);
  } else {
    h = seed + P5;
  }
  h += (uint64_t)len;
  for (; p + 8 <= end; p += 8) h = rotl(h ^ xx_round(0, le64(p)), 27) * P1 + P4;
  if (p + 4 <= end) {
    h = rotl(h ^ ((uint64_t)le32(p) * P1), 23) * P2 + P3;
    p += 4;
  }
  for (; p < end; ++p) h = rotl(h ^ ((uint64_t)(*p) * P5), 11) * P1;
  h ^= h >> 33;
  h *= P2;
  h ^= h >> 29;
  h *= P3;
  h ^= h >> 32;
  return h;
}

void put_le32(uint8_t* b, uint32_t v) {
  for (int i = 0; i < 4; ++i) b[i] = (uint8_t)(v >> (8 * i));
}

int write_all(int fd, const void* buf, size_t n) {
  const uint8_t* p = static_cast<const uint8_t*>(buf);
  while (n) {
    ssize_t rc = write(fd, p, n);
    if (rc < 0) {
      if (errno == EINTR) continue;
      kvcu_set_error("write failed: %s", strerror(errno));
      return KVCU_ERR_IO;
    }
    if (rc == 0) return KVCU_ERR_IO;
    p += rc;
    n -= (size_t)rc;
  }
  return KVCU_OK;
}

int read_no_eof(int fd, void* buf, size_t n) {
  uint8_t* p = static_cast<uint8_t*>(buf);
  while (n) {
    ssize_t rc = read(fd, p, n);
    if (rc < 0) {
      if (errno == EINTR) continue;
      kvcu_set_error("read failed: %s", strerror(errno));
      return KVCU_ERR_IO;
    }
    if (rc == 0) {
      kvcu_set_error("checkpoint truncated (end of stream)");
      return KVCU_ERR_EOF;
    }
    p += rc;
    n -= (size_t)rc;
  }
  return KVCU_OK;
}

struct Fd {
  int fd;
  explicit Fd(int f) : fd(f) {}
  ~Fd() {
    if (fd >= 0) close(fd);
  }
};

struct Seq {
  std::vector<uint32_t> table;
  uint32_t len = 0;
};

template <typename T>
int ensure_dev(T** ptr, size_t* cap, size_t n) {
  if (*cap >= n && *ptr) return KVCU_OK;
  size_t nc = std::max<size_t>(n, *cap * 2);
  if (nc < 16) nc = 16;
  cudaFree(*ptr);
  *ptr = nullptr;
  *cap = 0;
  KVCU_CUDA(cudaMalloc(ptr, nc * sizeof(T)));
  *cap = nc;
  return KVCU_OK;
}

// The device address of host buffer [p, p + bytes) when it is pinned, mapped
// into the device's address space and its allocation covers all `bytes`; null
// otherwise (pageable memory, an unmapped or shorter allocation, or a failed
// query), and the caller copies instead.
typedef CUresult (*PointerAttrFn)(void*, CUpointer_attribute, CUdeviceptr);
void* mapped_host_range(const void* p, size_t bytes) {
  static PointerAttrFn attr_fn = []() -> PointerAttrFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PointerAttrFn>(f);
  }();
  if (!attr_fn || !p || !bytes) return nullptr;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();  // a failed query leaves a (non-sticky) error behind: clear it
    return nullptr;
  }
  if (at.type != cudaMemoryTypeHost || !at.devicePointer) return nullptr;
  const CUdeviceptr dp = reinterpret_cast<CUdeviceptr>(at.devicePointer);
  CUdeviceptr start = 0;
  size_t size = 0;
  if (attr_fn(&start, CU_POINTER_ATTRIBUTE_RANGE_START_ADDR, dp) != CUDA_SUCCESS ||
      attr_fn(&size, CU_POINTER_ATTRIBUTE_RANGE_SIZE, dp) != CUDA_SUCCESS)
    return nullptr;
  if (dp < start || bytes > size || dp - start > size - bytes) return nullptr;
  return at.devicePointer;
}

}  // namespace

// A pinned host buffer that feeds one asynchronous upload at a time: `done`
// is recorded after the copy, and the buffer is refilled only once it fired.
struct HostStage {
  uint32_t* p = nullptr;
  size_t cap = 0;
  cudaEvent_t done = nullptr;
};

struct kvcache {
  int device = 0;
  uint32_t n_layers = 0, kv_rank = 0, rope_dim = 0, num_blocks = 0, block_size = 0;
  kvcu_pool* pool = nullptr;
  std::vector<uint32_t> ref_count;
  std::vector<uint64_t> hash;
  std::vector<uint32_t> free_list;  // LIFO: back() is handed out next
  std::unordered_map<uint64_t, uint32_t> hash_map;
  std::vector<Seq> seqs;
  cudaStream_t stream = nullptr;
  // device mirrors of the block tables (CSR by sequence id) and lengths
  uint32_t* d_toff = nullptr;
  size_t d_toff_cap = 0;
  uint32_t* d_tables = nullptr;
  size_t d_tables_cap = 0;
  uint32_t* d_lens = nullptr;
  size_t d_lens_cap = 0;
  bool tables_dirty = true, lens_dirty = true;
  std::vector<uint32_t> h_toff;
  // pinned staging of the table / length uploads (truly asynchronous copies)
  HostStage up_toff, up_tables, up_lens;
  HostStage up_rowidx;  // sequence ids and positions of a host-rows append
  // scratch for host-buffer calls
  float* d_f = nullptr;
  size_t d_f_cap = 0;
  float* d_f2 = nullptr;
  size_t d_f2_cap = 0;
  uint32_t* d_u = nullptr;
  size_t d_u_cap = 0;
  // scratch of the MLA step: q_abs, rows, latent, lse / seq ids, positions, history lengths
  float* d_step = nullptr;
  size_t d_step_cap = 0;
  uint32_t* d_stepu = nullptr;
  size_t d_stepu_cap = 0;
  // decode
  kvcu_decode_ws* ws = nullptr;
  uint32_t ws_batch = 0, ws_heads = 0, ws_layers = 0;
  uint32_t* d_seq_ids = nullptr;
  size_t d_seq_ids_cap = 0;
  std::vector<uint32_t> plan_ids;
  // the MLA step's plan (history lengths of its batch) is kept for the next
  // layer of the same step: valid while no other plan ran on the workspace
  std::vector<uint32_t> mla_plan_ids, mla_plan_hist;
  uint64_t plan_serial = 0, mla_plan_serial = ~0ull;
  uint64_t plan_epoch = ~0ull, epoch = 0;
  uint64_t plan_tokens = 0;
  uint32_t plan_layers = 0;  // layers the cached plan lists as one (1: a one-layer plan)
  uint32_t last_launches = 0;
  int decode_impl = KVCU_DECODE_AUTO;
  int last_mapped = 0;  // the last host-buffer decode read q / wrote out in place (pinned, mapped)
  int host_io = KVCACHE_HOST_IO_AUTO;
  // background save (kvcache_save_to_file_v2_async): the job in flight, and its
  // device staging and two pinned host buffers, kept for the next save
  kvcache_save* active_save = nullptr;
  uint8_t* save_stg = nullptr;
  uint8_t* save_host[2] = {nullptr, nullptr};

  bool quantized() const { return pool && pool->quantized; }
  uint32_t row_width() const { return kv_rank + rope_dim; }
};

namespace {

// Make h.p hold at least n words, once the previous upload from it has run
// (an event wait, normally long satisfied: the host stays ahead of the GPU).
int stage_acquire(HostStage& h, size_t n) {
  if (!h.done) KVCU_CUDA(cudaEventCreateWithFlags(&h.done, cudaEventDisableTiming));
  else KVCU_CUDA(cudaEventSynchronize(h.done));
  if (n > h.cap) {
    if (h.p) KVCU_CUDA(cudaFreeHost(h.p));
    h.p = nullptr;
    h.cap = 0;
    const size_t cap = std::max<size_t>(n + n / 4, 1024);
    KVCU_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h.p), cap * 4, cudaHostAllocDefault));
    h.cap = cap;
  }
  return KVCU_OK;
}

int stage_upload(HostStage& h, uint32_t* dst, size_t n, cudaStream_t st) {
  KVCU_CUDA(cudaMemcpyAsync(dst, h.p, n * 4, cudaMemcpyHostToDevice, st));
  KVCU_CUDA(cudaEventRecord(h.done, st));
  return KVCU_OK;
}

void stage_free(HostStage& h) {
  if (h.done) {
    cudaEventSynchronize(h.done);
    cudaEventDestroy(h.done);
  }
  if (h.p) cudaFreeHost(h.p);
  h = HostStage{};
}

// Block tables (CSR by sequence id) to the device, ordered on `st` before the
// kernels that read them.  Pinned staging: no stream drain on the host.
int sync_tables(kvcache* c, cudaStream_t st) {
  // a clean mirror may still be in flight on another stream: order `st` after it
  if (!c->tables_dirty) return c->up_tables.done ? kvcu_check_cuda(cudaStreamWaitEvent(st, c->up_tables.done, 0),
                                                                   "cudaStreamWaitEvent(tables)")
                                                 : KVCU_OK;
  const size_t nseq = c->seqs.size();
  size_t total = 0;
  for (size_t s = 0; s < nseq; ++s) total += c->seqs[s].table.size();
  const size_t nflat = std::max<size_t>(total, 1);
  int rc = stage_acquire(c->up_toff, nseq + 1);
  if (!rc) rc = stage_acquire(c->up_tables, nflat);
  if (!rc) rc = ensure_dev(&c->d_toff, &c->d_toff_cap, nseq + 1);
  if (!rc) rc = ensure_dev(&c->d_tables, &c->d_tables_cap, nflat);
  if (rc) return rc;
  uint32_t* toff = c->up_toff.p;
  uint32_t* flat = c->up_tables.p;
  size_t o = 0;
  for (size_t s = 0; s < nseq; ++s) {
    const auto& t = c->seqs[s].table;
    toff[s] = (uint32_t)o;
    if (!t.empty()) memcpy(flat + o, t.data(), t.size() * 4);
    o += t.size();
  }
  toff[nseq] = (uint32_t)o;
  if (total == 0) flat[0] = 0;
  c->h_toff.assign(toff, toff + nseq + 1);
  rc = stage_upload(c->up_toff, c->d_toff, nseq + 1, st);
  if (!rc) rc = stage_upload(c->up_tables, c->d_tables, nflat, st);
  if (rc) return rc;
  c->tables_dirty = false;
  return KVCU_OK;
}

int sync_lens(kvcache* c, cudaStream_t st) {
  if (!c->lens_dirty) return c->up_lens.done ? kvcu_check_cuda(cudaStreamWaitEvent(st, c->up_lens.done, 0),
                                                               "cudaStreamWaitEvent(lens)")
                                             : KVCU_OK;
  const size_t nseq = c->seqs.size();
  int rc = stage_acquire(c->up_lens, std::max<size_t>(nseq, 1));
  if (!rc) rc = ensure_dev(&c->d_lens, &c->d_lens_cap, nseq);
  if (rc) return rc;
  for (size_t s = 0; s < nseq; ++s) c->up_lens.p[s] = c->seqs[s].len;
  rc = stage_upload(c->up_lens, c->d_lens, nseq, st);
  if (rc) return rc;
  c->lens_dirty = false;
  return KVCU_OK;
}

int check_status(kvcache* c) {
  uint32_t st = 0;
  int rc = kvcu_pool_status(c->pool, &st, c->stream);
  if (rc) return rc;
  if (st) {
    kvcu_set_error("device status word 0x%x (bad table/block/sequence index)", st);
    return KVCU_ERR_DEVICE;
  }
  return KVCU_OK;
}

// src/kv_cache.zig:158-164
int allocate_block(kvcache* c, uint32_t* out) {
  if (c->free_list.empty()) {
    kvcu_set_error("OutOfKVCacheBlocks: all %u blocks in use", c->num_blocks);
    return KVCU_ERR_OUT_OF_BLOCKS;
  }
  const uint32_t id = c->free_list.back();
  c->free_list.pop_back();
  c->ref_count[id] = 1;
  c->hash[id] = kNoHash;
  *out = id;
  return KVCU_OK;
}

// src/kv_cache.zig:166-178
void release_block(kvcache* c, uint32_t id) {
  if (id >= c->num_blocks || c->ref_count[id] == 0) return;
  if (--c->ref_count[id] == 0) {
    if (c->hash[id] != kNoHash) {
      auto it = c->hash_map.find(c->hash[id]);
      if (it != c->hash_map.end()) c->hash_map.erase(it);
    }
    c->hash[id] = kNoHash;
    c->free_list.push_back(id);
  }
}

void retain_block(kvcache* c, uint32_t id) { c->ref_count[id] += 1; }

void take_off_free_list(kvcache* c, uint32_t id) {
  auto it = std::find(c->free_list.begin(), c->free_list.end(), id);
  if (it != c->free_list.end()) c->free_list.erase(it);
}

int seq_ensure(kvcache* c, uint32_t s, uint32_t n_tokens) {
  if (s >= c->seqs.size()) return KVCU_ERR_INVALID_ARG;
  const uint64_t needed = ((uint64_t)n_tokens + c->block_size - 1) / c->block_size;
  Seq& q = c->seqs[s];
  while (q.table.size() < needed) {
    uint32_t id;
    int rc = allocate_block(c, &id);
    if (rc) return rc;
    q.table.push_back(id);
    c->tables_dirty = true;
  }
  return KVCU_OK;
}

void seq_truncate(kvcache* c, uint32_t s, uint32_t n_tokens) {
  Seq& q = c->seqs[s];
  const uint64_t needed = ((uint64_t)n_tokens + c->block_size - 1) / c->block_size;
  while (q.table.size() > needed) {
    release_block(c, q.table.back());
    q.table.pop_back();
    c->tables_dirty = true;
  }
  if (n_tokens < q.len) {
    q.len = n_tokens;
    c->lens_dirty = true;
  }
  c->epoch++;
}

void seq_reset(kvcache* c, uint32_t s) {
  Seq& q = c->seqs[s];
  for (uint32_t id : q.table) release_block(c, id);
  q.table.clear();
  q.len = 0;
  c->tables_dirty = c->lens_dirty = true;
  c->epoch++;
}

kvcache* make_cache(int device, uint32_t n_layers, uint32_t kv_rank, uint32_t rope_dim,
                    uint32_t num_blocks, uint32_t block_size, int quantized) {
  if (num_blocks == 0) {
    kvcu_set_error("kvcache_init: zero blocks");
    return nullptr;
  }
  kvcache* c = new (std::nothrow) kvcache();
  if (!c) return nullptr;
  c->device = device;
  c->n_layers = n_layers;
  c->kv_rank = kv_rank;
  c->rope_dim = rope_dim;
  c->num_blocks = num_blocks;
  c->block_size = block_size;
  c->pool = kvcu_pool_create(device, n_layers, num_blocks, block_size, kv_rank, rope_dim, quantized);
  if (!c->pool) {
    delete c;
    return nullptr;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
    kvcu_set_error("cudaStreamCreate failed");
    kvcu_pool_destroy(c->pool);
    cudaSetDevice(prev);
    delete c;
    return nullptr;
  }
  cudaSetDevice(prev);
  c->ref_count.assign(num_blocks, 0);
  c->hash.assign(num_blocks, kNoHash);
  c->free_list.resize(num_blocks);
  for (uint32_t i = 0; i < num_blocks; ++i) c->free_list[i] = num_blocks - 1 - i;  // :89-91
  c->seqs.resize(1);
  return c;
}

struct DevScope {
  int prev = -1;
  explicit DevScope(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DevScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// Append host rows through the pool; positions already validated.
int append_host_rows(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                     const uint32_t* positions, const float* rows) {
  const uint32_t Wd = c->row_width();
  int rc = sync_tables(c, c->stream);
  if (!rc) rc = sync_lens(c, c->stream);
  if (!rc) rc = ensure_dev(&c->d_f, &c->d_f_cap, (size_t)n * Wd);
  if (!rc) rc = ensure_dev(&c->d_u, &c->d_u_cap, (size_t)2 * n);
  if (!rc) rc = stage_acquire(c->up_rowidx, (size_t)2 * n);
  if (rc) return rc;
  // rows by DMA (reading them in place from mapped host memory is slower: the
  // append kernel's row reads are latency-bound over PCIe); the row indices
  // through pinned staging
  KVCU_CUDA(cudaMemcpyAsync(c->d_f, rows, (size_t)n * Wd * 4, cudaMemcpyHostToDevice, c->stream));
  memcpy(c->up_rowidx.p, seq_ids, (size_t)n * 4);
  memcpy(c->up_rowidx.p + n, positions, (size_t)n * 4);
  rc = stage_upload(c->up_rowidx, c->d_u, (size_t)2 * n, c->stream);
  if (rc) return rc;
  rc = kvcu_append(c->pool, layer, n, c->d_f, Wd, c->d_f + c->kv_rank, Wd, c->d_u, c->d_u + n,
                   (uint32_t)c->seqs.size(), c->d_toff, c->d_tables, c->d_lens, c->stream);
  if (rc) return rc;
  c->last_launches = 1;
  return check_status(c);  // synchronises: the host buffers may be reused at return
}

int validate_positions(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                       const uint32_t* positions) {
  if (layer >= c->n_layers) {
    kvcu_set_error("LayerOutOfBounds: layer %u >= %u", layer, c->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  for (uint32_t r = 0; r < n; ++r) {
    if (seq_ids[r] >= c->seqs.size()) {
      kvcu_set_error("sequence %u does not exist", seq_ids[r]);
      return KVCU_ERR_INVALID_ARG;
    }
    if (positions[r] / c->block_size >= c->seqs[seq_ids[r]].table.size()) {
      kvcu_set_error("PositionOutOfBounds: seq %u pos %u beyond its %zu blocks", seq_ids[r],
                     positions[r], c->seqs[seq_ids[r]].table.size());
      return KVCU_ERR_POSITION_OOB;
    }
  }
  return KVCU_OK;
}

// Copy-on-write before writing (seq, pos): a block that is also held elsewhere
// (refcount > 1: another sequence reused it as a cached prefix) is first copied,
// all layers, to a fresh block that this sequence then owns alone, so shared
// prefix blocks stay read-only. The reference never writes into a shared
// block, because only full blocks are cached and reusePrefixBlocks moves len past
// them; this keeps that true after a truncate into a shared prefix as well.
// Runs after validate_positions, on the stream of the write that follows.
int cow_for_write(kvcache* c, uint32_t n, const uint32_t* seq_ids, const uint32_t* positions,
                  cudaStream_t st) {
  for (uint32_t r = 0; r < n; ++r) {
    Seq& q = c->seqs[seq_ids[r]];
    const uint32_t bi = positions[r] / c->block_size;
    const uint32_t old = q.table[bi];
    if (c->ref_count[old] <= 1) continue;
    uint32_t fresh;
    int rc = allocate_block(c, &fresh);
    if (rc) return rc;
    rc = kvcu_pool_copy_block(c->pool, old, fresh, st);
    if (rc) {
      release_block(c, fresh);
      return rc;
    }
    release_block(c, old);
    q.table[bi] = fresh;
    c->tables_dirty = true;
    c->epoch++;
  }
  return KVCU_OK;
}

void bump_lens(kvcache* c, uint32_t n, const uint32_t* seq_ids, const uint32_t* positions) {
  for (uint32_t r = 0; r < n; ++r) {
    Seq& q = c->seqs[seq_ids[r]];
    if (positions[r] >= q.len) q.len = positions[r] + 1;
  }
}

// getKVCompressed / getKPe checks (src/kv_cache.zig:225-230, :252-255)
int get_row(kvcache* c, uint32_t layer, uint32_t pos, float* kv_out, float* pe_out) {
  if (layer >= c->n_layers) {
    kvcu_set_error("LayerOutOfBounds: layer %u >= %u", layer, c->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  Seq& q = c->seqs[0];
  if (pos >= q.len) {
    kvcu_set_error("PositionNotWritten: pos %u >= len %u", pos, q.len);
    return KVCU_ERR_POSITION_NOT_WRITTEN;
  }
  if (pos / c->block_size >= q.table.size()) {
    kvcu_set_error("PositionOutOfBounds: pos %u", pos);
    return KVCU_ERR_POSITION_OOB;
  }
  const uint32_t Wd = c->row_width();
  int rc = sync_tables(c, c->stream);
  if (!rc) rc = ensure_dev(&c->d_f, &c->d_f_cap, Wd);
  if (!rc) rc = ensure_dev(&c->d_u, &c->d_u_cap, 2);
  if (rc) return rc;
  const uint32_t idx[2] = {0u, pos};
  KVCU_CUDA(cudaMemcpyAsync(c->d_u, idx, 8, cudaMemcpyHostToDevice, c->stream));
  rc = kvcu_gather_rows(c->pool, layer, 1, c->d_u, c->d_u + 1, (uint32_t)c->seqs.size(), c->d_toff,
                        c->d_tables, c->d_f, c->stream);
  if (rc) return rc;
  std::vector<float> row(Wd);
  KVCU_CUDA(cudaMemcpyAsync(row.data(), c->d_f, Wd * 4, cudaMemcpyDeviceToHost, c->stream));
  rc = check_status(c);
  if (rc) return rc;
  c->last_launches = 1;
  if (kv_out) memcpy(kv_out, row.data(), c->kv_rank * 4);
  if (pe_out) memcpy(pe_out, row.data() + c->kv_rank, c->rope_dim * 4);
  return KVCU_OK;
}

int ensure_ws(kvcache* c, uint32_t n, uint32_t n_heads, uint32_t n_layers = 1) {
  if (c->ws && c->ws_batch >= n && c->ws_heads >= n_heads && c->ws_layers >= n_layers) return KVCU_OK;
  kvcu_decode_ws_destroy(c->ws);
  c->ws = nullptr;
  c->ws_batch = std::max<uint32_t>(n, std::max<uint32_t>(c->ws_batch, 16));
  c->ws_heads = std::max<uint32_t>(n_heads, c->ws_heads);
  c->ws_layers = std::max<uint32_t>(n_layers, std::max<uint32_t>(c->ws_layers, 1));
  c->ws = kvcu_decode_ws_create_layers(c->device, c->ws_batch, c->ws_heads, c->ws_layers);
  if (!c->ws) return KVCU_ERR_NO_MEMORY;
  kvcu_decode_ws_set_impl(c->ws, c->decode_impl);
  c->plan_epoch = ~0ull;
  c->plan_ids.clear();
  ++c->plan_serial;
  return KVCU_OK;
}

// Decode layers [layer, layer + n_layers) of a batch (q / out of layer+i at
// + i * the stride, floats); n_layers > 1 runs as one multi-layer launch.
int decode_impl(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids, const float* q_dev,
                uint32_t n_heads, float scale, float* out_dev, cudaStream_t st, uint32_t n_layers = 1,
                uint64_t q_lstride = 0, uint64_t out_lstride = 0) {
  if (n_layers == 0 || layer >= c->n_layers || n_layers > c->n_layers - layer) {
    kvcu_set_error("LayerOutOfBounds: layers [%u, %u + %u) of %u", layer, layer, n_layers, c->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  for (uint32_t b = 0; b < n; ++b)
    if (seq_ids[b] >= c->seqs.size()) {
      kvcu_set_error("sequence %u does not exist", seq_ids[b]);
      return KVCU_ERR_INVALID_ARG;
    }
  int rc = ensure_ws(c, n, n_heads, n_layers);
  if (!rc) rc = sync_tables(c, st);
  if (!rc) rc = sync_lens(c, st);
  if (rc) return rc;
  uint32_t launches = 0;
  // Re-plan when the batch changed, a sequence shrank, or the tokens grew by
  // more than 1/8 since the plan (the open-ended last items absorb growth).
  uint64_t tokens = 0;
  for (uint32_t b = 0; b < n; ++b) tokens += c->seqs[seq_ids[b]].len;
  const bool same_ids = c->plan_ids.size() == n &&
                        std::equal(c->plan_ids.begin(), c->plan_ids.end(), seq_ids);
  // A multi-layer call on the tensor-core path balances all its (layer, entry)
  // pairs as one list, which splits far fewer entries than one layer's plan
  // repeated per layer.
  const uint32_t plan_layers =
      n_layers > 1 && kvcu_decode_layers_fused(c->ws, c->pool, n, n_heads) ? n_layers : 1u;
  if (!same_ids || c->plan_epoch != c->epoch || c->plan_layers != plan_layers ||
      tokens > c->plan_tokens + c->plan_tokens / 8) {
    rc = ensure_dev(&c->d_seq_ids, &c->d_seq_ids_cap, std::max<uint32_t>(n, 1));
    if (rc) return rc;
    if (!same_ids) {
      KVCU_CUDA(cudaMemcpyAsync(c->d_seq_ids, seq_ids, (size_t)n * 4, cudaMemcpyHostToDevice, st));
      KVCU_CUDA(cudaStreamSynchronize(st));
      c->plan_ids.assign(seq_ids, seq_ids + n);
    }
    rc = kvcu_decode_plan_layers(c->ws, c->pool, n, c->d_seq_ids, (uint32_t)c->seqs.size(), c->d_lens,
                                 plan_layers, st);
    ++c->plan_serial;
    if (rc) {
      c->plan_epoch = ~0ull;
      return rc;
    }
    launches += 1;
    c->plan_epoch = c->epoch;
    c->plan_tokens = tokens;
    c->plan_layers = plan_layers;
  }
  if (n_layers == 1)
    rc = kvcu_mla_decode(c->ws, c->pool, layer, n, c->d_seq_ids, (uint32_t)c->seqs.size(), c->d_toff,
                         c->d_tables, c->d_lens, q_dev, n_heads, scale, out_dev, st);
  else
    rc = kvcu_mla_decode_layers(c->ws, c->pool, layer, n_layers, n, c->d_seq_ids, (uint32_t)c->seqs.size(),
                                c->d_toff, c->d_tables, c->d_lens, q_dev, q_lstride, n_heads, scale, out_dev,
                                out_lstride, st);
  if (rc) return rc;
  c->last_launches = launches + kvcu_decode_last_launches(c->ws);
  return KVCU_OK;
}

// Causal multi-query attention over one sequence (mlaAttentionBatch,
// src/inference.zig:771-877): query i is position start_pos + i and attends
// positions [0, start_pos + i].  Stream-ordered on `st`.
int attention_batch_impl(kvcache* c, uint32_t layer, uint32_t seq, uint32_t start_pos, uint32_t n_pos,
                         const float* q_dev, uint32_t n_heads, float scale, float* out_dev, cudaStream_t st) {
  if (layer >= c->n_layers) {
    kvcu_set_error("LayerOutOfBounds: layer %u >= %u", layer, c->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if (seq >= c->seqs.size()) {
    kvcu_set_error("sequence %u does not exist", seq);
    return KVCU_ERR_INVALID_ARG;
  }
  if ((uint64_t)start_pos + n_pos > c->seqs[seq].len) {
    kvcu_set_error("PositionNotWritten: queries up to position %llu, sequence %u holds %u",
                   (unsigned long long)start_pos + n_pos - 1, seq, c->seqs[seq].len);
    return KVCU_ERR_POSITION_NOT_WRITTEN;
  }
  int rc = ensure_ws(c, n_pos, n_heads);
  if (!rc) rc = sync_tables(c, st);
  if (!rc) rc = sync_lens(c, st);
  if (!rc) rc = ensure_dev(&c->d_stepu, &c->d_stepu_cap, (size_t)2 * n_pos);
  if (!rc) rc = stage_acquire(c->up_rowidx, (size_t)2 * n_pos);
  if (rc) return rc;
  for (uint32_t i = 0; i < n_pos; ++i) {
    c->up_rowidx.p[i] = seq;
    c->up_rowidx.p[n_pos + i] = start_pos + i + 1;  // attended length of query i
  }
  rc = stage_upload(c->up_rowidx, c->d_stepu, (size_t)2 * n_pos, st);
  const uint32_t n_seqs = (uint32_t)c->seqs.size();
  if (!rc)
    rc = kvcu_decode_plan_causal(c->ws, c->pool, n_pos, c->d_stepu, n_seqs, c->d_lens, c->d_stepu + n_pos, st);
  ++c->plan_serial;
  c->plan_epoch = ~0ull;  // the cached decode plan no longer matches the workspace
  c->plan_ids.clear();
  if (!rc)
    rc = kvcu_mla_decode(c->ws, c->pool, layer, n_pos, c->d_stepu, n_seqs, c->d_toff, c->d_tables, c->d_lens, q_dev,
                         n_heads, scale, out_dev, st);
  if (rc) return rc;
  c->last_launches = 1 + kvcu_decode_last_launches(c->ws);
  return KVCU_OK;
}

}  // namespace

extern "C" {

int kvcache_mla_attention_batch_dev(kvcache* c, uint32_t layer, uint32_t seq, uint32_t start_pos, uint32_t n_pos,
                                    const float* q_dev, uint32_t n_heads, float scale, float* out_dev,
                                    void* stream) {
  if (!c || (n_pos && (!q_dev || !out_dev))) return KVCU_ERR_INVALID_ARG;
  if (!n_pos) return KVCU_OK;
  DevScope d(c->device);
  return attention_batch_impl(c, layer, seq, start_pos, n_pos, q_dev, n_heads, scale, out_dev, (cudaStream_t)stream);
}

int kvcache_mla_attention_batch(kvcache* c, uint32_t layer, uint32_t seq, uint32_t start_pos, uint32_t n_pos,
                                const float* q, uint32_t n_heads, float scale, float* out) {
  if (!c || (n_pos && (!q || !out))) return KVCU_ERR_INVALID_ARG;
  if (!n_pos) return KVCU_OK;
  DevScope d(c->device);
  const size_t qn = (size_t)n_pos * n_heads * c->row_width(), on = (size_t)n_pos * n_heads * c->kv_rank;
  const void* q_map = c->host_io == KVCACHE_HOST_IO_AUTO ? mapped_host_range(q, qn * 4) : nullptr;
  void* out_map = q_map ? mapped_host_range(out, on * 4) : nullptr;
  int rc;
  if (q_map && out_map) {
    rc = attention_batch_impl(c, layer, seq, start_pos, n_pos, static_cast<const float*>(q_map), n_heads, scale,
                              static_cast<float*>(out_map), c->stream);
    if (rc) return rc;
    return check_status(c);
  }
  rc = ensure_dev(&c->d_f, &c->d_f_cap, qn);
  if (!rc) rc = ensure_dev(&c->d_f2, &c->d_f2_cap, on);
  if (rc) return rc;
  KVCU_CUDA(cudaMemcpyAsync(c->d_f, q, qn * 4, cudaMemcpyHostToDevice, c->stream));
  rc = attention_batch_impl(c, layer, seq, start_pos, n_pos, c->d_f, n_heads, scale, c->d_f2, c->stream);
  if (rc) return rc;
  KVCU_CUDA(cudaMemcpyAsync(out, c->d_f2, on * 4, cudaMemcpyDeviceToHost, c->stream));
  return check_status(c);
}

kvcache* kvcache_init(int device, uint32_t n_layers, uint32_t kv_rank, uint32_t rope_dim,
                      uint32_t max_seq_len, uint32_t block_size) {
  if (block_size == 0) block_size = 16;  // BLOCK_SIZE, src/kv_cache.zig:14
  const uint32_t nb = (uint32_t)(((uint64_t)max_seq_len + block_size - 1) / block_size);  // :69
  return make_cache(device, n_layers, kv_rank, rope_dim, nb, block_size, 0);
}

kvcache* kvcache_init_blocks(int device, uint32_t n_layers, uint32_t kv_rank, uint32_t rope_dim,
                             uint32_t num_blocks, uint32_t block_size, int quantized) {
  return make_cache(device, n_layers, kv_rank, rope_dim, num_blocks, block_size, quantized);
}

void kvcache_deinit(kvcache* c) {
  if (!c) return;
  DevScope d(c->device);
  if (c->active_save) kvcache_save_wait(c->active_save);  // the worker reads the pool
  if (c->save_stg) cudaFree(c->save_stg);
  for (uint8_t* h : c->save_host)
    if (h) cudaFreeHost(h);
  if (c->stream) cudaStreamSynchronize(c->stream);
  kvcu_decode_ws_destroy(c->ws);
  kvcu_pool_destroy(c->pool);
  cudaFree(c->d_toff);
  cudaFree(c->d_tables);
  cudaFree(c->d_lens);
  cudaFree(c->d_f);
  cudaFree(c->d_f2);
  cudaFree(c->d_u);
  cudaFree(c->d_step);
  cudaFree(c->d_stepu);
  cudaFree(c->d_seq_ids);
  stage_free(c->up_toff);
  stage_free(c->up_tables);
  stage_free(c->up_lens);
  stage_free(c->up_rowidx);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

// src/kv_cache.zig:142-154.  The Q8_0 pool replaces the f32 pool (the
// reference keeps both; data written before the switch is not converted
// there either, its getters read the new Q8_0 pools afterwards).
int kvcache_enable_quantization(kvcache* c) {
  if (c && c->active_save) {
    kvcu_set_error("enableQuantization: a background save is reading the pool (kvcache_save_wait first)");
    return KVCU_ERR_INVALID_ARG;
  }
  if (!c) return KVCU_ERR_INVALID_ARG;
  if (c->quantized()) return KVCU_OK;
  DevScope d(c->device);
  kvcu_pool* q = kvcu_pool_create(c->device, c->n_layers, c->num_blocks, c->block_size, c->kv_rank,
                                  c->rope_dim, 1);
  if (!q) return KVCU_ERR_NO_MEMORY;
  cudaStreamSynchronize(c->stream);
  kvcu_pool_destroy(c->pool);
  c->pool = q;
  return KVCU_OK;
}

int kvcache_ensure_capacity(kvcache* c, uint32_t n_tokens) {
  return c ? seq_ensure(c, 0, n_tokens) : KVCU_ERR_INVALID_ARG;
}
void kvcache_truncate(kvcache* c, uint32_t n_tokens) {
  if (c) seq_truncate(c, 0, n_tokens);
}
void kvcache_reset(kvcache* c) {
  if (c) seq_reset(c, 0);
}

int kvcache_put(kvcache* c, uint32_t layer, uint32_t pos, const float* kv_comp, const float* k_pe) {
  if (!c || !kv_comp || !k_pe) return KVCU_ERR_INVALID_ARG;
  DevScope d(c->device);
  const uint32_t s0 = 0;
  int rc = validate_positions(c, layer, 1, &s0, &pos);
  if (!rc) rc = cow_for_write(c, 1, &s0, &pos, c->stream);
  if (rc) return rc;
  std::vector<float> row(c->row_width());
  memcpy(row.data(), kv_comp, c->kv_rank * 4);
  memcpy(row.data() + c->kv_rank, k_pe, c->rope_dim * 4);
  rc = append_host_rows(c, layer, 1, &s0, &pos, row.data());
  if (rc) return rc;
  bump_lens(c, 1, &s0, &pos);
  return KVCU_OK;
}

int kvcache_get_kv_compressed(kvcache* c, uint32_t layer, uint32_t pos, float* out) {
  if (!c || !out) return KVCU_ERR_INVALID_ARG;
  DevScope d(c->device);
  return get_row(c, layer, pos, out, nullptr);
}

int kvcache_get_kpe(kvcache* c, uint32_t layer, uint32_t pos, float* out) {
  if (!c || !out) return KVCU_ERR_INVALID_ARG;
  DevScope d(c->device);
  return get_row(c, layer, pos, nullptr, out);
}

uint32_t kvcache_len(const kvcache* c) { return c ? c->seqs[0].len : 0; }
uint32_t kvcache_num_blocks(const kvcache* c) { return c ? c->num_blocks : 0; }
uint32_t kvcache_block_size(const kvcache* c) { return c ? c->block_size : 0; }
int kvcache_quantized(const kvcache* c) { return c && c->quantized() ? 1 : 0; }
uint32_t kvcache_num_free_blocks(const kvcache* c) { return c ? (uint32_t)c->free_list.size() : 0; }
uint64_t kvcache_memory_usage(const kvcache* c) {
  // src/kv_cache.zig:439-443 reports the f32 pools' bytes
  return c ? (uint64_t)c->n_layers * c->num_blocks * c->block_size * c->row_width() * 4ull : 0;
}
uint32_t kvcache_block_table(const kvcache* c, uint32_t* out, uint32_t cap) {
  return kvcache_seq_block_table(c, 0, out, cap);
}
uint32_t kvcache_refcount(const kvcache* c, uint32_t id) {
  return c && id < c->num_blocks ? c->ref_count[id] : 0;
}
int kvcache_set_free_list(kvcache* c, const uint32_t* ids, uint32_t n) {
  if (!c || n > c->num_blocks || (n && !ids)) return KVCU_ERR_INVALID_ARG;
  for (uint32_t i = 0; i < n; ++i)
    if (ids[i] >= c->num_blocks || c->ref_count[ids[i]] != 0) return KVCU_ERR_INVALID_ARG;
  c->free_list.assign(ids, ids + n);
  return KVCU_OK;
}
kvcu_pool* kvcache_pool(kvcache* c) { return c ? c->pool : nullptr; }

// ---- prefix caching ----
uint64_t kvcache_compute_hash(const uint32_t* token_ids, uint32_t n, uint64_t prefix_hash) {
  std::vector<uint8_t> buf;
  buf.reserve(8 + 4 * (size_t)n);
  if (prefix_hash != kNoHash)
    for (int i = 0; i < 8; ++i) buf.push_back((uint8_t)(prefix_hash >> (8 * i)));
  for (uint32_t i = 0; i < n; ++i)
    for (int k = 0; k < 4; ++k) buf.push_back((uint8_t)(token_ids[i] >> (8 * k)));
  return xxh64(buf.data(), buf.size(), 0);
}

int kvcache_seq_cache_block(kvcache* c, uint32_t seq, uint32_t block_idx, const uint32_t* token_ids,
                            uint32_t n_tokens, uint64_t prefix_hash) {
  if (!c || seq >= c->seqs.size() || (n_tokens && !token_ids)) return KVCU_ERR_INVALID_ARG;
  Seq& q = c->seqs[seq];
  if (block_idx >= q.table.size() || n_tokens != c->block_size) return KVCU_OK;  // full blocks only
  const uint32_t id = q.table[block_idx];
  const uint64_t h = kvcache_compute_hash(token_ids, n_tokens, prefix_hash);
  auto it = c->hash_map.find(h);
  if (it != c->hash_map.end() && it->second != id) return KVCU_OK;  // collision: skip
  c->hash[id] = h;
  c->hash_map[h] = id;
  return KVCU_OK;
}

void kvcache_cache_block(kvcache* c, uint32_t block_idx, const uint32_t* token_ids,
                         uint32_t n_tokens, uint64_t prefix_hash) {
  if (c) kvcache_seq_cache_block(c, 0, block_idx, token_ids, n_tokens, prefix_hash);
}

uint32_t kvcache_find_prefix_blocks(kvcache* c, const uint32_t* tokens, uint32_t n) {
  if (!c) return 0;
  uint64_t prefix = kNoHash;
  uint32_t reusable = 0;
  const uint32_t bs = c->block_size;
  for (uint64_t start = 0; start + bs <= n; start += bs) {
    const uint64_t h = kvcache_compute_hash(tokens + start, bs, prefix);
    if (c->hash_map.find(h) == c->hash_map.end()) break;
    prefix = h;
    reusable += 1;
  }
  return reusable;
}

int kvcache_reuse_prefix_blocks(kvcache* c, const uint32_t* tokens, uint32_t n, uint32_t n_blocks) {
  return kvcache_seq_reuse_prefix_blocks(c, 0, tokens, n, n_blocks);
}

int kvcache_seq_reuse_prefix_blocks(kvcache* c, uint32_t seq, const uint32_t* tokens, uint32_t n,
                                    uint32_t n_blocks) {
  if (!c || seq >= c->seqs.size()) return KVCU_ERR_INVALID_ARG;
  if (n_blocks == 0) return KVCU_OK;
  const uint32_t bs = c->block_size;
  if ((uint64_t)n_blocks * bs > n || !tokens) return KVCU_ERR_INVALID_ARG;
  Seq& q = c->seqs[seq];
  uint64_t prefix = kNoHash;
  for (uint32_t bi = 0; bi < n_blocks; ++bi) {
    const uint64_t h = kvcache_compute_hash(tokens + (uint64_t)bi * bs, bs, prefix);
    auto it = c->hash_map.find(h);
    if (it == c->hash_map.end()) {
      kvcu_set_error("PrefixCacheMiss at block %u", bi);
      return KVCU_ERR_PREFIX_MISS;
    }
    const uint32_t cached = it->second;
    retain_block(c, cached);
    if (bi < q.table.size()) {
      release_block(c, q.table[bi]);
      q.table[bi] = cached;
    } else {
      q.table.push_back(cached);
    }
    prefix = h;
  }
  q.len = n_blocks * bs;
  c->tables_dirty = c->lens_dirty = true;
  c->epoch++;
  return KVCU_OK;
}

// ---- many sequences ----
int64_t kvcache_seq_create(kvcache* c) {
  if (!c) return KVCU_ERR_INVALID_ARG;
  c->seqs.emplace_back();
  c->tables_dirty = c->lens_dirty = true;
  return (int64_t)c->seqs.size() - 1;
}
uint32_t kvcache_num_seqs(const kvcache* c) { return c ? (uint32_t)c->seqs.size() : 0; }
int kvcache_seq_ensure_capacity(kvcache* c, uint32_t seq, uint32_t n_tokens) {
  return c ? seq_ensure(c, seq, n_tokens) : KVCU_ERR_INVALID_ARG;
}
int kvcache_seq_truncate(kvcache* c, uint32_t seq, uint32_t n_tokens) {
  if (!c || seq >= c->seqs.size()) return KVCU_ERR_INVALID_ARG;
  seq_truncate(c, seq, n_tokens);
  return KVCU_OK;
}
int kvcache_seq_reset(kvcache* c, uint32_t seq) {
  if (!c || seq >= c->seqs.size()) return KVCU_ERR_INVALID_ARG;
  seq_reset(c, seq);
  return KVCU_OK;
}
uint32_t kvcache_seq_len(const kvcache* c, uint32_t seq) {
  return c && seq < c->seqs.size() ? c->seqs[seq].len : 0;
}
uint32_t kvcache_seq_block_table(const kvcache* c, uint32_t seq, uint32_t* out, uint32_t cap) {
  if (!c || seq >= c->seqs.size()) return 0;
  const auto& t = c->seqs[seq].table;
  if (out) memcpy(out, t.data(), std::min<size_t>(cap, t.size()) * 4);
  return (uint32_t)t.size();
}

int kvcache_append_batch(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                         const uint32_t* positions, const float* rows) {
  if (!c || (n && (!seq_ids || !positions || !rows))) return KVCU_ERR_INVALID_ARG;
  if (!n) return KVCU_OK;
  DevScope d(c->device);
  int rc = validate_positions(c, layer, n, seq_ids, positions);
  if (!rc) rc = cow_for_write(c, n, seq_ids, positions, c->stream);
  if (rc) return rc;
  rc = append_host_rows(c, layer, n, seq_ids, positions, rows);
  if (rc) return rc;
  bump_lens(c, n, seq_ids, positions);
  return KVCU_OK;
}

int kvcache_append_batch_dev(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                             const uint32_t* positions, const uint32_t* seq_ids_dev,
                             const uint32_t* positions_dev, const float* rows_dev, void* stream) {
  if (!c || (n && (!seq_ids || !positions || !seq_ids_dev || !positions_dev || !rows_dev)))
    return KVCU_ERR_INVALID_ARG;
  if (!n) return KVCU_OK;
  DevScope d(c->device);
  int rc = validate_positions(c, layer, n, seq_ids, positions);
  if (!rc) rc = cow_for_write(c, n, seq_ids, positions, (cudaStream_t)stream);
  if (!rc) rc = sync_tables(c, (cudaStream_t)stream);
  if (!rc) rc = sync_lens(c, (cudaStream_t)stream);
  if (rc) return rc;
  const uint32_t Wd = c->row_width();
  rc = kvcu_append(c->pool, layer, n, rows_dev, Wd, rows_dev + c->kv_rank, Wd, seq_ids_dev,
                   positions_dev, (uint32_t)c->seqs.size(), c->d_toff, c->d_tables, c->d_lens,
                   stream);
  if (rc) return rc;
  c->last_launches = 1;
  bump_lens(c, n, seq_ids, positions);  // the kernel already advanced d_lens identically
  return KVCU_OK;
}

int kvcache_append_layers_dev(kvcache* c, uint32_t layer, uint32_t n_layers, uint32_t n, const uint32_t* seq_ids,
                              const uint32_t* positions, const uint32_t* seq_ids_dev, const uint32_t* positions_dev,
                              const float* rows_dev, uint64_t rows_layer_stride, void* stream) {
  if (!c || (n && (!seq_ids || !positions || !seq_ids_dev || !positions_dev || !rows_dev)))
    return KVCU_ERR_INVALID_ARG;
  if (n_layers == 0 || layer >= c->n_layers || n_layers > c->n_layers - layer) {
    kvcu_set_error("LayerOutOfBounds: layers [%u, %u + %u) of %u", layer, layer, n_layers, c->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if (!n) return KVCU_OK;
  DevScope d(c->device);
  const cudaStream_t st = (cudaStream_t)stream;
  int rc = validate_positions(c, layer, n, seq_ids, positions);
  if (!rc) rc = cow_for_write(c, n, seq_ids, positions, st);
  if (!rc) rc = sync_tables(c, st);
  if (!rc) rc = sync_lens(c, st);
  if (rc) return rc;
  const uint32_t Wd = c->row_width();
  rc = kvcu_append_layers(c->pool, layer, n_layers, n, rows_dev, Wd, rows_layer_stride, rows_dev + c->kv_rank, Wd,
                          rows_layer_stride, seq_ids_dev, positions_dev, (uint32_t)c->seqs.size(), c->d_toff,
                          c->d_tables, c->d_lens, stream);
  if (rc) return rc;
  c->last_launches = 1;
  bump_lens(c, n, seq_ids, positions);  // the kernel already advanced d_lens identically
  return KVCU_OK;
}

int kvcache_mla_decode_layers_dev(kvcache* c, uint32_t layer, uint32_t n_layers, uint32_t n,
                                  const uint32_t* seq_ids, const float* q_dev, uint64_t q_layer_stride,
                                  uint32_t n_heads, float scale, float* out_dev, uint64_t out_layer_stride,
                                  void* stream) {
  if (!c || (n && (!seq_ids || !q_dev || !out_dev))) return KVCU_ERR_INVALID_ARG;
  if (!n) return KVCU_OK;
  DevScope d(c->device);
  return decode_impl(c, layer, n, seq_ids, q_dev, n_heads, scale, out_dev, (cudaStream_t)stream, n_layers,
                     q_layer_stride, out_layer_stride);
}

int kvcache_append_decode_layers(kvcache* c, uint32_t layer, uint32_t n_layers, uint32_t n, const uint32_t* seq_ids,
                                 const uint32_t* positions, const float* rows, const float* q, uint32_t n_heads,
                                 float scale, float* out) {
  if (!c || (n && (!seq_ids || !positions || !rows || !q || !out))) return KVCU_ERR_INVALID_ARG;
  if (n_layers == 0 || layer >= c->n_layers || n_layers > c->n_layers - layer) {
    kvcu_set_error("LayerOutOfBounds: layers [%u, %u + %u) of %u", layer, layer, n_layers, c->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if (!n) return KVCU_OK;
  DevScope d(c->device);
  const cudaStream_t st = c->stream;
  const uint32_t Wd = c->row_width();
  // ---- the appends: rows by one DMA, row indices through pinned staging, one launch for all layers
  int rc = validate_positions(c, layer, n, seq_ids, positions);
  if (!rc) rc = cow_for_write(c, n, seq_ids, positions, st);
  if (!rc) rc = sync_tables(c, st);
  if (!rc) rc = sync_lens(c, st);
  const size_t rows_n = (size_t)n_layers * n * Wd;
  if (!rc) rc = ensure_dev(&c->d_step, &c->d_step_cap, rows_n);
  if (!rc) rc = ensure_dev(&c->d_u, &c->d_u_cap, (size_t)2 * n);
  if (!rc) rc = stage_acquire(c->up_rowidx, (size_t)2 * n);
  if (rc) return rc;
  KVCU_CUDA(cudaMemcpyAsync(c->d_step, rows, rows_n * 4, cudaMemcpyHostToDevice, st));
  memcpy(c->up_rowidx.p, seq_ids, (size_t)n * 4);
  memcpy(c->up_rowidx.p + n, positions, (size_t)n * 4);
  rc = stage_upload(c->up_rowidx, c->d_u, (size_t)2 * n, st);
  if (!rc)
    rc = kvcu_append_layers(c->pool, layer, n_layers, n, c->d_step, Wd, (uint64_t)n * Wd, c->d_step + c->kv_rank,
                            Wd, (uint64_t)n * Wd, c->d_u, c->d_u + n, (uint32_t)c->seqs.size(), c->d_toff,
                            c->d_tables, c->d_lens, st);
  if (rc) return rc;
  bump_lens(c, n, seq_ids, positions);
  uint32_t launches = 1;
  // ---- the decode of every layer: q / out in place when pinned and mapped, else copied
  const uint64_t qs = (uint64_t)n * n_heads * Wd, os = (uint64_t)n * n_heads * c->kv_rank;
  const void* q_map =
      c->host_io == KVCACHE_HOST_IO_AUTO ? mapped_host_range(q, (size_t)n_layers * qs * 4) : nullptr;
  void* out_map = q_map ? mapped_host_range(out, (size_t)n_layers * os * 4) : nullptr;
  if (c->host_io == KVCACHE_HOST_IO_COPY_IN) {
    // q by DMA before the kernels, out written in place by them
    out_map = mapped_host_range(out, (size_t)n_layers * os * 4);
    if (out_map) {
      rc = ensure_dev(&c->d_f, &c->d_f_cap, (size_t)n_layers * qs);
      if (rc) return rc;
      KVCU_CUDA(cudaMemcpyAsync(c->d_f, q, (size_t)n_layers * qs * 4, cudaMemcpyHostToDevice, st));
      q_map = c->d_f;
    }
  }
  c->last_mapped = (q_map && out_map) ? 1 : 0;
  if (c->last_mapped) {
    rc = decode_impl(c, layer, n, seq_ids, static_cast<const float*>(q_map), n_heads, scale,
                     static_cast<float*>(out_map), st, n_layers, qs, os);
    if (rc) return rc;
  } else {
    rc = ensure_dev(&c->d_f, &c->d_f_cap, (size_t)n_layers * qs);
    if (!rc) rc = ensure_dev(&c->d_f2, &c->d_f2_cap, (size_t)n_layers * os);
    if (rc) return rc;
    KVCU_CUDA(cudaMemcpyAsync(c->d_f, q, (size_t)n_layers * qs * 4, cudaMemcpyHostToDevice, st));
    rc = decode_impl(c, layer, n, seq_ids, c->d_f, n_heads, scale, c->d_f2, st, n_layers, qs, os);
    if (rc) return rc;
    KVCU_CUDA(cudaMemcpyAsync(out, c->d_f2, (size_t)n_layers * os * 4, cudaMemcpyDeviceToHost, st));
  }
  c->last_launches += launches;
  return check_status(c);  // the one synchronise: out is complete, rows / q may be reused
}

int kvcache_gather(kvcache* c, uint32_t layer, uint32_t seq, float* out) {
  if (!c || seq >= c->seqs.size()) return KVCU_ERR_INVALID_ARG;
  if (layer >= c->n_layers) return KVCU_ERR_LAYER_OOB;
  DevScope d(c->device);
  const Seq& q = c->seqs[seq];
  if (q.len == 0) return KVCU_OK;
  if (!out) return KVCU_ERR_INVALID_ARG;
  const uint32_t Wd = c->row_width();
  int rc = sync_tables(c, c->stream);
  if (!rc) rc = ensure_dev(&c->d_f, &c->d_f_cap, (size_t)q.len * Wd);
  if (rc) return rc;
  rc = kvcu_gather(c->pool, layer, c->d_tables + c->h_toff[seq], (uint32_t)q.table.size(), q.len,
                   c->d_f, c->stream);
  if (rc) return rc;
  KVCU_CUDA(cudaMemcpyAsync(out, c->d_f, (size_t)q.len * Wd * 4, cudaMemcpyDeviceToHost, c->stream));
  c->last_launches = 1;
  return check_status(c);
}

int kvcache_mla_decode(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                       const float* q, uint32_t n_heads, float scale, float* out) {
  if (!c || (n && (!seq_ids || !q || !out))) return KVCU_ERR_INVALID_ARG;
  if (!n) return KVCU_OK;
  DevScope d(c->device);
  const size_t qn = (size_t)n * n_heads * c->row_width(), on = (size_t)n * n_heads * c->kv_rank;
  // Pinned, mapped host buffers that hold the whole q / out: the kernels read
  // q and write out over the bus themselves, overlapped with the decode.
  const void* q_map = c->host_io == KVCACHE_HOST_IO_AUTO ? mapped_host_range(q, qn * 4) : nullptr;
  void* out_map = q_map ? mapped_host_range(out, on * 4) : nullptr;
  c->last_mapped = (q_map && out_map) ? 1 : 0;
  if (c->last_mapped) {
    int rc = decode_impl(c, layer, n, seq_ids, static_cast<const float*>(q_map), n_heads, scale,
                         static_cast<float*>(out_map), c->stream);
    if (rc) return rc;
    return check_status(c);  // synchronises: out is complete in host memory
  }
  int rc = ensure_dev(&c->d_f, &c->d_f_cap, qn);
  if (!rc) rc = ensure_dev(&c->d_f2, &c->d_f2_cap, on);
  if (rc) return rc;
  KVCU_CUDA(cudaMemcpyAsync(c->d_f, q, qn * 4, cudaMemcpyHostToDevice, c->stream));
  rc = decode_impl(c, layer, n, seq_ids, c->d_f, n_heads, scale, c->d_f2, c->stream);
  if (rc) return rc;
  KVCU_CUDA(cudaMemcpyAsync(out, c->d_f2, on * 4, cudaMemcpyDeviceToHost, c->stream));
  return check_status(c);  // synchronises; bad indices / timeouts become KVCU_ERR_DEVICE
}

int kvcache_mla_decode_dev(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                           const float* q_dev, uint32_t n_heads, float scale, float* out_dev,
                           void* stream) {
  if (!c || (n && (!seq_ids || !q_dev || !out_dev))) return KVCU_ERR_INVALID_ARG;
  if (!n) return KVCU_OK;
  DevScope d(c->device);
  return decode_impl(c, layer, n, seq_ids, q_dev, n_heads, scale, out_dev, (cudaStream_t)stream);
}

int kvcache_mla_step_dev(kvcache* c, uint32_t layer, uint32_t n, const uint32_t* seq_ids,
                         const uint32_t* positions, const float* q_dev, const float* kv_a_dev,
                         const float* norm_w_dev, float eps, float rope_base, const float* k_b_dev,
                         const float* v_b_dev, uint32_t n_heads, uint32_t qk_nope, uint32_t v_dim,
                         float scale, float* attn_dev, void* stream) {
  if (!c || (n && (!seq_ids || !positions || !q_dev || !kv_a_dev || !norm_w_dev || !k_b_dev ||
                   !v_b_dev || !attn_dev)))
    return KVCU_ERR_INVALID_ARG;
  if (!n) return KVCU_OK;
  DevScope d(c->device);
  const cudaStream_t st = (cudaStream_t)stream;
  int rc = validate_positions(c, layer, n, seq_ids, positions);
  if (!rc) rc = cow_for_write(c, n, seq_ids, positions, st);
  if (rc) return rc;
  const uint32_t R = c->kv_rank, Wd = c->row_width(), n_seqs = (uint32_t)c->seqs.size();
  // scratch: q_abs [n][H][W], rows [n][W], latent [n][H][R], lse [n][H], merge weights [n][H][3]
  const size_t q_abs_n = (size_t)n * n_heads * Wd, rows_n = (size_t)n * Wd, lat_n = (size_t)n * n_heads * R;
  rc = ensure_dev(&c->d_step, &c->d_step_cap, q_abs_n + rows_n + lat_n + (size_t)n * n_heads * 4);
  if (!rc) rc = ensure_dev(&c->d_stepu, &c->d_stepu_cap, 2 * (size_t)n + n_seqs);
  if (!rc) rc = sync_tables(c, st);
  if (!rc) rc = sync_lens(c, st);
  if (!rc) rc = ensure_ws(c, n, n_heads);
  if (rc) return rc;
  float* q_abs = c->d_step;
  float* rows = q_abs + q_abs_n;
  float* latent = rows + rows_n;
  float* lse = latent + lat_n;
  float* mrg_w = lse + (size_t)n * n_heads;  // [n][H][3] merge weights
  uint32_t* d_ids = c->d_stepu;
  uint32_t* d_pos = d_ids + n;
  uint32_t* d_hist = d_pos + n;
  // the decode covers each entry's history, positions < pos (the newest token
  // is merged by kvcu_mla_finish as the reference treats it)
  std::vector<uint32_t> hist(n_seqs, 0);
  std::vector<char> seen(n_seqs, 0);
  for (uint32_t b = 0; b < n; ++b) {
    if (seen[seq_ids[b]]) {
      kvcu_set_error("kvcache_mla_step_dev: sequence %u appears twice in the batch", seq_ids[b]);
      return KVCU_ERR_INVALID_ARG;
    }
    seen[seq_ids[b]] = 1;
    hist[seq_ids[b]] = positions[b];
  }
  KVCU_CUDA(cudaMemcpyAsync(d_ids, seq_ids, (size_t)n * 4, cudaMemcpyHostToDevice, st));
  KVCU_CUDA(cudaMemcpyAsync(d_pos, positions, (size_t)n * 4, cudaMemcpyHostToDevice, st));
  KVCU_CUDA(cudaMemcpyAsync(d_hist, hist.data(), (size_t)n_seqs * 4, cudaMemcpyHostToDevice, st));
  rc = kvcu_mla_prepare(c->pool, n, n_heads, qk_nope, q_dev, kv_a_dev, d_pos, norm_w_dev, eps, rope_base,
                        k_b_dev, q_abs, rows, st);
  if (!rc)
    rc = kvcu_append(c->pool, layer, n, rows, Wd, rows + R, Wd, d_ids, d_pos, n_seqs, c->d_toff, c->d_tables,
                     c->d_lens, st);
  if (rc) return rc;
  bump_lens(c, n, seq_ids, positions);  // the append kernel advanced d_lens identically
  // The plan depends only on the batch and its history lengths, which the
  // layers of one step share: the first layer plans, the others reuse it.
  const bool same_plan = c->mla_plan_serial == c->plan_serial && c->mla_plan_ids.size() == n &&
                         std::equal(c->mla_plan_ids.begin(), c->mla_plan_ids.end(), seq_ids) &&
                         std::equal(c->mla_plan_hist.begin(), c->mla_plan_hist.end(), positions);
  if (!same_plan) {
    rc = kvcu_decode_plan(c->ws, c->pool, n, d_ids, n_seqs, d_hist, st);
    c->plan_epoch = ~0ull;  // the cached decode plan no longer matches the workspace
    c->mla_plan_serial = rc ? ~0ull : ++c->plan_serial;
    c->mla_plan_ids.assign(seq_ids, seq_ids + n);
    c->mla_plan_hist.assign(positions, positions + n);
  }
  if (!rc)
    rc = kvcu_mla_decode_lse(c->ws, c->pool, layer, n, d_ids, n_seqs, c->d_toff, c->d_tables, d_hist, q_abs,
                             n_heads, scale, latent, lse, st);
  if (!rc)
    rc = kvcu_mla_finish_fused(c->pool, n, n_heads, v_dim, q_abs, rows, latent, lse, mrg_w, scale, v_b_dev, attn_dev,
                               st);
  if (rc) return rc;
  // rows, gemm (prepare) + append + plan + decode + merge, gemm (finish). The
  // three host arrays above are pageable: each cudaMemcpyAsync returned only
  // after staging them, so they may go out of scope now.
  c->last_launches = 2 + 1 + (same_plan ? 0 : 1) + kvcu_decode_last_launches(c->ws) + 2;
  return KVCU_OK;
}

uint32_t kvcache_last_launches(const kvcache* c) { return c ? c->last_launches : 0; }

int kvcache_last_decode_mapped(const kvcache* c) { return c ? c->last_mapped : 0; }

int kvcache_set_host_io(kvcache* c, int mode) {
  if (!c || mode < KVCACHE_HOST_IO_AUTO || mode > KVCACHE_HOST_IO_COPY_IN) return KVCU_ERR_INVALID_ARG;
  c->host_io = mode;
  return KVCU_OK;
}

int kvcache_set_decode_impl(kvcache* c, int impl) {
  if (!c || impl < KVCU_DECODE_AUTO || impl > KVCU_DECODE_TENSOR_CORE) return KVCU_ERR_INVALID_ARG;
  c->decode_impl = impl;
  return c->ws ? kvcu_decode_ws_set_impl(c->ws, impl) : KVCU_OK;
}

int kvcache_last_decode_impl(const kvcache* c) { return c && c->ws ? kvcu_decode_last_impl(c->ws) : 0; }

// ---- checkpoints ----
namespace {

constexpr size_t kIoChunk = 64ull << 20;

// Two host buffers for the pool section of a checkpoint, pinned so that the
// device copies run at full bus speed (pageable ones if pinning fails).
struct IoBuffers {
  uint8_t* pinned[2] = {nullptr, nullptr};
  std::vector<uint8_t> pageable[2];
  explicit IoBuffers(size_t n) {
    for (int i = 0; i < 2; ++i)
      if (cudaHostAlloc(reinterpret_cast<void**>(&pinned[i]), n, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        pinned[i] = nullptr;
        pageable[i].resize(n);
      }
  }
  ~IoBuffers() {
    for (int i = 0; i < 2; ++i)
      if (pinned[i]) cudaFreeHost(pinned[i]);
  }
  uint8_t* operator[](int i) { return pinned[i] ? pinned[i] : pageable[i].data(); }
};

// Save: while a helper thread writes chunk k to the file, the device packs and
// copies chunk k+1 into the other buffer.
int write_pool(kvcache* c, int fd) {
  kvcu_pool_desc desc;
  int rc = kvcu_pool_describe(c->pool, &desc);
  if (rc) return rc;
  const uint64_t total = desc.checkpoint_bytes;
  const size_t chunk = (size_t)std::min<uint64_t>(kIoChunk, std::max<uint64_t>(total, 1));
  IoBuffers bufs(chunk);
  std::thread writer;
  int wrc = KVCU_OK;
  uint64_t k = 0;
  for (uint64_t off = 0; off < total; off += chunk, ++k) {
    const uint64_t n = std::min<uint64_t>(chunk, total - off);
    uint8_t* b = bufs[(int)(k & 1)];
    rc = kvcu_pool_read_checkpoint(c->pool, off, n, b, c->stream);  // returns with b filled
    if (writer.joinable()) writer.join();  // chunk k-1, in the other buffer, is written
    if (rc || wrc) break;
    writer = std::thread([&wrc, fd, b, n]() { wrc = write_all(fd, b, n); });
  }
  if (writer.joinable()) writer.join();
  if (!rc && wrc) kvcu_set_error("checkpoint write failed");
  return rc ? rc : wrc;
}

// Load: while chunk k goes to the device, a helper thread reads chunk k+1 from
// the file into the other buffer.
int read_pool(kvcache* c, int fd) {
  kvcu_pool_desc desc;
  int rc = kvcu_pool_describe(c->pool, &desc);
  if (rc) return rc;
  const uint64_t total = desc.checkpoint_bytes;
  if (!total) return KVCU_OK;
  const size_t chunk = (size_t)std::min<uint64_t>(kIoChunk, total);
  IoBuffers bufs(chunk);
  rc = read_no_eof(fd, bufs[0], (size_t)std::min<uint64_t>(chunk, total));
  if (rc) return rc;
  int rrc = KVCU_OK;
  uint64_t k = 0;
  for (uint64_t off = 0; off < total; off += chunk, ++k) {
    const uint64_t n = std::min<uint64_t>(chunk, total - off);
    std::thread reader;
    if (off + chunk < total) {
      uint8_t* nb = bufs[(int)((k + 1) & 1)];
      const uint64_t nn = std::min<uint64_t>(chunk, total - off - chunk);
      reader = std::thread([&rrc, fd, nb, nn]() { rrc = read_no_eof(fd, nb, nn); });
    }
    rc = kvcu_pool_write_checkpoint(c->pool, off, n, bufs[(int)(k & 1)], c->stream);
    if (reader.joinable()) reader.join();
    if (rc) return rc;
    if (rrc) {
      kvcu_set_error("checkpoint truncated or unreadable");
      return rrc;
    }
  }
  return KVCU_OK;
}

// Rebuild refcounts / free list from the sequences' tables (v2 load).
void rebuild_allocator(kvcache* c) {
  std::fill(c->ref_count.begin(), c->ref_count.end(), 0u);
  std::fill(c->hash.begin(), c->hash.end(), kNoHash);
  c->hash_map.clear();
  for (auto& s : c->seqs)
    for (uint32_t id : s.table) c->ref_count[id] += 1;
  c->free_list.clear();
  for (uint32_t i = c->num_blocks; i-- > 0;)
    if (c->ref_count[i] == 0) c->free_list.push_back(i);  // pops hand out the lowest id first
}

}  // namespace

// src/kv_cache.zig:453-494 (CheckpointHeader :549-560: magic@0 version@4 len@8
// quantized@12 pad@13..15 block_table_len@16 num_layers@20 num_blocks@24
// block_size@28 kv_rank@32 rope_dim@36).
int kvcache_save_to_file(kvcache* c, const char* path) {
  if (!c || !path) return KVCU_ERR_INVALID_ARG;
  DevScope d(c->device);
  int rc = cudaStreamSynchronize(c->stream) == cudaSuccess ? KVCU_OK : KVCU_ERR_CUDA;
  if (rc) return rc;
  Fd f(open(path, O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644));
  if (f.fd < 0) {
    kvcu_set_error("open(%s): %s", path, strerror(errno));
    return KVCU_ERR_IO;
  }
  const Seq& q = c->seqs[0];
  uint8_t h[40];
  memset(h, 0, sizeof(h));
  memcpy(h, "KVCK", 4);
  put_le32(h + 4, 1);
  put_le32(h + 8, q.len);
  h[12] = c->quantized() ? 1 : 0;
  put_le32(h + 16, (uint32_t)q.table.size());
  put_le32(h + 20, c->n_layers);
  put_le32(h + 24, c->num_blocks);
  put_le32(h + 28, c->block_size);
  put_le32(h + 32, c->kv_rank);
  put_le32(h + 36, c->rope_dim);
  rc = write_all(f.fd, h, sizeof(h));
  if (rc) return rc;
  std::vector<uint8_t> tb(q.table.size() * 4);
  for (size_t i = 0; i < q.table.size(); ++i) put_le32(tb.data() + 4 * i, q.table[i]);
  if (!tb.empty()) rc = write_all(f.fd, tb.data(), tb.size());
  if (rc) return rc;
  return write_pool(c, f.fd);
}

// src/kv_cache.zig:497-546 with block-id validation and free-list removal.
int kvcache_load_from_file(kvcache* c, const char* path) {
  if (!c || !path) return KVCU_ERR_INVALID_ARG;
  if (c->active_save) {
    kvcu_set_error("loadFromFile: a background save is reading the pool (kvcache_save_wait first)");
    return KVCU_ERR_INVALID_ARG;
  }
  // A v1 file holds one sequence and overwrites the whole pool; with other
  // sequences holding blocks it would clobber their rows and could hand one of
  // their blocks to sequence 0 as well.  The reference's cache has a single
  // sequence, so refuse instead of guessing (the v2 format keeps them all).
  for (size_t s = 1; s < c->seqs.size(); ++s)
    if (!c->seqs[s].table.empty() || c->seqs[s].len) {
      kvcu_set_error("loadFromFile: sequence %zu of this cache holds blocks; a v1 checkpoint restores a "
                     "single-sequence cache (use kvcache_load_from_file_v2)",
                     s);
      return KVCU_ERR_INVALID_ARG;
    }
  DevScope d(c->device);
  Fd f(open(path, O_RDONLY | O_CLOEXEC));
  if (f.fd < 0) {
    kvcu_set_error("open(%s): %s", path, strerror(errno));
    return KVCU_ERR_IO;
  }
  uint8_t h[40];
  int rc = read_no_eof(f.fd, h, sizeof(h));
  if (rc) return rc;
  if (memcmp(h, "KVCK", 4) != 0) {
    kvcu_set_error("InvalidCheckpointMagic");
    return KVCU_ERR_BAD_MAGIC;
  }
  if (le32(h + 4) != 1) {
    kvcu_set_error("UnsupportedCheckpointVersion %u (v1 loader)", le32(h + 4));
    return KVCU_ERR_BAD_VERSION;
  }
  if (le32(h + 20) != c->n_layers || le32(h + 24) != c->num_blocks ||
      le32(h + 28) != c->block_size || le32(h + 32) != c->kv_rank || le32(h + 36) != c->rope_dim) {
    kvcu_set_error("CheckpointShapeMismatch");
    return KVCU_ERR_SHAPE_MISMATCH;
  }
  const uint32_t len = le32(h + 8), tlen = le32(h + 16);
  const bool quant = h[12] == 1;
  if (tlen > c->num_blocks || (uint64_t)len > (uint64_t)tlen * c->block_size ||
      (!quant && c->quantized())) {
    kvcu_set_error("CheckpointShapeMismatch (table %u, len %u, quantized %d)", tlen, len, (int)quant);
    return KVCU_ERR_SHAPE_MISMATCH;
  }
  std::vector<uint32_t> ids(tlen);
  if (tlen) {
    std::vector<uint8_t> tb(4 * (size_t)tlen);
    rc = read_no_eof(f.fd, tb.data(), tb.size());
    if (rc) return rc;
    for (uint32_t i = 0; i < tlen; ++i) {
      ids[i] = le32(tb.data() + 4 * i);
      if (ids[i] >= c->num_blocks) {
        kvcu_set_error("checkpoint block id %u >= num_blocks %u", ids[i], c->num_blocks);
        return KVCU_ERR_BAD_BLOCK_ID;
      }
    }
  }
  if (quant && !c->quantized()) {
    rc = kvcache_enable_quantization(c);
    if (rc) return rc;
  }
  rc = read_pool(c, f.fd);
  if (rc) return rc;
  Seq& q = c->seqs[0];
  for (uint32_t id : q.table) release_block(c, id);
  q.table.clear();
  for (uint32_t id : ids) {
    if (c->ref_count[id] == 0) take_off_free_list(c, id);
    retain_block(c, id);
    q.table.push_back(id);
  }
  q.len = len;
  c->tables_dirty = c->lens_dirty = true;
  c->epoch++;
  return KVCU_OK;
}

// v2 (many sequences): magic "KVCK", version 2 @4, n_seqs @8, quantized @12,
// pad @13..15, num_layers @16, num_blocks @20, block_size @24, kv_rank @28,
// rope_dim @32, total table entries @36, reserved u64 @40 (48 bytes); then
// n_seqs x (len u32, table_len u32); then all tables (u32 LE); then the pool
// section in the v1 order.
int kvcache_save_to_file_v2(kvcache* c, const char* path) {
  if (!c || !path) return KVCU_ERR_INVALID_ARG;
  DevScope d(c->device);
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return KVCU_ERR_CUDA;
  Fd f(open(path, O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644));
  if (f.fd < 0) {
    kvcu_set_error("open(%s): %s", path, strerror(errno));
    return KVCU_ERR_IO;
  }
  uint64_t total = 0;
  for (auto& s : c->seqs) total += s.table.size();
  uint8_t h[48];
  memset(h, 0, sizeof(h));
  memcpy(h, "KVCK", 4);
  put_le32(h + 4, 2);
  put_le32(h + 8, (uint32_t)c->seqs.size());
  h[12] = c->quantized() ? 1 : 0;
  put_le32(h + 16, c->n_layers);
  put_le32(h + 20, c->num_blocks);
  put_le32(h + 24, c->block_size);
  put_le32(h + 28, c->kv_rank);
  put_le32(h + 32, c->rope_dim);
  put_le32(h + 36, (uint32_t)total);
  int rc = write_all(f.fd, h, sizeof(h));
  if (rc) return rc;
  std::vector<uint8_t> meta(8 * c->seqs.size() + 4 * total);
  size_t o = 0;
  for (auto& s : c->seqs) {
    put_le32(meta.data() + o, s.len);
    put_le32(meta.data() + o + 4, (uint32_t)s.table.size());
    o += 8;
  }
  for (auto& s : c->seqs)
    for (uint32_t id : s.table) {
      put_le32(meta.data() + o, id);
      o += 4;
    }
  if (!meta.empty()) rc = write_all(f.fd, meta.data(), meta.size());
  if (rc) return rc;
  return write_pool(c, f.fd);
}

int kvcache_load_from_file_v2(kvcache* c, const char* path) {
  if (!c || !path) return KVCU_ERR_INVALID_ARG;
  if (c->active_save) {
    kvcu_set_error("loadFromFile: a background save is reading the pool (kvcache_save_wait first)");
    return KVCU_ERR_INVALID_ARG;
  }
  DevScope d(c->device);
  Fd f(open(path, O_RDONLY | O_CLOEXEC));
  if (f.fd < 0) {
    kvcu_set_error("open(%s): %s", path, strerror(errno));
    return KVCU_ERR_IO;
  }
  uint8_t h[48];
  int rc = read_no_eof(f.fd, h, sizeof(h));
  if (rc) return rc;
  if (memcmp(h, "KVCK", 4) != 0) return KVCU_ERR_BAD_MAGIC;
  if (le32(h + 4) != 2) {
    kvcu_set_error("UnsupportedCheckpointVersion %u (v2 loader)", le32(h + 4));
    return KVCU_ERR_BAD_VERSION;
  }
  if (le32(h + 16) != c->n_layers || le32(h + 20) != c->num_blocks ||
      le32(h + 24) != c->block_size || le32(h + 28) != c->kv_rank || le32(h + 32) != c->rope_dim)
    return KVCU_ERR_SHAPE_MISMATCH;
  const uint32_t n_seqs = le32(h + 8), total = le32(h + 36);
  const bool quant = h[12] == 1;
  if (n_seqs == 0 || (!quant && c->quantized())) return KVCU_ERR_SHAPE_MISMATCH;
  std::vector<uint8_t> meta(8ull * n_seqs + 4ull * total);
  rc = read_no_eof(f.fd, meta.data(), meta.size());
  if (rc) return rc;
  std::vector<Seq> seqs(n_seqs);
  uint64_t sum = 0;
  for (uint32_t s = 0; s < n_seqs; ++s) {
    seqs[s].len = le32(meta.data() + 8 * s);
    const uint32_t tl = le32(meta.data() + 8 * s + 4);
    seqs[s].table.resize(tl);
    sum += tl;
    if ((uint64_t)seqs[s].len > (uint64_t)tl * c->block_size) return KVCU_ERR_SHAPE_MISMATCH;
  }
  if (sum != total) return KVCU_ERR_SHAPE_MISMATCH;
  size_t o = 8ull * n_seqs;
  for (auto& s : seqs)
    for (auto& id : s.table) {
      id = le32(meta.data() + o);
      o += 4;
      if (id >= c->num_blocks) return KVCU_ERR_BAD_BLOCK_ID;
    }
  if (quant && !c->quantized()) {
    rc = kvcache_enable_quantization(c);
    if (rc) return rc;
  }
  rc = read_pool(c, f.fd);
  if (rc) return rc;
  c->seqs = std::move(seqs);
  rebuild_allocator(c);
  c->tables_dirty = c->lens_dirty = true;
  c->epoch++;
  return KVCU_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- background save
// A v2 checkpoint written while serving goes on.  At the call, the header and
// every sequence's length and block table are captured and every block in
// those tables is retained once more, so (i) no block of the snapshot returns
// to the free list and (ii) any write into one of them first copies it to a
// fresh block (copy-on-write, as for shared prefix blocks).  The snapshot's
// rows therefore stay as they were while a worker thread copies the pool
// section device -> pinned host -> file on its own stream, overlapped with
// the caller's kernels; kvcache_save_wait joins it and drops the extra refs.
struct kvcache_save {
  kvcache* c = nullptr;
  std::thread worker;
  std::atomic<int> done{0};
  int rc = KVCU_OK;
  char err[512] = {0};
  std::vector<uint32_t> held;  // blocks retained for the snapshot
  uint64_t bytes = 0;
};

namespace {

constexpr size_t kSaveChunk = 64ull << 20;

void save_worker(kvcache_save* job, int device, kvcu_pool* pool, std::string path, std::vector<uint8_t> head,
                 cudaEvent_t start, uint8_t* stg, uint8_t* hbuf0, uint8_t* hbuf1) {
  int rc = kvcu_check_cuda(cudaSetDevice(device), "cudaSetDevice(save worker)");
  cudaStream_t st = nullptr;
  if (!rc) rc = kvcu_check_cuda(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate(save)");
  // the pool section is read only after the work queued before the call
  if (!rc) rc = kvcu_check_cuda(cudaStreamWaitEvent(st, start, 0), "cudaStreamWaitEvent(save)");
  Fd f(rc ? -1 : open(path.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644));
  if (!rc && f.fd < 0) {
    kvcu_set_error("open(%s): %s", path.c_str(), strerror(errno));
    rc = KVCU_ERR_IO;
  }
  if (!rc) rc = write_all(f.fd, head.data(), head.size());
  uint64_t written = head.size();
  kvcu_pool_desc desc;
  if (!rc) rc = kvcu_pool_describe(pool, &desc);
  if (!rc) {
    // chunk k is copied into one buffer while the file write of chunk k-1 from
    // the other runs in a helper thread
    uint8_t* bufs[2] = {hbuf0, hbuf1};
    const uint64_t total = desc.checkpoint_bytes;
    std::thread writer;
    int wrc = KVCU_OK;
    uint64_t k = 0;
    for (uint64_t off = 0; off < total; off += kSaveChunk, ++k) {
      const uint64_t n = std::min<uint64_t>(kSaveChunk, total - off);
      uint8_t* b = bufs[k & 1];
      rc = kvcu_pool_read_checkpoint_staged(pool, off, n, b, st, stg, kSaveChunk);
      if (writer.joinable()) writer.join();
      if (rc || wrc) break;
      writer = std::thread([&wrc, fd = f.fd, b, n]() { wrc = write_all(fd, b, n); });
      written += n;
    }
    if (writer.joinable()) writer.join();
    if (!rc && wrc) {
      kvcu_set_error("checkpoint write failed");
      rc = wrc;
    }
  }
  if (st) cudaStreamDestroy(st);
  cudaEventDestroy(start);
  job->rc = rc;
  job->bytes = written;
  if (rc) snprintf(job->err, sizeof(job->err), "%s", kvcu_get_last_error());
  job->done.store(1);
}

}  // namespace

extern "C" {

int kvcache_save_to_file_v2_async(kvcache* c, const char* path, void* stream, kvcache_save** job_out) {
  if (!c || !path || !job_out) return KVCU_ERR_INVALID_ARG;
  *job_out = nullptr;
  if (c->active_save) {
    kvcu_set_error("a background save of this cache is already running");
    return KVCU_ERR_INVALID_ARG;
  }
  DevScope d(c->device);
  // buffers kept across saves: device staging for the Q8_0 repacking, two pinned chunks
  if (!c->save_stg) KVCU_CUDA(cudaMalloc(&c->save_stg, kSaveChunk));
  for (auto& h : c->save_host)
    if (!h) KVCU_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h), kSaveChunk, cudaHostAllocDefault));
  // start after the caller's stream and the cache's own stream
  cudaEvent_t start = nullptr;
  KVCU_CUDA(cudaEventCreateWithFlags(&start, cudaEventDisableTiming));
  if (stream) {
    KVCU_CUDA(cudaEventRecord(start, (cudaStream_t)stream));
    KVCU_CUDA(cudaStreamWaitEvent(c->stream, start, 0));
  }
  KVCU_CUDA(cudaEventRecord(start, c->stream));
  // header and tables as kvcache_save_to_file_v2 writes them, captured now
  uint64_t total = 0;
  for (auto& s : c->seqs) total += s.table.size();
  std::vector<uint8_t> head(48 + 8 * c->seqs.size() + 4 * total, 0);
  uint8_t* h = head.data();
  memcpy(h, "KVCK", 4);
  put_le32(h + 4, 2);
  put_le32(h + 8, (uint32_t)c->seqs.size());
  h[12] = c->quantized() ? 1 : 0;
  put_le32(h + 16, c->n_layers);
  put_le32(h + 20, c->num_blocks);
  put_le32(h + 24, c->block_size);
  put_le32(h + 28, c->kv_rank);
  put_le32(h + 32, c->rope_dim);
  put_le32(h + 36, (uint32_t)total);
  size_t o = 48;
  for (auto& s : c->seqs) {
    put_le32(h + o, s.len);
    put_le32(h + o + 4, (uint32_t)s.table.size());
    o += 8;
  }
  kvcache_save* job = new (std::nothrow) kvcache_save();
  if (!job) {
    cudaEventDestroy(start);
    return KVCU_ERR_NO_MEMORY;
  }
  job->c = c;
  job->held.reserve(total);
  for (auto& s : c->seqs)
    for (uint32_t id : s.table) {
      put_le32(h + o, id);
      o += 4;
      retain_block(c, id);  // the snapshot's own reference
      job->held.push_back(id);
    }
  c->active_save = job;
  job->worker = std::thread(save_worker, job, c->device, c->pool, std::string(path), std::move(head), start,
                            c->save_stg, c->save_host[0], c->save_host[1]);
  *job_out = job;
  return KVCU_OK;
}

int kvcache_save_done(const kvcache_save* job) { return job ? job->done.load() : 1; }

int kvcache_save_wait(kvcache_save* job) {
  if (!job) return KVCU_ERR_INVALID_ARG;
  if (job->worker.joinable()) job->worker.join();
  kvcache* c = job->c;
  for (uint32_t id : job->held) release_block(c, id);  // blocks no sequence holds any more go back
  if (c->active_save == job) c->active_save = nullptr;
  const int rc = job->rc;
  if (rc) kvcu_set_error("%s", job->err);
  delete job;
  return rc;
}

}  // extern "C"
