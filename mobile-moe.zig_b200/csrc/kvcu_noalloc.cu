// kvcu_noalloc.cu — MLA decode that allocates nothing (kvcu_mla_decode_noalloc).
//
// For callers that cannot allocate device memory when they decode: the split-KV
// scratch that kvcu_decode_ws_create would cudaMalloc (work items, the plan's
// per-entry item ranges, per-item partial outputs and softmax statistics) is a
// fixed array compiled into this translation unit, one per device.  CUDA loads
// a module's device memory lazily (on first use), so kvcu_init (which every
// pool creation calls) looks the array up on its device: that is the moment
// the memory is reserved, before any serving starts.  The call plans and decodes with
// the same kernels as kvcu_decode_plan + kvcu_mla_decode; only where the
// scratch lives, and the plan's range count (bounded by the array), differ.
//
// Nothing in the scratch needs clearing between calls: the plan kernel writes
// every field the decode reads (item list, item count, CTA ranges, per-entry
// first item and item count), and the decode writes every partial before the
// combine reads it.
#include <cuda_runtime.h>

#include <mutex>

#include "kvcu_internal.h"

namespace {

constexpr uint32_t kMaxBatch = KVCU_NOALLOC_MAX_BATCH;
constexpr uint32_t kMaxHeads = KVCU_NOALLOC_MAX_HEADS;
constexpr uint32_t kMaxItems = KVCU_NOALLOC_MAX_ITEMS;
constexpr int kMaxDevices = 64;

// Scratch layout (byte offsets inside the array); every part 256-aligned.
constexpr size_t align256(size_t x) { return (x + 255) / 256 * 256; }
constexpr size_t kPartO = 0;                                                  // f32 [items][heads][512]
constexpr size_t kPartMl = align256(kPartO + (size_t)kMaxItems * kMaxHeads * 512 * 4);  // f32 [items][heads][2]
constexpr size_t kItems = align256(kPartMl + (size_t)kMaxItems * kMaxHeads * 2 * 4);   // kvcu_item [items]
constexpr size_t kMeta = align256(kItems + (size_t)kMaxItems * sizeof(kvcu_item));     // u32 [4]
constexpr size_t kRanges = align256(kMeta + 4 * 4);                                   // u32 [items + 1]
constexpr size_t kSeqFirst = align256(kRanges + ((size_t)kMaxItems + 1) * 4);         // u32 [batch]
constexpr size_t kSeqCount = align256(kSeqFirst + (size_t)kMaxBatch * 4);            // u32 [batch]
constexpr size_t kScratchBytes = align256(kSeqCount + (size_t)kMaxBatch * 4);
static_assert(sizeof(kvcu_item) == 16, "item layout");
static_assert(kScratchBytes >= (size_t)KVCU_NOALLOC_SCRATCH_BYTES &&
                  kScratchBytes <= (size_t)KVCU_NOALLOC_SCRATCH_BYTES + 7 * 256,
              "the header's stated scratch size");

}  // namespace

// The scratch itself: device memory reserved with the module, never allocated
// or freed by this library.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

namespace {

std::mutex g_setup_mutex;
unsigned char* g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's scratch (looked up once per device, with the
// device current).
int scratch_for_device(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) {
    kvcu_set_error("kvcu_mla_decode_noalloc: device %d outside [0, %d)", device, kMaxDevices);
    return KVCU_ERR_INVALID_ARG;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[device]) {
    void* ptr = nullptr;
    const int rc = kvcu_check_cuda(cudaGetSymbolAddress(&ptr, g_noalloc_scratch),
                                   "cudaGetSymbolAddress(no-alloc decode scratch)");
    if (rc) return rc;
    g_scratch_ptr[device] = static_cast<unsigned char*>(ptr);
  }
  *out = g_scratch_ptr[device];
  return KVCU_OK;
}

}  // namespace

// Called by kvcu_init with `device` current: loads the module that holds the
// scratch and resolves its address, so the reservation happens at set-up.
int kvcu_noalloc_prepare(int device) {
  unsigned char* base = nullptr;
  return scratch_for_device(device, &base);
}

extern "C" int kvcu_mla_decode_noalloc(kvcu_pool* p, uint32_t layer, uint32_t n,
                                       const uint32_t* seq_ids, uint32_t n_seqs,
                                       const uint32_t* table_offsets, const uint32_t* tables,
                                       const uint32_t* lens, const float* q, uint32_t n_heads,
                                       float scale, float* out, void* stream) {
  if (!p || !(p->kv || p->qs)) return KVCU_ERR_INVALID_ARG;
  if (layer >= p->n_layers) {
    kvcu_set_error("kvcu_mla_decode_noalloc: layer %u >= n_layers %u", layer, p->n_layers);
    return KVCU_ERR_LAYER_OOB;
  }
  if (n > kMaxBatch) {
    kvcu_set_error("kvcu_mla_decode_noalloc: batch %u exceeds the fixed scratch limit %u", n, kMaxBatch);
    return KVCU_ERR_INVALID_ARG;
  }
  if (n_heads == 0 || n_heads > kMaxHeads) {
    kvcu_set_error("kvcu_mla_decode_noalloc: n_heads=%u outside [1, %u]", n_heads, kMaxHeads);
    return KVCU_ERR_INVALID_ARG;
  }
  if (n && (!table_offsets || !tables || !lens || !q || !out)) return KVCU_ERR_INVALID_ARG;

  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (prev != p->device) {
    const int rc = kvcu_check_cuda(cudaSetDevice(p->device), "cudaSetDevice");
    if (rc) return rc;
  }
  int rc = KVCU_OK;
  unsigned char* base = nullptr;
  rc = scratch_for_device(p->device, &base);
  if (!rc) {
    // a workspace view of the fixed scratch (host-side struct on the stack)
    kvcu_decode_ws ws = {};
    ws.device = p->device;
    ws.max_batch = kMaxBatch;
    ws.max_heads = kMaxHeads;
    ws.max_items = kMaxItems;
    ws.max_ranges = kMaxItems;
    ws.items = reinterpret_cast<kvcu_item*>(base + kItems);
    ws.meta = reinterpret_cast<uint32_t*>(base + kMeta);
    ws.ranges = reinterpret_cast<uint32_t*>(base + kRanges);
    ws.seq_first = reinterpret_cast<uint32_t*>(base + kSeqFirst);
    ws.seq_count = reinterpret_cast<uint32_t*>(base + kSeqCount);
    ws.part_o = reinterpret_cast<float*>(base + kPartO);
    ws.part_ml = reinterpret_cast<float*>(base + kPartMl);
    ws.impl = KVCU_DECODE_AUTO;
    rc = kvcu_decode_setup(&ws);
    if (!rc && n) {
      // at most n + ranges - 1 items: keep them within the array
      uint32_t ranges = (uint32_t)ws.decode_ctas;
      if (ranges > kMaxItems - n) ranges = kMaxItems - n;
      const cudaStream_t st = (cudaStream_t)stream;
      rc = kvcu_launch_plan_target(&ws, p, n, seq_ids, n_seqs, lens, ranges, st);
      if (!rc)
        rc = kvcu_launch_decode(&ws, p, layer, n, seq_ids, n_seqs, table_offsets, tables, lens, q,
                                n_heads, scale, out, nullptr, st);
    }
  }
  if (prev >= 0 && prev != p->device) cudaSetDevice(prev);
  return rc;
}
