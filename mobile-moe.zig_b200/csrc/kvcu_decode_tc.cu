// kvcu_decode_tc.cu — paged MLA decode on the sm_100a tensor cores (tcgen05 + TMA).
//
// Same contract as k_decode in kvcu_decode.cu (the attention core of
// src/inference.zig:518-660 in absorbed form, over a Q8_0 pool), same work
// items and partial format, so k_plan / k_combine are shared.  One persistent
// CTA per SM, 16 warps in 4 warpgroups with fixed roles:
//
//   warp 0      TMA producer: per 128-token tile, the Q8_0 payload rows of the
//               sequence's physical blocks (2-D tensor maps over the pool,
//               128B swizzle for the 512 latent bytes, 64B for the 64 rope
//               bytes) and the f16 scales (1-D bulk copies) -> raw stage ring (2).
//   warp 1      TMEM owner + QK issuer: 18 x tcgen05.mma.kind::i8 per tile, one
//               per Q8_0 block (A = the raw int8 tile [128 tok x 32], B = the
//               query as two int8 digits [2H x 32]): exact int32 dot products
//               per block into a ring of 3 TMEM slot pairs.
//   warp 2      PV issuer: per 16-token V chunk, four tcgen05.mma.kind::f16
//               (M = 128 latent columns, N = 32 heads, K = 16 tokens):
//               O^T += V^T P^T, accumulated in TMEM across the whole work item,
//               and l = ones x P^T by one more MMA.
//   warps 4-11  epilogue (two halves of the heads, each over all 128 token
//               rows): combine the 18 per-block dot products with the block
//               scales, online softmax over the tile (lazy rescale of O / l in
//               TMEM only when a head's max grows by > 2^14), P (f16) -> shared
//               memory; at item end O / l -> output (or the split partial).
//   warps 12-15 converter: V = f16(d * q) for the tile's 512 latent columns in
//               16 KB chunks through a 2-deep ring, in the MN-major f16 layout.
//
// The issue warps run converged and issue through one elected lane: an
// mbarrier wait costs ~100+ cycles even when the phase is complete, so they
// wait once per block pair / V chunk rather than once per MMA.
//
// The QK path is exact (int32 accumulation per 32-element Q8_0 block), so the
// only roundings are the query's two-digit int8 form (|err| <= amax/65024),
// V and P in f16, and f32 accumulation.  Every mbarrier wait is bounded
// (~1 s of clocks); on timeout the CTA sets KVCU_STATUS_TIMEOUT, every role
// unwinds, in-flight copies and MMAs are waited for (bounded) and TMEM is freed.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "kvcu_internal.h"
#include "kvcu_tcgen05.cuh"

namespace {
using namespace kvtc;

constexpr int R = 512, P = 64, W = 576;
constexpr int TILE = 128;            // tokens per tile (MMA M for QK)
constexpr int NBLK = 18;             // Q8_0 blocks per row (16 latent + 2 rope)
constexpr int NQK_MAX = 48;          // QK N: 2 digits x up to 24 heads
constexpr int HMAX = NQK_MAX / 2;    // heads supported by the tensor-core kernel
constexpr int NPV = 32;              // PV N: heads padded to 32
constexpr int QK_GROUPS = 2;         // TMEM ring of QK accumulator groups (cols 0..287)
constexpr int GB = 3;                // Q8_0 blocks per group (one TMEM round trip of the epilogue)
constexpr int NGRP = NBLK / GB;      // 6 block groups per tile
constexpr int PV_COL = 352;          // O^T accumulator: 4 M-tiles x 32 cols = [352, 480)
constexpr int L_COL = 480;           // softmax denominators l[h] (ones x P^T) = [480, 512)
constexpr int TMEM_COLS = 512;
static_assert(QK_GROUPS * GB * NQK_MAX <= PV_COL && NBLK % GB == 0, "TMEM map");
constexpr int VCH = 16;              // tokens per V chunk (one f16 MMA K-step)
constexpr int NCH = TILE / VCH;      // 8 token chunks per tile
constexpr int V_SLOTS = 2;           // V chunk ring depth
constexpr uint32_t VU_BYTES = 4096;  // one V unit: 16 tokens x 128 columns (one M-tile) x f16
constexpr uint32_t VCH_BYTES = 4 * VU_BYTES;  // one V chunk: 16 tokens x 512 columns
constexpr int NTHREADS = 512;        // 4 warpgroups: issue, epilogue x2, converter
constexpr int EPI_WARPS = 8;
constexpr float RESCALE_LOG2 = 14.0f;        // lazy rescale threshold (factor 16384; P stays < f16 max)
constexpr uint32_t STATUS_TIMEOUT = KVCU_STATUS_TIMEOUT;

// ---- shared memory map (offsets from a 1024-aligned base) ----
constexpr uint32_t ST_LAT = 0;                   // [16 row groups][4 column chunks][8 rows][128 B], SW128
constexpr uint32_t LAT_GROUP = 4096;             // bytes per 8-row group (the QK A operand's SBO)
constexpr uint32_t ST_ROPE = 4 * 16384;          // [128 rows][64 B], SW64
constexpr uint32_t ST_SC = ST_ROPE + 8192;       // [128][18] u16 scales
constexpr uint32_t STAGE_BYTES = 79872;          // 78,336 rounded up to 1024
constexpr uint32_t OFF_QD = 2 * STAGE_BYTES;     // query digits: 4 x [<=48][128 B] + [<=48][64 B]
constexpr uint32_t QD_LAT_BYTES = NQK_MAX * 128;  // 6144 per latent region
constexpr uint32_t OFF_QD_ROPE = OFF_QD + 4 * QD_LAT_BYTES;
constexpr uint32_t OFF_VR = OFF_QD + 4 * QD_LAT_BYTES + 3072;  // 187392: V chunk ring (2 x 16 KB)
constexpr uint32_t OFF_P = OFF_VR + V_SLOTS * VCH_BYTES;        // P^T: 2 regions x [32][128 B]
constexpr uint32_t OFF_MISC = OFF_P + 8192;                     // 228352
// misc: mbarriers, then small words and arrays
// The raw stage is loaded and handed back in slices of whole V chunks.
// Measured on config 5 (block size 64): 64-row slices with early hand-back
// 3.78 G ctx-tok/s, one 128-row slice 3.74 G, 32-row 3.59 G, 16-row 2.19 G
// (TMA boxes under 32 rows cost more per byte than they save in waiting).
constexpr uint32_t SLICE = 64;
constexpr int NSL = TILE / SLICE;
constexpr uint32_t CPS = SLICE / VCH;  // V chunks per slice
constexpr uint32_t ROW_BYTES = 4u * 128u + 64u + 36u;  // latent + rope + scales
static_assert(SLICE % VCH == 0 && TILE % SLICE == 0, "a slice is a whole number of V chunks");
constexpr int B_KV_FULL = 0, B_SL_EMPTY = 2 /* 2 stages x NSL slices */, B_QK_FULL = 2 + 2 * NSL,
              B_QK_EMPTY = B_QK_FULL + QK_GROUPS, B_V_FULL = B_QK_EMPTY + QK_GROUPS,
              B_V_EMPTY = B_V_FULL + V_SLOTS, B_P_FULL = B_V_EMPTY + V_SLOTS, B_P_EMPTY = B_P_FULL + 1,
              B_PV_DONE = B_P_EMPTY + 1, B_PV_EMPTY = B_PV_DONE + 1, B_Q_FULL = B_PV_EMPTY + 1,
              B_FINAL = B_Q_FULL + 1, B_FINAL_PV = B_FINAL + 1, B_EPI = B_FINAL_PV + 1 /* 2: one per head half */,
              NUM_BARS = B_EPI + 2;
static_assert(NUM_BARS * 8 <= 352, "mbarriers overlap the misc words");
constexpr uint32_t OFF_TMEM_BASE = OFF_MISC + 352;            // u32
constexpr uint32_t OFF_ABORT = OFF_MISC + 368;                // u32, followed by the wait limit
constexpr uint32_t OFF_WAIT_LIMIT = OFF_MISC + 376;           // i64: clocks a bounded wait may take
constexpr uint32_t OFF_CUR_ITEM = OFF_MISC + 360;             // u32: the epilogue's current item
constexpr uint32_t ITEMS_DONE = 0xFFFFFFFFu;
constexpr uint32_t OFF_ONES = OFF_MISC + 384;                 // 128 B of f16 1.0 (l = ones x P^T)
static_assert(OFF_WAIT_LIMIT == OFF_ABORT + 8 && OFF_WAIT_LIMIT % 8 == 0 && OFF_WAIT_LIMIT + 8 <= OFF_ONES,
              "the wait limit sits two words after the abort flag");
constexpr uint32_t OFF_QSCALE = OFF_MISC + 512;               // float[24]
constexpr uint32_t OFF_REDMAX = OFF_MISC + 640;               // float[2][8 warps][24]
constexpr uint32_t OFF_VOTE = OFF_REDMAX + 2 * EPI_WARPS * 24 * 4;  // u32[2][8 warps] rescale votes
constexpr uint32_t SMEM_USED = OFF_VOTE + 2 * EPI_WARPS * 4;
constexpr uint32_t SMEM_ALLOC = SMEM_USED + 1024;             // slack for 1024 alignment
static_assert(SMEM_ALLOC <= 232448, "shared memory budget");

struct TcArgs {
  uint32_t layer, num_blocks, block_size, box_rows;
  const uint16_t* sc;  // f16 scale pool [rows][18]
  uint32_t* status;
  uint32_t n;
  const uint32_t* seq_ids;
  uint32_t n_seqs;
  const uint32_t* toff;
  const uint32_t* tables;
  const uint32_t* lens;
  const float* q;
  uint32_t n_heads;
  float scale_log2;    // softmax scale * log2(e)
  float* out;
  const kvcu_item* items;
  const uint32_t* meta;
  const uint32_t* ranges;
  const uint32_t* seq_count;
  float* part_o;
  float* part_ml;
  uint32_t ws_heads;
  float* lse;  // optional [n][H] log-sum-exp (natural log) of single-item entries
  // Layers [layer, layer + n_layers_call) in one launch: layer layer+i reads
  // q + i*q_lstride and writes out + i*out_lstride (floats), its lse at
  // + i*lse_lstride.  A one-layer plan runs once per layer (unit_layers =
  // n_layers_call), layer i's partials at item index i*part_lstride + item; a
  // layered plan runs once (unit_layers = 1), each item carrying its layer
  // offset, and plan entry layer*n + b holds entry b's item count.
  uint32_t n_layers_call, unit_layers;
  uint64_t q_lstride, out_lstride, part_lstride, lse_lstride;
  const uint32_t* entry_lens;  // optional per-entry attended length (capped by lens[seq]); from the plan
  long long wait_limit;        // clocks a bounded wait may take before the CTA gives up
  uint32_t withhold_plus1;     // test hook: 0, or 1 + the tile whose first slice the producer withholds
};

// Work unit u of a CTA whose plan range holds `cnt` items from `it_begin`:
// repeat li = u / cnt, item it_begin + u % cnt (layer-major, so each layer's
// items run in plan order).  With a layered plan there is one repeat (li = 0)
// and the item gives the layer.
struct Unit {
  uint32_t li, it;
};
__device__ __forceinline__ Unit unit_of(uint32_t u, uint32_t it_begin, uint32_t cnt) {
  const uint32_t li = u / cnt;  // callers only ask for u < unit_layers * cnt, so cnt > 0
  return Unit{li, it_begin + (u - li * cnt)};
}

// ------------------------------------------------------------------ PTX helpers
// Bounded wait: gives up after the CTA's wait limit (the 64-bit word two
// words after the abort flag; ~2^31 clocks, about a second, unless the host
// set another) or when another role has aborted; any give-up records a
// timeout in the status word.
// (Inlined: a call would have to run under several setmaxnreg budgets.)
__device__ __forceinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity,
                                            volatile uint32_t* abort_flag, uint32_t* status) {
  const long long t0 = clock64();
  const long long limit = *reinterpret_cast<const volatile long long*>(abort_flag + 2);
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag || clock64() - t0 > limit) {
      *abort_flag = 1u;
      atomicOr(status, STATUS_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                          uint32_t* status) {
  return mbar_try(bar, parity) || mbar_wait_slow(bar, parity, abort_flag, status);
}
// Warp-wide wait with one verdict for the whole warp (the issue warps run
// converged so that their MMA operands stay warp-uniform).
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                               uint32_t* status) {
  const bool ok = mbar_wait(bar, parity, abort_flag, status);
  return __all_sync(0xffffffffu, ok);
}
// Per-warpgroup register budgets (setmaxnreg).  The block launches with 128
// registers per thread (checked on the host before the first launch); the
// split below never asks for more than that total, so every .inc completes.
constexpr uint32_t LAUNCH_REGS = 128, ISSUE_REGS = 56, EPI_REGS = 184, CVT_REGS = 88;
static_assert(128 * ISSUE_REGS + 256 * EPI_REGS + 128 * CVT_REGS <= NTHREADS * LAUNCH_REGS,
              "register split exceeds the launch allocation");
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
// Wait for this CTA's own asynchronous work (copies, MMAs) to retire: bounded
// by time only, so it still waits after another role has aborted.
__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity, uint32_t* status, long long limit) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (clock64() - t0 > limit) {
      atomicOr(status, STATUS_TIMEOUT);
      return;
    }
  }
}

// 4-D tile: coordinates innermost first
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_load_hint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}
// L2 prefetches of the same boxes (no shared memory, no barrier)
__device__ __forceinline__ void tma_prefetch_4d(const CUtensorMap* map, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_prefetch(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// L2 policy for data read once (the KV stream): evicted first, so that what is
// reused (queries, partials, block tables) stays
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void prefetch_l2_keep(const void* p) {
  asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}

// Instruction descriptors: kind::i8 (s8 x s8 -> s32, both K-major, M=128, N=nqk),
// kind::f16 (f16 x f16 -> f32, A MN-major, B K-major, M=128, N=32) for PV, and
// the same with a K-major A for the l accumulation (A = all ones, zero strides:
// every row and K index reads the same 128 bytes of 1.0).
constexpr uint32_t idesc_qk(int nqk) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(nqk >> 3) << 17) | ((uint32_t)(TILE >> 4) << 24);
}
constexpr uint32_t IDESC_PV = (1u << 4) | (1u << 15) | ((uint32_t)(NPV >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t IDESC_L = (1u << 4) | ((uint32_t)(NPV >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

// Head bucket HK (8, 16, 20 or 24 heads per kernel instance).  Each epilogue
// half owns HH = HK/2 heads.  Query digit rows (= QK accumulator columns) of
// half f start at f*NQH, head-local hl's digits d at f*NQH + 2hl + d, so each
// half drains one 8-column-aligned run of 2HH columns per block.  P rows (= PV
// accumulator columns) of half f start at 16f.
template <int HK>
struct Cfg {
  static constexpr int HH = HK / 2;
  static constexpr int NQH = (2 * HH + 7) / 8 * 8;
  static constexpr int NQK = 2 * NQH;
  static_assert(NQK <= NQK_MAX && NQK % 16 == 0 && HK % 2 == 0 && HH <= 16, "head bucket");
};

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
struct Item {
  uint32_t b, s, t0, t1, tok0, tok1;  // entry, sequence, table range, token range
  uint32_t ntiles;
  uint32_t li;  // layer offset from the call's first layer
  uint32_t e;   // plan entry (item count in seq_count)
};

__device__ __forceinline__ Item load_item(const TcArgs& a, const Unit& un) {
  const kvcu_item ki = a.items[un.it];
  Item r;
  r.b = ki.b;
  r.li = un.li + ki.layer;
  r.e = ki.layer * a.n + ki.b;
  r.s = a.seq_ids ? a.seq_ids[ki.b] : ki.b;
  r.t0 = r.t1 = 0;
  uint32_t len = 0;
  if (r.s < a.n_seqs) {
    r.t0 = a.toff[r.s];
    r.t1 = a.toff[r.s + 1];
    if (r.t1 < r.t0) r.t1 = r.t0;
    len = a.lens[r.s];
    const uint64_t cap = (uint64_t)(r.t1 - r.t0) * a.block_size;
    if (len > cap) len = (uint32_t)cap;
    if (a.entry_lens) len = min(len, a.entry_lens[ki.b]);
  }
  r.tok0 = ki.start;
  r.tok1 = min(ki.end, len);
  r.ntiles = r.tok1 > r.tok0 ? (r.tok1 - r.tok0 + TILE - 1) / TILE : 0u;
  return r;
}

// ------------------------------------------------------------------ the kernel
template <int HK>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_decode_tc(const __grid_constant__ CUtensorMap map_lat, const __grid_constant__ CUtensorMap map_rope,
                TcArgs a) {
  constexpr int NQ = Cfg<HK>::NQK;
  constexpr int HH = Cfg<HK>::HH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  auto bar = [&](int i) { return sbase + OFF_MISC + 8u * (uint32_t)i; };
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + OFF_ABORT);
  const uint32_t H = a.n_heads;

  // ---- set-up: barriers, constant operands, TMEM
  if (threadIdx.x == 0) {
    mbar_init(bar(B_KV_FULL + 0), NSL);  // one arrival per slice, loaded or not
    mbar_init(bar(B_KV_FULL + 1), NSL);
    for (int i = 0; i < 2 * NSL; ++i) mbar_init(bar(B_SL_EMPTY + i), 4);  // the 4 converter warps
    for (int i = 0; i < QK_GROUPS; ++i) {
      mbar_init(bar(B_QK_FULL + i), 1);
      mbar_init(bar(B_QK_EMPTY + i), EPI_WARPS);
    }
    for (int i = 0; i < V_SLOTS; ++i) {
      mbar_init(bar(B_V_FULL + i), 4);
      mbar_init(bar(B_V_EMPTY + i), 1);
    }
    mbar_init(bar(B_P_FULL), EPI_WARPS);
    mbar_init(bar(B_P_EMPTY), 1);
    mbar_init(bar(B_PV_DONE), 1);
    mbar_init(bar(B_PV_EMPTY), EPI_WARPS);
    mbar_init(bar(B_Q_FULL), EPI_WARPS);
    mbar_init(bar(B_FINAL), 1);
    mbar_init(bar(B_FINAL_PV), 1);
    mbar_init(bar(B_EPI + 0), EPI_WARPS / 2);
    mbar_init(bar(B_EPI + 1), EPI_WARPS / 2);
    *abort_flag = 0u;
    *reinterpret_cast<volatile long long*>(smem + OFF_WAIT_LIMIT) = a.wait_limit;
    uint32_t* ones = reinterpret_cast<uint32_t*>(smem + OFF_ONES);
    for (int i = 0; i < 32; ++i) ones[i] = 0x3C003C00u;  // f16 1.0 pairs
    fence_proxy_async();
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     sbase + OFF_TMEM_BASE),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Everything above is independent of earlier kernels in the stream (under a
  // programmatic launch it overlaps their tail); the plan, the lengths and the
  // pool rows are read only after this wait.
  kvcu_pdl_wait();
  // this CTA's range of work items (the plan cuts the batch into equal-cost
  // ranges, one per CTA)
  const uint32_t n_items = a.meta[0], n_ranges = a.meta[1];
  const uint32_t it_begin = blockIdx.x < n_ranges ? min(a.ranges[blockIdx.x], n_items) : n_items;
  const uint32_t it_end = blockIdx.x < n_ranges ? min(a.ranges[blockIdx.x + 1], n_items) : n_items;
  const uint32_t cnt = it_end > it_begin ? it_end - it_begin : 0u;
  const uint32_t n_units = cnt * a.unit_layers;
  if (blockIdx.x == 0 && threadIdx.x == 0 && n_ranges > gridDim.x) atomicOr(a.status, KVCU_STATUS_BAD_PLAN);
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(smem + OFF_CUR_ITEM) = 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + OFF_TMEM_BASE);

  // Register split by warpgroup (set once, with each warpgroup converged): the
  // issue and converter warpgroups hand registers to the two epilogue ones.
  if (warp < 4) {
    setmaxnreg_dec<ISSUE_REGS>();
  if (warp == 0) {
    // ================================================================ producer
    // Slice i of a tile is refilled as soon as the converter hands back the
    // same slice of the tile two earlier, so the next tile streams in while
    // this one's PV runs.  Every slice arrives once on the stage's full
    // barrier, with its bytes, or with none past the item end.
    if (lane == 0) {
      uint32_t g = 0;  // tiles whose NSL arrivals are all made
      bool live = true;
      const uint64_t once = policy_evict_first();
      const uint32_t br = a.box_rows;
      // The rows of tile k of an item go to L2 (no shared memory, no barrier),
      // so that its copy, issued once the converter hands a slot back, reads L2.
      auto prefetch_tile = [&](const Item& pi, uint64_t player, uint32_t pk) {
        const uint32_t p0 = pi.tok0 + pk * TILE, p1 = min(p0 + TILE, pi.tok1);
        for (uint32_t pos = p0; pos < p1; pos += br) {
          const uint32_t blk = a.tables[pi.t0 + pos / a.block_size];
          if (blk >= a.num_blocks || pos % a.block_size + br > a.block_size) continue;
          const uint64_t row = (player * a.num_blocks + blk) * a.block_size + pos % a.block_size;
          tma_prefetch_4d(&map_lat, 0, 0, 0, (int)(row >> 3));
          tma_prefetch_2d(&map_rope, 512, (int)row);
          bulk_prefetch(a.sc + row * NBLK, br * 36u);
        }
      };
      for (uint32_t u = 0; u < n_units && live; ++u) {
        const Item im = load_item(a, unit_of(u, it_begin, cnt));
        const uint64_t layer = (uint64_t)a.layer + im.li;
        for (uint32_t k = 0; k < im.ntiles && live; ++k) {
          const uint32_t s = g & 1u;
          const uint32_t tt0 = im.tok0 + k * TILE;
          const uint32_t tt1 = min(tt0 + TILE, im.tok1);
          // one tile ahead: the next tile of this item, or the first of the
          // next non-empty unit (looking a few units ahead)
          if (k + 1 < im.ntiles) {
            prefetch_tile(im, layer, k + 1);
          } else {
            for (uint32_t u2 = u + 1; u2 < n_units && u2 < u + 4; ++u2) {
              const Item im2 = load_item(a, unit_of(u2, it_begin, cnt));
              if (im2.ntiles) {
                prefetch_tile(im2, (uint64_t)a.layer + im2.li, 0);
                break;
              }
            }
          }
          const uint32_t stage = sbase + s * STAGE_BYTES;
          const uint32_t full = bar(B_KV_FULL + s);
          bool started = false;
#pragma unroll 1
          for (uint32_t i = 0; i < (uint32_t)NSL; ++i) {
            if (live && !mbar_wait(bar(B_SL_EMPTY + NSL * s + i), ((g >> 1) & 1u) ^ 1u, abort_flag, a.status))
              live = false;
            // Stop before the first slice; after it, the remaining slices still
            // arrive (without bytes) so that the drain below sees the phase end.
            if (!live && !started) break;
            started = true;
            // test hook (kvcu_decode_ws_test_withhold): no copy and no arrival
            // for this slice, so the tile never lands and every wait on it runs out
            if (a.withhold_plus1 && g + 1u == a.withhold_plus1 && i == 0) continue;
            // every segment is one box of br rows inside one physical block (the
            // plan aligns items to max(128, block size); anything else is refused)
            uint32_t bytes = 0;
            for (uint32_t off = i * SLICE; live && off < (i + 1) * SLICE && tt0 + off < tt1; off += br) {
              const uint32_t pos = tt0 + off;
              const uint32_t blk = a.tables[im.t0 + pos / a.block_size];
              if (blk >= a.num_blocks) atomicOr(a.status, KVCU_STATUS_BAD_BLOCK);
              else if (pos % a.block_size + br > a.block_size) atomicOr(a.status, KVCU_STATUS_MISALIGNED);
              else bytes += br * ROW_BYTES;
            }
            mbar_arrive_tx(full, bytes);
            for (uint32_t off = i * SLICE; bytes && off < (i + 1) * SLICE && tt0 + off < tt1; off += br) {
              const uint32_t pos = tt0 + off;
              const uint32_t blk = a.tables[im.t0 + pos / a.block_size];
              if (blk >= a.num_blocks || pos % a.block_size + br > a.block_size) continue;
              const uint64_t row = (layer * a.num_blocks + blk) * a.block_size + pos % a.block_size;
              // the segment's whole latent (4 column chunks) in one box
              tma_load_4d(stage + ST_LAT + (off >> 3) * LAT_GROUP, &map_lat, 0, 0, 0, (int)(row >> 3), full, once);
              tma_load_2d_hint(stage + ST_ROPE + off * 64u, &map_rope, 512, (int)row, full, once);
              bulk_load_hint(stage + ST_SC + off * 36u, a.sc + row * NBLK, br * 36u, full, once);
            }
          }
          if (started) ++g;
        }
      }
      // wait (bounded) for the copies of the last two stages to land
      for (uint32_t k = (g >= 2 ? g - 2 : 0); k < g; ++k)
        mbar_wait_drain(bar(B_KV_FULL + (k & 1u)), (k >> 1) & 1u, a.status, a.wait_limit);
    }
  } else if (warp == 1) {
    // ================================================================ QK issuer
    // The whole warp runs the loop (warp-uniform operands); one elected lane
    // issues each MMA / commit.  One wait per pair of Q8_0 blocks.
    uint32_t g = 0, item_no = 0;
    bool ok = true;
    for (uint32_t u = 0; u < n_units && ok; ++u) {
      const Item im = load_item(a, unit_of(u, it_begin, cnt));
      if (im.ntiles == 0) continue;
      if (!mbar_wait_warp(bar(B_Q_FULL), item_no & 1u, abort_flag, a.status)) break;
      tc_fence_after();
      for (uint32_t k = 0; k < im.ntiles; ++k, ++g) {
        const uint32_t s = g & 1u;
        if (!mbar_wait_warp(bar(B_KV_FULL + s), (g >> 1) & 1u, abort_flag, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t stage = sbase + s * STAGE_BYTES;
        for (uint32_t gi = 0; gi < (uint32_t)NGRP; ++gi) {
          const uint32_t kk = g * NGRP + gi, slot = kk % QK_GROUPS;
          if (!mbar_wait_warp(bar(B_QK_EMPTY + slot), ((kk / QK_GROUPS) & 1u) ^ 1u, abort_flag, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
#pragma unroll
            for (uint32_t e = 0; e < (uint32_t)GB; ++e) {
              const uint32_t b = GB * gi + e;
              uint64_t ad, bd;
              if (b < 16) {
                ad = smem_desc(stage + ST_LAT + (b >> 2) * 1024u + (b & 3u) * 32u, 16, LAT_GROUP, LAYOUT_SW128);
                bd = smem_desc(sbase + OFF_QD + (b >> 2) * QD_LAT_BYTES + (b & 3u) * 32u, 16, 1024,
                               LAYOUT_SW128);
              } else {
                ad = smem_desc(stage + ST_ROPE + (b - 16u) * 32u, 16, 512, LAYOUT_SW64);
                bd = smem_desc(sbase + OFF_QD_ROPE + (b - 16u) * 32u, 16, 512, LAYOUT_SW64);
              }
              mma_i8(tmem + (GB * slot + e) * NQ, ad, bd, idesc_qk(NQ), 0u);  // fresh int32 dots
            }
            mma_commit(bar(B_QK_FULL + slot));
          }
          __syncwarp();
        }
        if (!ok) break;
      }
      ++item_no;
    }
    // all issued tcgen05 work retires before TMEM is freed
    if (elect_one()) mma_commit(bar(B_FINAL));
    __syncwarp();
    mbar_wait_drain(bar(B_FINAL), 0, a.status, a.wait_limit);
  } else if (warp == 2) {
    // ================================================================ PV issuer
    // Converged warp, elected issue lane; one wait per 16-token V chunk.
    uint32_t g = 0, item_ord = 0;
    bool ok = true;
    const uint64_t ones_desc = smem_desc(sbase + OFF_ONES, 0, 0, LAYOUT_NONE);
    for (uint32_t u = 0; u < n_units && ok; ++u) {
      const Item im = load_item(a, unit_of(u, it_begin, cnt));
      if (im.ntiles == 0) continue;
      for (uint32_t k = 0; k < im.ntiles && ok; ++k, ++g) {
        if (k == 0 && item_ord > 0) {
          // the epilogue has drained the previous item's O and l
          if (!mbar_wait_warp(bar(B_PV_EMPTY), (item_ord - 1) & 1u, abort_flag, a.status)) {
            ok = false;
            break;
          }
        }
        if (!mbar_wait_warp(bar(B_P_FULL), g & 1u, abort_flag, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (uint32_t c = 0; c < NCH; ++c) {
          const uint32_t v = g * NCH + c, vs = v % V_SLOTS;
          if (!mbar_wait_warp(bar(B_V_FULL + vs), (v / V_SLOTS) & 1u, abort_flag, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
            const uint64_t bdesc = smem_desc(sbase + OFF_P + (c >> 2) * 4096u + (c & 3u) * 32u, 16, 1024,
                                             LAYOUT_SW128);
            const uint32_t acc_flag = (k == 0 && c == 0) ? 0u : 1u;
            mma_f16(tmem + L_COL, ones_desc, bdesc, IDESC_L, acc_flag);
            const uint32_t vbase = sbase + OFF_VR + vs * VCH_BYTES;
#pragma unroll
            for (uint32_t mt = 0; mt < 4; ++mt)
              mma_f16(tmem + PV_COL + mt * NPV, smem_desc(vbase + mt * VU_BYTES, 2048, 1024, LAYOUT_SW128), bdesc,
                      IDESC_PV, acc_flag);
            mma_commit(bar(B_V_EMPTY + vs));
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) {
          mma_commit(bar(B_PV_DONE));
          mma_commit(bar(B_P_EMPTY));
        }
        __syncwarp();
      }
      ++item_ord;
    }
    if (elect_one()) mma_commit(bar(B_FINAL_PV));
    __syncwarp();
    mbar_wait_drain(bar(B_FINAL_PV), 0, a.status, a.wait_limit);
  } else {
    // ================================================================ query prefetcher
    // While the epilogue runs item n, pull item n+1's query into L2 (kept
    // against the KV stream), so that its staging does not wait on a cold read:
    // DRAM, or PCIe when q is in mapped host memory.  Best effort: the poll is
    // bounded and gives up quietly, it never aborts the CTA.
    const volatile uint32_t* cur = reinterpret_cast<const volatile uint32_t*>(smem + OFF_CUR_ITEM);
    const long long t0 = clock64();
    for (uint32_t nx = 1; nx < n_units; ++nx) {
      bool go = false;
      while (true) {
        const uint32_t c = *cur;
        if (c == ITEMS_DONE || *abort_flag) break;
        if (c + 1u >= nx) {
          go = true;
          break;
        }
        if (clock64() - t0 > (1ll << 32)) break;
        __nanosleep(256);
      }
      if (!go) break;
      const Item im = load_item(a, unit_of(nx, it_begin, cnt));
      if (im.ntiles == 0) continue;
      const uint8_t* qb = reinterpret_cast<const uint8_t*>(a.q + im.li * a.q_lstride + (uint64_t)im.b * H * W);
      for (uint32_t off = lane * 128u; off < H * (uint32_t)W * 4u; off += 32u * 128u) prefetch_l2_keep(qb + off);
    }
  }
  } else if (warp < 12) {
    setmaxnreg_inc<EPI_REGS>();
    // ================================================================ epilogue
    const uint32_t ew = warp - 4u;             // 0..7
    const uint32_t hf = ew >> 2;               // head half
    const uint32_t h0 = hf * HH;               // first head of this half
    const uint32_t q4 = warp & 3u;             // TMEM lane quarter
    const uint32_t trow = 32u * q4 + lane;     // token row in the tile / latent row in an M-tile
    const uint32_t lane_addr = (32u * q4) << 16;
    float* qscale = reinterpret_cast<float*>(smem + OFF_QSCALE);
    float* redmax = reinterpret_cast<float*>(smem + OFF_REDMAX);
    uint32_t g = 0, esync = 0;
    bool ok = true;
    // bounded barrier among the 4 epilogue warps of this half (an mbarrier, so
    // a timeout elsewhere cannot strand a warp in bar.sync)
    auto epi_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_EPI + hf));
      const bool r = mbar_wait(bar(B_EPI + hf), esync & 1u, abort_flag, a.status);
      ++esync;
      return r;
    };
    // ---- query -> two int8 digits per element (x = s_h * (d0 + d1/256)), per-head
    // scale; each half's 4 warps encode that half's heads.  The next item's
    // query is staged as soon as this item's last P is out (its QK MMAs are all
    // done then), so the next item's first QK overlaps this item's drain.
    uint32_t staged_u = 0xFFFFFFFFu;
    auto stage_q = [&](const Item& si) -> bool {
      const float* qb = a.q + si.li * a.q_lstride + (uint64_t)si.b * H * W;
      for (uint32_t hl = ew & 3u; hl < (uint32_t)HH; hl += 4) {
        const uint32_t h = h0 + hl;
        float amax = 0.f;
        float v[18];
#pragma unroll
        for (int j = 0; j < 18; ++j) {
          v[j] = h < H ? qb[(uint64_t)h * W + lane + 32 * j] : 0.f;
          amax = fmaxf(amax, fabsf(v[j]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float sh = amax > 0.f ? amax / 127.0f : 1.0f;
        const float inv = 1.0f / sh;
        const uint32_t qrow = hf * Cfg<HK>::NQH + 4u * (hl >> 1) + (hl & 1u);  // digit-0 row
#pragma unroll
        for (int j = 0; j < 18; ++j) {
          const uint32_t kcol = lane + 32u * j;
          const float x = v[j] * inv;
          const float d0 = fminf(fmaxf(rintf(x), -127.f), 127.f);
          const float d1 = fminf(fmaxf(rintf((x - d0) * 256.f), -127.f), 127.f);
          uint8_t* base;
          uint32_t o0, o1;
          if (kcol < 512) {
            base = smem + OFF_QD + (kcol >> 7) * QD_LAT_BYTES;
            o0 = sw128_off(qrow, kcol & 127u);
            o1 = sw128_off(qrow + 2u, kcol & 127u);
          } else {
            base = smem + OFF_QD_ROPE;
            o0 = sw64_off(qrow, kcol - 512u);
            o1 = sw64_off(qrow + 2u, kcol - 512u);
          }
          base[o0] = (uint8_t)(int8_t)(int)d0;
          base[o1] = (uint8_t)(int8_t)(int)d1;
        }
        if (lane == 0) qscale[h] = sh * (1.0f / 256.0f) * a.scale_log2;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_Q_FULL));
      return epi_sync();  // this half's qscale visible to its 4 warps
    };
    volatile uint32_t* cur_item = reinterpret_cast<volatile uint32_t*>(smem + OFF_CUR_ITEM);
    for (uint32_t u = 0; u < n_units && ok; ++u) {
      if (ew == 0 && lane == 0) *cur_item = u;
      const Unit un = unit_of(u, it_begin, cnt);
      const Item im = load_item(a, un);
      const bool single = a.seq_count[im.e] == 1;
      // this unit's partial slot (item index); its output rows and lse, those
      // of entry b in layer offset im.li, are addressed where they are written
      // (a pointer formed here would stay live across the item and spill)
      const uint64_t pit = un.li * a.part_lstride + un.it;
      if (im.ntiles == 0) {
        // empty item: zeros, or an empty partial
        for (uint32_t i = ew * 32 + lane; i < H * (uint32_t)R; i += 32 * EPI_WARPS) {
          const uint32_t h = i / R, c = i % R;
          if (single) a.out[im.li * a.out_lstride + ((uint64_t)im.b * H + h) * R + c] = 0.f;
          else a.part_o[(pit * a.ws_heads + h) * R + c] = 0.f;
        }
        if (!single && ew == 0 && lane < H) {
          a.part_ml[(pit * a.ws_heads + lane) * 2 + 0] = -INFINITY;
          a.part_ml[(pit * a.ws_heads + lane) * 2 + 1] = 0.f;
        }
        if (single && a.lse && ew == 0 && lane < H) a.lse[im.li * a.lse_lstride + (uint64_t)im.b * H + lane] = -INFINITY;
        continue;
      }
      if (staged_u != u) {
        if (!stage_q(im)) {
          ok = false;
          break;
        }
        staged_u = u;
      }
      // running reference max per head (log2 domain), identical in the 4 warps of the half
      float mref[HH];
#pragma unroll
      for (int h = 0; h < HH; ++h) mref[h] = -INFINITY;
      const float2* qsc2 = reinterpret_cast<const float2*>(qscale + h0);  // h0 is even
      for (uint32_t k = 0; k < im.ntiles && ok; ++k, ++g) {
        const uint32_t s = g & 1u;
        const uint32_t tt0 = im.tok0 + k * TILE;
        const bool valid = tt0 + trow < im.tok1;
        // raw stage s holds this tile's block scales (read before this tile's P
        // is published; the converter hands the stage back after that)
        if (!mbar_wait(bar(B_KV_FULL + s), (g >> 1) & 1u, abort_flag, a.status)) {
          ok = false;
          break;
        }
        const uint16_t* scrow =
            reinterpret_cast<const uint16_t*>(smem + s * STAGE_BYTES + ST_SC) + trow * NBLK;
        // per head: sum over blocks of d_b * (256 x0 + x1)
        float2 acc2[HH / 2];  // heads (2p, 2p+1)
#pragma unroll
        for (int p = 0; p < HH / 2; ++p) acc2[p] = make_float2(0.f, 0.f);
        // Three Q8_0 blocks per TMEM round trip (18 blocks -> 6 groups); this
        // half reads its 2HH digit columns of each slot, per head pair
        // [digit0 h, digit0 h+1, digit1 h, digit1 h+1].
        // Software-pipelined over groups: the TMEM loads of group gi+1 are in
        // flight while group gi is combined (two register sets, a and b).
        uint32_t ra[3][2 * HH], rb[3][2 * HH];
        auto grp_issue = [&](uint32_t gi, uint32_t(&r)[3][2 * HH]) -> bool {
          const uint32_t kk = g * NGRP + gi, slot = kk % QK_GROUPS;
          if (!mbar_wait(bar(B_QK_FULL + slot), (kk / QK_GROUPS) & 1u, abort_flag, a.status)) return false;
          tc_fence_after();
          const uint32_t ta = tmem + lane_addr + GB * slot * NQ + hf * Cfg<HK>::NQH;
          tmem_ld<2 * HH>(ta, r[0]);
          tmem_ld<2 * HH>(ta + NQ, r[1]);
          tmem_ld<2 * HH>(ta + 2 * NQ, r[2]);
          return true;
        };
        // the values are in registers: the slot can take the next group's MMAs now
        auto grp_land = [&](uint32_t gi, uint32_t(&r)[3][2 * HH]) {
          tmem_wait_ld();
          reg_fence(r[0]);
          reg_fence(r[1]);
          reg_fence(r[2]);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_QK_EMPTY + (g * NGRP + gi) % QK_GROUPS));
        };
        // Per head: 256 x0 + x1 exactly in int32 (|x0| <= 32 * 127^2 < 2^19),
        // one rounding to f32, then the block scale, two heads per packed
        // f32x2 FMA (each lane is one fused multiply-add, as fmaf). Head pair p
        // has digit-0 columns 4p, 4p+1 and digit-1 columns 4p+2, 4p+3.  (An
        // exact conversion by the 1.5 * 2^23 bias, avoiding the int->float
        // unit, measured 8% slower: it needs more instructions per value.)
        auto grp_math = [&](uint32_t gi, const uint32_t(&r)[3][2 * HH]) {
          const float d0 = __half2float(__ushort_as_half(scrow[GB * gi]));
          const float d1 = __half2float(__ushort_as_half(scrow[GB * gi + 1]));
          const float d2 = __half2float(__ushort_as_half(scrow[GB * gi + 2]));
          const float2 dd0 = make_float2(d0, d0), dd1 = make_float2(d1, d1), dd2 = make_float2(d2, d2);
#pragma unroll
          for (int p = 0; p < HH / 2; ++p) {
            const int c = 4 * p;
            const float2 f0 = make_float2(__int2float_rn((int)r[0][c] * 256 + (int)r[0][c + 2]),
                                          __int2float_rn((int)r[0][c + 1] * 256 + (int)r[0][c + 3]));
            const float2 f1 = make_float2(__int2float_rn((int)r[1][c] * 256 + (int)r[1][c + 2]),
                                          __int2float_rn((int)r[1][c + 1] * 256 + (int)r[1][c + 3]));
            const float2 f2 = make_float2(__int2float_rn((int)r[2][c] * 256 + (int)r[2][c + 2]),
                                          __int2float_rn((int)r[2][c + 1] * 256 + (int)r[2][c + 3]));
            acc2[p] = __ffma2_rn(dd0, f0, acc2[p]);
            acc2[p] = __ffma2_rn(dd1, f1, acc2[p]);
            acc2[p] = __ffma2_rn(dd2, f2, acc2[p]);
          }
        };
        static_assert(NGRP % 2 == 0, "groups are combined in pairs");
        if constexpr (HH > 10) {
          // 21-24 heads: the second register set does not fit, one group at a time
          for (uint32_t gi = 0; gi < (uint32_t)NGRP && ok; ++gi) {
            if (!grp_issue(gi, ra)) {
              ok = false;
              break;
            }
            grp_land(gi, ra);
            grp_math(gi, ra);
          }
          if (!ok) break;
        } else {
        if (!grp_issue(0, ra)) {
          ok = false;
          break;
        }
        grp_land(0, ra);
        for (uint32_t gp = 0; gp < (uint32_t)NGRP; gp += 2) {
          if (!grp_issue(gp + 1, rb)) {
            ok = false;
            break;
          }
          grp_math(gp, ra);
          grp_land(gp + 1, rb);
          const bool more = gp + 2 < (uint32_t)NGRP;
          if (more && !grp_issue(gp + 2, ra)) {
            ok = false;
            break;
          }
          grp_math(gp + 1, rb);
          if (more) grp_land(gp + 2, ra);
        }
        }
        if (!ok) break;
        // ---- online softmax over the tile (log2 domain)
        float sc[HH];
#pragma unroll
        for (int p = 0; p < HH / 2; ++p) {
          const float2 q2 = qsc2[p];
          const float2 v2 = __fmul2_rn(acc2[p], q2);
          const float vx = v2.x, vy = v2.y;
          sc[2 * p] = (valid && h0 + 2 * p < H && vx == vx) ? vx : -INFINITY;
          sc[2 * p + 1] = (valid && h0 + 2 * p + 1 < H && vy == vy) ? vy : -INFINITY;
        }
        // lazy rescale: a head's reference max moves only when some score of
        // the tile exceeds it by more than 2^14 (so P <= 16384 otherwise, inside f16).  Each
        // warp votes per head; the half combines the 4 votes after one sync.
        uint32_t bits = 0;
#pragma unroll
        for (int h = 0; h < HH; ++h) bits |= (sc[h] > mref[h] + RESCALE_LOG2) ? (1u << h) : 0u;
        bits = __reduce_or_sync(0xffffffffu, bits);
        uint32_t* vote = reinterpret_cast<uint32_t*>(smem + OFF_VOTE) + (g & 1u) * EPI_WARPS;
        if (lane == 0) vote[ew] = bits;
        if (!epi_sync()) {
          ok = false;
          break;
        }
        const uint4 vw = *reinterpret_cast<const uint4*>(vote + 4 * hf);  // ordered by the mbarrier wait
        const uint32_t flagged = vw.x | vw.y | vw.z | vw.w;
        if (flagged) {
          // exact tile max of the flagged heads over the half's 128 rows
          float* rm = redmax + (g & 1u) * (EPI_WARPS * 24);
#pragma unroll
          for (int h = 0; h < HH; ++h) {
            float m = sc[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) rm[ew * 24 + h] = m;
          }
          if (!epi_sync()) {
            ok = false;
            break;
          }
          const float* rmh = rm + hf * 4 * 24;  // the 4 warps of this half
          float tmax[HH];
          bool need_rescale = false;
#pragma unroll
          for (int h = 0; h < HH; ++h) {
            tmax[h] = fmaxf(fmaxf(rmh[h], rmh[24 + h]), fmaxf(rmh[48 + h], rmh[72 + h]));
            need_rescale |= ((flagged >> h) & 1u) && mref[h] != -INFINITY;
          }
          if (need_rescale) {
            // O holds the PV of this item's earlier tiles: retire it, then scale
            if (!mbar_wait(bar(B_PV_DONE), (g - 1) & 1u, abort_flag, a.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll 1
            for (uint32_t mt = 0; mt < 5; ++mt) {  // 4 O^T M-tiles, then l
              uint32_t o[HH];
              const uint32_t ta = tmem + lane_addr + (mt < 4 ? PV_COL + mt * NPV : L_COL) + 16u * hf;
              tmem_ld<HH>(ta, o);
              tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < HH; ++h)
                if (((flagged >> h) & 1u) && mref[h] != -INFINITY)
                  o[h] = __float_as_uint(__uint_as_float(o[h]) * exp2f(mref[h] - tmax[h]));
              tmem_st<HH>(ta, o);
              tmem_wait_st();
            }
            tc_fence_before();
          }
#pragma unroll
          for (int h = 0; h < HH; ++h)
            if ((flagged >> h) & 1u) mref[h] = tmax[h];
        }
        // ---- P (f16) -> shared memory, K-major 128B-swizzled [head][token];
        // the values are formed before the wait for the buffer (the previous
        // tile's PV)
        __half ph[HH];
#pragma unroll
        for (int h = 0; h < HH; ++h) ph[h] = __float2half_rn(sc[h] == -INFINITY ? 0.f : exp2f(sc[h] - mref[h]));
        if (!mbar_wait(bar(B_P_EMPTY), (g & 1u) ^ 1u, abort_flag, a.status)) {
          ok = false;
          break;
        }
        {
          uint8_t* pb = smem + OFF_P + (trow >> 6) * 4096u;
          const uint32_t tb = (trow & 63u) * 2u;
#pragma unroll
          for (int h = 0; h < HH; ++h) *reinterpret_cast<__half*>(pb + sw128_off(16u * hf + (uint32_t)h, tb)) = ph[h];
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_P_FULL));
      }
      if (!ok) break;
      for (uint32_t u2 = u + 1; u2 < n_units; ++u2) {
        const Item im2 = load_item(a, unit_of(u2, it_begin, cnt));
        if (im2.ntiles == 0) continue;
        if (!stage_q(im2)) ok = false;
        staged_u = u2;
        break;
      }
      if (!ok) break;
      // ---- item end: l (every TMEM lane holds it), drain O, write the output or the partial
      {
        if (!mbar_wait(bar(B_PV_DONE), (g - 1) & 1u, abort_flag, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float ltot[HH];
        {
          uint32_t lv[HH];
          tmem_ld<HH>(tmem + lane_addr + L_COL + 16u * hf, lv);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < HH; ++h) ltot[h] = __uint_as_float(lv[h]);
        }
#pragma unroll 1
        for (uint32_t mt = 0; mt < 4; ++mt) {
          uint32_t o[HH];
          tmem_ld<HH>(tmem + lane_addr + PV_COL + mt * NPV + 16u * hf, o);
          tmem_wait_ld();
          const uint32_t c = mt * 128u + trow;
#pragma unroll
          for (int h = 0; h < HH; ++h) {
            const uint32_t hg = h0 + h;
            if (hg >= H) continue;
            const float v = __uint_as_float(o[h]);
            if (single) a.out[im.li * a.out_lstride + ((uint64_t)im.b * H + hg) * R + c] = ltot[h] > 0.f ? v / ltot[h] : 0.f;
            else a.part_o[(pit * a.ws_heads + hg) * R + c] = v;
          }
        }
        if (!single && q4 == 0 && lane < HH && h0 + lane < H) {
          float lh = 0.f, mh = 0.f;
#pragma unroll
          for (int h = 0; h < HH; ++h)
            if ((uint32_t)h == lane) {
              lh = ltot[h];
              mh = mref[h];
            }
          a.part_ml[(pit * a.ws_heads + h0 + lane) * 2 + 0] = mh * 0.69314718055994531f;
          a.part_ml[(pit * a.ws_heads + h0 + lane) * 2 + 1] = lh;
        }
        if (single && a.lse && q4 == 0 && lane < HH && h0 + lane < H) {
          float lh = 0.f, mh = 0.f;
#pragma unroll
          for (int h = 0; h < HH; ++h)
            if ((uint32_t)h == lane) {
              lh = ltot[h];
              mh = mref[h];
            }
          // mref is in log2 units of the scaled score, l = sum 2^(s - mref)
          a.lse[im.li * a.lse_lstride + (uint64_t)im.b * H + h0 + lane] = lh > 0.f ? (mh + log2f(lh)) * 0.69314718055994531f : -INFINITY;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_PV_EMPTY));
      }
    }
    if (ew == 0 && lane == 0) *cur_item = ITEMS_DONE;
  } else {
    setmaxnreg_dec<CVT_REGS>();
    // ================================================================ converter
    const uint32_t tid = (warp - 12u) * 32u + lane;  // 0..127
    const uint32_t tl = tid & 15u;                   // token within the 16-token chunk
    const uint32_t j = tid >> 4;                     // 16-column group within the M-tile, 0..7
    uint32_t g = 0;
    bool ok = true;
    for (uint32_t u = 0; u < n_units && ok; ++u) {
      const Item im = load_item(a, unit_of(u, it_begin, cnt));
      for (uint32_t k = 0; k < im.ntiles && ok; ++k, ++g) {
        const uint32_t s = g & 1u;
        const uint32_t tt0 = im.tok0 + k * TILE;
        if (!mbar_wait(bar(B_KV_FULL + s), (g >> 1) & 1u, abort_flag, a.status)) {
          ok = false;
          break;
        }
        const uint8_t* stage = smem + s * STAGE_BYTES;
        for (uint32_t c = 0; c < NCH; ++c) {
          const uint32_t t = c * VCH + tl;  // token row in the tile
          const bool valid = tt0 + t < im.tok1;
          // dequantize the whole chunk into registers first, so that the wait
          // for a free slot overlaps this work: this thread covers token t,
          // latent columns 128mt + 16j .. +15 (one raw 16-byte chunk) of each M-tile mt
          // Branch-free: rows past the sequence end (stale stage bytes) get a
          // zero scale, so their V is exactly 0 ((1152+q)-1152 is finite).
          uint4 raw[4];
          uint16_t dsc[4];
#pragma unroll
          for (uint32_t mt = 0; mt < 4; ++mt) {
            raw[mt] = *reinterpret_cast<const uint4*>(stage + ST_LAT + (t >> 3) * LAT_GROUP + mt * 1024u +
                                                      sw128_off(t & 7u, j * 16u));
            dsc[mt] = *reinterpret_cast<const uint16_t*>(stage + ST_SC + t * 36u + (4u * mt + (j >> 1)) * 2u);
          }
          uint32_t hv[4][8];
          const __half2 bias = __float2half2_rn(1152.0f);
#pragma unroll
          for (uint32_t mt = 0; mt < 4; ++mt) {
            const __half2 dd = __half2half2(__ushort_as_half(valid ? dsc[mt] : (uint16_t)0));
            const uint32_t w[4] = {raw[mt].x, raw[mt].y, raw[mt].z, raw[mt].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t uu = w[e] ^ 0x80808080u;  // q + 128 per byte
              const uint32_t lo = __byte_perm(uu, 0x64646464u, 0x4140u);
              const uint32_t hi = __byte_perm(uu, 0x64646464u, 0x4342u);
              __half2 a0 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&lo), bias), dd);
              __half2 a1 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&hi), bias), dd);
              hv[mt][2 * e] = *reinterpret_cast<uint32_t*>(&a0);
              hv[mt][2 * e + 1] = *reinterpret_cast<uint32_t*>(&a1);
            }
          }
          const uint32_t v = g * NCH + c, vs = v % V_SLOTS;
          if (!mbar_wait(bar(B_V_EMPTY + vs), ((v / V_SLOTS) & 1u) ^ 1u, abort_flag, a.status)) {
            ok = false;
            break;
          }
          // From chunk 2 on, this slot was freed by a PV MMA of this tile, so
          // the epilogue has published the tile's P: it has read the stage's
          // scales and waited for the QK MMAs.  The raw rows of the chunks read
          // so far (into registers) go back to the producer.
          // Slices [lo, hi) are whole after chunk c and were not handed back yet.
          const uint32_t lo = c == 2 ? 0u : c / CPS, hi = c >= 2 ? (c + 1) / CPS : 0u;
          if (hi > lo) {
            __syncwarp();
            if (lane == 0)
              for (uint32_t j = lo; j < hi; ++j) mbar_arrive(bar(B_SL_EMPTY + NSL * s + j));
          }
          // unit mt of the chunk: MN atom j/4, chunks 2(j%4), 2(j%4)+1 of atom row t%8, K atom t/8
          uint8_t* vrow = smem + OFF_VR + vs * VCH_BYTES + (j >> 2) * 2048u + (tl >> 3) * 1024u + (tl & 7u) * 128u;
          const uint32_t ch0 = 2u * (j & 3u);
#pragma unroll
          for (uint32_t mt = 0; mt < 4; ++mt) {
            *reinterpret_cast<uint4*>(vrow + mt * VU_BYTES + (((ch0 ^ tl) & 7u) << 4)) =
                make_uint4(hv[mt][0], hv[mt][1], hv[mt][2], hv[mt][3]);
            *reinterpret_cast<uint4*>(vrow + mt * VU_BYTES + ((((ch0 + 1u) ^ tl) & 7u) << 4)) =
                make_uint4(hv[mt][4], hv[mt][5], hv[mt][6], hv[mt][7]);
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_V_FULL + vs));
        }
        if (!ok) break;
      }
    }
  }

  // ---- teardown (the combine that follows may start launching now)
  kvcu_pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_maps(const kvcu_pool* p, uint32_t box_rows, CUtensorMap* lat, CUtensorMap* rope) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    kvcu_set_error("cuTensorMapEncodeTiled unavailable");
    return KVCU_ERR_CUDA;
  }
  const uint64_t rows = p->rows();
  const cuuint64_t dims[2] = {(cuuint64_t)W, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)W};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const cuuint32_t box_rope[2] = {64, box_rows};
  // Latent as (byte in chunk, row in group, 128 B chunk, 8-row group), so one
  // box lands as [group][chunk][8 rows x 128 B]: the 128B-swizzled K-major
  // layout of all four chunks, 4096 B per 8-row group.  Rows are a multiple of
  // 16 (the block size is), so the groups tile the pool exactly.
  const cuuint64_t dims_lat[4] = {128, 8, 4, (cuuint64_t)(rows / 8)};
  const cuuint64_t strides_lat[3] = {(cuuint64_t)W, 128, 8 * (cuuint64_t)W};
  const cuuint32_t box_lat[4] = {128, 8, 4, box_rows / 8};
  CUresult r = enc(lat, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, p->qs, dims_lat, strides_lat, box_lat, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    kvcu_set_error("cuTensorMapEncodeTiled(latent) failed: %d", (int)r);
    return KVCU_ERR_CUDA;
  }
  r = enc(rope, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p->qs, dims, strides, box_rope, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    kvcu_set_error("cuTensorMapEncodeTiled(rope) failed: %d", (int)r);
    return KVCU_ERR_CUDA;
  }
  return KVCU_OK;
}

// Per-device set-up of one head bucket's kernel (run once per device by
// kvcu_configure_once).
template <int HK>
int setup_tc(const void*) {
  // the setmaxnreg split assumes exactly LAUNCH_REGS registers per thread at
  // launch; with fewer, an epilogue .inc could wait forever, so refuse
  cudaFuncAttributes fa;
  int rc = kvcu_check_cuda(cudaFuncGetAttributes(&fa, k_decode_tc<HK>), "cudaFuncGetAttributes(decode_tc)");
  if (rc) return rc;
  if (fa.numRegs != (int)LAUNCH_REGS) {
    kvcu_set_error("decode_tc: built with %d registers per thread, the register split needs %u", fa.numRegs,
                   LAUNCH_REGS);
    return KVCU_ERR_UNSUPPORTED;
  }
  return kvcu_check_cuda(
      cudaFuncSetAttribute(k_decode_tc<HK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_ALLOC),
      "cudaFuncSetAttribute(decode_tc)");
}

template <int HK>
int launch_tc(int grid, const CUtensorMap& lat, const CUtensorMap& rope, const TcArgs& a, cudaStream_t st) {
  const int rc = kvcu_configure_once(reinterpret_cast<const void*>(&k_decode_tc<HK>), setup_tc<HK>, nullptr);
  if (rc) return rc;
  // programmatic launch: the prologue overlaps the previous kernel's tail
  return kvcu_check_cuda(kvcu_launch_pdl(k_decode_tc<HK>, dim3(grid), dim3(NTHREADS), SMEM_ALLOC, st, lat, rope, a),
                         "decode_tc kernel launch");
}

}  // namespace

// Whether the tensor-core kernel handles this pool / head count.
bool kvcu_decode_tc_supported(const kvcu_pool* p, uint32_t n_heads) {
  if (!p->quantized || p->kv_rank != (uint32_t)R || p->rope_dim != (uint32_t)P) return false;
  if (n_heads == 0 || n_heads > (uint32_t)HMAX) return false;
  if (p->block_size % 16 != 0) return false;
  if (p->block_size < TILE && TILE % p->block_size != 0) return false;
  if (p->block_size > TILE && p->block_size % TILE != 0) return false;
  if (p->rows() > 0x7FFFFFFFull) return false;  // TMA coordinates are int32
  return true;
}

int kvcu_launch_decode_tc(kvcu_decode_ws* ws, kvcu_pool* p, uint32_t layer, uint32_t n_layers_call, uint32_t n,
                          const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* toff,
                          const uint32_t* tables, const uint32_t* lens, const float* q, uint64_t q_lstride,
                          uint32_t n_heads, float scale, float* out, uint64_t out_lstride, float* lse,
                          uint64_t lse_lstride, cudaStream_t st) {
  // one box per slice, or per block where blocks are smaller than a slice
  const uint32_t box_rows = p->block_size < SLICE ? p->block_size : SLICE;
  CUtensorMap lat, rope;
  int rc = make_maps(p, box_rows, &lat, &rope);
  if (rc) return rc;
  TcArgs a;
  a.layer = layer;
  a.num_blocks = p->num_blocks;
  a.block_size = p->block_size;
  a.box_rows = box_rows;
  a.sc = p->sc;
  a.status = p->status;
  a.n = n;
  a.seq_ids = seq_ids;
  a.n_seqs = n_seqs;
  a.toff = toff;
  a.tables = tables;
  a.lens = lens;
  a.q = q;
  a.n_heads = n_heads;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = out;
  a.items = ws->items;
  a.meta = ws->meta;
  a.ranges = ws->ranges;
  a.seq_count = ws->seq_count;
  a.part_o = ws->part_o;
  a.part_ml = ws->part_ml;
  a.ws_heads = ws->max_heads;
  a.lse = lse;
  a.n_layers_call = n_layers_call;
  a.unit_layers = ws->plan_layers > 1 ? 1u : n_layers_call;  // a layered plan already lists every layer
  a.q_lstride = q_lstride;
  a.out_lstride = out_lstride;
  a.part_lstride = ws->max_items;
  a.lse_lstride = lse_lstride;
  a.entry_lens = ws->entry_lens;
  a.wait_limit = ws->wait_limit ? (long long)ws->wait_limit : (1ll << 31);
  a.withhold_plus1 = ws->withhold_plus1;
  if (n_heads <= 8) return launch_tc<8>(ws->decode_ctas, lat, rope, a, st);
  if (n_heads <= 16) return launch_tc<16>(ws->decode_ctas, lat, rope, a, st);
  if (n_heads <= 20) return launch_tc<20>(ws->decode_ctas, lat, rope, a, st);
  return launch_tc<24>(ws->decode_ctas, lat, rope, a, st);
}
