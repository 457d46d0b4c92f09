// kvcu_decode.cu — paged MLA decode attention (split-KV) over the block pool.
//
// Restates the attention core of InferenceEngine.mlaAttention
// (src/inference.zig:518-660) in absorbed form (q is 576 wide, K is the cached
// latent ++ rope row, V is the latent): online softmax over the sequence's
// cached positions read through its block table, Q8_0 rows dequantized on the
// fly exactly as getKVCompressed/getKPe do (src/kv_cache.zig:232-246).
//
// Structure (one decode = three stream-ordered launches, or two when the plan
// is reused across layers):
//   k_plan      one CTA: cuts the batch into one equal-cost range of work
//               items per decode CTA, splitting a sequence where a cut falls;
//   k_decode    persistent CTAs (one per SM) run their range of items; each
//               streams its KV tile-by-tile through shared memory and keeps
//               (m, l, o[512]) per head; single-item sequences write the final
//               output, the others write partials to the workspace;
//   k_combine   merges the partials of split sequences (log-sum-exp rescale).
#include <cuda_runtime.h>
#include <math.h>

#include "kvcu_internal.h"
#include "kvcu_numeric.cuh"

namespace {

constexpr int R = 512;           // kv_rank (latent, also V width)
constexpr int P = 64;            // rope_dim
constexpr int W = R + P;         // K row width
constexpr int TT = 32;           // tokens per tile
constexpr int KS = W + 4;        // padded smem row stride (conflict-free float4)
constexpr int NT = 256;          // threads per CTA
constexpr int NW = NT / 32;      // warps
constexpr int KSLICE = W / NW;   // 72 K elements per warp in the QK stage

struct DecodeArgs {
  uint32_t layer, num_blocks, block_size, nblk;
  const float* kv;
  const float* pe;
  const int8_t* qs;
  const uint16_t* sc;
  uint32_t* status;
  uint32_t n;
  const uint32_t* seq_ids;
  uint32_t n_seqs;
  const uint32_t* toff;
  const uint32_t* tables;
  const uint32_t* lens;
  const float* q;
  uint32_t n_heads;
  float scale;
  float* out;
  const kvcu_item* items;
  const uint32_t* meta;
  const uint32_t* ranges;
  const uint32_t* seq_count;
  float* part_o;
  float* part_ml;
  uint32_t ws_heads;
  float* lse;  // optional [n][H] log-sum-exp of the scaled scores (natural log)
  const uint32_t* entry_lens;  // optional per-entry attended length (capped by lens[seq]); from the plan
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------ plan
// Balanced split-KV plan. Every entry b costs PLAN_UNIT per `align`-token unit
// of its length plus PLAN_ITEM for finishing an item (draining O, writing the
// output or a partial). The entries are laid end to end on a cost line of
// length T in batch order, and the line is cut into G equal ranges, one per
// decode CTA: range c is [P_c, P_{c+1}) with P_c = floor(c T / G). A cut that
// falls inside an entry's units splits the entry there (rounded up to a unit),
// so every CTA gets the same cost within one unit and at most G - 1 entries are
// split. Items are numbered in batch order; CTA c runs items
// [ranges[c], ranges[c+1]).
//
// A layered plan (n_layers = L > 1) lays the L x n (layer, entry) pairs of one
// multi-layer decode on the line as plan entries e = layer * n + b, so the
// whole launch splits at most G - 1 of them; a one-layer plan, repeated by a
// multi-layer decode for each layer, splits up to G - 1 in every layer. Every
// item records its layer offset, and seq_first / seq_count are indexed by e.
//
// Items start at multiples of `align` (= max(128, block size)), so every
// 128-token tile of the tensor-core kernel covers whole physical blocks (or a
// 128-row-aligned part of one). An entry's last item is open-ended: decode
// clips it to the live length, so a plan stays valid while appends grow the
// sequences.
// Relative costs measured on B200 with the tensor-core kernel (config 5): an
// item's set-up and finish take about 2.5 tiles; 16..24 gave the same speed,
// 4 was 5% and 64 was 6% slower.
constexpr uint32_t PLAN_UNIT = 8;   // cost of one align-token unit
constexpr uint32_t PLAN_ITEM = 20;  // cost of one item besides its units

__device__ __forceinline__ unsigned long long ceil_div_u64(unsigned long long x, unsigned long long y) {
  return (x + y - 1) / y;
}

// entry_lens (nullable): entry b attends min(entry_lens[b], lens[seq]) positions
// instead of the sequence's whole length (causal multi-query attention).
__global__ void __launch_bounds__(1024) k_plan(uint32_t n, uint32_t n_layers, const uint32_t* __restrict__ seq_ids,
                                               uint32_t n_seqs, const uint32_t* __restrict__ lens,
                                               const uint32_t* __restrict__ entry_lens,
                                               uint32_t max_ranges, uint32_t align, uint32_t max_items,
                                               kvcu_item* __restrict__ items,
                                               uint32_t* __restrict__ meta,
                                               uint32_t* __restrict__ ranges,
                                               uint32_t* __restrict__ seq_first,
                                               uint32_t* __restrict__ seq_count) {
  __shared__ unsigned long long s_total;
  __shared__ unsigned long long s_wcost[32];
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_carry;           // items of the earlier chunks
  __shared__ unsigned long long s_ccarry;  // cost of the earlier chunks
  const uint32_t tid = threadIdx.x, lane = tid & 31u, wid = tid >> 5, nw = blockDim.x >> 5;
  kvcu_pdl_trigger();  // a programmatically launched decode may start its prologue
  if (tid == 0) {
    s_total = 0;
    s_carry = 0;
    s_ccarry = 0;
  }
  __syncthreads();
  const uint32_t N = n * n_layers;  // plan entries e = layer * n + b
  auto units_of = [&](uint32_t e) -> uint32_t {
    const uint32_t b = e % n;  // only called for e < N, so n > 0
    const uint32_t s = seq_ids ? seq_ids[b] : b;
    uint32_t len = s < n_seqs ? lens[s] : 0u;
    if (entry_lens) len = min(len, entry_lens[b]);
    return (uint32_t)ceil_div_u64(len, align);
  };
  unsigned long long local = 0;
  for (uint32_t e = tid; e < N; e += blockDim.x)
    local += (unsigned long long)PLAN_UNIT * units_of(e) + PLAN_ITEM;
  atomicAdd(&s_total, local);
  __syncthreads();
  const unsigned long long T = s_total;
  // ranges at least PLAN_UNIT apart, so two cuts never land in one unit
  unsigned long long g = T / PLAN_UNIT;
  if (g > max_ranges) g = max_ranges;
  if (g < 1) g = 1;
  const uint32_t G = (uint32_t)g;
  for (uint32_t base = 0; base < N; base += blockDim.x) {
    const uint32_t e = base + tid;
    const bool valid = e < N;
    const uint32_t U = valid ? units_of(e) : 0u;
    const unsigned long long cost = valid ? (unsigned long long)PLAN_UNIT * U + PLAN_ITEM : 0ull;
    // block-wide exclusive scan of the cost
    unsigned long long xc = cost;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, xc, o);
      if (lane >= (uint32_t)o) xc += y;
    }
    if (lane == 31) s_wcost[wid] = xc;
    __syncthreads();
    if (wid == 0) {
      unsigned long long w = lane < nw ? s_wcost[lane] : 0ull;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= (uint32_t)o) w += y;
      }
      s_wcost[lane] = w;
    }
    __syncthreads();
    const unsigned long long S = s_ccarry + (wid ? s_wcost[wid - 1] : 0ull) + xc - cost;
    const unsigned long long E = S + cost;
    // cuts c with S <= P_c < E (only cuts 1 .. G-1 can split anything)
    uint32_t c_lo = 1, c_hi = 1;
    if (valid && T) {
      c_lo = (uint32_t)max(1ull, ceil_div_u64(S * G, T));
      c_hi = (uint32_t)min((unsigned long long)G, ceil_div_u64(E * G, T));
    }
    // the unit a cut splits at, or 0 when it does not split (cut in the item
    // cost or in the last unit)
    auto split_unit = [&](uint32_t c) -> uint32_t {
      const unsigned long long Pc = (unsigned long long)c * T / G;
      if (Pc <= S + PLAN_ITEM) return 0u;
      const unsigned long long u = ceil_div_u64(Pc - S - PLAN_ITEM, PLAN_UNIT);
      return u < U ? (uint32_t)u : 0u;
    };
    uint32_t cnt = valid ? 1u : 0u;
    for (uint32_t c = c_lo; c < c_hi; ++c) cnt += split_unit(c) ? 1u : 0u;
    // block-wide exclusive scan of the item counts
    uint32_t x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= (uint32_t)o) x += y;
    }
    if (lane == 31) s_warp[wid] = x;
    __syncthreads();
    if (wid == 0) {
      uint32_t w = lane < nw ? s_warp[lane] : 0u;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= (uint32_t)o) w += y;
      }
      s_warp[lane] = w;  // inclusive per-warp totals
    }
    __syncthreads();
    const uint32_t first = s_carry + (wid ? s_warp[wid - 1] : 0u) + x - cnt;
    if (valid) {
      seq_first[e] = first;
      seq_count[e] = cnt;
      const uint32_t layer = e / n;
      // item k covers units [u_k, u_{k+1}); u_0 = 0, the last one is open
      uint32_t k = 0, u_start = 0;
      for (uint32_t c = c_lo; c <= c_hi; ++c) {
        const uint32_t u = c < c_hi ? split_unit(c) : 0u;
        if (c < c_hi) {
          // range c starts after the entry's items that begin before the cut;
          // the first item counts as beginning after its item cost, so a cut
          // that lands in that cost hands the whole first item to range c
          const unsigned long long Pc = (unsigned long long)c * T / G;
          ranges[c] = first + (Pc > S + PLAN_ITEM ? 1u : 0u) + k;
        }
        if (c < c_hi && !u) continue;
        if (first + k < max_items) {
          kvcu_item it;
          it.b = e - layer * n;
          it.start = u_start * align;
          it.end = (c == c_hi) ? 0xFFFFFFFFu : u * align;
          it.layer = layer;
          items[first + k] = it;
        }
        ++k;
        u_start = u;
      }
    }
    __syncthreads();
    if (tid == 0) {
      s_carry += s_warp[nw - 1];
      s_ccarry += s_wcost[nw - 1];
    }
    __syncthreads();
  }
  if (tid == 0) {
    const uint32_t n_items = min(s_carry, max_items);
    meta[0] = n_items;
    meta[1] = G;
    ranges[0] = 0;
    ranges[G] = n_items;
  }
}

// ------------------------------------------------------------------ decode
// Resolve the pool row of position `pos` of the sequence with table [t0, t1);
// -1 (and a status bit) when out of range.
__device__ __forceinline__ long long pool_row(const DecodeArgs& a, uint32_t t0, uint32_t t1,
                                              uint32_t pos) {
  const uint32_t bi = pos / a.block_size;
  if (bi >= t1 - t0) {
    atomicOr(a.status, KVCU_STATUS_BAD_TABLE);
    return -1;
  }
  const uint32_t blk = a.tables[t0 + bi];
  if (blk >= a.num_blocks) {
    atomicOr(a.status, KVCU_STATUS_BAD_BLOCK);
    return -1;
  }
  return (long long)(((uint64_t)a.layer * a.num_blocks + blk) * a.block_size + pos % a.block_size);
}

template <bool QUANT, int NH>
__global__ void __launch_bounds__(NT, 1) k_decode(DecodeArgs a) {
  extern __shared__ __align__(16) float smem[];
  float* q_s = smem;                     // [NH][W]
  float* k_s = q_s + NH * W;             // [TT][KS]
  float* red = k_s + TT * KS;            // [NW][NH][TT]
  float* p_s = red + NW * NH * TT;       // [NH][TT]
  float* m_s = p_s + NH * TT;            // [NH]
  float* l_s = m_s + NH;                 // [NH]
  float* c_s = l_s + NH;                 // [NH]

  const uint32_t tid = threadIdx.x, lane = tid & 31u, wid = tid >> 5;
  constexpr int HH = NH / 2;             // heads per PV thread group
  const uint32_t c4 = tid & 127u;        // PV: output columns 4*c4 .. +3
  const uint32_t hg = tid >> 7;          // PV: head group
  const uint32_t n_items = a.meta[0], n_ranges = a.meta[1];
  const uint32_t H = a.n_heads;
  if (blockIdx.x == 0 && tid == 0 && n_ranges > gridDim.x) atomicOr(a.status, KVCU_STATUS_BAD_PLAN);
  const uint32_t it0 = blockIdx.x < n_ranges ? min(a.ranges[blockIdx.x], n_items) : n_items;
  const uint32_t it1 = blockIdx.x < n_ranges ? min(a.ranges[blockIdx.x + 1], n_items) : n_items;

  for (uint32_t it = it0; it < it1; ++it) {
    const kvcu_item item = a.items[it];
    const uint32_t b = item.b;
    const uint32_t s = a.seq_ids ? a.seq_ids[b] : b;
    uint32_t t0 = 0, t1 = 0, len = 0;
    if (s < a.n_seqs) {
      t0 = a.toff[s];
      t1 = a.toff[s + 1];
      if (t1 < t0) t1 = t0;
      len = a.lens[s];
      const uint64_t cap = (uint64_t)(t1 - t0) * a.block_size;
      if (len > cap) {
        if (tid == 0) atomicOr(a.status, KVCU_STATUS_BAD_LEN);
        len = (uint32_t)cap;
      }
      if (a.entry_lens) len = min(len, a.entry_lens[b]);
    } else if (tid == 0) {
      atomicOr(a.status, KVCU_STATUS_BAD_SEQ);
    }
    const uint32_t start = item.start;
    const uint32_t end = min(item.end, len);

    // q for this batch entry (heads >= H are zero)
    const float* qb = a.q + (uint64_t)b * H * W;
    for (uint32_t i = tid; i < NH * (W / 4); i += NT) {
      const uint32_t h = i / (W / 4), e = i % (W / 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (h < H) v = reinterpret_cast<const float4*>(qb + (uint64_t)h * W)[e];
      reinterpret_cast<float4*>(q_s + h * W)[e] = v;
    }
    if (tid < NH) {
      m_s[tid] = -INFINITY;
      l_s[tid] = 0.f;
    }
    float acc[HH][4];
#pragma unroll
    for (int j = 0; j < HH; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    __syncthreads();

    for (uint32_t tb = start; tb < end; tb += TT) {
      const uint32_t tl = min((uint32_t)TT, end - tb);
      // ---- stage the tile (dequantized) into k_s
      if (QUANT) {
        // 16-byte units: 36 per row (32 latent+rope payload halves of 16 B)
        for (uint32_t u = tid; u < TT * (W / 16); u += NT) {
          const uint32_t t = u / (W / 16), h16 = u % (W / 16);
          float* dst = k_s + t * KS + 16 * h16;
          long long row = -1;
          if (t < tl) row = pool_row(a, t0, t1, tb + t);
          if (row < 0) {
#pragma unroll
            for (int k = 0; k < 16; k += 4)
              *reinterpret_cast<float4*>(dst + k) = make_float4(0.f, 0.f, 0.f, 0.f);
            continue;
          }
          const int4 raw =
              *reinterpret_cast<const int4*>(a.qs + (uint64_t)row * (32u * a.nblk) + 16u * h16);
          const float d = kvcu::f16_to_f32(a.sc[(uint64_t)row * a.nblk + h16 / 2]);
          const int8_t* q8 = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
          for (int k = 0; k < 16; k += 4) {
            float4 v;
            v.x = d * (float)q8[k + 0];
            v.y = d * (float)q8[k + 1];
            v.z = d * (float)q8[k + 2];
            v.w = d * (float)q8[k + 3];
            *reinterpret_cast<float4*>(dst + k) = v;
          }
        }
      } else {
        for (uint32_t u = tid; u < TT * (W / 4); u += NT) {
          const uint32_t t = u / (W / 4), e4 = u % (W / 4);
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          long long row = -1;
          if (t < tl) row = pool_row(a, t0, t1, tb + t);
          if (row >= 0) {
            if (e4 < R / 4)
              v = reinterpret_cast<const float4*>(a.kv + (uint64_t)row * R)[e4];
            else
              v = reinterpret_cast<const float4*>(a.pe + (uint64_t)row * P)[e4 - R / 4];
          }
          *reinterpret_cast<float4*>(k_s + t * KS + 4 * e4) = v;
        }
      }
      __syncthreads();

      // ---- QK: warp wid covers K elements [72*wid, 72*wid+72); lane = token
      {
        float sacc[NH];
#pragma unroll
        for (int h = 0; h < NH; ++h) sacc[h] = 0.f;
        const float* krow = k_s + lane * KS + KSLICE * wid;
        const float* qcol = q_s + KSLICE * wid;
#pragma unroll 2
        for (int i = 0; i < KSLICE; i += 4) {
          const float4 kv4 = *reinterpret_cast<const float4*>(krow + i);
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            const float4 q4 = *reinterpret_cast<const float4*>(qcol + h * W + i);
            sacc[h] = fmaf(q4.x, kv4.x, sacc[h]);
            sacc[h] = fmaf(q4.y, kv4.y, sacc[h]);
            sacc[h] = fmaf(q4.z, kv4.z, sacc[h]);
            sacc[h] = fmaf(q4.w, kv4.w, sacc[h]);
          }
        }
#pragma unroll
        for (int h = 0; h < NH; ++h) red[(wid * NH + h) * TT + lane] = sacc[h];
      }
      __syncthreads();
      for (uint32_t i = tid; i < NH * TT; i += NT) {
        const uint32_t h = i / TT, t = i % TT;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) sum += red[(w * NH + h) * TT + t];
        p_s[h * TT + t] = t < tl ? sum * a.scale : -INFINITY;
      }
      __syncthreads();
      // ---- online softmax per head (warp per head)
      for (uint32_t h = wid; h < (uint32_t)NH; h += NW) {
        const float sv = p_s[h * TT + lane];
        const float mt = warp_max(sv);
        const float m_old = m_s[h];
        const float m_new = fmaxf(m_old, mt);
        const float pv = lane < tl ? expf(sv - m_new) : 0.f;
        const float ls = warp_sum(pv);
        p_s[h * TT + lane] = pv;
        if (lane == 0) {
          const float corr = expf(m_old - m_new);
          c_s[h] = corr;
          l_s[h] = l_s[h] * corr + ls;
          m_s[h] = m_new;
        }
      }
      __syncthreads();
      // ---- PV: thread owns columns 4*c4..+3 of heads [hg*HH, hg*HH+HH)
      {
#pragma unroll
        for (int j = 0; j < HH; ++j) {
          const float cr = c_s[hg * HH + j];
          acc[j][0] *= cr;
          acc[j][1] *= cr;
          acc[j][2] *= cr;
          acc[j][3] *= cr;
        }
        for (uint32_t t = 0; t < tl; ++t) {
          const float4 v4 = *reinterpret_cast<const float4*>(k_s + t * KS + 4 * c4);
#pragma unroll
          for (int j = 0; j < HH; ++j) {
            const float pw = p_s[(hg * HH + j) * TT + t];
            acc[j][0] = fmaf(pw, v4.x, acc[j][0]);
            acc[j][1] = fmaf(pw, v4.y, acc[j][1]);
            acc[j][2] = fmaf(pw, v4.z, acc[j][2]);
            acc[j][3] = fmaf(pw, v4.w, acc[j][3]);
          }
        }
      }
      __syncthreads();
    }

    // ---- epilogue: final output or split partial
    const bool single = a.seq_count[b] == 1;
#pragma unroll
    for (int j = 0; j < HH; ++j) {
      const uint32_t h = hg * HH + j;
      if (h >= H) continue;
      const float m = m_s[h], l = l_s[h];
      if (single) {
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        float4 o = make_float4(acc[j][0] * inv, acc[j][1] * inv, acc[j][2] * inv, acc[j][3] * inv);
        if (!(l > 0.f)) o = make_float4(0.f, 0.f, 0.f, 0.f);
        reinterpret_cast<float4*>(a.out + ((uint64_t)b * H + h) * R)[c4] = o;
        if (a.lse && c4 == 0) a.lse[(uint64_t)b * H + h] = l > 0.f ? m + logf(l) : -INFINITY;
      } else {
        reinterpret_cast<float4*>(a.part_o + ((uint64_t)it * a.ws_heads + h) * R)[c4] =
            make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
        if (c4 == 0) {
          a.part_ml[((uint64_t)it * a.ws_heads + h) * 2 + 0] = m;
          a.part_ml[((uint64_t)it * a.ws_heads + h) * 2 + 1] = l;
        }
      }
    }
    __syncthreads();  // m_s/l_s/q_s reused by the next item
  }
}

// ------------------------------------------------------------------ combine
// One CTA of 128 threads per (entry, head): merge the entry's partials.
// One warp per (cut, head).  An entry split into several items has its second
// item start exactly at the CTA range boundary of its first cut inside it
// (ranges[c] == seq_first[b] + 1), so the cuts 1 .. G-1 enumerate the split
// entries without a list; entries decoded as one item were written by the
// decode kernel.  A fixed grid of warps strides over the (G-1) x H tasks.
// Several layers decoded with one one-layer plan (task_layers > 1): the tasks
// of layer i read partials at item index i * part_lstride + item; the tasks of
// all layers share the grid.  A layered plan (task_layers = 1) holds every
// layer's items in one list, and each item carries its layer offset.  Entry
// b's output / lse of layer offset l sit at + l * out_lstride / lse_lstride
// floats, and its item range at plan entry l * plan_n + b.
constexpr int COMBINE_WARPS = 4;
__global__ void __launch_bounds__(32 * COMBINE_WARPS) k_combine(uint32_t H, uint32_t ws_heads,
                                                                const uint32_t* __restrict__ meta,
                                                                const uint32_t* __restrict__ ranges,
                                                                const kvcu_item* __restrict__ items,
                                                                const uint32_t* __restrict__ seq_first,
                                                                const uint32_t* __restrict__ seq_count,
                                                                const float* __restrict__ part_o_all,
                                                                const float* __restrict__ part_ml_all,
                                                                float* __restrict__ out_all, float* __restrict__ lse_all,
                                                                uint32_t task_layers, uint32_t plan_n,
                                                                uint64_t part_lstride, uint64_t out_lstride,
                                                                uint64_t lse_lstride) {
  kvcu_pdl_wait();     // launched programmatically after the decode kernel
  kvcu_pdl_trigger();  // the next layer's append may start launching
  const uint32_t n_items = meta[0], G = meta[1];
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t per_layer = G > 1 ? (G - 1) * H : 0u;
  const uint32_t tasks = per_layer * task_layers;
  for (uint32_t t = blockIdx.x * COMBINE_WARPS + (threadIdx.x >> 5); t < tasks;
       t += gridDim.x * COMBINE_WARPS) {
    const uint32_t lt = t / per_layer, tl = t - lt * per_layer;
    const float* part_o = part_o_all + lt * part_lstride * ws_heads * R;
    const float* part_ml = part_ml_all + lt * part_lstride * ws_heads * 2;
    const uint32_t c = 1 + tl / H, h = tl % H;
    const uint32_t i = ranges[c];
    if (i == 0 || i >= n_items) continue;
    const kvcu_item ki = items[i];
    const uint32_t b = ki.b, li = lt + ki.layer;
    float* out = out_all + li * out_lstride;
    float* lse = lse_all ? lse_all + li * lse_lstride : nullptr;
    const uint32_t e = ki.layer * plan_n + b;
    const uint32_t cnt = seq_count[e], first = seq_first[e];
    if (cnt <= 1 || first + 1 != i) continue;  // no split here, or not the entry's first cut
    float m = -INFINITY;
    for (uint32_t k = 0; k < cnt; ++k) m = fmaxf(m, part_ml[((uint64_t)(first + k) * ws_heads + h) * 2]);
    float l = 0.f;
    float4 o[R / 128];
#pragma unroll
    for (int j = 0; j < R / 128; ++j) o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t k = 0; k < cnt; ++k) {
      const uint64_t base = (uint64_t)(first + k) * ws_heads + h;
      const float mk = part_ml[base * 2], lk = part_ml[base * 2 + 1];
      const float f = (lk > 0.f) ? expf(mk - m) : 0.f;
      l += lk * f;
      const float4* src = reinterpret_cast<const float4*>(part_o + base * R);
#pragma unroll
      for (int j = 0; j < R / 128; ++j) {
        const float4 v = src[lane + 32 * j];
        o[j].x += v.x * f;
        o[j].y += v.y * f;
        o[j].z += v.z * f;
        o[j].w += v.w * f;
      }
    }
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    float4* dst = reinterpret_cast<float4*>(out + ((uint64_t)b * H + h) * R);
#pragma unroll
    for (int j = 0; j < R / 128; ++j)
      dst[lane + 32 * j] = l > 0.f ? make_float4(o[j].x * inv, o[j].y * inv, o[j].z * inv, o[j].w * inv)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    if (lse && lane == 0) lse[(uint64_t)b * H + h] = l > 0.f ? m + logf(l) : -INFINITY;
  }
}

int launch_combine(kvcu_decode_ws* ws, uint32_t n_heads, uint32_t n, float* out, float* lse, cudaStream_t st,
                   uint32_t n_layers_call = 1, uint64_t out_lstride = 0, uint64_t lse_lstride = 0) {
  // the plan makes at most min(max_ranges, decode CTAs) ranges
  uint32_t G = ws->max_ranges;
  if (ws->decode_ctas > 0 && (uint32_t)ws->decode_ctas < G) G = (uint32_t)ws->decode_ctas;
  // a layered plan's cuts already cover every layer
  const uint32_t task_layers = ws->plan_layers > 1 ? 1u : n_layers_call;
  const uint32_t tasks = (G > 1 ? G - 1 : 1) * n_heads * task_layers;
  uint32_t grid = (tasks + COMBINE_WARPS - 1) / COMBINE_WARPS;
  const uint32_t cap = 8u * (uint32_t)(ws->num_sms > 0 ? ws->num_sms : 148);
  if (grid > cap) grid = cap;
  if (grid == 0) grid = 1;
  return kvcu_check_cuda(kvcu_launch_pdl(k_combine, dim3(grid), dim3(32 * COMBINE_WARPS), 0, st, n_heads,
                                         ws->max_heads, (const uint32_t*)ws->meta, (const uint32_t*)ws->ranges,
                                         (const kvcu_item*)ws->items, (const uint32_t*)ws->seq_first,
                                         (const uint32_t*)ws->seq_count, (const float*)ws->part_o,
                                         (const float*)ws->part_ml, out, lse, task_layers, n,
                                         (uint64_t)ws->max_items, out_lstride, lse_lstride),
                         "combine kernel launch");
}

size_t decode_smem(int nh) {
  return sizeof(float) * ((size_t)nh * W + (size_t)TT * KS + (size_t)NW * nh * TT + (size_t)nh * TT +
                          3 * (size_t)nh);
}

// Per-device set-up of one instance (run once per device by kvcu_configure_once).
template <bool QUANT, int NH>
int setup_decode(const void*) {
  return kvcu_check_cuda(cudaFuncSetAttribute(k_decode<QUANT, NH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)decode_smem(NH)),
                         "cudaFuncSetAttribute(decode)");
}

template <bool QUANT, int NH>
int launch_decode_t(kvcu_decode_ws* ws, const DecodeArgs& a, cudaStream_t st) {
  const size_t smem = decode_smem(NH);
  const int rc =
      kvcu_configure_once(reinterpret_cast<const void*>(&k_decode<QUANT, NH>), setup_decode<QUANT, NH>, nullptr);
  if (rc) return rc;
  k_decode<QUANT, NH><<<ws->decode_ctas, NT, smem, st>>>(a);
  return kvcu_check_cuda(cudaGetLastError(), "decode kernel launch");
}

template <bool QUANT>
int launch_decode_q(kvcu_decode_ws* ws, const DecodeArgs& a, cudaStream_t st) {
  const uint32_t H = a.n_heads;
  if (H <= 4) return launch_decode_t<QUANT, 4>(ws, a, st);
  if (H <= 8) return launch_decode_t<QUANT, 8>(ws, a, st);
  if (H <= 16) return launch_decode_t<QUANT, 16>(ws, a, st);
  if (H <= 20) return launch_decode_t<QUANT, 20>(ws, a, st);
  if (H <= 24) return launch_decode_t<QUANT, 24>(ws, a, st);
  return launch_decode_t<QUANT, 32>(ws, a, st);
}

}  // namespace

int kvcu_decode_setup(kvcu_decode_ws* ws) {
  int sms = 0;
  KVCU_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ws->device));
  ws->num_sms = sms > 0 ? sms : 148;
  ws->decode_ctas = ws->num_sms;  // one 256-thread CTA per SM (smem-limited)
  return KVCU_OK;
}

int kvcu_launch_plan(kvcu_decode_ws* ws, const kvcu_pool* p, uint32_t n, const uint32_t* seq_ids,
                     uint32_t n_seqs, const uint32_t* lens, cudaStream_t st, const uint32_t* entry_lens) {
  return kvcu_launch_plan_target(ws, p, n, seq_ids, n_seqs, lens, (uint32_t)ws->decode_ctas, st, entry_lens);
}

// The plan with at most `ranges` CTA ranges. It makes at most n * n_layers +
// ranges - 1 items, so ws->max_items >= n + ranges per layer keeps every item;
// the decode grid (ws->decode_ctas) must be >= ranges.  n_layers > 1 (a
// layered plan) needs ws->max_layers >= n_layers: the items, the per-entry
// ranges and the partials then use the room of that many layers.
int kvcu_launch_plan_target(kvcu_decode_ws* ws, const kvcu_pool* p, uint32_t n,
                            const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* lens,
                            uint32_t ranges, cudaStream_t st, const uint32_t* entry_lens, uint32_t n_layers) {
  if (n_layers < 1 || (n_layers > 1 && n_layers > ws->max_layers)) {
    kvcu_set_error("decode plan: %u layers, the workspace holds %u", n_layers, ws->max_layers);
    return KVCU_ERR_INVALID_ARG;
  }
  const uint32_t align = p->block_size > 128u ? p->block_size : 128u;
  if (ranges > ws->max_ranges) ranges = ws->max_ranges;
  if (ranges > (uint32_t)ws->decode_ctas) ranges = (uint32_t)ws->decode_ctas;
  if (ranges < 1) ranges = 1;
  ws->entry_lens = entry_lens;  // the decodes that use this plan read the same per-entry lengths
  k_plan<<<1, 1024, 0, st>>>(n, n_layers, seq_ids, n_seqs, lens, entry_lens, ranges, align,
                             ws->max_items * n_layers, ws->items, ws->meta, ws->ranges, ws->seq_first,
                             ws->seq_count);
  const int rc = kvcu_check_cuda(cudaGetLastError(), "plan kernel launch");
  // after a failed launch the device holds an older plan of unknown shape: no
  // decode may use it until a plan succeeds
  ws->plan_layers = rc ? 0xFFFFFFFFu : n_layers;
  ws->plan_n = rc ? 0xFFFFFFFFu : n;
  return rc;
}

bool kvcu_decode_layers_fused(const kvcu_decode_ws* ws, const kvcu_pool* p, uint32_t n, uint32_t n_heads) {
  return kvcu_decode_tc_supported(p, n_heads) && n_heads <= ws->max_heads && n <= ws->max_batch &&
         ws->impl != KVCU_DECODE_CUDA_CORE;
}

int kvcu_launch_decode(kvcu_decode_ws* ws, kvcu_pool* p, uint32_t layer, uint32_t n,
                       const uint32_t* seq_ids, uint32_t n_seqs, const uint32_t* toff,
                       const uint32_t* tables, const uint32_t* lens, const float* q,
                       uint32_t n_heads, float scale, float* out, float* lse, cudaStream_t st) {
  if (ws->plan_layers > 1) {
    kvcu_set_error("mla_decode: the workspace's plan covers %u layers as one list; a one-layer decode "
                   "needs kvcu_decode_plan", ws->plan_layers);
    return KVCU_ERR_INVALID_ARG;
  }
  if (n && n != ws->plan_n) {
    kvcu_set_error("mla_decode: batch of %u entries, the workspace's last plan covers %u", n, ws->plan_n);
    return KVCU_ERR_INVALID_ARG;
  }
  const bool tc_ok = kvcu_decode_tc_supported(p, n_heads) && n_heads <= ws->max_heads &&
                     n <= ws->max_batch;
  if (ws->impl == KVCU_DECODE_TENSOR_CORE && !tc_ok) {
    kvcu_set_error("mla_decode: the tensor-core kernel needs a Q8_0 pool with kv_rank 512, rope_dim "
                   "64, <= 24 heads and a block size dividing (or a multiple of) 128");
    return KVCU_ERR_UNSUPPORTED;
  }
  if (tc_ok && ws->impl != KVCU_DECODE_CUDA_CORE) {
    ws->last_launches = 0;
    if (n == 0) return KVCU_OK;
    int rc = kvcu_launch_decode_tc(ws, p, layer, 1, n, seq_ids, n_seqs, toff, tables, lens, q, 0, n_heads,
                                   scale, out, 0, lse, 0, st);
    if (rc) return rc;
    rc = launch_combine(ws, n_heads, n, out, lse, st);
    if (rc) return rc;
    ws->last_launches = 2;
    ws->last_impl = KVCU_DECODE_TENSOR_CORE;
    return KVCU_OK;
  }
  ws->last_impl = KVCU_DECODE_CUDA_CORE;
  if (p->kv_rank != (uint32_t)R || p->rope_dim != (uint32_t)P) {
    kvcu_set_error("mla_decode: kernels are built for kv_rank=%d, rope_dim=%d (pool has %u, %u)", R,
                   P, p->kv_rank, p->rope_dim);
    return KVCU_ERR_UNSUPPORTED;
  }
  if (n_heads == 0 || n_heads > 32 || n_heads > ws->max_heads) {
    kvcu_set_error("mla_decode: n_heads=%u outside [1, min(32, workspace %u)]", n_heads,
                   ws->max_heads);
    return KVCU_ERR_UNSUPPORTED;
  }
  if (n > ws->max_batch) {
    kvcu_set_error("mla_decode: batch %u exceeds workspace capacity %u", n, ws->max_batch);
    return KVCU_ERR_INVALID_ARG;
  }
  ws->last_launches = 0;
  if (n == 0) return KVCU_OK;
  DecodeArgs a;
  a.layer = layer;
  a.num_blocks = p->num_blocks;
  a.block_size = p->block_size;
  a.nblk = p->nblk;
  a.kv = p->kv;
  a.pe = p->pe;
  a.qs = p->qs;
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
  a.scale = scale;
  a.out = out;
  a.items = ws->items;
  a.meta = ws->meta;
  a.ranges = ws->ranges;
  a.seq_count = ws->seq_count;
  a.part_o = ws->part_o;
  a.part_ml = ws->part_ml;
  a.lse = lse;
  a.ws_heads = ws->max_heads;
  a.entry_lens = ws->entry_lens;
  int rc = p->quantized ? launch_decode_q<true>(ws, a, st) : launch_decode_q<false>(ws, a, st);
  if (rc) return rc;
  rc = launch_combine(ws, n_heads, n, out, lse, st);
  if (rc) return rc;
  ws->last_launches = 2;
  return KVCU_OK;
}

int kvcu_launch_decode_layers(kvcu_decode_ws* ws, kvcu_pool* p, uint32_t layer, uint32_t n_layers_call,
                              uint32_t n, const uint32_t* seq_ids, uint32_t n_seqs,
                              const uint32_t* toff, const uint32_t* tables, const uint32_t* lens,
                              const float* q, uint64_t q_lstride, uint32_t n_heads, float scale, float* out,
                              uint64_t out_lstride, float* lse, uint64_t lse_lstride, cudaStream_t st) {
  if (n_layers_call > ws->max_layers) {
    kvcu_set_error("mla_decode: %u layers in one call, the workspace holds %u", n_layers_call, ws->max_layers);
    return KVCU_ERR_INVALID_ARG;
  }
  if (n && n != ws->plan_n) {
    kvcu_set_error("mla_decode: batch of %u entries, the workspace's last plan covers %u", n, ws->plan_n);
    return KVCU_ERR_INVALID_ARG;
  }
  const bool fused = kvcu_decode_layers_fused(ws, p, n, n_heads);
  if (ws->plan_layers > 1 && (ws->plan_layers != n_layers_call || !fused)) {
    kvcu_set_error("mla_decode: the workspace's plan covers %u layers as one list, the call %u layers%s",
                   ws->plan_layers, n_layers_call, fused ? "" : " on the CUDA-core path (one-layer plans only)");
    return KVCU_ERR_INVALID_ARG;
  }
  if (n_layers_call > 1 && fused) {
    // one persistent launch for all layers: every CTA runs its plan range once
    // per layer, or once in all with a layered plan
    ws->last_launches = 0;
    if (n == 0) return KVCU_OK;
    int rc = kvcu_launch_decode_tc(ws, p, layer, n_layers_call, n, seq_ids, n_seqs, toff, tables, lens, q,
                                   q_lstride, n_heads, scale, out, out_lstride, lse, lse_lstride, st);
    if (rc) return rc;
    rc = launch_combine(ws, n_heads, n, out, lse, st, n_layers_call, out_lstride, lse_lstride);
    if (rc) return rc;
    ws->last_launches = 2;
    ws->last_impl = KVCU_DECODE_TENSOR_CORE;
    return KVCU_OK;
  }
  uint32_t launches = 0;
  for (uint32_t i = 0; i < n_layers_call; ++i) {
    const int rc = kvcu_launch_decode(ws, p, layer + i, n, seq_ids, n_seqs, toff, tables, lens, q + i * q_lstride,
                                      n_heads, scale, out + i * out_lstride, lse ? lse + i * lse_lstride : nullptr,
                                      st);
    if (rc) return rc;
    launches += ws->last_launches;
  }
  ws->last_launches = launches;
  return KVCU_OK;
}
