// kvcu_kernels.cu — append (f32 -> Q8_0 quantize + block-table scatter),
// block-table gather/dequant, checkpoint repacking and the seeded generator.
//
// Reference behaviour restated:
//   append  = KVCache.put            src/kv_cache.zig:279-361
//   gather  = getKVCompressed/getKPe src/kv_cache.zig:225-277
//   repack  = the BlockQ8_0 byte order of saveToFile/loadFromFile
//             (src/kv_cache.zig:484-492, :535-545; BlockQ8_0 src/dequant.zig:372-377)
//
// All three are HBM-bound byte/integer work with a little f32 arithmetic:
// one warp owns one 32-element Q8_0 block (one 128-byte coalesced f32 read,
// one 32-byte int8 write, a 5-step shuffle max), grids are sized in multiples
// of the SM count and loop grid-stride.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kvcu_internal.h"
#include "kvcu_numeric.cuh"

namespace {

struct PoolArgs {
  uint32_t layer, num_blocks, block_size, kv_rank, rope_dim, nbk, nbp, nblk;
  uint32_t bs_log2;  // log2(block_size) when it is a power of two, else 32
  float* kv;
  float* pe;
  int8_t* qs;
  uint16_t* sc;
  uint32_t* status;
};

PoolArgs pool_args(kvcu_pool* p, uint32_t layer) {
  PoolArgs a;
  a.layer = layer;
  a.num_blocks = p->num_blocks;
  a.block_size = p->block_size;
  a.bs_log2 = 32;
  for (uint32_t k = 0; k < 32; ++k)
    if ((1u << k) == p->block_size) a.bs_log2 = k;
  a.kv_rank = p->kv_rank;
  a.rope_dim = p->rope_dim;
  a.nbk = p->nbk;
  a.nbp = p->nbp;
  a.nblk = p->nblk;
  a.kv = p->kv;
  a.pe = p->pe;
  a.qs = p->qs;
  a.sc = p->sc;
  a.status = p->status;
  return a;
}

int grid_for(uint64_t warps, int threads) {
  const int sms = kvcu_current_sm_count();
  uint64_t blocks = (warps * 32 + threads - 1) / threads;
  uint64_t cap = (uint64_t)sms * 16;  // 16 resident 256-thread CTAs per SM at most
  if (blocks > cap) blocks = cap;
  if (blocks == 0) blocks = 1;
  return (int)blocks;
}

// Resolve (sequence, position) -> pool row; returns false (and flags the
// status word once per warp) when an index is out of range.
__device__ __forceinline__ bool resolve_row(const PoolArgs& a, uint32_t s, uint32_t pos,
                                            uint32_t n_seqs, const uint32_t* __restrict__ toff,
                                            const uint32_t* __restrict__ tables, uint32_t lane,
                                            uint64_t* row) {
  if (s >= n_seqs) {
    if (lane == 0) atomicOr(a.status, KVCU_STATUS_BAD_SEQ);
    return false;
  }
  uint32_t t0 = toff[s], t1 = toff[s + 1];
  // a shift and a mask for power-of-two block sizes (a uniform branch)
  const uint32_t bi = a.bs_log2 < 32 ? pos >> a.bs_log2 : pos / a.block_size;
  const uint32_t off = a.bs_log2 < 32 ? pos & (a.block_size - 1u) : pos % a.block_size;
  if (t1 < t0 || bi >= t1 - t0) {
    if (lane == 0) atomicOr(a.status, KVCU_STATUS_BAD_TABLE);
    return false;
  }
  uint32_t blk = tables[t0 + bi];
  if (blk >= a.num_blocks) {
    if (lane == 0) atomicOr(a.status, KVCU_STATUS_BAD_BLOCK);
    return false;
  }
  *row = ((uint64_t)a.layer * a.num_blocks + blk) * a.block_size + off;
  return true;
}

// One warp per (row, 32-element block).  Q8_0: amax over the block,
// d = amax/127, d16 = f32ToF16(d), q = clamp(round(x/d)), tail zero-fill.
template <bool QUANT>
__global__ void __launch_bounds__(256) k_append(PoolArgs a, uint32_t n_rows,
                                                const float* __restrict__ latent, uint64_t ls,
                                                const float* __restrict__ rope, uint64_t ps,
                                                const uint32_t* __restrict__ row_seq,
                                                const uint32_t* __restrict__ row_pos,
                                                uint32_t n_seqs, const uint32_t* __restrict__ toff,
                                                const uint32_t* __restrict__ tables,
                                                uint32_t* __restrict__ lens) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const uint32_t W = a.kv_rank + a.rope_dim;
  const uint32_t nper = QUANT ? a.nblk : (W + 31u) / 32u;
  const uint64_t total = (uint64_t)n_rows * nper;
  for (uint64_t wi = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < total;
       wi += nwarps) {
    const uint32_t r = (uint32_t)(wi / nper), b = (uint32_t)(wi % nper);
    uint64_t row;
    if (!resolve_row(a, row_seq[r], row_pos[r], n_seqs, toff, tables, lane, &row)) continue;
    // len = max(len, pos + 1), src/kv_cache.zig:358-360 (once per row)
    if (lens && b == 0 && lane == 0) atomicMax(lens + row_seq[r], row_pos[r] + 1u);
    if (QUANT) {
      const float* src;
      uint32_t cnt;
      if (b < a.nbk) {
        src = latent + (uint64_t)r * ls + 32u * b;
        cnt = min(32u, a.kv_rank - 32u * b);
      } else {
        src = rope + (uint64_t)r * ps + 32u * (b - a.nbk);
        cnt = min(32u, a.rope_dim - 32u * (b - a.nbk));
      }
      const float x = lane < cnt ? src[lane] : 0.0f;
      float amax = fabsf(x);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float d = kvcu::q8_scale(amax);
      const int8_t q = (d > 0.0f && lane < cnt) ? kvcu::q8_value(x, d) : (int8_t)0;
      a.qs[row * (32u * a.nblk) + 32u * b + lane] = q;
      if (lane == 0) a.sc[row * a.nblk + b] = kvcu::f32_to_f16(d);
    } else {
      const uint32_t e = 32u * b + lane;
      if (e < a.kv_rank) a.kv[row * a.kv_rank + e] = latent[(uint64_t)r * ls + e];
      else if (e < W) a.pe[row * a.rope_dim + (e - a.kv_rank)] = rope[(uint64_t)r * ps + (e - a.kv_rank)];
    }
  }
}

// Fast append for the usual shapes (kv_rank and rope_dim multiples of 32,
// 16-byte aligned source rows): one warp per row, so the row's sequence /
// table lookups happen once; each 8-lane group owns one 32-element block per
// step (one float4 per lane, a 3-step shuffle max, one 4-byte store per lane).
// Same bytes as k_append.
// WHOLE_ROW: each row (up to 4 x APPEND_PREFETCH_GROUPS Q8_0 blocks, i.e.
// kv_rank + rope_dim <= 1024) is loaded whole before its table lookup.  That
// hides the lookup for small, latency-bound batches (one token per sequence);
// large batches keep the leaner form, whose lower register count keeps more
// warps resident.
constexpr int APPEND_PREFETCH_GROUPS = 8;
constexpr uint32_t APPEND_WHOLE_ROW_MAX_ROWS = 16384;

// Layers: rows of layer a.layer + i come from latent + i*llat / rope + i*lrope
// (n_layers_call >= 1); every (row, layer) pair is one warp's work.
template <bool QUANT, bool WHOLE_ROW>
__global__ void __launch_bounds__(256) k_append_rows(PoolArgs a, uint32_t n_rows,
                                                     const float* __restrict__ latent, uint64_t ls,
                                                     const float* __restrict__ rope, uint64_t ps,
                                                     const uint32_t* __restrict__ row_seq,
                                                     const uint32_t* __restrict__ row_pos,
                                                     uint32_t n_seqs, const uint32_t* __restrict__ toff,
                                                     const uint32_t* __restrict__ tables,
                                                     uint32_t* __restrict__ lens, uint32_t n_layers_call,
                                                     uint64_t llat, uint64_t lrope) {
  const uint32_t lane = threadIdx.x & 31u, grp = lane >> 3, sub = lane & 7u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const uint32_t nblk = a.nbk + a.nbp;
  kvcu_pdl_wait();     // the previous kernel may still read the rows this one writes
  kvcu_pdl_trigger();  // a programmatically launched decode may start its prologue
  // one 4-block group of the row: 8 lanes per block, a float4 each
  auto put_group = [&](uint64_t r, uint64_t row, uint32_t b, bool act, float4 x) {
    if (QUANT) {
      float amax = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float d = kvcu::q8_scale(amax);
      const float inv = d > 0.0f ? __frcp_rn(d) : 0.0f;
      char4 q = make_char4(0, 0, 0, 0);
      if (d > 0.0f) {
        q.x = kvcu::q8_value_fast(x.x, d, inv);
        q.y = kvcu::q8_value_fast(x.y, d, inv);
        q.z = kvcu::q8_value_fast(x.z, d, inv);
        q.w = kvcu::q8_value_fast(x.w, d, inv);
      }
      if (act) {
        *reinterpret_cast<char4*>(a.qs + row * (32u * nblk) + 32u * b + 4u * sub) = q;
        // the hardware RNE conversion gives the same bits as f32_to_f16 for
        // every non-NaN d (normal, subnormal, overflow to inf)
        if (sub == 0) a.sc[row * nblk + b] = d == d ? __half_as_ushort(__float2half_rn(d)) : kvcu::f32_to_f16(d);
      }
    } else if (act) {
      float* dst = b < a.nbk ? a.kv + row * a.kv_rank + 32u * b + 4u * sub
                             : a.pe + row * a.rope_dim + 32u * (b - a.nbk) + 4u * sub;
      *reinterpret_cast<float4*>(dst) = x;
    }
  };
  const uint64_t layer_rows = (uint64_t)a.num_blocks * a.block_size;
  const uint64_t total = (uint64_t)n_rows * n_layers_call;
  for (uint64_t ra = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; ra < total; ra += nwarps) {
    const uint64_t li = ra / n_rows, r = ra - li * n_rows;
    const float* lat_l = latent + li * llat;
    const float* rope_l = rope + li * lrope;
    auto load_group = [&](uint64_t r, uint32_t b) -> float4 {
      const float* src = b < a.nbk ? lat_l + r * ls + 32u * b + 4u * sub
                                   : rope_l + r * ps + 32u * (b - a.nbk) + 4u * sub;
      return __ldg(reinterpret_cast<const float4*>(src));
    };
    const uint32_t s = row_seq[r], pos = row_pos[r];
    if (WHOLE_ROW) {
      // The whole row is loaded first, so that its loads overlap the block
      // table lookup below (the input does not depend on the table).
      float4 xs[APPEND_PREFETCH_GROUPS];
#pragma unroll
      for (uint32_t g = 0; g < (uint32_t)APPEND_PREFETCH_GROUPS; ++g) {
        const uint32_t b = 4u * g + grp;
        xs[g] = b < nblk ? load_group(r, b) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      uint64_t row;
      if (!resolve_row(a, s, pos, n_seqs, toff, tables, lane, &row)) continue;
      row += li * layer_rows;
      // len = max(len, pos + 1), src/kv_cache.zig:358-360
      if (lens && li == 0 && lane == 0) atomicMax(lens + s, pos + 1u);
#pragma unroll
      for (uint32_t g = 0; g < (uint32_t)APPEND_PREFETCH_GROUPS; ++g)
        if (4u * g < nblk) put_group(r, row, 4u * g + grp, 4u * g + grp < nblk, xs[g]);  // warp-uniform test
    } else {
      uint64_t row;
      if (!resolve_row(a, s, pos, n_seqs, toff, tables, lane, &row)) continue;
      row += li * layer_rows;
      if (lens && li == 0 && lane == 0) atomicMax(lens + s, pos + 1u);
      for (uint32_t b0 = 0; b0 < nblk; b0 += 4) {
        const uint32_t b = b0 + grp;
        const bool act = b < nblk;
        put_group(r, row, b, act, act ? load_group(r, b) : make_float4(0.f, 0.f, 0.f, 0.f));
      }
    }
  }
}

// Q8_0 append for rows of whole 32-element blocks (kv_rank and rope_dim
// multiples of 32, 16-byte aligned sources, at most 8*NS blocks a row): one
// warp per (row, layer).  A 4-lane group quantizes one block per step, 8
// values a lane (two float4 loads, a 2-step shuffle max, one 8-byte store), so
// a 576-wide row is 3 steps and the per-block work (scale division, f16
// conversion, scale store) is shared by 4 lanes instead of 8.  The whole row
// is loaded before its block-table lookup, so both latencies overlap.  Same
// bytes as k_append.
template <int NS>
__global__ void __launch_bounds__(256) k_append_q8(PoolArgs a, uint32_t n_rows, const float* __restrict__ latent,
                                                   uint64_t ls, const float* __restrict__ rope, uint64_t ps,
                                                   const uint32_t* __restrict__ row_seq,
                                                   const uint32_t* __restrict__ row_pos, uint32_t n_seqs,
                                                   const uint32_t* __restrict__ toff,
                                                   const uint32_t* __restrict__ tables, uint32_t* __restrict__ lens,
                                                   uint32_t n_layers_call, uint64_t llat, uint64_t lrope) {
  const uint32_t lane = threadIdx.x & 31u, grp = lane >> 2, sub = lane & 3u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const uint32_t nblk = a.nbk + a.nbp;
  kvcu_pdl_wait();     // the previous kernel may still read the rows this one writes
  kvcu_pdl_trigger();  // a programmatically launched decode may start its prologue
  const uint64_t layer_rows = (uint64_t)a.num_blocks * a.block_size;
  // (layer, row) pairs in layer-major order without a division per row: the
  // warp's first pair, then steps of nwarps carried across layers
  const uint32_t w0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (uint32_t)nwarps;
  uint32_t li = w0 / n_rows, r = w0 - li * n_rows;
  const uint32_t step_l = nw / n_rows, step_r = nw - step_l * n_rows;
  for (; li < n_layers_call; li += step_l, r += step_r) {
    if (r >= n_rows) {
      r -= n_rows;
      if (++li >= n_layers_call) break;
    }
    const float* lat_r = latent + li * llat + r * ls;
    const float* rope_r = rope + li * lrope + r * ps;
    const uint32_t s = row_seq[r], pos = row_pos[r];
    float4 xa[NS], xb[NS];
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      const uint32_t b = 8u * k + grp, e = 32u * b + 8u * sub;
      xa[k] = xb[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (b < nblk) {
        const float* src = e < a.kv_rank ? lat_r + e : rope_r + (e - a.kv_rank);
        xa[k] = __ldg(reinterpret_cast<const float4*>(src));
        xb[k] = __ldg(reinterpret_cast<const float4*>(src + 4));
      }
    }
    uint64_t row;
    if (!resolve_row(a, s, pos, n_seqs, toff, tables, lane, &row)) continue;
    row += li * layer_rows;
    // len = max(len, pos + 1), src/kv_cache.zig:358-360
    if (lens && li == 0 && lane == 0) atomicMax(lens + s, pos + 1u);
    int8_t* qrow = a.qs + row * (32u * nblk);
    uint16_t* srow = a.sc + row * nblk;
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      if (8u * k >= nblk) break;  // warp-uniform
      const uint32_t b = 8u * k + grp;
      const float v[8] = {xa[k].x, xa[k].y, xa[k].z, xa[k].w, xb[k].x, xb[k].y, xb[k].z, xb[k].w};
      float amax = fabsf(v[0]);
#pragma unroll
      for (int i = 1; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const float d = kvcu::q8_scale(amax);
      // round(x/d) through a multiply (q8_value_fast's argument) for all 8
      // values without a branch each; if any lane of the warp met a value near a
      // half-integer (or a NaN / inf), the whole warp redoes its values with the
      // IEEE quotient (rare), so the common path has no divergence
      const float inv = d > 0.0f ? kvcu::rcp_approx(d) : 0.0f;
      int qv[8];
      bool near_tie = false;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float t = v[i] * inv;
        const float r = rintf(t);
        near_tie |= !(fabsf(t - r) < 0.4999f);
        qv[i] = (int)r;
      }
      if (__any_sync(0xffffffffu, near_tie && d > 0.0f)) {
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[i] = d > 0.0f ? kvcu::q8_value(v[i], d) : 0;
      }
      uint32_t w[2] = {0u, 0u};
      if (d > 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i >> 2] |= (uint32_t)(uint8_t)(int8_t)qv[i] << (8 * (i & 3));
      }
      if (b < nblk) {
        *reinterpret_cast<uint2*>(qrow + 32u * b + 8u * sub) = make_uint2(w[0], w[1]);
        // the hardware RNE conversion gives the same bits as f32_to_f16 for
        // every non-NaN d (normal, subnormal, overflow to inf)
        if (sub == 0) srow[b] = d == d ? __half_as_ushort(__float2half_rn(d)) : kvcu::f32_to_f16(d);
      }
    }
  }
}

// One warp per (row, 32-element block): out = f16ToF32(d) * q, or the f32 row.
// Rows come either from one table (table != nullptr, row r = position r) or
// from (row_seq[r], row_pos[r]) through the CSR tables.
template <bool QUANT>
__global__ void __launch_bounds__(256) k_gather(PoolArgs a, uint32_t n_rows,
                                                const uint32_t* __restrict__ row_seq,
                                                const uint32_t* __restrict__ row_pos,
                                                uint32_t n_seqs, const uint32_t* __restrict__ toff,
                                                const uint32_t* __restrict__ tables,
                                                const uint32_t* __restrict__ table,
                                                uint32_t table_len, float* __restrict__ out) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const uint32_t W = a.kv_rank + a.rope_dim;
  const uint32_t nper = QUANT ? a.nblk : (W + 31u) / 32u;
  const uint64_t total = (uint64_t)n_rows * nper;
  for (uint64_t wi = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < total;
       wi += nwarps) {
    const uint32_t r = (uint32_t)(wi / nper), b = (uint32_t)(wi % nper);
    uint64_t row;
    if (table) {
      const uint32_t bi = r / a.block_size;
      if (bi >= table_len) {
        if (lane == 0) atomicOr(a.status, KVCU_STATUS_BAD_TABLE);
        continue;
      }
      const uint32_t blk = table[bi];
      if (blk >= a.num_blocks) {
        if (lane == 0) atomicOr(a.status, KVCU_STATUS_BAD_BLOCK);
        continue;
      }
      row = ((uint64_t)a.layer * a.num_blocks + blk) * a.block_size + r % a.block_size;
    } else if (!resolve_row(a, row_seq[r], row_pos[r], n_seqs, toff, tables, lane, &row)) {
      continue;
    }
    float* dst = out + (uint64_t)r * W;
    if (QUANT) {
      uint32_t e, cnt;
      if (b < a.nbk) {
        e = 32u * b;
        cnt = min(32u, a.kv_rank - e);
      } else {
        e = a.kv_rank + 32u * (b - a.nbk);
        cnt = min(32u, a.rope_dim - 32u * (b - a.nbk));
      }
      if (lane < cnt) {
        const float d = kvcu::f16_to_f32(a.sc[row * a.nblk + b]);
        const float q = (float)a.qs[row * (32u * a.nblk) + 32u * b + lane];
        dst[e + lane] = __fmul_rn(d, q);
      }
    } else {
      const uint32_t e = 32u * b + lane;
      if (e < a.kv_rank) dst[e] = a.kv[row * a.kv_rank + e];
      else if (e < W) dst[e] = a.pe[row * a.rope_dim + (e - a.kv_rank)];
    }
  }
}

// Fast gather for the usual shapes (kv_rank and rope_dim multiples of 32, the
// output 16-byte aligned): one warp per row, so the row's table lookup happens
// once; each step covers 128 consecutive elements of the row, lane l the four
// at 4l (a 4-byte Q8_0 load, its block's scale, one float4 store), so loads
// and stores are coalesced.  Same values as k_gather: f16ToF32(d) * q rounded
// once (the product of an 11-bit and an 8-bit integer is exact in f32).
template <bool QUANT>
__global__ void __launch_bounds__(256) k_gather_rows(PoolArgs a, uint32_t n_rows,
                                                     const uint32_t* __restrict__ row_seq,
                                                     const uint32_t* __restrict__ row_pos,
                                                     uint32_t n_seqs, const uint32_t* __restrict__ toff,
                                                     const uint32_t* __restrict__ tables,
                                                     const uint32_t* __restrict__ table,
                                                     uint32_t table_len, float* __restrict__ out) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const uint32_t W = a.kv_rank + a.rope_dim;
  const uint32_t nblk = a.nbk + a.nbp;
  for (uint64_t r = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n_rows; r += nwarps) {
    uint64_t row;
    if (table) {
      const uint32_t bi = (uint32_t)(r / a.block_size);
      if (bi >= table_len) {
        if (lane == 0) atomicOr(a.status, KVCU_STATUS_BAD_TABLE);
        continue;
      }
      const uint32_t blk = table[bi];
      if (blk >= a.num_blocks) {
        if (lane == 0) atomicOr(a.status, KVCU_STATUS_BAD_BLOCK);
        continue;
      }
      row = ((uint64_t)a.layer * a.num_blocks + blk) * a.block_size + r % a.block_size;
    } else if (!resolve_row(a, row_seq[r], row_pos[r], n_seqs, toff, tables, lane, &row)) {
      continue;
    }
    float* dst = out + r * W;
    if (QUANT) {
      const int8_t* src = a.qs + row * (32u * nblk);  // latent blocks then rope blocks: W bytes
      const uint16_t* sc = a.sc + row * nblk;
      for (uint32_t e = 4u * lane; e < W; e += 128u) {
        const char4 q = *reinterpret_cast<const char4*>(src + e);
        const float d = kvcu::f16_to_f32(sc[e >> 5]);
        *reinterpret_cast<float4*>(dst + e) =
            make_float4(__fmul_rn(d, (float)q.x), __fmul_rn(d, (float)q.y), __fmul_rn(d, (float)q.z),
                        __fmul_rn(d, (float)q.w));
      }
    } else {
      for (uint32_t e = 4u * lane; e < W; e += 128u) {
        const float* s = e < a.kv_rank ? a.kv + row * a.kv_rank + e : a.pe + row * a.rope_dim + (e - a.kv_rank);
        *reinterpret_cast<float4*>(dst + e) = __ldg(reinterpret_cast<const float4*>(s));
      }
    }
  }
}

// Checkpoint repacking between the device layout (qs / sc split) and the
// reference's 34-byte BlockQ8_0 order.  part 0 = latent blocks of every row,
// part 1 = rope blocks of every row.  One warp per 34-byte block.
__global__ void __launch_bounds__(256) k_pack_q8(PoolArgs a, int part, uint64_t blk0,
                                                 uint64_t nblocks, uint8_t* __restrict__ dst) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const uint32_t per = part == 0 ? a.nbk : a.nbp;
  for (uint64_t wi = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < nblocks;
       wi += nwarps) {
    const uint64_t k = blk0 + wi;
    const uint64_t row = k / per;
    const uint32_t j = (uint32_t)(k % per) + (part == 0 ? 0u : a.nbk);
    uint8_t* o = dst + wi * 34u;
    o[2 + lane] = (uint8_t)a.qs[row * (32u * a.nblk) + 32u * j + lane];
    if (lane == 0) {
      const uint16_t d = a.sc[row * a.nblk + j];
      o[0] = (uint8_t)(d & 0xFFu);
      o[1] = (uint8_t)(d >> 8);
    }
  }
}

__global__ void __launch_bounds__(256) k_unpack_q8(PoolArgs a, int part, uint64_t blk0,
                                                   uint64_t nblocks, const uint8_t* __restrict__ src) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const uint32_t per = part == 0 ? a.nbk : a.nbp;
  for (uint64_t wi = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < nblocks;
       wi += nwarps) {
    const uint64_t k = blk0 + wi;
    const uint64_t row = k / per;
    const uint32_t j = (uint32_t)(k % per) + (part == 0 ? 0u : a.nbk);
    const uint8_t* s = src + wi * 34u;
    a.qs[row * (32u * a.nblk) + 32u * j + lane] = (int8_t)s[2 + lane];
    if (lane == 0) a.sc[row * a.nblk + j] = (uint16_t)(s[0] | ((uint16_t)s[1] << 8));
  }
}

__global__ void __launch_bounds__(256) k_synth(uint64_t seed, uint64_t a, uint32_t n_rows,
                                               const uint32_t* __restrict__ b,
                                               const uint32_t* __restrict__ c, uint32_t width,
                                               float outlier_p, float* __restrict__ out) {
  const uint64_t total = (uint64_t)n_rows * width;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t r = (uint32_t)(i / width), e = (uint32_t)(i % width);
    out[i] = kvcu::gen_normal(seed, a, b[r], (uint64_t)c[r] * 1024u + e, outlier_p);
  }
}

}  // namespace

int kvcu_launch_append(kvcu_pool* p, uint32_t layer, uint32_t n_rows, const float* latent,
                       uint64_t ls, const float* rope, uint64_t ps, const uint32_t* row_seq,
                       const uint32_t* row_pos, uint32_t n_seqs, const uint32_t* toff,
                       const uint32_t* tables, uint32_t* lens, cudaStream_t st) {
  return kvcu_launch_append_layers(p, layer, 1, n_rows, latent, ls, 0, rope, ps, 0, row_seq, row_pos, n_seqs, toff,
                                   tables, lens, st);
}

int kvcu_launch_append_layers(kvcu_pool* p, uint32_t layer, uint32_t n_layers_call, uint32_t n_rows,
                              const float* latent, uint64_t ls, uint64_t llat, const float* rope, uint64_t ps,
                              uint64_t lrope, const uint32_t* row_seq, const uint32_t* row_pos, uint32_t n_seqs,
                              const uint32_t* toff, const uint32_t* tables, uint32_t* lens, cudaStream_t st) {
  if (n_rows == 0 || n_layers_call == 0) return KVCU_OK;
  PoolArgs a = pool_args(p, layer);
  const bool rows_ok = p->kv_rank % 32 == 0 && p->rope_dim % 32 == 0 && ls % 4 == 0 && ps % 4 == 0 &&
                       llat % 4 == 0 && lrope % 4 == 0 && (reinterpret_cast<uintptr_t>(latent) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(rope) & 15) == 0;
  if (rows_ok && p->quantized && p->nblk <= 32u) {
    const uint64_t pairs = (uint64_t)n_rows * n_layers_call;
    const int g = grid_for(pairs, 256);
    auto kern = p->nblk <= 24u ? (p->nblk <= 16u ? k_append_q8<2> : k_append_q8<3>) : k_append_q8<4>;
    return kvcu_check_cuda(kvcu_launch_pdl(kern, dim3(g), dim3(256), 0, st, a, n_rows, latent, ls, rope, ps,
                                           row_seq, row_pos, n_seqs, toff, tables, lens, n_layers_call, llat,
                                           lrope),
                           "append kernel launch");
  }
  if (rows_ok) {
    const uint64_t pairs = (uint64_t)n_rows * n_layers_call;
    const int g = grid_for(pairs, 256);
    // programmatic launch: it waits for the previous kernel before any access
    const bool whole = pairs <= APPEND_WHOLE_ROW_MAX_ROWS && p->nblk <= 4u * APPEND_PREFETCH_GROUPS;
    auto kern = p->quantized ? (whole ? k_append_rows<true, true> : k_append_rows<true, false>)
                             : (whole ? k_append_rows<false, true> : k_append_rows<false, false>);
    return kvcu_check_cuda(kvcu_launch_pdl(kern, dim3(g), dim3(256), 0, st, a, n_rows, latent, ls, rope, ps,
                                           row_seq, row_pos, n_seqs, toff, tables, lens, n_layers_call, llat,
                                           lrope),
                           "append kernel launch");
  }
  const uint32_t nper = p->quantized ? p->nblk : (p->kv_rank + p->rope_dim + 31) / 32;
  const int g = grid_for((uint64_t)n_rows * nper, 256);
  for (uint32_t i = 0; i < n_layers_call; ++i) {
    a.layer = layer + i;
    if (p->quantized)
      k_append<true><<<g, 256, 0, st>>>(a, n_rows, latent + i * llat, ls, rope + i * lrope, ps, row_seq, row_pos,
                                        n_seqs, toff, tables, lens);
    else
      k_append<false><<<g, 256, 0, st>>>(a, n_rows, latent + i * llat, ls, rope + i * lrope, ps, row_seq, row_pos,
                                         n_seqs, toff, tables, lens);
    const int rc = kvcu_check_cuda(cudaGetLastError(), "append kernel launch");
    if (rc) return rc;
  }
  return KVCU_OK;
}

int kvcu_launch_gather_rows(kvcu_pool* p, uint32_t layer, uint32_t n_rows, const uint32_t* row_seq,
                            const uint32_t* row_pos, uint32_t n_seqs, const uint32_t* toff,
                            const uint32_t* tables, const uint32_t* table, uint32_t table_len,
                            float* out, cudaStream_t st) {
  if (n_rows == 0) return KVCU_OK;
  PoolArgs a = pool_args(p, layer);
  if (p->kv_rank % 32 == 0 && p->rope_dim % 32 == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
    const int gr = grid_for(n_rows, 256);
    if (p->quantized)
      k_gather_rows<true><<<gr, 256, 0, st>>>(a, n_rows, row_seq, row_pos, n_seqs, toff, tables, table, table_len,
                                              out);
    else
      k_gather_rows<false><<<gr, 256, 0, st>>>(a, n_rows, row_seq, row_pos, n_seqs, toff, tables, table, table_len,
                                               out);
    return kvcu_check_cuda(cudaGetLastError(), "gather kernel launch");
  }
  const uint32_t nper = p->quantized ? p->nblk : (p->kv_rank + p->rope_dim + 31) / 32;
  const int g = grid_for((uint64_t)n_rows * nper, 256);
  if (p->quantized)
    k_gather<true><<<g, 256, 0, st>>>(a, n_rows, row_seq, row_pos, n_seqs, toff, tables, table,
                                      table_len, out);
  else
    k_gather<false><<<g, 256, 0, st>>>(a, n_rows, row_seq, row_pos, n_seqs, toff, tables, table,
                                       table_len, out);
  return kvcu_check_cuda(cudaGetLastError(), "gather kernel launch");
}

int kvcu_launch_pack_q8(kvcu_pool* p, int part, uint64_t blk0, uint64_t nblocks, uint8_t* dst,
                        cudaStream_t st) {
  if (!nblocks) return KVCU_OK;
  k_pack_q8<<<grid_for(nblocks, 256), 256, 0, st>>>(pool_args(p, 0), part, blk0, nblocks, dst);
  return kvcu_check_cuda(cudaGetLastError(), "pack kernel launch");
}

int kvcu_launch_unpack_q8(kvcu_pool* p, int part, uint64_t blk0, uint64_t nblocks,
                          const uint8_t* src, cudaStream_t st) {
  if (!nblocks) return KVCU_OK;
  k_unpack_q8<<<grid_for(nblocks, 256), 256, 0, st>>>(pool_args(p, 0), part, blk0, nblocks, src);
  return kvcu_check_cuda(cudaGetLastError(), "unpack kernel launch");
}

int kvcu_launch_synth(uint64_t seed, uint64_t a, uint32_t n_rows, const uint32_t* b,
                      const uint32_t* c, uint32_t width, float outlier_p, float* out,
                      cudaStream_t st) {
  const uint64_t total = (uint64_t)n_rows * width;
  if (!total) return KVCU_OK;
  k_synth<<<grid_for((total + 31) / 32, 256), 256, 0, st>>>(seed, a, n_rows, b, c, width,
                                                           outlier_p, out);
  return kvcu_check_cuda(cudaGetLastError(), "synth kernel launch");
}
