// kvcu_mla.cu — the MLA decode step around the cache, in absorbed form.
//
// Per new token at position pos, the reference (src/inference.zig:492-513,
// 518-660) computes
//   c     = RMSNorm(kv_a[0:R]) * w                       (src/math.zig:7-35)
//   k_pe  = RoPE(kv_a[R:R+P], pos)                        (src/math.zig:197-240)
//   q_h   = [q_nope_h, RoPE(q_rope_h, pos)]               per head h
//   put(layer, pos, c, k_pe)
//   for p <= pos: k_nope_p = k_b_h c_p, v_p = v_b_h c_p   (matVecMul, math.zig:79-99)
//                 s_p = (q_nope_h . k_nope_p + q_rope_h . k_pe_p) / sqrt(head_dim)
//   out_h = sum_p softmax(s)_p v_p
// where c_pos is the unquantized c and every k_pe_p, and c_p for p < pos,
// come from the cache. Moving k_b to the query and v_b to the output
// (absorption) reads the cache once as 576-wide rows:
//   q_abs_h = [k_b_h^T q_nope_h, RoPE(q_rope_h, pos)],  s_p = q_abs_h . [c_p, k_pe_p] * scale
//   out_h   = v_b_h (sum_p softmax(s)_p c_p)
// The step is three calls around the existing append and decode:
//   kvcu_mla_prepare  rows[b] = [c, k_pe], q_abs              k_mla_rows + k_head_gemm
//   kvcu_append(rows) at pos; kvcu_mla_decode_lse over p < pos (the history)
//   kvcu_mla_finish   merges the newest token as the reference treats it
//                     (unquantized c, k_pe as the cache holds it), then v_b
//                     k_mla_merge + k_head_gemm; the cache's own step uses
//                     k_mla_merge_w + a v_b GEMM that applies the merge weights
//                     while it loads the latent (kvcu_mla_finish_fused)
// The two per-head products are small f32 GEMMs (k_b: n x qk_nope x R, v_b:
// n x R x v_dim per head), ~1.3 GFLOP each at a 512-sequence batch. They run
// on the tensor cores as 3xTF32 (k_head_gemm_tc, f32-level error) where the
// shapes allow, else on the CUDA cores in f32, as exact as the reference's
// matVecMul.
#include <cuda_runtime.h>
#include <math.h>

#include "kvcu_internal.h"
#include "kvcu_numeric.cuh"

namespace {

constexpr int ROWS_THREADS = 256;

// One CTA per batch entry: RMSNorm of the latent, RoPE of k_pe and of every
// head's q_rope. Multiplies and adds are _rn so that no FMA contraction
// changes a rounding against the reference's f32 arithmetic.
__global__ void __launch_bounds__(ROWS_THREADS)
    k_mla_rows(uint32_t H, uint32_t qk_nope, uint32_t R, uint32_t P, const float* __restrict__ q,
               const float* __restrict__ kv_a, const uint32_t* __restrict__ pos,
               const float* __restrict__ norm_w, float eps, float rope_base, float* __restrict__ q_abs,
               float* __restrict__ rows) {
  __shared__ float red[ROWS_THREADS / 32];
  kvcu_pdl_wait();     // launched programmatically: the previous kernel may still be finishing
  kvcu_pdl_trigger();  // the k_b product may start its set-up
  const uint32_t b = blockIdx.x, tid = threadIdx.x;
  const float* x = kv_a + (uint64_t)b * (R + P);
  float* row = rows + (uint64_t)b * (R + P);
  // sum of squares (math.zig:14-24)
  float ss = 0.f;
  for (uint32_t i = tid; i < R; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  if ((tid & 31u) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (uint32_t w = 0; w < blockDim.x / 32; ++w) tot = __fadd_rn(tot, red[w]);
  // ss / n + eps, inv = 1 / sqrt(.), out = x * inv * w (math.zig:25-34)
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)R), eps)));
  for (uint32_t i = tid; i < R; i += blockDim.x) row[i] = __fmul_rn(__fmul_rn(x[i], inv), norm_w[i]);
  // RoPE on pairs (2i, 2i+1), i < P/2 (math.zig:227-238): k_pe, then each head's q_rope
  const float pf = (float)pos[b];
  const uint32_t half = P / 2;
  for (uint32_t t = tid; t < (H + 1) * half; t += blockDim.x) {
    const uint32_t v = t / half, i = t % half;
    const float freq = __fdiv_rn(1.0f, powf(rope_base, __fdiv_rn((float)(2 * i), (float)P)));
    const float theta = __fmul_rn(pf, freq);
    const float cs = cosf(theta), sn = sinf(theta);
    const float* src = v < H ? q + ((uint64_t)b * H + v) * (qk_nope + P) + qk_nope : x + R;
    float* dst = v < H ? q_abs + ((uint64_t)b * H + v) * (R + P) + R : row + R;
    const float x0 = src[2 * i], x1 = src[2 * i + 1];
    dst[2 * i] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
    dst[2 * i + 1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
  }
}

// Per-head f32 GEMM C[m][n] = sum_k A[m][k] * B(k, n) for head z = blockIdx.z,
// B(k, n) = TRANS_B ? Bm[n * ldb + k] : Bm[k * ldb + n]. 128 x 64 output tile
// per CTA, 16-deep K slices through shared memory; each thread owns 8 rows x 4
// columns and reads its operands from shared memory as float4.
constexpr int GM = 128, GN = 64, GK = 16;
template <bool TRANS_B>
__global__ void __launch_bounds__(256)
    k_head_gemm(uint32_t M, uint32_t N, uint32_t K, const float* __restrict__ A, uint32_t lda,
                uint64_t a_hs, const float* __restrict__ B, uint32_t ldb, uint64_t b_hs,
                float* __restrict__ C, uint32_t ldc, uint64_t c_hs) {
  __shared__ __align__(16) float As[GK][GM + 4];
  __shared__ __align__(16) float Bs[GK][GN + 4];
  const uint32_t z = blockIdx.z, tid = threadIdx.x;
  A += z * a_hs;
  B += z * b_hs;
  C += z * c_hs;
  const uint32_t m0 = blockIdx.y * GM, n0 = blockIdx.x * GN;
  const uint32_t tx = tid % 16, ty = tid / 16;  // columns tx*4.., rows ty*8..
  constexpr int RA = (GM * GK) / 256, RB = (GN * GK) / 256;
  // The next K tile is loaded into registers while the current one is used,
  // so the global loads' latency overlaps the FMAs.
  float ra[RA], rb[RB];
  auto load_tile = [&](uint32_t k0) {
#pragma unroll
    for (int r = 0; r < RA; ++r) {
      const uint32_t e = tid + 256u * r, mm = e / GK, kk = e % GK;
      const uint32_t gm = m0 + mm, gk = k0 + kk;
      ra[r] = (gm < M && gk < K) ? A[(uint64_t)gm * lda + gk] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const uint32_t e = tid + 256u * r;
      uint32_t kk, nn;
      if (TRANS_B) {
        nn = e / GK;
        kk = e % GK;
      } else {
        kk = e / GN;
        nn = e % GN;
      }
      const uint32_t gk = k0 + kk, gn = n0 + nn;
      float v = 0.f;
      if (gk < K && gn < N) v = TRANS_B ? B[(uint64_t)gn * ldb + gk] : B[(uint64_t)gk * ldb + gn];
      rb[r] = v;
    }
  };
  // A tile [GM][GK] -> As[k][m], B tile [GK][GN] -> Bs[k][n]
  auto store_tile = [&]() {
#pragma unroll
    for (int r = 0; r < RA; ++r) {
      const uint32_t e = tid + 256u * r;
      As[e % GK][e / GK] = ra[r];
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const uint32_t e = tid + 256u * r;
      if (TRANS_B) Bs[e % GK][e / GK] = rb[r];
      else Bs[e / GN][e % GN] = rb[r];
    }
  };
  // accumulators in column pairs: one packed f32x2 FMA is two fmaf
  float2 acc[8][2];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
  load_tile(0);
  for (uint32_t k0 = 0; k0 < K; k0 += GK) {
    store_tile();
    __syncthreads();
    if (k0 + GK < K) load_tile(k0 + GK);
#pragma unroll
    for (int kk = 0; kk < GK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * 8 + 4]);
      const float4 b4 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float2 b01 = make_float2(b4.x, b4.y), b23 = make_float2(b4.z, b4.w);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 aa = make_float2(a[i], a[i]);
        acc[i][0] = __ffma2_rn(aa, b01, acc[i][0]);
        acc[i][1] = __ffma2_rn(aa, b23, acc[i][1]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t gm = m0 + ty * 8 + i;
    if (gm >= M) continue;
    const float v[4] = {acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t gn = n0 + tx * 4 + j;
      if (gn < N) C[(uint64_t)gm * ldc + gn] = v[j];
    }
  }
}

template <bool TRANS_B>
int launch_head_gemm_cc(uint32_t heads, uint32_t M, uint32_t N, uint32_t K, const float* A, uint32_t lda,
                        uint64_t a_hs, const float* B, uint32_t ldb, uint64_t b_hs, float* C, uint32_t ldc,
                        uint64_t c_hs, cudaStream_t st) {
  const dim3 grid((N + GN - 1) / GN, (M + GM - 1) / GM, heads);
  k_head_gemm<TRANS_B><<<grid, 256, 0, st>>>(M, N, K, A, lda, a_hs, B, ldb, b_hs, C, ldc, c_hs);
  return kvcu_check_cuda(cudaGetLastError(), "head gemm launch");
}

// The per-head GEMM of the step: the tensor-core 3xTF32 kernel when the shapes
// fit its tiles (the model's: N = 512 or 128, K = 128 or 512), else the
// CUDA-core f32 kernel.
template <bool TRANS_B>
int launch_head_gemm(uint32_t heads, uint32_t M, uint32_t N, uint32_t K, const float* A, uint32_t lda,
                     uint64_t a_hs, const float* B, uint32_t ldb, uint64_t b_hs, float* C, uint32_t ldc,
                     uint64_t c_hs, uint32_t* status, cudaStream_t st) {
  const int rc =
      kvcu_launch_head_gemm_tc(TRANS_B, heads, M, N, K, A, lda, a_hs, B, ldb, b_hs, C, ldc, c_hs, status, st);
  if (rc != KVCU_ERR_UNSUPPORTED) return rc;
  return launch_head_gemm_cc<TRANS_B>(heads, M, N, K, A, lda, a_hs, B, ldb, b_hs, C, ldc, c_hs, st);
}

// The MLA step's merge of the newest token into the history output, in two
// parts.  k_mla_merge_w, one CTA per entry: the newest token's k_pe as the
// cache holds it (once for all heads) and its unquantized latent go to shared
// memory, then one warp per head forms the token's score and the log-sum-exp
// weights (wh, wc, inv) of out = (history * wh + latent * wc) * inv.  The
// weights are applied by the v_b GEMM while it loads its A operand, or, where
// that kernel does not fit the shapes, by k_mla_merge_apply in place.
constexpr int MERGE_THREADS = 128;
__global__ void __launch_bounds__(MERGE_THREADS)
    k_mla_merge_w(uint32_t H, uint32_t R, uint32_t P, int kpe_q8, const float* __restrict__ q_abs,
                  const float* __restrict__ rows, const float* __restrict__ lse, float scale,
                  float* __restrict__ w) {
  extern __shared__ float msh[];  // [R] latent of the newest token, then [P] its k_pe
  kvcu_pdl_wait();     // launched programmatically after the decode's combine
  kvcu_pdl_trigger();  // the v_b product may start its set-up
  float* cs = msh;
  float* kpe = msh + R;
  const uint32_t b = blockIdx.x, tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const float* row = rows + (uint64_t)b * (R + P);
  for (uint32_t c = tid; c < R; c += blockDim.x) cs[c] = row[c];
  // k_pe of the newest token as stored: the Q8_0 round trip of the append
  // (d = amax/127, f16 scale, clamp(round(x/d)), dequant f16(d) * q)
  if (warp == 0) {
    for (uint32_t blk = 0; blk * 32 < P; ++blk) {
      const uint32_t e = blk * 32 + lane;
      const float v = e < P ? row[R + e] : 0.f;
      float out = v;
      if (kpe_q8) {
        float amax = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = kvcu::q8_scale(amax);
        const int8_t qv = d > 0.f ? kvcu::q8_value(v, d) : (int8_t)0;
        out = __fmul_rn(kvcu::f16_to_f32(kvcu::f32_to_f16(d)), (float)qv);
      }
      if (e < P) kpe[e] = out;
    }
  }
  __syncthreads();
  for (uint32_t h = warp; h < H; h += blockDim.x / 32) {
    const float* qa = q_abs + ((uint64_t)b * H + h) * (R + P);
    float dot = 0.f;
#pragma unroll 4
    for (uint32_t c = lane; c < R; c += 32) dot = fmaf(qa[c], cs[c], dot);
    for (uint32_t r = lane; r < P; r += 32) dot = fmaf(qa[R + r], kpe[r], dot);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0) {
      const float s = dot * scale;
      const float lh = lse[(uint64_t)b * H + h];
      const float m = fmaxf(lh, s);
      const float wh = lh == -INFINITY ? 0.f : expf(lh - m);
      const float wc = expf(s - m);
      float* wr = w + ((uint64_t)b * H + h) * 3;
      wr[0] = wh;
      wr[1] = wc;
      wr[2] = 1.0f / (wh + wc);
    }
  }
}

// The merge in place, for the CUDA-core GEMM: one CTA per (entry, head).
__global__ void __launch_bounds__(MERGE_THREADS)
    k_mla_merge_apply(uint32_t H, uint32_t R, uint32_t P, const float* __restrict__ rows, const float* __restrict__ w,
                      float* __restrict__ latent) {
  kvcu_pdl_wait();  // launched programmatically after the weights kernel
  kvcu_pdl_trigger();
  const uint32_t b = blockIdx.x / H, h = blockIdx.x % H;
  const float* row = rows + (uint64_t)b * (R + P);
  const float* wr = w + ((uint64_t)b * H + h) * 3;
  const float wh = wr[0], wc = wr[1], inv = wr[2];
  float* lat = latent + ((uint64_t)b * H + h) * R;
  for (uint32_t c = threadIdx.x; c < R; c += blockDim.x) {
    const float hv = wh > 0.f ? lat[c] * wh : 0.f;
    lat[c] = (hv + row[c] * wc) * inv;
  }
}

// The whole merge in place, one CTA per (entry, head), for kvcu_mla_finish,
// whose caller passes no room for the weights: the newest token's score with
// the unquantized latent and k_pe as the cache holds it, then its log-sum-exp
// merge into the history's normalised output.
__global__ void __launch_bounds__(MERGE_THREADS)
    k_mla_merge(uint32_t H, uint32_t R, uint32_t P, int kpe_q8, const float* __restrict__ q_abs,
                const float* __restrict__ rows, float* __restrict__ latent, const float* __restrict__ lse,
                float scale) {
  __shared__ float kpe[256];
  __shared__ float red[MERGE_THREADS / 32];
  const uint32_t b = blockIdx.x / H, h = blockIdx.x % H, tid = threadIdx.x;
  const float* row = rows + (uint64_t)b * (R + P);
  const float* qa = q_abs + ((uint64_t)b * H + h) * (R + P);
  // k_pe of the newest token as stored: the Q8_0 round trip of the append
  // (d = amax/127, f16 scale, clamp(round(x/d)), dequant f16(d) * q)
  if (tid < 32) {
    for (uint32_t blk = 0; blk * 32 < P; ++blk) {
      const uint32_t e = blk * 32 + tid;
      const float v = e < P ? row[R + e] : 0.f;
      float out = v;
      if (kpe_q8) {
        float amax = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = kvcu::q8_scale(amax);
        const int8_t qv = d > 0.f ? kvcu::q8_value(v, d) : (int8_t)0;
        out = __fmul_rn(kvcu::f16_to_f32(kvcu::f32_to_f16(d)), (float)qv);
      }
      if (e < P) kpe[e] = out;
    }
  }
  __syncthreads();
  float dot = 0.f;
  for (uint32_t c = tid; c < R; c += blockDim.x) dot = fmaf(qa[c], row[c], dot);
  for (uint32_t r = tid; r < P; r += blockDim.x) dot = fmaf(qa[R + r], kpe[r], dot);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if ((tid & 31u) == 0) red[tid >> 5] = dot;
  __syncthreads();
  float s = 0.f;
  for (uint32_t w = 0; w < blockDim.x / 32; ++w) s += red[w];
  s *= scale;
  const float lh = lse[(uint64_t)b * H + h];
  const float m = fmaxf(lh, s);
  const float wh = lh == -INFINITY ? 0.f : expf(lh - m);
  const float wc = expf(s - m);
  const float inv = 1.0f / (wh + wc);
  float* lat = latent + ((uint64_t)b * H + h) * R;
  for (uint32_t c = tid; c < R; c += blockDim.x) {
    const float hv = wh > 0.f ? lat[c] * wh : 0.f;
    lat[c] = (hv + row[c] * wc) * inv;
  }
}

bool valid_dims(const kvcu_pool* p, uint32_t n_heads, uint32_t d) {
  return p && n_heads >= 1 && n_heads <= 128 && d >= 1 && d <= 1024 && p->rope_dim % 2 == 0 &&
         p->rope_dim <= 256 && p->kv_rank >= 1;
}

struct DevScope {
  int prev = -1, rc = 0;
  explicit DevScope(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) rc = kvcu_check_cuda(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~DevScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int kvcu_mla_prepare(kvcu_pool* pool, uint32_t n, uint32_t n_heads, uint32_t qk_nope,
                                const float* q, const float* kv_a, const uint32_t* positions,
                                const float* norm_w, float eps, float rope_base, const float* k_b,
                                float* q_abs, float* rows, void* stream) {
  if (!valid_dims(pool, n_heads, qk_nope)) {
    kvcu_set_error("kvcu_mla_prepare: unsupported n_heads %u / qk_nope %u / pool dims", n_heads, qk_nope);
    return KVCU_ERR_INVALID_ARG;
  }
  if (!n) return KVCU_OK;
  if (!q || !kv_a || !positions || !norm_w || !k_b || !q_abs || !rows) return KVCU_ERR_INVALID_ARG;
  DevScope d(pool->device);
  if (d.rc) return d.rc;
  const uint32_t R = pool->kv_rank, P = pool->rope_dim;
  const cudaStream_t st = (cudaStream_t)stream;
  int rc = kvcu_check_cuda(kvcu_launch_pdl(k_mla_rows, dim3(n), dim3(ROWS_THREADS), 0, st, n_heads, qk_nope, R, P,
                                           q, kv_a, positions, norm_w, eps, rope_base, q_abs, rows),
                           "mla rows launch");
  if (rc) return rc;
  // q_abs[b][h][0:R] = q_nope[b][h] (n x qk_nope) x k_b_h (qk_nope x R)
  return launch_head_gemm<false>(n_heads, n, R, qk_nope, q, n_heads * (qk_nope + P), qk_nope + P, k_b, R,
                                 (uint64_t)qk_nope * R, q_abs, n_heads * (R + P), R + P, pool->status, st);
}

extern "C" int kvcu_mla_finish(kvcu_pool* pool, uint32_t n, uint32_t n_heads, uint32_t v_dim,
                               const float* q_abs, const float* rows, float* latent, const float* lse,
                               float scale, const float* v_b, float* attn, void* stream) {
  if (!valid_dims(pool, n_heads, v_dim)) {
    kvcu_set_error("kvcu_mla_finish: unsupported n_heads %u / v_dim %u / pool dims", n_heads, v_dim);
    return KVCU_ERR_INVALID_ARG;
  }
  if (!n) return KVCU_OK;
  if (!q_abs || !rows || !latent || !lse || !v_b || !attn) return KVCU_ERR_INVALID_ARG;
  DevScope d(pool->device);
  if (d.rc) return d.rc;
  const uint32_t R = pool->kv_rank, P = pool->rope_dim;
  const cudaStream_t st = (cudaStream_t)stream;
  k_mla_merge<<<n * n_heads, MERGE_THREADS, 0, st>>>(n_heads, R, P, pool->quantized ? 1 : 0, q_abs, rows,
                                                     latent, lse, scale);
  int rc = kvcu_check_cuda(cudaGetLastError(), "mla merge launch");
  if (rc) return rc;
  // attn[b][h][j] = latent[b][h] (n x R) x v_b_h^T, v_b_h = v_b[h*v_dim .. +v_dim][0:R]
  return launch_head_gemm<true>(n_heads, n, v_dim, R, latent, n_heads * R, R, v_b, R, (uint64_t)v_dim * R,
                                attn, n_heads * v_dim, v_dim, pool->status, st);
}

// kvcu_mla_finish with scratch for the merge weights w [n][H][3]: the weights
// kernel, then the v_b GEMM that merges its A operand as it loads it (no pass
// over the latent in between); the in-place merge and the CUDA-core GEMM where
// the tensor-core kernel does not fit the shapes.
int kvcu_mla_finish_fused(kvcu_pool* pool, uint32_t n, uint32_t n_heads, uint32_t v_dim, const float* q_abs,
                          const float* rows, float* latent, const float* lse, float* w, float scale,
                          const float* v_b, float* attn, cudaStream_t st) {
  if (!valid_dims(pool, n_heads, v_dim)) {
    kvcu_set_error("kvcu_mla_finish: unsupported n_heads %u / v_dim %u / pool dims", n_heads, v_dim);
    return KVCU_ERR_INVALID_ARG;
  }
  if (!n) return KVCU_OK;
  if (!q_abs || !rows || !latent || !lse || !w || !v_b || !attn) return KVCU_ERR_INVALID_ARG;
  DevScope d(pool->device);
  if (d.rc) return d.rc;
  const uint32_t R = pool->kv_rank, P = pool->rope_dim;
  if ((uint64_t)(R + P) * sizeof(float) > 48u * 1024u)  // the weights kernel's shared latent and k_pe
    return kvcu_mla_finish(pool, n, n_heads, v_dim, q_abs, rows, latent, lse, scale, v_b, attn, st);
  int rc = kvcu_check_cuda(kvcu_launch_pdl(k_mla_merge_w, dim3(n), dim3(MERGE_THREADS), (R + P) * sizeof(float), st,
                                           n_heads, R, P, pool->quantized ? 1 : 0, q_abs, rows, lse, scale, w),
                           "mla merge launch");
  if (rc) return rc;
  const kvcu_gemm_merge mrg{rows, R + P, w};
  rc = kvcu_launch_head_gemm_tc(true, n_heads, n, v_dim, R, latent, n_heads * R, R, v_b, R, (uint64_t)v_dim * R,
                                attn, n_heads * v_dim, v_dim, pool->status, st, &mrg);
  if (rc != KVCU_ERR_UNSUPPORTED) return rc;
  rc = kvcu_check_cuda(kvcu_launch_pdl(k_mla_merge_apply, dim3(n * n_heads), dim3(MERGE_THREADS), 0, st, n_heads, R,
                                       P, rows, w, latent),
                       "mla merge launch");
  if (rc) return rc;
  return launch_head_gemm_cc<true>(n_heads, n, v_dim, R, latent, n_heads * R, R, v_b, R, (uint64_t)v_dim * R, attn,
                                   n_heads * v_dim, v_dim, st);
}

// Per-head batched GEMM entry point (the step's two contractions, exposed so a
// caller, or a test, can run either kernel): impl 0 = the tensor-core 3xTF32
// kernel where the shapes fit it, else CUDA cores; 1 = CUDA cores; 2 = tensor
// cores or KVCU_ERR_UNSUPPORTED.
extern "C" int kvcu_head_gemm(int trans_b, uint32_t heads, uint32_t M, uint32_t N, uint32_t K, const float* A,
                              uint32_t lda, uint64_t a_hs, const float* B, uint32_t ldb, uint64_t b_hs, float* C,
                              uint32_t ldc, uint64_t c_hs, int impl, kvcu_pool* pool, void* stream) {
  if (!pool || !(pool->kv || pool->qs) || impl < 0 || impl > 2) return KVCU_ERR_INVALID_ARG;
  if (M && heads && (!A || !B || !C)) return KVCU_ERR_INVALID_ARG;
  DevScope d(pool->device);
  if (d.rc) return d.rc;
  const cudaStream_t st = (cudaStream_t)stream;
  if (impl != 1) {
    const int rc = kvcu_launch_head_gemm_tc(trans_b != 0, heads, M, N, K, A, lda, a_hs, B, ldb, b_hs, C, ldc, c_hs,
                                            pool->status, st);
    if (rc != KVCU_ERR_UNSUPPORTED || impl == 2) {
      if (rc == KVCU_ERR_UNSUPPORTED)
        kvcu_set_error("kvcu_head_gemm: the tensor-core kernel needs N %% 128 == 0, K %% 32 == 0 and 16-byte rows");
      return rc;
    }
  }
  return trans_b ? launch_head_gemm_cc<true>(heads, M, N, K, A, lda, a_hs, B, ldb, b_hs, C, ldc, c_hs, st)
                 : launch_head_gemm_cc<false>(heads, M, N, K, A, lda, a_hs, B, ldb, b_hs, C, ldc, c_hs, st);
}
