// kvcu_gemm_tc.cu — the per-head GEMMs of the MLA step (k_b absorption and
// v_b, src/inference.zig:524-550 and :663-665 in absorbed form) on the sm_100a
// tcgen05 tensor cores, at f32-level accuracy.
//
// Per head z: C[m][n] = sum_k A[m][k] * B(k, n).  TF32 keeps 10 mantissa
// bits, so every f32 operand x is split into x_hi = x with its low 13 mantissa
// bits cleared (exactly a TF32 value) and x_lo = x - x_hi (exact in f32), and
// C = A_hi B_hi + A_hi B_lo + A_lo B_hi ("3xTF32"): the dropped A_lo B_lo and
// the TF32 rounding of the lo parts are below 2^-20 of each product, against
// 2^-24 for an f32 product, and the sums accumulate in f32 in TMEM.
//
// One CTA per (128-row M tile, NT-column N tile, head), 256 threads: all
// threads stage each 32-deep K slice of A and B into shared memory (split into
// hi / lo, 128B-swizzled K-major layout, two stages; the next slice's global
// loads are in flight meanwhile), one elected thread issues
// 4 K-steps x 3 tcgen05.mma.kind::tf32 (M = 128, N = NT, K = 8) per slice, and
// the accumulator (128 lanes x NT f32 columns of TMEM) is read back by the 8
// warps at the end.  Every wait is bounded; a timeout sets the pool's status
// word, waits (bounded) for the MMAs already issued and frees TMEM.
#include <cuda_runtime.h>

#include "kvcu_internal.h"
#include "kvcu_tcgen05.cuh"

namespace {
using namespace kvtc;

constexpr int TM = 128;   // rows per CTA (the MMA's M)
constexpr int TK = 32;    // K per stage: one 128-byte swizzle row of f32
constexpr int NTHR = 256;
constexpr int STAGES = 2;
constexpr long long WAIT_LIMIT = 1ll << 31;  // ~1 s of clocks

template <int NT>
struct Layout {
  static constexpr uint32_t A_BYTES = TM * TK * 4;  // 16 KB (hi or lo)
  static constexpr uint32_t B_BYTES = NT * TK * 4;  // 16 / 32 KB (hi or lo)
  static constexpr uint32_t STAGE = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr uint32_t OFF_BAR = STAGES * STAGE;      // mbarriers: free[STAGES], done
  static constexpr uint32_t OFF_TMEM = OFF_BAR + 64;       // TMEM base address
  static constexpr uint32_t ALLOC = OFF_TMEM + 16 + 1024;  // + slack for 1024 alignment
  static_assert(ALLOC <= 232448, "shared memory budget");
};

struct GemmArgs {
  uint32_t M, N, K;
  const float* A;
  uint32_t lda;
  uint64_t a_hs;
  const float* B;
  uint32_t ldb;
  uint64_t b_hs;
  float* C;
  uint32_t ldc;
  uint64_t c_hs;
  uint32_t* status;
  kvcu_gemm_merge mrg;  // mrg.w == nullptr: plain A
  uint32_t heads;
};

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Bounded wait; false (and the status bit) after WAIT_LIMIT clocks.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, uint32_t* status) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (clock64() - t0 > WAIT_LIMIT) {
      atomicOr(status, KVCU_STATUS_TIMEOUT);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// Store the hi / lo parts of 4 consecutive K values (16 bytes) of row r.
__device__ __forceinline__ void put4(uint8_t* hi, uint8_t* lo, uint32_t r, uint32_t chunk, float4 v) {
  const uint32_t off = sw128_off(r, chunk * 16u);
  const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
  *reinterpret_cast<float4*>(hi + off) = h;
  *reinterpret_cast<float4*>(lo + off) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
}

template <int NT, bool TRANS_B>
__global__ void __launch_bounds__(NTHR, 1) k_head_gemm_tc(GemmArgs g) {
  using L = Layout<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  const uint32_t z = blockIdx.z, m0 = blockIdx.y * TM, n0 = blockIdx.x * NT;
  const float* A = g.A + z * g.a_hs;
  const float* B = g.B + z * g.b_hs;
  const bool merge = g.mrg.w != nullptr;  // uniform
  float* C = g.C + z * g.c_hs;
  auto bar = [&](int i) { return sbase + L::OFF_BAR + 8u * (uint32_t)i; };
  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) mbar_init(bar(i), 1);
    mbar_init(bar(STAGES), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + L::OFF_TMEM),
                 "r"((uint32_t)NT)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L::OFF_TMEM);
  // programmatic launch: the set-up above overlaps the previous kernel's tail;
  // A, B and the merge operands are read only after this wait
  kvcu_pdl_wait();
  kvcu_pdl_trigger();  // the next kernel may start its own set-up
  // kind::tf32: D f32 (bit 4), A and B TF32 (format 2 at bits 7 and 10), both
  // K-major, N >> 3 at bit 17, M >> 4 at bit 24
  constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(NT >> 3) << 17) |
                             ((uint32_t)(TM >> 4) << 24);
  const uint32_t nk = g.K / TK;
  // The next K slice is read from global memory into registers while the
  // current one is stored, synchronised and multiplied.
  constexpr int NA = TM * 8 / NTHR, NB = NT * 8 / NTHR;
  float4 pa[NA], pb[NB];
  // merge: the rows' weights once, and the newest token's latent beside A
  float4 px[NA];
  float mw[NA][3];
  if (merge) {
#pragma unroll
    for (int i = 0; i < NA; ++i) {
      const uint32_t r = (tid + NTHR * i) >> 3;
      mw[i][0] = mw[i][1] = mw[i][2] = 0.f;
      if (m0 + r < g.M) {
        const float* wr = g.mrg.w + ((uint64_t)(m0 + r) * g.heads + z) * 3;
        mw[i][0] = __ldg(wr);
        mw[i][1] = __ldg(wr + 1);
        mw[i][2] = __ldg(wr + 2);
      }
    }
  }
  auto load_slice = [&](uint32_t c) {
    const uint32_t k0 = c * TK;
#pragma unroll
    for (int i = 0; i < NA; ++i) {
      const uint32_t e = tid + NTHR * i, r = e >> 3, ch = e & 7u;
      pa[i] = px[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m0 + r >= g.M) continue;
      pa[i] = __ldg(reinterpret_cast<const float4*>(A + (uint64_t)(m0 + r) * g.lda + k0 + 4 * ch));
      if (merge)
        px[i] = __ldg(reinterpret_cast<const float4*>(g.mrg.rows + (uint64_t)(m0 + r) * g.mrg.ldr + k0 + 4 * ch));
    }
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const uint32_t e = tid + NTHR * i;
      if (TRANS_B)  // B(k, n) = B[n * ldb + k]: rows n, K contiguous, like A
        pb[i] = __ldg(reinterpret_cast<const float4*>(B + (uint64_t)(n0 + (e >> 3)) * g.ldb + k0 + 4 * (e & 7u)));
      else  // B(k, n) = B[k * ldb + n]: 4 consecutive n of one k
        pb[i] = __ldg(reinterpret_cast<const float4*>(B + (uint64_t)(k0 + e / (NT / 4)) * g.ldb + n0 +
                                                      4 * (e % (NT / 4))));
    }
  };
  load_slice(0);
  bool ok = true;
  for (uint32_t c = 0; c < nk && ok; ++c) {
    const uint32_t s = c % STAGES;
    if (c >= STAGES) ok = wait_bounded(bar(s), ((c / STAGES) - 1) & 1u, g.status);  // MMAs of c - STAGES done
    if (!__syncthreads_and(ok)) {
      ok = false;
      break;
    }
    uint8_t* st = smem + s * L::STAGE;
    uint8_t *a_hi = st, *a_lo = st + L::A_BYTES, *b_hi = st + 2 * L::A_BYTES, *b_lo = b_hi + L::B_BYTES;
#pragma unroll
    for (int i = 0; i < NA; ++i) {
      const uint32_t e = tid + NTHR * i;
      float4 v = pa[i];
      if (merge) {
        // the MLA step's merge, in the order of the in-place merge kernel (the
        // history term is dropped, not multiplied, where its weight is 0)
        const float wh = mw[i][0], wc = mw[i][1], inv = mw[i][2];
        const float4 h = wh > 0.f ? make_float4(v.x * wh, v.y * wh, v.z * wh, v.w * wh) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 x = px[i];
        v = make_float4((h.x + x.x * wc) * inv, (h.y + x.y * wc) * inv, (h.z + x.z * wc) * inv, (h.w + x.w * wc) * inv);
      }
      put4(a_hi, a_lo, e >> 3, e & 7u, v);
    }
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const uint32_t e = tid + NTHR * i;
      if (TRANS_B) {
        put4(b_hi, b_lo, e >> 3, e & 7u, pb[i]);
      } else {
        // 4 consecutive n of one k go to 4 rows
        const uint32_t kk = e / (NT / 4), n4 = e % (NT / 4);
        const float x[4] = {pb[i].x, pb[i].y, pb[i].z, pb[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t off = sw128_off(4 * n4 + j, 4 * kk);
          const float h = tf32_hi(x[j]);
          *reinterpret_cast<float*>(b_hi + off) = h;
          *reinterpret_cast<float*>(b_lo + off) = x[j] - h;
        }
      }
    }
    if (c + 1 < nk) load_slice(c + 1);
    fence_proxy_async();  // the generic-proxy stores, seen by the tensor cores
    __syncthreads();
    if (warp == 0) {
      tc_fence_after();
      if (elect_one()) {
        const uint32_t sa = sbase + s * L::STAGE;
        const uint32_t ah = sa, al = sa + L::A_BYTES, bh = sa + 2 * L::A_BYTES, bl = bh + L::B_BYTES;
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk) {  // 8 f32 = 32 bytes per K-step
          const uint64_t dah = smem_desc(ah + 32u * kk, 16, 1024, LAYOUT_SW128);
          const uint64_t dal = smem_desc(al + 32u * kk, 16, 1024, LAYOUT_SW128);
          const uint64_t dbh = smem_desc(bh + 32u * kk, 16, 1024, LAYOUT_SW128);
          const uint64_t dbl = smem_desc(bl + 32u * kk, 16, 1024, LAYOUT_SW128);
          mma_tf32(tmem, dah, dbh, IDESC, (c | kk) != 0u);
          mma_tf32(tmem, dah, dbl, IDESC, 1u);
          mma_tf32(tmem, dal, dbh, IDESC, 1u);
        }
        mma_commit(bar(s));
      }
      __syncwarp();
    }
  }
  // all issued MMAs retire (also after a timeout) before TMEM is read or freed
  if (warp == 0) {
    if (elect_one()) mma_commit(bar(STAGES));
    __syncwarp();
  }
  const bool done = wait_bounded(bar(STAGES), 0, g.status);
  tc_fence_after();
  if (__syncthreads_and(ok && done)) {
    // lanes = rows: warp w reads lane quarter w % 4, column half w / 4
    const uint32_t row = m0 + 32u * (warp & 3u) + lane;
    const uint32_t col0 = (warp >> 2) * (NT / 2);
    const uint32_t ta = tmem + ((32u * (warp & 3u)) << 16) + col0;
#pragma unroll 1
    for (uint32_t cc = 0; cc < (uint32_t)(NT / 2); cc += 16) {
      uint32_t r[16];
      tmem_ld<16>(ta + cc, r);
      tmem_wait_ld();
      reg_fence(r);
      if (row < g.M) {
        float4* dst = reinterpret_cast<float4*>(C + (uint64_t)row * g.ldc + n0 + col0 + cc);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)NT) : "memory");
  }
}

template <int NT, bool TRANS_B>
int setup_gemm(const void*) {
  return kvcu_check_cuda(cudaFuncSetAttribute(k_head_gemm_tc<NT, TRANS_B>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Layout<NT>::ALLOC),
                         "cudaFuncSetAttribute(head_gemm_tc)");
}

template <int NT, bool TRANS_B>
int launch(const GemmArgs& g, uint32_t heads, cudaStream_t st) {
  int rc = kvcu_configure_once(reinterpret_cast<const void*>(&k_head_gemm_tc<NT, TRANS_B>), setup_gemm<NT, TRANS_B>,
                               nullptr);
  if (rc) return rc;
  const dim3 grid(g.N / NT, (g.M + TM - 1) / TM, heads);
  return kvcu_check_cuda(kvcu_launch_pdl(k_head_gemm_tc<NT, TRANS_B>, grid, dim3(NTHR), Layout<NT>::ALLOC, st, g),
                         "head_gemm_tc launch");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Tensor-core per-head GEMM; KVCU_ERR_UNSUPPORTED when the shapes or strides do
// not fit its tiles (N a multiple of 128, K of 32, 16-byte aligned rows), so
// the caller can use the CUDA-core kernel instead.
int kvcu_launch_head_gemm_tc(bool trans_b, uint32_t heads, uint32_t M, uint32_t N, uint32_t K, const float* A,
                             uint32_t lda, uint64_t a_hs, const float* B, uint32_t ldb, uint64_t b_hs, float* C,
                             uint32_t ldc, uint64_t c_hs, uint32_t* status, cudaStream_t st,
                             const kvcu_gemm_merge* mrg) {
  if (M == 0 || heads == 0) return KVCU_OK;
  if (N % 128 != 0 || K % TK != 0 || K == 0 || lda % 4 || ldb % 4 || ldc % 4 || a_hs % 4 || b_hs % 4 || c_hs % 4 ||
      !aligned16(A) || !aligned16(B) || !aligned16(C) || !status ||
      (mrg && (!mrg->w || mrg->ldr % 4 || !aligned16(mrg->rows))))
    return KVCU_ERR_UNSUPPORTED;
  GemmArgs g{M, N, K, A, lda, a_hs, B, ldb, b_hs, C, ldc, c_hs, status,
             mrg ? *mrg : kvcu_gemm_merge{nullptr, 0, nullptr}, heads};
  // one CTA per SM (shared memory): pick the N tile whose waves of CTAs cover
  // the fewest columns per SM
  const uint64_t sms = (uint64_t)kvcu_current_sm_count(), mt = (M + TM - 1) / TM;
  const uint64_t waves256 = (N / 256 * mt * heads + sms - 1) / sms, waves128 = (N / 128 * mt * heads + sms - 1) / sms;
  if (N % 256 == 0 && waves256 * 256 <= waves128 * 128)
    return trans_b ? launch<256, true>(g, heads, st) : launch<256, false>(g, heads, st);
  return trans_b ? launch<128, true>(g, heads, st) : launch<128, false>(g, heads, st);
}
