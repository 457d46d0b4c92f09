// kvcu_numeric.cuh — bit-exact scalar numerics shared by the kernels.
//
// Every routine here must produce the same bits as mobile-moe.zig's CPU code:
//   f16_to_f32 / f32_to_f16  : src/dequant.zig:19-95 (bit routines, not the
//                              hardware conversion, so NaN payloads, f32
//                              subnormal flushing and overflow match)
//   q8 quantization           : src/kv_cache.zig:294-349
// The f16-subnormal branch of f32ToF16 is computed with correct IEEE
// round-to-nearest-even (the reference's shift at src/dequant.zig:76-77
// overflows u16), and a NaN quotient x/d quantizes to 0 (undefined in the
// reference).  All float operations use explicit _rn intrinsics so that no
// FMA contraction or fast-math rewrite can change a bit.
#pragma once

#include <stdint.h>

namespace kvcu {

__host__ __device__ __forceinline__ float bits_f32(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}
__host__ __device__ __forceinline__ uint32_t f32_bits(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  __builtin_memcpy(&u, &f, 4);
  return u;
#endif
}

// f16 bits -> f32, exact (src/dequant.zig:19-47).
__host__ __device__ __forceinline__ float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  if (e == 0) {
    if (m == 0) return bits_f32(sign);
    // subnormal: value = m * 2^-24, exact in f32 via an integer-to-float
    // conversion (m < 2^10) and a power-of-two scale.
    float v = (float)m * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  if (e == 31) return bits_f32(sign | 0x7F800000u | (m << 13));
  return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

// f32 -> f16 bits, round to nearest even; f32 subnormals -> signed zero,
// overflow -> inf, NaN keeps its top mantissa bits (forced non-zero).
__host__ __device__ __forceinline__ uint16_t f32_to_f16(float v) {
  uint32_t bits = f32_bits(v);
  uint32_t sign = (bits >> 31) & 1u;
  uint32_t exp_raw = (bits >> 23) & 0xFFu;
  uint32_t mant = bits & 0x7FFFFFu;
  uint32_t e, m;
  if (exp_raw == 0) {
    e = 0;
    m = 0;
  } else if (exp_raw == 0xFFu) {
    e = 0x1F;
    m = mant >> 13;
    if (mant != 0 && m == 0) m = 1;
  } else {
    int exp16 = (int)exp_raw - 112;
    if (exp16 >= 31) {
      e = 0x1F;
      m = 0;
    } else if (exp16 <= 0) {
      e = 0;
      if (exp16 < -10) {
        m = 0;
      } else {
        uint32_t full = mant | 0x800000u;
        uint32_t shift = (uint32_t)(14 - exp16);
        uint32_t q = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q += 1u;
        m = q;  // a carry to 0x400 is the smallest normal, as IEEE requires
      }
    } else {
      e = (uint32_t)exp16;
      m = mant >> 13;
      uint32_t rb = mant & 0x1FFFu;
      if (rb > 0x1000u || (rb == 0x1000u && (m & 1u))) {
        m += 1u;
        if (m == 0x400u) {
          m = 0;
          e += 1;
        }
      }
    }
  }
  return (uint16_t)((sign << 15) | (e << 10) | m);
}

#ifdef __CUDACC__
// Quantized value of x for scale d > 0: clamp(round_half_away(x / d), +-127),
// NaN -> 0.  __fdiv_rn is the IEEE quotient the reference's f32 `/` produces.
__device__ __forceinline__ int8_t q8_value(float x, float d) {
  float r = roundf(__fdiv_rn(x, d));
  if (r != r) return 0;
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return (int8_t)(int)r;
}

// q8_value through a multiply: for any inv within 2^-22 (relative) of 1/d,
// t = x * inv lies within |x/d| * 2^-21 <= 6.1e-5 of RN(x/d) for |x/d| <= 128,
// so both round to the same integer unless t is within 1e-4 of a
// half-integer; there (and for NaN / inf, e.g. from a reciprocal that
// overflowed) the IEEE quotient decides.  Away from half-integers, round-half-even
// (rintf) and the reference's round-half-away agree.  For |x| <= amax of its
// block (d = RN(amax/127)), |t| <= 127 * (1 + 3 * 2^-24), so the result needs
// no clamp.  Same results as q8_value for such x.
__device__ __forceinline__ int8_t q8_value_fast(float x, float d, float inv) {
  const float t = x * inv;
  const float r = rintf(t);
  if (!(fabsf(t - r) < 0.4999f)) return q8_value(x, d);
  return (int8_t)(int)r;
}

// Hardware approximate reciprocal (PTX rcp.approx.f32: at most 1 ulp of error,
// subnormal inputs kept), accurate enough for q8_value_fast's `inv`.
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Block scale from the block's max |x| (NaN-free max): d = amax/127 or 0.
__device__ __forceinline__ float q8_scale(float amax) {
  return amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 0.0f;
}

// ---- seeded synthetic inputs (same bits as oracle/kvoracle.c) ----
// SplitMix64 (Steele, Lea & Flood, OOPSLA 2014).
__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// ln(s), s in (0,1): s = 2^e m, ln m = 2 atanh((m-1)/(m+1)) by its Taylor
// series to t^13, evaluated with explicitly rounded operations.
__device__ __forceinline__ float log_det(float s) {
  uint32_t bits = __float_as_uint(s);
  int e = (int)((bits >> 23) & 0xFF) - 127;
  float m = __uint_as_float((bits & 0x7FFFFFu) | 0x3F800000u);
  if (m > 1.41421356f) {
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  float t = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  float t2 = __fmul_rn(t, t);
  float p = 0.0769230769f;
  p = __fadd_rn(__fmul_rn(p, t2), 0.0909090909f);
  p = __fadd_rn(__fmul_rn(p, t2), 0.111111111f);
  p = __fadd_rn(__fmul_rn(p, t2), 0.142857143f);
  p = __fadd_rn(__fmul_rn(p, t2), 0.2f);
  p = __fadd_rn(__fmul_rn(p, t2), 0.333333333f);
  p = __fadd_rn(__fmul_rn(p, t2), 1.0f);
  float lnm = __fmul_rn(__fadd_rn(t, t), p);
  float el = __fmul_rn((float)e, 0.693147181f);
  return __fadd_rn(el, lnm);
}

__device__ __forceinline__ float gen_normal(uint64_t seed, uint64_t a, uint64_t b, uint64_t c,
                                            float outlier_p) {
  uint64_t key = splitmix64(seed ^ splitmix64(a));
  key = splitmix64(key ^ b);
  key = splitmix64(key ^ c);
  float z = 0.0f;
  for (uint32_t j = 0; j < 64; ++j) {
    uint64_t r = splitmix64(key + j);
    uint32_t ux = (uint32_t)(r >> 41);
    uint32_t uy = (uint32_t)(r >> 18) & 0x7FFFFFu;
    float x = __fsub_rn(__fmul_rn((float)(2u * ux + 1u), 1.1920928955078125e-07f), 1.0f);
    float y = __fsub_rn(__fmul_rn((float)(2u * uy + 1u), 1.1920928955078125e-07f), 1.0f);
    float s = __fadd_rn(__fmul_rn(x, x), __fmul_rn(y, y));
    if (s >= 1.0f) continue;
    float ls = log_det(s);
    float ratio = __fdiv_rn(__fmul_rn(-2.0f, ls), s);
    z = __fmul_rn(x, __fsqrt_rn(ratio));
    break;
  }
  if (outlier_p > 0.0f) {
    uint64_t r = splitmix64(key ^ 0xD1B54A32D192ED03ull);
    float u = __fmul_rn((float)(uint32_t)(r >> 40), 5.9604644775390625e-08f);
    if (u < outlier_p) z = __fmul_rn(z, 20.0f);
  }
  return z;
}
#endif  // __CUDACC__

}  // namespace kvcu
