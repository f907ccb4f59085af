// spb_exact.cuh -- exact integer / IEEE-op helpers shared by the sm_100a kernels.
//
// Every helper here reproduces one rule of the byte-exact numeric contract bit for
// bit: round-half-away llround of a double, the OK_Q4B f16 block scale as an integer
// (value = k * 2^-24), the activation quantizer (sp_frob_quant1, frobenius_lift.c:27-35),
// 128-bit products/shifts with the truncation semantics of the reference islands'
// (int64_t)((__int128)a*b >> 30) casts (exact_islands.c:38-45,112-124), the island exp
// / tanh primitives, and the 128/64 divisions the RMSNorm island and the attention
// V-sum need. Float ops use the _rn intrinsics so nvcc never contracts them into FMAs.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "spb_kernels.cuh"

namespace spb {

constexpr int FB = 30;
constexpr int64_t ONE = int64_t(1) << FB;
constexpr int64_t K_LOG2E = 1549082005LL;   // round(log2(e) * 2^30)
constexpr int64_t K_GELU_K = 856722024LL;   // round(sqrt(2/pi) * 2^30)
constexpr int64_t K_GELU_A = 48012366LL;    // round(0.044715 * 2^30)

__device__ __forceinline__ void raise_err(uint32_t *err, uint32_t bit) {
  if (err) atomicOr(err, bit);
}

// llround(v): nearest integer, halfway cases away from zero (C99 llround).
__device__ __forceinline__ int64_t llround_d(double v) {
  double t = trunc(v);
  double f = __dsub_rn(v, t);           // exact: the fractional bits of v
  int64_t r = __double2ll_rz(t);
  if (f >= 0.5) r += 1;
  else if (f <= -0.5) r -= 1;
  return r;
}

// f16 block scale -> (m, sh, neg) with |value| = m * 2^sh * 2^-24 (m < 2^11, sh < 30).
__device__ __forceinline__ void f16_scale_parts(uint32_t h, int32_t &m, int32_t &sh) {
  uint32_t e = (h >> 10) & 31u, mant = h & 1023u;
  m = (int32_t)(e ? (mant | 1024u) : mant);
  sh = e ? (int32_t)e - 1 : 0;
  if (h & 0x8000u) m = -m;
}

// sp_frob_quant1: x = v / s * 127 (two IEEE ops), round half away via floorf/ceilf of
// x +- 0.5f, clamp to +-127.
__device__ __forceinline__ int32_t quant1(float v, float s) {
  if (s == 0.0f) return 0;
  float x = __fmul_rn(__fdiv_rn(v, s), 127.0f);
  float r = (x >= 0.0f) ? floorf(__fadd_rn(x, 0.5f)) : ceilf(__fsub_rn(x, 0.5f));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return (int32_t)r;
}

// floor(a*b / 2^30) truncated to int64 (the islands' 128-bit mulshift).
__device__ __forceinline__ int64_t mulshr30(int64_t a, int64_t b) {
  uint64_t lo = (uint64_t)a * (uint64_t)b;
  int64_t hi = __mul64hi(a, b);
  return (int64_t)((lo >> 30) | ((uint64_t)hi << 34));
}

__device__ __forceinline__ int64_t exp2_frac(int64_t r) {
  const int64_t C[7] = {1073741824LL, 744261118LL, 257941248LL, 59597083LL,
                        10327387LL, 1431680LL, 165394LL};
  int64_t acc = C[6];
#pragma unroll
  for (int k = 5; k >= 0; k--) acc = ((acc * r) >> FB) + C[k];
  return acc;
}

// e^(d / 2^30) for d <= 0, 2^30 fixed point.
__device__ __forceinline__ int64_t exp_fixed(int64_t d) {
  int64_t g = -mulshr30(d, K_LOG2E);
  int64_t n = g >> FB, r = g - (n << FB);
  if (n >= 32) return 0;
  if (r != 0) return exp2_frac(ONE - r) >> (n + 1);
  return ONE >> n;
}

__device__ __forceinline__ int64_t tanh_fixed(int64_t t) {
  int64_t a = t >= 0 ? t : -t;
  int64_t e2 = exp_fixed(-(2 * a));
  int64_t th = ONE - ((2 * e2) << FB) / (ONE + e2);
  return t >= 0 ? th : -th;
}

__device__ __forceinline__ float gelu_exact(float x) {
  int64_t xq = llround_d((double)x * 65536.0);
  int64_t X = (xq * ONE) >> 16;
  int64_t X2 = mulshr30(X, X);
  int64_t X3 = mulshr30(X2, X);
  int64_t inner = mulshr30(K_GELU_K, X + mulshr30(K_GELU_A, X3));
  int64_t t = tanh_fixed(inner);
  int64_t g = mulshr30(X >> 1, ONE + t);
  return __double2float_rn(__dmul_rn(__ll2double_rn(g), 0x1p-30));
}

__device__ __forceinline__ float silu_exact(float x) {
  int64_t xq = llround_d((double)x * 65536.0);
  int64_t X = (xq * ONE) >> 16;
  int64_t sig;
  if (X >= 0) {
    int64_t e = exp_fixed(-X);
    sig = (ONE << FB) / (ONE + e);
  } else {
    int64_t e = exp_fixed(X);
    sig = (e << FB) / (ONE + e);
  }
  int64_t g = mulshr30(X, sig);
  return __double2float_rn(__dmul_rn(__ll2double_rn(g), 0x1p-30));
}

// floor(sqrt(v)): a correctly rounded double sqrt gives the answer to within one or
// two units; the integer checks s*s <= v < (s+1)^2 then make it exact.
__device__ __forceinline__ uint64_t isqrt_u64(uint64_t v) {
  if (v == 0) return 0;
  uint64_t s = (uint64_t)__dsqrt_rn(__ull2double_rn(v));
  if (s > 0xFFFFFFFFull) s = 0xFFFFFFFFull;
  while (s * s > v) s--;
  while (s < 0xFFFFFFFFull && (s + 1) * (s + 1) <= v) s++;
  return s;
}

// (hi:lo) / d for unsigned 128-bit numerator, 64-bit divisor; returns the low 64 bits
// of the quotient (restoring long division over 128 bits).
__device__ __forceinline__ uint64_t udiv128_lo(uint64_t hi, uint64_t lo, uint64_t d) {
  // quotient high word contributes nothing to the truncated low 64 bits except through
  // the remainder, so first reduce hi modulo d.
  uint64_t r = hi % d;
  uint64_t q = 0;
#pragma unroll 1
  for (int i = 63; i >= 0; i--) {
    uint64_t top = r >> 63;
    r = (r << 1) | ((lo >> i) & 1ull);
    q <<= 1;
    if (top || r >= d) { r -= d; q |= 1ull; }
  }
  return q;
}

// floor((hi:lo) / d) when hi < d and the quotient is below 2^62: a double-precision
// estimate, one residual-based refinement, and exact +-1 steps on the 128-bit residual.
// Returns false (caller falls back to the long division) outside that range.
__device__ __forceinline__ bool udiv128_fast(uint64_t hi, uint64_t lo, uint64_t d, uint64_t &q_out) {
  if (hi >= d) return false;
  const double dd = __ull2double_rn(d);
  const double nd = __dadd_rn(__dmul_rn(__ull2double_rn(hi), 18446744073709551616.0), __ull2double_rn(lo));
  const double qe = __ddiv_rn(nd, dd);
  if (!(qe < 4611686018427387904.0)) return false;   // 2^62
  uint64_t q = (uint64_t)qe;
  for (int it = 0; it < 2; it++) {
    // residual r = N - q*d as a signed 128-bit value
    const uint64_t plo = q * d, phi = __umul64hi(q, d);
    const uint64_t rlo = lo - plo;
    const int64_t rhi = (int64_t)(hi - phi - (lo < plo ? 1ull : 0ull));
    if (rhi == 0 && rlo < d) { q_out = q; return true; }
    if (it == 1) {
      // final exact steps: the estimate is now within a few units
      int64_t h = rhi;
      uint64_t l = rlo;
      for (int k = 0; k < 8; k++) {
        if (h < 0) {              // r < 0: q -= 1, r += d
          const uint64_t nl = l + d;
          h += (nl < l) ? 1 : 0;
          l = nl;
          q -= 1;
        } else if (h > 0 || l >= d) {   // r >= d: q += 1, r -= d
          const uint64_t nl = l - d;
          h -= (l < d) ? 1 : 0;
          l = nl;
          q += 1;
        } else {
          q_out = q;
          return true;
        }
      }
      return false;
    }
    const double rd = __dadd_rn(__dmul_rn(__ll2double_rn(rhi), 18446744073709551616.0), __ull2double_rn(rlo));
    const double corr = floor(__ddiv_rn(rd, dd));
    q = (uint64_t)((int64_t)q + __double2ll_rz(corr));
  }
  return false;
}

// floor(n * 2^72 / ss) truncated to 64 bits (the RMSNorm island's uint64 quotient).
__device__ __forceinline__ uint64_t rms_quotient(uint32_t n, uint64_t ss) {
  uint64_t q;
  if (udiv128_fast((uint64_t)n << 8, 0ull, ss, q)) return q;
  return udiv128_lo((uint64_t)n << 8, 0ull, ss);
}

// floor((hi:lo) / d) for a signed 128-bit numerator whose quotient fits int64, d > 0.
__device__ __forceinline__ int64_t floordiv_s128(int64_t hi, uint64_t lo, uint64_t d) {
  bool neg = hi < 0;
  uint64_t ahi = (uint64_t)hi, alo = lo;
  if (neg) {   // |n| = ~n + 1
    alo = ~lo + 1ull;
    ahi = ~(uint64_t)hi + (alo == 0 ? 1ull : 0ull);
  }
  uint64_t q = 0, r = 0;
  if (udiv128_fast(ahi, alo, d, q)) {
    r = alo - q * d;   // the true remainder is < d < 2^64, so its low word is exact
  } else {
    r = ahi % d;
#pragma unroll 1
    for (int i = 63; i >= 0; i--) {
      uint64_t top = r >> 63;
      r = (r << 1) | ((alo >> i) & 1ull);
      q <<= 1;
      if (top || r >= d) { r -= d; q |= 1ull; }
    }
  }
  if (!neg) return (int64_t)q;
  return r ? -(int64_t)q - 1 : -(int64_t)q;
}

// ---- 128-bit signed accumulator (two's complement hi:lo) ----
struct acc128 {
  uint64_t lo;
  int64_t hi;
};
__device__ __forceinline__ void acc128_add(acc128 &a, int64_t v) {
  uint64_t lo = a.lo + (uint64_t)v;
  a.hi += (v >> 63) + (lo < a.lo ? 1 : 0);
  a.lo = lo;
}
__device__ __forceinline__ void acc128_add(acc128 &a, const acc128 &b) {
  uint64_t lo = a.lo + b.lo;
  a.hi += b.hi + (lo < a.lo ? 1 : 0);
  a.lo = lo;
}

// ---- warp reductions ----
__device__ __forceinline__ int64_t warp_sum_i64(int64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int32_t warp_sum_i32(int32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int32_t warp_max_i32(int32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace spb
