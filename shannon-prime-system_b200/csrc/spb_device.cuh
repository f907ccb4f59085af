// spb_device.cuh -- element-level device helpers of the kernels: the OK_Q4B block dot and
// block-scale accumulation, the RMSNorm island's per-element pieces, the CORDIC rotation and
// the greedy-argmax key.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#include "spb_exact.cuh"
#include "spb_kernels.cuh"

namespace spb {

// llround(x * 2^16) for |x| < 32768: x * 2^16 is exact in fp32 and below 2^31, its
// fractional part is exact too, so this equals the islands' llround((double)x * 65536.0)
__device__ __forceinline__ int32_t q16_round(float x) {
  const float v = __fmul_rn(x, 65536.0f);
  const float t = truncf(v);
  const float f = __fsub_rn(v, t);
  return (int32_t)t + (f >= 0.5f ? 1 : 0) - (f <= -0.5f ? 1 : 0);
}

// exact int32 dot of one 32-column block: 16 code bytes against the 8 activation words
// (x0: words 0-3, x1: words 4-7; each 8-column group is [even cols][odd cols])
__device__ __forceinline__ int32_t block_dot(const uint4 cw, const int4 x0, const int4 x1) {
  const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
  const int32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  int32_t s = 0;
#pragma unroll
  for (int g = 0; g < 4; g++) {
    const int32_t lo = (int32_t)((w[g] & 0x0F0F0F0Fu) ^ 0x08080808u);
    const int32_t hi = (int32_t)(((w[g] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u);
    s = __dp4a(lo, xv[2 * g], s);
    s = __dp4a(hi, xv[2 * g + 1], s);
  }
  return s;
}

// d = c + sum of the 4 unsigned bytes of a times the 4 signed bytes of b
__device__ __forceinline__ int32_t dp4a_us(uint32_t a, int32_t b, int32_t c) {
  int32_t d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// block_dot(cw, x0, x1) + corr with one mask-and-flip per nibble half and no shift: even columns
// (w & 0x0F) ^ 0x08 = code + 8 per byte; odd columns (w & 0xF0) ^ 0x80 = 16 (code + 8) per
// unsigned byte, so that half's sum is exactly 16 times its block sum (an arithmetic shift by 4)
__device__ __forceinline__ int32_t block_dot_corr(const uint4 cw, const int4 x0, const int4 x1, int32_t corr) {
  const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
  const int32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  int32_t lo = corr, hi = 0;
#pragma unroll
  for (int g = 0; g < 4; g++) {
    lo = dp4a_us((w[g] & 0x0F0F0F0Fu) ^ 0x08080808u, xv[2 * g], lo);
    hi = dp4a_us((w[g] & 0xF0F0F0F0u) ^ 0x80808080u, xv[2 * g + 1], hi);
  }
  return lo + (hi >> 4);
}

// acc += k * isum with the f16 block scale as k = m * 2^sh (|m| < 2^11, sh < 30):
// one 32-bit multiply (|m*isum| < 2^26) and one widening multiply-add by 2^sh.
__device__ __forceinline__ void scale_acc(int64_t &acc, uint32_t h, int32_t isum) {
  const uint32_t e = (h >> 10) & 31u;
  int32_t m = (int32_t)(e ? ((h & 1023u) | 1024u) : (h & 1023u));
  if (h & 0x8000u) m = -m;
  const int32_t pw = 1 << (e ? e - 1 : 0);
  acc += (int64_t)(m * isum) * (int64_t)pw;
}

// Greedy-argmax key: f32 bits mapped to an order-preserving uint32 in the high word, the
// complemented row index in the low word, so a 64-bit max picks the largest value and,
// among equal values, the lowest index (the first maximum).
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}

// interleaved byte position of column c inside its 32-column block
__device__ __forceinline__ int perm_pos(int c) {
  const int p = c & 7;
  return (c & ~7) + ((p & 1) << 2) + (p >> 1);
}

__device__ __forceinline__ uint64_t rms_inv(const acc128 &tot, int n, uint32_t *err) {
  if (tot.hi != 0 || (tot.lo >> 63)) {
    raise_err(err, ERR_NORM_RANGE);
    return 0;
  }
  return tot.lo ? isqrt_u64(rms_quotient((uint32_t)n, tot.lo)) : 0ull;
}

__device__ __forceinline__ float rms_apply(float x, float w, uint64_t inv, uint32_t *err) {
  if (!(fabsf(w) < 32768.0f)) { raise_err(err, ERR_NORM_RANGE); w = 0.0f; }
  const int64_t xi = q16_round(fabsf(x) < 32768.0f ? x : 0.0f), wi = q16_round(w);
  const int64_t yi = (int64_t)((uint64_t)xi * inv * (uint64_t)wi);
  return __double2float_rn(__dmul_rn(__ll2double_rn(yi), 0x1p-52));
}

// CORDIC-RoPE rotation of one (a, b) pair onto the 2^16 score grid; UNROLL sets how far the
// 30 micro-rotations are unrolled (code size against loop overhead)
constexpr int CORDIC_ITERS = 30;

template <int UNROLL = CORDIC_ITERS>
__device__ __forceinline__ void cordic_rotate(float a, float b, uint64_t phase, const uint64_t *T, uint64_t gain,
                                              int32_t &oa, int32_t &ob, uint32_t *err) {
  if (!(fabsf(a) < 256.0f) || !(fabsf(b) < 256.0f)) { raise_err(err, ERR_ROPE_RANGE); a = 0.0f; b = 0.0f; }
  const int64_t A = llround_d((double)a * 1073741824.0);
  const int64_t B = llround_d((double)b * 1073741824.0);
  const uint64_t ph = phase + (1ull << 61);
  const unsigned quad = (unsigned)(ph >> 62);
  int64_t z = (int64_t)(ph & ((1ull << 62) - 1)) - (1ll << 61);
  int64_t X, Y;
  switch (quad) {
    case 0: X = A; Y = B; break;
    case 1: X = -B; Y = A; break;
    case 2: X = -A; Y = -B; break;
    default: X = B; Y = -A; break;
  }
#pragma unroll UNROLL
  for (int k = 0; k < CORDIC_ITERS; k++) {
    const int64_t xs = X >> k, ys = Y >> k;
    const int64_t tk = (int64_t)T[k];
    if (z >= 0) { X -= ys; Y += xs; z -= tk; }
    else { X += ys; Y -= xs; z += tk; }
  }
  // round((X * gain) / 2^76), half up: the high word of the 128-bit product plus 2^75
  const int64_t rx = (__mul64hi(X, (int64_t)gain) + 2048) >> 12;
  const int64_t ry = (__mul64hi(Y, (int64_t)gain) + 2048) >> 12;
  if (rx >= (1 << 24) || rx <= -(1 << 24) || ry >= (1 << 24) || ry <= -(1 << 24)) {
    raise_err(err, ERR_ROPE_RANGE);
    oa = 0; ob = 0;
    return;
  }
  oa = (int32_t)rx;
  ob = (int32_t)ry;
}

// exact f16 -> f32 (the hardware conversion is exact for every finite f16)
__device__ __forceinline__ float f16_value(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)h));
}

}  // namespace spb
