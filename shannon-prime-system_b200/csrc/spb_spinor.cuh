// spb_spinor.cuh -- the reference's frozen 63-byte Spinor KV block on the device: a K or V
// head row of HD values kept as ceil(HD / 55) blocks (header[7] = f32 scale little-endian,
// exponent 0, basis 0, 0; body[55] = int8 coefficients at Mobius slots (17 i) mod 55; CRC-8
// of header || body), include/sp/spinor_block.h:93-97 and core/vht2/{vht2,spinor_block,
// mobius_reorder}.c. Encode: scale = max |v| over the chunk (1 when 0), coefficient =
// quant1(v, scale) (the same v / s * 127, round-half-away, +-127 op sequence). Decode:
// mul = scale / 127.0f, value = coefficient * mul. The exact path keeps the attention's
// integers: a K row is encoded from its 2^16-grid values times 2^-16, a V row from its float
// projections, and the grid value attention reads is __float2int_rn(decoded * 65536).
#pragma once
#include <cstdint>

#include "spb_exact.cuh"

namespace spb {

constexpr int SPIN_BODY = 55;
constexpr int SPIN_BYTES = 63;

// the frozen balanced split of HD coordinates into NB chunks (the first EXTRA one longer)
template <int HD>
struct SpinGeom {
  static constexpr int NB = HD <= SPIN_BODY ? 1 : (HD + SPIN_BODY - 1) / SPIN_BODY;
  static constexpr int BASE = HD / NB, EXTRA = HD % NB;
  static constexpr int RB = NB * SPIN_BYTES;   // bytes of one head row
  __host__ __device__ static constexpr int start(int b) { return b * BASE + (b < EXTRA ? b : EXTRA); }
  __host__ __device__ static constexpr int len(int b) { return BASE + (b < EXTRA ? 1 : 0); }
  // chunk b and index i of coordinate d
  __device__ static void locate(int d, int &b, int &i) {
    constexpr int T = EXTRA * (BASE + 1);
    if (d < T) {
      b = d / (BASE + 1);
      i = d - b * (BASE + 1);
    } else {
      const int e = d - T;
      b = EXTRA + e / BASE;
      i = e - (b - EXTRA) * BASE;
    }
  }
};
inline int spin_row_bytes(int hd) { return (hd <= SPIN_BODY ? 1 : (hd + SPIN_BODY - 1) / SPIN_BODY) * SPIN_BYTES; }

// CRC-8/SMBus (poly 0x07, init 0, no reflection, xorout 0) in slices of four bytes: for a
// linear CRC, crc after bytes b0..b3 = T4[crc ^ b0] ^ T3[b1] ^ T2[b2] ^ T1[b3], Tk = the byte
// table applied k times. The four tables are built once per CTA into shared memory.
__device__ __forceinline__ uint32_t crc8_byte_table(uint32_t x) {
  for (int b = 0; b < 8; b++) x = (x & 0x80u) ? ((x << 1) ^ 0x07u) & 0xFFu : (x << 1) & 0xFFu;
  return x;
}
// tab: 1024 bytes of shared memory; every thread of the CTA calls this (nthreads >= 32)
__device__ __forceinline__ void crc8_tables_build(uint8_t *tab, int tid, int nthreads) {
  for (int x = tid; x < 256; x += nthreads) {
    uint32_t t = crc8_byte_table((uint32_t)x);
    tab[x] = (uint8_t)t;                // T1
    t = crc8_byte_table(t);
    tab[256 + x] = (uint8_t)t;          // T2
    t = crc8_byte_table(t);
    tab[512 + x] = (uint8_t)t;          // T3
    t = crc8_byte_table(t);
    tab[768 + x] = (uint8_t)t;          // T4
  }
}
__device__ __forceinline__ uint32_t crc8_62(const uint8_t *m, const uint8_t *tab) {
  uint32_t c = 0;
  for (int j = 0; j < 60; j += 4)
    c = tab[768 + (c ^ m[j])] ^ tab[512 + m[j + 1]] ^ tab[256 + m[j + 2]] ^ tab[m[j + 3]];
  c = tab[c ^ m[60]];
  c = tab[c ^ m[61]];
  return c;
}

// One warp encodes chunk values v (lane i holds v[i] and v[i + 32] for i < len) into the
// 63-byte block `img` (shared memory, 64 bytes, written whole) and returns each lane's two
// decoded grid values (for its i and i + 32). tab: the CRC tables. Caller syncs the warp
// before reading img.
__device__ __forceinline__ void spin_encode_warp(float v0, float v1, int len, uint8_t *img, const uint8_t *tab,
                                                 int32_t &g0, int32_t &g1) {
  const int lane = threadIdx.x & 31;
  const bool h0 = lane < len, h1 = lane + 32 < len;
  float m = fmaxf(h0 ? fabsf(v0) : 0.0f, h1 ? fabsf(v1) : 0.0f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float scale = m > 0.0f ? m : 1.0f;
  if (lane < 16) reinterpret_cast<uint32_t *>(img)[lane] = 0u;
  __syncwarp();
  const int32_t q0 = h0 ? quant1(v0, scale) : 0, q1 = h1 ? quant1(v1, scale) : 0;
  if (h0) img[7 + (17 * lane) % SPIN_BODY] = (uint8_t)(int8_t)q0;
  if (h1) img[7 + (17 * (lane + 32)) % SPIN_BODY] = (uint8_t)(int8_t)q1;
  if (lane == 0) {
    const uint32_t u = __float_as_uint(scale);
    img[0] = (uint8_t)u;
    img[1] = (uint8_t)(u >> 8);
    img[2] = (uint8_t)(u >> 16);
    img[3] = (uint8_t)(u >> 24);
  }
  __syncwarp();
  if (lane == 0) img[62] = (uint8_t)crc8_62(img, tab);
  const float mul = __fdiv_rn(scale, 127.0f);
  g0 = __float2int_rn(__fmul_rn(__fmul_rn((float)q0, mul), 65536.0f));
  g1 = __float2int_rn(__fmul_rn(__fmul_rn((float)q1, mul), 65536.0f));
  __syncwarp();
}

// A head row of hd values (v: K grid values when kgrid, else V floats) encoded by the warps of
// the CTA, chunk b by warp b % nwarps: the blocks go to dst (global, hd's row bytes), the
// decoded grid values to grid (shared or global). V values must be below 16384 in magnitude
// before and after the round trip (ERR_V_RANGE). imgs: 64 bytes of shared memory per warp.
__device__ __forceinline__ void spin_encode_row(const void *v, bool kgrid, int hd, uint8_t *dst, int32_t *grid,
                                                uint8_t *imgs, const uint8_t *tab, uint32_t *err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int nb = hd <= SPIN_BODY ? 1 : (hd + SPIN_BODY - 1) / SPIN_BODY, base = hd / nb, extra = hd % nb;
  uint8_t *img = imgs + warp * 64;
  for (int b = warp; b < nb; b += nw) {
    const int off = b * base + min(b, extra), len = base + (b < extra ? 1 : 0);
    float x[2] = {0.0f, 0.0f};
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int i = lane + 32 * r;
      if (i < len) {
        if (kgrid) {
          x[r] = __fmul_rn((float)reinterpret_cast<const int32_t *>(v)[off + i], 1.0f / 65536.0f);
        } else {
          x[r] = reinterpret_cast<const float *>(v)[off + i];
          if (!(fabsf(x[r]) < 16384.0f)) { raise_err(err, ERR_V_RANGE); x[r] = 0.0f; }
        }
      }
    }
    int32_t g0, g1;
    spin_encode_warp(x[0], x[1], len, img, tab, g0, g1);
    for (int j = lane; j < SPIN_BYTES; j += 32) dst[b * SPIN_BYTES + j] = img[j];
    if (!kgrid && (g0 >= (1 << 30) || g0 <= -(1 << 30) || g1 >= (1 << 30) || g1 <= -(1 << 30)))
      raise_err(err, ERR_V_RANGE);
    if (grid && lane < len) grid[off + lane] = g0;
    if (grid && lane + 32 < len) grid[off + lane + 32] = g1;
    __syncwarp();
  }
}

// the f32 scale of a block (bytes 0..3, little-endian) as the decode multiplier scale / 127
__device__ __forceinline__ float spin_block_mul(const uint8_t *blk) {
  const uint32_t u = (uint32_t)blk[0] | ((uint32_t)blk[1] << 8) | ((uint32_t)blk[2] << 16) | ((uint32_t)blk[3] << 24);
  return __fdiv_rn(__uint_as_float(u), 127.0f);
}

// grid value of coefficient byte c under multiplier mul
__device__ __forceinline__ int32_t spin_grid(uint8_t c, float mul) {
  return __float2int_rn(__fmul_rn(__fmul_rn((float)(int8_t)c, mul), 65536.0f));
}

}  // namespace spb
