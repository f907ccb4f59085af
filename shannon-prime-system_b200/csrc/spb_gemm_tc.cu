// spb_gemm_tc.cu -- the token-batch OK_Q4B GEMM on the fifth-generation tensor cores:
// tcgen05.mma kind::i8 (int8 x int8 -> int32) with the accumulators in tensor memory, the
// activation tiles staged by TMA (cp.async.bulk.tensor, 128-byte swizzle), one elected thread
// issuing the MMAs. It replaces the n_tok > 1 branch of matmul_arena (forward_dispatch.c:74-84)
// for large token batches (prefill chunks), with exactly the integers of the dequant-GEMV.
//
// The per-32-column f16 block scales are folded into the weights as 8-bit digit planes. A
// row's block scale is k_b = m_b * 2^s_b (m_b the signed 11-bit mantissa, s_b = max(e - 1, 0));
// with sigma = the row's smallest s_b over nonzero blocks (DevQ4B::shift), every weight becomes
// the integer W_i = code_i * m_b * 2^(s_b - sigma), and the exact accumulator of the GEMV is
//     acc = sum_b k_b * sum_{i in b} code_i x_i = 2^sigma * sum_i W_i x_i.
// W_i fits 8P-bit two's complement for the row spreads s_b - sigma that DevQ4B::planes covers
// (P = 2: spread <= 1, 3: <= 9, 4: <= 17), so W_i = sum_d 256^d D_d,i with bytes D_0..D_{P-2}
// unsigned and D_{P-1} signed. Each plane is one plain int8 GEMM over the full K into an int32
// accumulator in tensor memory (exact: |x| <= 127, |D| <= 255, K <= 16384 -> |sum| < 2^31), and
// the epilogue rebuilds acc = 2^sigma * sum_d 256^d P_d in 64-bit two's complement (exact modulo
// 2^64, and the true value is inside int64 by the upload bound). The planes are produced in
// shared memory from the packed codes by converter warps, so HBM still reads 0.5625 bytes per
// weight; the activation rows are the GEMV's quantized rows (the column order inside each
// 8-column group, even then odd, is the same on both operands, so it cancels).
//
// CTA: 128 weight rows x N token rows (N = 256 / 160 / 128 / 80 for P x matrices = 2 / 3 / 4 / 6),
// a ring of S stages of 128 columns. Warp 0: TMA producer of the activation tiles; warp 1:
// tensor-memory allocation and the MMA issuer; warps 2-9: converters (codes -> planes), then
// the epilogue (tensor memory -> int64 -> f32), two warps per tensor-memory lane quarter, each
// taking every other 16-column chunk. Every mbarrier wait is bounded
// (ERR_TIMEOUT), the tensor memory is freed on every path, and no load uses cluster multicast.
#include <cuda.h>

#include "spb_async.cuh"
#include "spb_device.cuh"
#include "spb_exact.cuh"
#include "spb_kernels.cuh"

#include <mutex>

namespace spb {

namespace {

constexpr int TC_BM = 128;          // weight rows per CTA (the MMA's M)
constexpr int TC_BK = 128;          // columns per stage: one 128-byte swizzle atom per row
constexpr int TC_CONV_WARPS = 8;    // converter warps (2..9)
constexpr int TC_THREADS = 32 * (2 + TC_CONV_WARPS);
constexpr int TC_PLANE = TC_BM * TC_BK;   // bytes of one plane tile
constexpr int TC_SMEM_BUDGET = 225 * 1024;

// SN 1: the 64-token tile for batches of at most 64 rows (the multi-session decode step), where
// the larger tiles would mostly multiply zero rows; SN 2 (two planes of one matrix): a 128-token
// tile with two stages, so that two CTAs share an SM (256 tensor-memory columns and ~97 KB of
// shared memory each) and one CTA's epilogue overlaps the other's main loop
template <int P, int NM, int SN = 0>
struct TcShape {
  static constexpr int PM = P * NM;
  static constexpr int N = SN == 1 ? 64 : SN == 2 ? 128 : PM == 2 ? 256 : PM == 3 ? 160 : PM == 4 ? 128 : 80;
  static constexpr int COLS = PM * N;                                             // tensor-memory columns used
  static constexpr int TMEM_COLS = COLS <= 256 ? 256 : 512;
  static constexpr int A_BYTES = PM * TC_PLANE;
  static constexpr int B_BYTES = N * TC_BK;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int S0 = (TC_SMEM_BUDGET - 1024) / STAGE;
  static constexpr int S = SN == 2 ? 2 : S0 > 4 ? 4 : S0;
  static constexpr int CTAS_PER_SM = SN == 2 ? 2 : 1;
  static constexpr int SMEM = S * STAGE + 1024;   // + alignment slack (stages start 1024-aligned)
  static_assert(COLS <= 512, "tensor memory holds 512 columns");
  static_assert(S >= 2, "at least two stages");
  static_assert(B_BYTES % 1024 == 0 && A_BYTES % 1024 == 0, "stage parts stay 1024-aligned");
};

__device__ __forceinline__ void pdl_wait_tc() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger_tc() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// K-major operand tile in shared memory with the 128-byte swizzle: 8-row groups of 1024 bytes
// (stride-dimension offset), rows of 128 bytes; start address, LBO 1 (unused for swizzled
// K-major), SBO 1024 bytes, descriptor version 1, layout SWIZZLE_128B
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// instruction descriptor of kind::i8: int32 accumulator, A unsigned or signed bytes, B signed
// bytes, both K-major, M = 128, N
__device__ __forceinline__ uint32_t idesc_i8(int n, bool a_signed) {
  return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// 16 consecutive accumulator columns of this warp's 32 tensor-memory lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) { return __byte_perm(a, b, s); }

// byte offset of 16-byte chunk c (0..7) of row r inside a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// The multiplier of one block for its row: m * 2^(s - sigma) (0 for a zero block)
__device__ __forceinline__ int32_t block_mult(uint32_t h, int sigma) {
  const uint32_t e = (h >> 10) & 31u;
  const int32_t m = (int32_t)(e ? ((h & 1023u) | 1024u) : (h & 1023u));
  if (m == 0) return 0;
  const int d = (e ? (int)e - 1 : 0) - sigma;   // 0 .. spread (the row's prepared shift)
  const int32_t v = m << d;
  return (h & 0x8000u) ? -v : v;
}

// 32 weights (one 16-byte code vector, one block) -> P plane chunks of 32 bytes (two 16-byte
// halves each: words 0-1 then words 2-3 of the code vector), in the activation's column order
template <int P>
__device__ __forceinline__ void convert_block(const uint4 cw, int32_t mult, uint32_t (&out)[P][8]) {
  const uint32_t wv[4] = {cw.x, cw.y, cw.z, cw.w};
  if (P == 2) {
    // two 16-bit lanes per register: u * |mult| stays below 2^16 (u <= 15, |mult| <= 4094), and
    // the offset 2^15 -/+ 8|mult| keeps each lane in [0, 2^16) with no carry or borrow between
    // lanes; flipping bit 15 of each lane then gives the int16 two's complement of W = (u - 8) * mult
    const bool neg = mult < 0;
    const uint32_t am = (uint32_t)(neg ? -mult : mult);
    const uint32_t c = neg ? (0x8000u + 8u * am) : (0x8000u - 8u * am);
    const uint32_t cc = c | (c << 16);
#pragma unroll
    for (int g = 0; g < 4; g++) {
      const uint32_t u = wv[g] ^ 0x88888888u;
      const uint32_t lo = u & 0x0F0F0F0Fu, hi = (u >> 4) & 0x0F0F0F0Fu;
      uint32_t h4[4] = {prmt(lo, 0, 0x4140), prmt(lo, 0, 0x4342), prmt(hi, 0, 0x4140), prmt(hi, 0, 0x4342)};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const uint32_t x = h4[j] * am;
        h4[j] = (neg ? (cc - x) : (x + cc)) ^ 0x80008000u;
      }
      out[0][2 * g] = prmt(h4[0], h4[1], 0x6420);
      out[1][2 * g] = prmt(h4[0], h4[1], 0x7531);
      out[0][2 * g + 1] = prmt(h4[2], h4[3], 0x6420);
      out[1][2 * g + 1] = prmt(h4[2], h4[3], 0x7531);
    }
  } else {
    // one 32-bit two's-complement W per weight: W = u * mult - 8 * mult (|W| < 2^31 for P <= 4;
    // u * mult alone may pass 2^31, so the arithmetic is modulo 2^32, where the sum is exact)
    const uint32_t c = 0u - 8u * (uint32_t)mult, um = (uint32_t)mult;
#pragma unroll
    for (int g = 0; g < 4; g++) {
      const uint32_t u = wv[g] ^ 0x88888888u;
      uint32_t W[8];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        W[j] = ((u >> (8 * j)) & 15u) * um + c;           // even columns (low nibbles)
        W[4 + j] = ((u >> (8 * j + 4)) & 15u) * um + c;   // odd columns (high nibbles)
      }
#pragma unroll
      for (int d = 0; d < P; d++) {
        const uint32_t sel = (uint32_t)d | ((uint32_t)(d + 4) << 4);
        const uint32_t a = prmt(prmt(W[0], W[1], sel), prmt(W[2], W[3], sel), 0x5410);
        const uint32_t b = prmt(prmt(W[4], W[5], sel), prmt(W[6], W[7], sel), 0x5410);
        out[d][2 * g] = a;
        out[d][2 * g + 1] = b;
      }
    }
  }
}

// APL: the weight planes come precomputed (DevQ4B::pl) by TMA (tma0 / tma1 over [P x rows][K]
// bytes, the same 128-byte swizzle), and the converter warps only run the epilogue
template <int P, int NM, int EPI, int SN, bool APL = false>
__global__ void __launch_bounds__(TC_THREADS, TcShape<P, NM, SN>::CTAS_PER_SM)
k_gemm_tc(const __grid_constant__ CUtensorMap tmb, const __grid_constant__ CUtensorMap tma0,
          const __grid_constant__ CUtensorMap tma1, DevQ4B w, DevQ4B w2, DevAct act, int ntok, int ks, float *y,
          int ldy, uint32_t *err, uint32_t *ymax, unsigned long long *amax) {
  using SH = TcShape<P, NM, SN>;
  constexpr int N = SH::N, S = SH::S;
  constexpr int PF = 2;   // stages of codes and scales in flight in the converters' registers
  extern __shared__ uint8_t tsm_raw[];
  __shared__ __align__(8) uint64_t full_a[S], full_b[S], empty[S], tfull;
  __shared__ uint32_t tmem_base_sh;
  __shared__ double dsc[N];
  __shared__ float tmax[N];
  __shared__ unsigned long long tkey[N];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_addr(tsm_raw);
  uint8_t *tsm = tsm_raw + ((1024u - (raw & 1023u)) & 1023u);
  const int K = w.cols, rows = w.rows;
  const int t0 = blockIdx.x * N, row0 = blockIdx.y * TC_BM, part = blockIdx.z;
  const int kper = K / ks, kbase = part * kper, nk = kper / TC_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full_a[s], APL ? 1 : TC_CONV_WARPS);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&tfull, 1);
    mbar_init_fence();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmb) : "memory");
    if (APL) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tma0) : "memory");
      if (NM == 2) asm volatile("prefetch.tensormap [%0];" ::"l"(&tma1) : "memory");
    }
  }
  if (warp == 1) {   // the whole warp allocates; the base column address lands in shared memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base_sh)),
                 "r"(SH::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  for (int t = threadIdx.x; t < N; t += TC_THREADS) {
    tmax[t] = 0.0f;
    tkey[t] = 0ull;
  }
  pdl_trigger_tc();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ---- TMA producer: the activation tile [N tokens][128 columns] of every stage (the warp
    // walks the loop together, lane 0 issues)
    pdl_wait_tc();
    for (int kt = 0; kt < nk; kt++) {
      const int s = kt % S, r = kt / S;
      if (lane == 0) {
        mbar_wait(&empty[s], (r & 1) ^ 1, err);
        uint8_t *B = tsm + s * SH::STAGE + SH::A_BYTES;
        mbar_arrive_expect_tx(&full_b[s], SH::B_BYTES);
        tma_load_2d(B, &tmb, kbase + kt * TC_BK, t0, &full_b[s]);
        if (APL) {   // the stage's plane tiles: plane d of matrix m at rows d * rows + row0
          uint8_t *A = tsm + s * SH::STAGE;
          mbar_arrive_expect_tx(&full_a[s], SH::A_BYTES);
#pragma unroll
          for (int q = 0; q < SH::PM; q++)
            tma_load_2d(A + q * TC_PLANE, q / P ? &tma1 : &tma0, kbase + kt * TC_BK, (q % P) * rows + row0,
                        &full_a[s]);
        }
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ---- MMA issuer: per stage, 4 K-steps of 32 columns x (matrices x planes) accumulators
    const uint32_t id_u = idesc_i8(N, false), id_s = idesc_i8(N, true);
    for (int kt = 0; kt < nk; kt++) {
      const int s = kt % S, r = kt / S;
      if (lane == 0) {
        mbar_wait(&full_a[s], r & 1, err);
        mbar_wait(&full_b[s], r & 1, err);
        tc_fence_after();
        const uint32_t sa = smem_addr(tsm + s * SH::STAGE), sb = sa + SH::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < TC_BK / 32; kk++) {
          const uint64_t bdesc = umma_desc(sb + kk * 32);
#pragma unroll
          for (int q = 0; q < SH::PM; q++) {   // q = m * P + d
            const uint64_t adesc = umma_desc(sa + q * TC_PLANE + kk * 32);
            mma_i8(tmem + q * N, adesc, bdesc, (q % P) == P - 1 ? id_s : id_u, (kt | kk) != 0);
          }
        }
        mma_commit(&empty[s]);   // the stage is free once these MMAs have read it
      }
      __syncwarp();
    }
    if (lane == 0) mma_commit(&tfull);   // every accumulator is final
    __syncwarp();
  } else {
    // ---- converters: thread ct takes row ct / 2 and the two 32-column blocks (ct & 1) * 2 + {0,1}
    const int ct = threadIdx.x - 64, row = ct >> 1, hb = ct & 1;
    if (!APL) {
    const int grow = row0 + row;
    const bool valid = grow < rows;
    const size_t rb = (size_t)(valid ? grow : 0);
    const uint8_t *cp[NM];
    const uint16_t *sp[NM];
    int sig[NM];
#pragma unroll
    for (int m = 0; m < NM; m++) {
      const DevQ4B &q = m ? w2 : w;
      cp[m] = q.codes + rb * (size_t)(K >> 1) + (kbase >> 1) + hb * 32;
      sp[m] = q.scales + rb * (size_t)(K >> 5) + (kbase >> 5) + hb * 2;
      sig[m] = valid ? q.shift[rb] : 0;
    }
    // register ring of PF stages of codes and scales: stage kt + PF is loading while stage kt
    // converts
    uint4 cw[PF][NM][2];
    uint32_t sc[PF][NM];
    auto fetch = [&](int kt, uint4 (&c)[NM][2], uint32_t (&h)[NM]) {
#pragma unroll
      for (int m = 0; m < NM; m++) {
        if (valid) {
          c[m][0] = __ldg(reinterpret_cast<const uint4 *>(cp[m] + (size_t)kt * 64));
          c[m][1] = __ldg(reinterpret_cast<const uint4 *>(cp[m] + (size_t)kt * 64 + 16));
          h[m] = __ldg(reinterpret_cast<const uint32_t *>(sp[m] + (size_t)kt * 4));
        } else {
          c[m][0] = c[m][1] = make_uint4(0u, 0u, 0u, 0u);
          h[m] = 0u;
        }
      }
    };
#pragma unroll
    for (int f = 0; f < PF; f++)
      if (f < nk) fetch(f, cw[f], sc[f]);
    for (int kt0 = 0; kt0 < nk; kt0 += PF) {
#pragma unroll
      for (int u = 0; u < PF; u++) {
        const int kt = kt0 + u;
        if (kt >= nk) break;
        const int s = kt % S, r = kt / S;
        uint4 cur[NM][2];
        uint32_t scur[NM];
#pragma unroll
        for (int m = 0; m < NM; m++) {
          cur[m][0] = cw[u][m][0];
          cur[m][1] = cw[u][m][1];
          scur[m] = sc[u][m];
        }
        if (kt + PF < nk) fetch(kt + PF, cw[u], sc[u]);
        mbar_wait(&empty[s], (r & 1) ^ 1, err);
        uint8_t *A = tsm + s * SH::STAGE;
#pragma unroll
        for (int m = 0; m < NM; m++) {
#pragma unroll
          for (int j = 0; j < 2; j++) {
            const uint32_t h = (scur[m] >> (16 * j)) & 0xFFFFu;
            uint32_t pl[P][8];
            convert_block<P>(cur[m][j], block_mult(h, sig[m]), pl);
            const int blk = hb * 2 + j;   // block inside the stage: chunks 2 blk, 2 blk + 1
#pragma unroll
            for (int d = 0; d < P; d++) {
              uint8_t *T = A + (m * P + d) * TC_PLANE;
              *reinterpret_cast<uint4 *>(T + swz(row, 2 * blk)) = make_uint4(pl[d][0], pl[d][1], pl[d][2], pl[d][3]);
              *reinterpret_cast<uint4 *>(T + swz(row, 2 * blk + 1)) = make_uint4(pl[d][4], pl[d][5], pl[d][6], pl[d][7]);
            }
          }
        }
        fence_proxy_async_smem();   // the generic-proxy stores become visible to the tensor cores
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
      }
    }
    }   // !APL

    // ---- epilogue (all converter warps): warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (its
    // weight rows) and every other 16-column chunk (eh = 0: warps 2-5, 1: warps 6-9)
    {
      const int sub = warp & 3, eh = (warp - 2) >> 2, erow = sub * 32 + lane, egrow = row0 + erow;
      const bool evalid = egrow < rows;
      pdl_wait_tc();
      const int et = threadIdx.x - 64;   // 0..255
      for (int t = et; t < N; t += 32 * TC_CONV_WARPS)
        dsc[t] = (t0 + t < ntok) ? __dmul_rn(__ddiv_rn((double)act.scale[t0 + t], 127.0), 0x1p-24) : 0.0;
      asm volatile("bar.sync 1, %0;" ::"n"(32 * TC_CONV_WARPS) : "memory");
      mbar_wait(&tfull, 0, err);
      tc_fence_after();
      int esig[NM];
#pragma unroll
      for (int m = 0; m < NM; m++) esig[m] = evalid ? (m ? w2 : w).shift[egrow] : 0;
      const uint32_t lane_base = tmem + ((uint32_t)(sub * 32) << 16);
      for (int c = eh * 16; c < N; c += 32) {
        uint64_t acc[NM][16];
        int32_t v[NM][P][16];
#pragma unroll
        for (int m = 0; m < NM; m++)
#pragma unroll
          for (int d = 0; d < P; d++) tmem_ld16(lane_base + (uint32_t)((m * P + d) * N + c), v[m][d]);
        tmem_wait_ld();   // one wait for all the chunk's loads
#pragma unroll
        for (int m = 0; m < NM; m++)
#pragma unroll
          for (int i = 0; i < 16; i++) {
            uint64_t a = 0ull;
#pragma unroll
            for (int d = 0; d < P; d++) a += (uint64_t)(int64_t)v[m][d][i] << (8 * d);
            acc[m][i] = a;
          }
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int tl = c + i, t = t0 + tl;
          const bool ok = evalid && t < ntok;
          const int64_t a0 = (int64_t)(acc[0][i] << esig[0]);
          float v = 0.0f;
          if (EPI == EPI_I64) {
            if (ok) reinterpret_cast<int64_t *>(y)[((size_t)part * ntok + t) * ldy + egrow] = a0;
            continue;
          }
          v = __double2float_rn(__dmul_rn(__ll2double_rn(a0), dsc[tl]));
          if (epi_pair(EPI)) {
            const int64_t a1 = (int64_t)(acc[NM - 1][i] << esig[NM - 1]);
            const float u = __double2float_rn(__dmul_rn(__ll2double_rn(a1), dsc[tl]));
            if (!(fabsf(v) < 2048.0f)) {
              if (ok) raise_err(err, ERR_ACT_RANGE);
              v = 0.0f;
            }
            v = __fmul_rn(EPI == EPI_GELU_MUL ? gelu_exact(v) : silu_exact(v), u);
          }
          if (ok) y[(size_t)t * ldy + egrow] = v;
          if (ymax) {
            float mv = ok ? fabsf(v) : 0.0f;
            if (ok && !(mv <= 3.402823466e38f)) { raise_err(err, ERR_ACT_RANGE); mv = 0.0f; }
            mv = warp_max_f(mv);
            if (lane == 0 && mv > 0.0f) atomicMax(reinterpret_cast<unsigned int *>(&tmax[tl]), __float_as_uint(mv));
          }
          if (amax) {
            unsigned long long k = ok ? argmax_key(v, egrow) : 0ull;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
              const unsigned long long ok2 = __shfl_xor_sync(0xffffffffu, k, o);
              k = ok2 > k ? ok2 : k;
            }
            if (lane == 0 && k) atomicMax(&tkey[tl], k);
          }
        }
      }
      tc_fence_before();
      asm volatile("bar.sync 1, %0;" ::"n"(32 * TC_CONV_WARPS) : "memory");
      for (int t = et; t < N; t += 32 * TC_CONV_WARPS) {
        if (t0 + t >= ntok) continue;
        if (ymax && tmax[t] > 0.0f) atomicMax(ymax + t0 + t, __float_as_uint(tmax[t]));
        if (amax && tkey[t]) atomicMax(amax + t0 + t, tkey[t]);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {   // free the tensor memory once every read of it has completed
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(SH::TMEM_COLS) : "memory");
  }
}

// One thread per (row, 32-column block): the block's P digit planes (convert_block, the
// converters' arithmetic) stored row-major, block b at bytes 32 b .. 32 b + 31 of each plane row
template <int P>
__global__ void __launch_bounds__(256) k_q4b_planes(DevQ4B w, uint8_t *out) {
  const int nblk = w.cols >> 5;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)w.rows * nblk) return;
  const int row = (int)(i / nblk), b = (int)(i - (long long)row * nblk);
  const uint4 cw = *reinterpret_cast<const uint4 *>(w.codes + (size_t)row * (w.cols >> 1) + (size_t)b * 16);
  const uint32_t h = w.scales[(size_t)row * nblk + b];
  uint32_t pl[P][8];
  convert_block<P>(cw, block_mult(h, w.shift[row]), pl);
#pragma unroll
  for (int d = 0; d < P; d++) {
    uint4 *dst = reinterpret_cast<uint4 *>(out + ((size_t)d * w.rows + row) * w.cols + (size_t)b * 32);
    dst[0] = make_uint4(pl[d][0], pl[d][1], pl[d][2], pl[d][3]);
    dst[1] = make_uint4(pl[d][4], pl[d][5], pl[d][6], pl[d][7]);
  }
}

// ---- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool tc_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_TC");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}

// a 2-D TMA map over [P x rows][K] plane bytes: 128-byte boxes of 128 rows, 128-byte swizzle
static bool plane_map(EncodeTiledFn enc, CUtensorMap *tm, const DevQ4B &w, int P) {
  const cuuint64_t gdim[2] = {(cuuint64_t)w.cols, (cuuint64_t)P * (cuuint64_t)w.rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)w.cols};
  const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)TC_BM};
  const cuuint32_t estr[2] = {1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)w.pl, gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int P, int NM, int EPI, int SN, bool APL = false>
cudaError_t tc_launch_sn(const DevQ4B &w, const DevQ4B &w2, const DevAct &act, int ntok, float *y, int ldy, uint32_t *err,
                      uint32_t *ymax, unsigned long long *amax, cudaStream_t st, int ks, bool pdl) {
  using SH = TcShape<P, NM, SN>;
  auto kern = k_gemm_tc<P, NM, EPI, SN, APL>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SH::SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap tm;
  const cuuint64_t gdim[2] = {(cuuint64_t)w.cols, (cuuint64_t)ntok};
  const cuuint64_t gstride[1] = {(cuuint64_t)w.cols};
  const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)SH::N};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)act.q, gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  CUtensorMap ta0 = tm, ta1 = tm;   // (unused without APL)
  if (APL && (!plane_map(enc, &ta0, w, P) || (NM == 2 && !plane_map(enc, &ta1, w2, P)))) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((ntok + SH::N - 1) / SH::N, (w.rows + TC_BM - 1) / TC_BM, ks);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = SH::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, tm, ta0, ta1, w, w2, act, ntok, ks, y, ldy, err, ymax, amax);
}

template <int P, int NM, int EPI>
cudaError_t tc_launch(const DevQ4B &w, const DevQ4B &w2, const DevAct &act, int ntok, float *y, int ldy, uint32_t *err,
                      uint32_t *ymax, unsigned long long *amax, cudaStream_t st, int ks, bool pdl) {
  const bool apl = w.pl && w.planes == P && (NM == 1 || (w2.pl && w2.planes == P));
  if (ntok <= 64) {
    // the 64-token tile loads the precomputed planes too (measured on the 12B batch-64 decode
    // step: 3723 -> 3968 tok/s); SPB_TC_PLANES_SMALL=0 keeps its converter warps
    static int small = -1;
    if (small < 0) {
      const char *e = getenv("SPB_TC_PLANES_SMALL");
      small = (e && e[0] == '0') ? 0 : 1;
    }
    if (apl && small) return tc_launch_sn<P, NM, EPI, 1, true>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
    return tc_launch_sn<P, NM, EPI, 1>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
  }
  // precomputed planes (each matrix's own plane count equal to the launch's) for larger batches
  if (apl) {
    // two planes of one matrix: the two-CTA 128-token tile (SPB_TC_N128=0: the 256-token tile;
    // measured at M = 2048: 3840 x 3840 144.5 -> 132.3 us, 15360 x 3840 357.8 -> 314.4 us,
    // 3840 x 15360 unchanged)
    static int n128 = -1;
    if (n128 < 0) {
      const char *e = getenv("SPB_TC_N128");
      n128 = (e && e[0] == '0') ? 0 : 1;
    }
    if (P * NM == 2 && n128)
      return tc_launch_sn<P, NM, EPI, (P * NM == 2 ? 2 : 0), true>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks,
                                                                    pdl);
    return tc_launch_sn<P, NM, EPI, 0, true>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
  }
  return tc_launch_sn<P, NM, EPI, 0>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
}

template <int EPI>
cudaError_t tc_planes(int P, const DevQ4B &w, const DevQ4B &w2, const DevAct &act, int ntok, float *y, int ldy,
                      uint32_t *err, uint32_t *ymax, unsigned long long *amax, cudaStream_t st, int ks, bool pdl) {
  constexpr int NM = epi_pair(EPI) ? 2 : 1;
  switch (P) {
    case 2: return tc_launch<2, NM, EPI>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
    case 3: return tc_launch<3, NM, EPI>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
    default:
      if (NM == 1) return tc_launch<4, 1, EPI>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
      return cudaErrorNotSupported;
  }
}

}  // namespace

int gemm_tc_covers(const DevQ4B &w, const DevQ4B *w2, int epi, int ntok) {
  if (!tc_enabled() || !w.shift || w.planes < 2 || (w.cols % TC_BK) || w.cols > 16384 || ntok < 1) return 0;
  if (((uintptr_t)w.codes & 15) || ((uintptr_t)w.scales & 3)) return 0;
  int P = w.planes;
  if (epi_pair(epi)) {
    if (!w2 || !w2->shift || w2->planes < 2) return 0;
    if (((uintptr_t)w2->codes & 15) || ((uintptr_t)w2->scales & 3)) return 0;
    P = P > w2->planes ? P : w2->planes;
    if (P > 3) return 0;   // two matrices of four planes do not fit the tensor memory with a useful N
  }
  return P;
}

cudaError_t launch_q4b_planes(const DevQ4B &w, uint8_t *pl, cudaStream_t st) {
  if (!w.shift || w.planes < 2 || w.planes > 4 || (w.cols & 31) || w.rows <= 0 || ((uintptr_t)w.codes & 15))
    return cudaErrorInvalidValue;
  const long long n = (long long)w.rows * (w.cols >> 5);
  const dim3 grid((unsigned)((n + 255) / 256));
  switch (w.planes) {
    case 2: k_q4b_planes<2><<<grid, 256, 0, st>>>(w, pl); break;
    case 3: k_q4b_planes<3><<<grid, 256, 0, st>>>(w, pl); break;
    default: k_q4b_planes<4><<<grid, 256, 0, st>>>(w, pl); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_gemm_tc(const DevQ4B &w, const DevQ4B *w2, const DevAct &act, int ntok, float *y, int ldy, int epi,
                           uint32_t *err, cudaStream_t st, uint32_t *ymax, unsigned long long *amax, int ks, bool pdl) {
  const int P = gemm_tc_covers(w, w2, epi, ntok);
  if (!P) return cudaErrorNotSupported;
  if (ks < 1 || (w.cols / TC_BK) % ks) return cudaErrorInvalidValue;
  if (ks > 1 && epi != EPI_I64) return cudaErrorInvalidValue;
  const DevQ4B ww2 = w2 ? *w2 : w;
  switch (epi) {
    case EPI_STORE: return tc_planes<EPI_STORE>(P, w, ww2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
    case EPI_GELU_MUL: return tc_planes<EPI_GELU_MUL>(P, w, ww2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
    case EPI_SILU_MUL: return tc_planes<EPI_SILU_MUL>(P, w, ww2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
    case EPI_I64: return tc_planes<EPI_I64>(P, w, ww2, act, ntok, y, ldy, err, ymax, amax, st, ks, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace spb
