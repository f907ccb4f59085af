// spb_kernels.cu -- the byte-exact OK_Q4B forward kernels for sm_100a.
//
// Each kernel implements one rule of the exact numeric contract (the CPU checker
// under oracle/ states the same rules in C and the parity tests compare bytes):
//
//   k_gemv     OK_Q4B dequant-matvec/GEMM replacing matmul_arena's Q4B branch
//              (forward_dispatch.c:69-86). Each warp owns a group of rows; every lane
//              issues all of its 16-byte code vectors for the whole group before using any
//              (one 32-column scale block per vector), so a warp keeps ~4-8 KB in flight.
//              Nibbles are unpacked in registers (nibble ^ 8 = code + 8 in [0,15]; the
//              -8 * sum(x) correction is the per-block activation sum), multiplied with the
//              int8 activations by dp4a into an exact int32 block sum, scaled by the f16 block
//              scale taken as integer mantissa and shift, accumulated exactly in int64, and
//              reduced by warp shuffles; one rounding per output.
//   k_quant_*  activation quantizer sp_frob_quant1 over max|u| (frobenius_lift.c:27-35);
//              the max comes from the producing kernel (atomicMax of the f32 bits).
//   k_norm     residual add + exact RMSNorm island (exact_islands.c:60-79) + quantizer.
//   k_rope_kv  QK-norm island + CORDIC-RoPE onto the 2^16 score grid + KV-cache store
//              (replaces sp_rope_neox, forward_kernels.c:31-41, and the KV memcpy,
//              sp_session.c:433-436).
//   k_attn     session-resident KV-decode attention (sp_attn_head, forward_kernels.c:
//              59-81) with exact int64 scores, the softmax island's integer exponentials
//              (exact_islands.c:82-97) and an exact 128-bit V-sum. One thread-block cluster
//              per KV head splits the positions; each CTA streams its K then V slice through
//              a ring of shared-memory stages filled by TMA bulk copies; the cluster
//              exchanges the integer max and the partial sums through distributed shared
//              memory.
#include "spb_async.cuh"
#include "spb_device.cuh"
#include "spb_exact.cuh"
#include "spb_kernels.cuh"
#include "spb_spinor.cuh"

#include <algorithm>
#include <cooperative_groups.h>
#include <cuda_fp16.h>

namespace cg = cooperative_groups;

namespace spb {

// ------------------------------------------------------------------------------ launch helpers
// Programmatic dependent launch: every kernel of the schedule lets its successor be
// scheduled as soon as all of its own CTAs have started (griddepcontrol.launch_dependents),
// and waits for its predecessor's completion (griddepcontrol.wait, a hardware wait, not a
// spin) only right before it reads the predecessor's output. GEMVs issue their first weight
// loads before that wait, so the weight stream overlaps the previous kernel's tail. Without
// the launch attribute both instructions are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

static int pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_PDL");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on;
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  if (cluster > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------------------------ GEMV
constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

__device__ __forceinline__ uint4 ld_stream_u4(const uint8_t *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// warps sharing one row at batch 1 (KSF: forced, 0 = the default rule)
template <int NT, int NM, int NCH, int RPW, int KSF>
__host__ __device__ constexpr int gemv_ks() {
  return KSF ? KSF : (NT == 1 && RPW == 1 && NCH * NM >= 8) ? 2 : 1;
}

// NT token rows, epilogue EPI, NCH 16-byte vectors per lane per row (cols <= 1024*NCH),
// RPW rows per warp group, KSF warps per row (0: the default rule).
// ymax (nullable): per-token max |y| via atomicMax of f32 bits.
template <int NT, int EPI, int NCH, int RPW, int KSF = 0>
__global__ void __launch_bounds__(GEMV_THREADS)
k_gemv(DevQ4B w, DevQ4B w2, DevAct act, float *__restrict__ y, int ldy, uint32_t *err, uint32_t *ymax,
       unsigned long long *amax) {
  constexpr int NM = epi_pair(EPI) ? 2 : 1;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ float wmax[GEMV_WARPS][NT];
  const int K = w.cols, nblk = K >> 5, kw = K >> 2;
  int32_t *xw = reinterpret_cast<int32_t *>(smem_raw);                    // [NT][K/4]
  int32_t *xs = xw + NT * kw;                                               // [NT][nblk]
  double *dsc = reinterpret_cast<double *>(xs + ((NT * nblk + 1) & ~1));   // [NT]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // KS = 2 (single rows of >= 8 code vectors per lane: the FFN down projection, the gate/up
  // pair at K > 1024), or 4 where forced: the KS warps of a group take KS parts of a row's
  // 32-column blocks, so each holds 1/KS of the code vectors (fewer registers: more resident
  // warps); the other warps hand their exact int64 parts to the group's first warp through
  // shared memory under a named barrier of the group, and only first warps finish rows
  constexpr int KS = gemv_ks<NT, NM, NCH, RPW, KSF>();
  constexpr int NCHW = NCH / KS;   // code vectors per lane per row held by one warp
  const int half = warp % KS, pair = warp / KS;
  __shared__ int64_t ks_part[GEMV_WARPS / KS][KS][NM];
  const int rows = w.rows;
  const size_t rstride = (size_t)(K >> 1);
  const int ngroups = (rows + RPW - 1) / RPW;
  const int gstride = gridDim.x * (GEMV_WARPS / KS);
  int g = blockIdx.x * (GEMV_WARPS / KS) + pair;

  typedef uint4 CodeBuf[NM][RPW][NCHW];
  typedef uint32_t ScaleBuf[NM][RPW][NCHW];
  CodeBuf cw;
  ScaleBuf hw;
  auto load_into = [&](int grp, CodeBuf &cw, ScaleBuf &hw) {
#pragma unroll
    for (int r = 0; r < RPW; r++) {
      const int row = grp * RPW + r;
#pragma unroll
      for (int j = 0; j < NCHW; j++) {
        const int b = lane + 32 * (half * NCHW + j);
        if (row < rows && b < nblk) {
          cw[0][r][j] = ld_stream_u4(w.codes + (size_t)row * rstride + (size_t)b * 16);
          hw[0][r][j] = __ldg(w.scales + (size_t)row * nblk + b);
          if (NM == 2) {
            cw[NM - 1][r][j] = ld_stream_u4(w2.codes + (size_t)row * rstride + (size_t)b * 16);
            hw[NM - 1][r][j] = __ldg(w2.scales + (size_t)row * nblk + b);
          }
        } else {
          cw[0][r][j] = make_uint4(0u, 0u, 0u, 0u);
          hw[0][r][j] = 0u;
          if (NM == 2) { cw[NM - 1][r][j] = make_uint4(0u, 0u, 0u, 0u); hw[NM - 1][r][j] = 0u; }
        }
      }
    }
  };
  pdl_trigger();
  if (g < ngroups) load_into(g, cw, hw);   // weight loads are in flight while the predecessor drains
  pdl_wait();

  {
    const int4 *src = reinterpret_cast<const int4 *>(act.q);
    int4 *dst = reinterpret_cast<int4 *>(xw);
    for (int i = threadIdx.x; i < NT * (K >> 4); i += GEMV_THREADS) dst[i] = src[i];
    for (int i = threadIdx.x; i < NT * nblk; i += GEMV_THREADS) xs[i] = act.bsum[i];
    if (threadIdx.x < NT)
      dsc[threadIdx.x] = __dmul_rn(__ddiv_rn((double)act.scale[threadIdx.x], 127.0), 0x1p-24);
  }
  __syncthreads();

  float lmax[NT];
  unsigned long long lkey[NT];   // greedy argmax: orderable (value, ~row) key per token
#pragma unroll
  for (int t = 0; t < NT; t++) { lmax[t] = 0.0f; lkey[t] = 0ull; }
  // deferred epilogue: lane j keeps the j-th reduced output of this warp until 32 are
  // pending, then all lanes convert (and apply GELU/SiLU * up) in parallel
  int64_t pa = 0, pa2 = 0;
  int prow = -1, ptok = 0, npend = 0;
  auto flush = [&]() {
    if (EPI == EPI_I64) {
      if (prow >= 0) reinterpret_cast<int64_t *>(y)[(size_t)ptok * ldy + prow] = pa;
    } else if (prow >= 0) {
      const double d = dsc[ptok];
      float v = __double2float_rn(__dmul_rn(__ll2double_rn(pa), d));
      if (epi_pair(EPI)) {
        const float u = __double2float_rn(__dmul_rn(__ll2double_rn(pa2), d));
        if (!(fabsf(v) < 2048.0f)) { raise_err(err, ERR_ACT_RANGE); v = 0.0f; }
        const float gv = (EPI == EPI_GELU_MUL) ? gelu_exact(v) : silu_exact(v);
        v = __fmul_rn(gv, u);
      }
      y[(size_t)ptok * ldy + prow] = v;
      const unsigned long long key = argmax_key(v, prow);
#pragma unroll
      for (int t = 0; t < NT; t++)
        if (ptok == t) {
          lmax[t] = fmaxf(lmax[t], fabsf(v));
          if (key > lkey[t]) lkey[t] = key;
        }
    }
    prow = -1;
    npend = 0;
  };

  typedef int64_t AccBuf[NM][RPW][NT];
  // the group's exact int32 block sums, scaled and accumulated in int64
  auto dots = [&](const CodeBuf &cw, const ScaleBuf &hw, AccBuf &acc) {
#pragma unroll
    for (int m = 0; m < NM; m++)
#pragma unroll
      for (int r = 0; r < RPW; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[m][r][t] = 0;
#pragma unroll
    for (int j = 0; j < NCHW; j++) {
      const int b = lane + 32 * (half * NCHW + j);
      if (b < nblk) {
#pragma unroll
        for (int t = 0; t < NT; t++) {
          const int4 *xb = reinterpret_cast<const int4 *>(xw + t * kw + b * 8);
          const int4 x0 = xb[0], x1 = xb[1];
          const int32_t corr = -8 * xs[t * nblk + b];
          // the leaner block sum where instruction issue bounds the kernel (4 vectors per lane:
          // Q|K|V, O, gate/up, LM head); the down projection (16) is bound by latency, and
          // measured slower with it
#pragma unroll
          for (int m = 0; m < NM; m++)
#pragma unroll
            for (int r = 0; r < RPW; r++)
              scale_acc(acc[m][r][t], hw[m][r][j],
                        NCH <= 4 ? block_dot_corr(cw[m][r][j], x0, x1, corr) : block_dot(cw[m][r][j], x0, x1) + corr);
        }
      }
    }
  };
  // warp reduction (and the pair's exchange), then the deferred epilogue's bookkeeping
  auto finish = [&](int g0, AccBuf &acc) {
#pragma unroll
    for (int r = 0; r < RPW; r++) {
      const int row = g0 * RPW + r;
#pragma unroll
      for (int t = 0; t < NT; t++) {
#pragma unroll
        for (int m = 0; m < NM; m++) acc[m][r][t] = warp_sum_i64(acc[m][r][t]);
        if (KS > 1) {   // (KS > 1 only with RPW = 1, NT = 1)
#pragma unroll
          for (int m = 0; m < NM; m++)
            if (half > 0 && lane == 0) ks_part[pair][half][m] = acc[m][r][t];
          asm volatile("bar.sync %0, %1;" ::"r"(1 + pair), "n"(32 * KS) : "memory");
#pragma unroll
          for (int m = 0; m < NM; m++)
            if (half == 0)
#pragma unroll
              for (int h = 1; h < KS; h++) acc[m][r][t] += ks_part[pair][h][m];
          asm volatile("bar.sync %0, %1;" ::"r"(1 + pair), "n"(32 * KS) : "memory");   // the slots are free again
          if (half > 0) continue;
        }
        if (lane == npend && row < rows) {
          pa = acc[0][r][t];
          pa2 = acc[NM - 1][r][t];
          prow = row;
          ptok = t;
        }
        if (++npend == 32) flush();
      }
    }
  };

  for (; g < ngroups; g += gstride) {
    AccBuf acc;
    dots(cw, hw, acc);
    if (g + gstride < ngroups) load_into(g + gstride, cw, hw);   // next group's loads overlap the reduction
    finish(g, acc);
  }
  flush();
  if (ymax) {   // per-token max |y| of this CTA -> one atomic per token
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const float mt = warp_max_f(lmax[t]);   // every lane owns outputs after the deferred epilogue
      if (lane == 0) wmax[warp][t] = mt;
    }
    __syncthreads();
    if (threadIdx.x < NT) {
      float m = 0.0f;
      for (int i = 0; i < GEMV_WARPS; i++) m = fmaxf(m, wmax[i][threadIdx.x]);
      if (!(m <= 3.402823466e38f)) raise_err(err, ERR_ACT_RANGE);
      else atomicMax(ymax + threadIdx.x, __float_as_uint(m));
    }
  }
  if (amax) {   // per-token greedy argmax of this CTA -> one 64-bit atomic per token
    __shared__ unsigned long long wkey[GEMV_WARPS][NT];
#pragma unroll
    for (int t = 0; t < NT; t++) {
      unsigned long long k = lkey[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
        k = ok > k ? ok : k;
      }
      if (lane == 0) wkey[warp][t] = k;
    }
    __syncthreads();
    if (threadIdx.x < NT) {
      unsigned long long k = 0ull;
      for (int i = 0; i < GEMV_WARPS; i++) k = wkey[i][threadIdx.x] > k ? wkey[i][threadIdx.x] : k;
      atomicMax(amax + threadIdx.x, k);
    }
  }
}

template <int NT, int EPI, int NCH, int RPW, int KSF = 0>
static cudaError_t gemv_launch(const DevQ4B &w, const DevQ4B &w2, const DevAct &act, float *y, int ldy,
                               uint32_t *err, uint32_t *ymax, unsigned long long *amax, cudaStream_t st,
                               int grid_limit) {
  const int K = w.cols, nblk = K >> 5;
  const size_t smem = (size_t)NT * K + (size_t)(((NT * nblk + 1) & ~1)) * 4 + (size_t)NT * 8;
  auto kern = k_gemv<NT, EPI, NCH, RPW, KSF>;
  static int occ = 0, nsm = 0;
  static size_t occ_smem = 0;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  if (occ == 0 || occ_smem != smem) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, GEMV_THREADS, smem);
    if (occ < 1) occ = 1;
    occ_smem = smem;
  }
  const int ngroups = (w.rows + RPW - 1) / RPW;
  constexpr int NM = epi_pair(EPI) ? 2 : 1;
  constexpr int KS = gemv_ks<NT, NM, NCH, RPW, KSF>();   // as in k_gemv
  constexpr int GPC = GEMV_WARPS / KS;                                      // row groups per CTA round
  int grid = (ngroups + GPC - 1) / GPC;
  const int resident = nsm * occ;
  if (grid > resident) grid = resident;       // persistent: each warp walks several groups
  if (grid_limit > 0 && grid > grid_limit) grid = grid_limit;
  return launch_k(kern, dim3(grid), dim3(GEMV_THREADS), smem, st, 1, w, w2, act, y, ldy, err, ymax, amax);
}

// one row per warp group: the most warps (and CTAs) per matrix, and the fewest registers (64 for
// a single matrix at K <= 4096, 79 for the gate/up pair, against ~126 at 2-4 rows), so 4 CTAs
// instead of 2 fit an SM. Measured per decode step at the 12B shape: 257-259 vs 251-255 tok/s.
template <int NT, int EPI, int NCH>
static cudaError_t gemv_rpw(const DevQ4B &w, const DevQ4B &w2, const DevAct &act, float *y, int ldy,
                            uint32_t *err, uint32_t *ymax, unsigned long long *amax, cudaStream_t st,
                            int grid_limit) {
  return gemv_launch<NT, EPI, NCH, 1>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
}

// warps per row at batch 1, per matrix kind (SPB_GEMV_KS1 single matrices of <= 4 vectors per
// lane, default 1; SPB_GEMV_KSG gate/up pairs of <= 4, default 2; SPB_GEMV_KS16 single matrices
// of 9-16, default 4): fewer code registers per warp, more resident warps
static int gemv_ks_env(const char *name, int dflt) {
  const char *e = getenv(name);
  const int v = e ? atoi(e) : dflt;
  return (v == 1 || v == 2 || v == 4 || v == 8) ? v : dflt;
}

template <int NT, int EPI>
static cudaError_t gemv_nch(const DevQ4B &w, const DevQ4B &w2, const DevAct &act, float *y, int ldy,
                            uint32_t *err, uint32_t *ymax, unsigned long long *amax, cudaStream_t st,
                            int grid_limit) {
  static int ks1 = 0, ksg = 0, ks16 = 0;
  if (!ks1) {
    ks1 = gemv_ks_env("SPB_GEMV_KS1", 1);
    ksg = gemv_ks_env("SPB_GEMV_KSG", 2);
    ks16 = gemv_ks_env("SPB_GEMV_KS16", 4);
  }
  const int per_lane = ((w.cols >> 5) + 31) / 32;
  if (per_lane <= 1) return gemv_rpw<NT, EPI, 1>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
  if (per_lane <= 4) {
    if (NT == 1 && !epi_pair(EPI) && ks1 == 2)
      return gemv_launch<NT, EPI, 4, 1, 2>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
    if (NT == 1 && epi_pair(EPI) && ksg == 4)
      return gemv_launch<NT, EPI, 4, 1, 4>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
    return gemv_rpw<NT, EPI, 4>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
  }
  if (per_lane <= 16) {
    if (NT == 1 && !epi_pair(EPI) && ks16 == 4)
      return gemv_launch<NT, EPI, 16, 1, 4>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
    if (NT == 1 && !epi_pair(EPI) && ks16 == 8)
      return gemv_launch<NT, EPI, 16, 1, 8>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
    return gemv_rpw<NT, EPI, 16>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
  }
  return cudaErrorInvalidValue;
}

template <int EPI>
static cudaError_t gemv_nt(const DevQ4B &w, const DevQ4B &w2, const DevAct &act, int ntok, float *y, int ldy,
                           uint32_t *err, uint32_t *ymax, unsigned long long *amax, cudaStream_t st,
                           int grid_limit) {
  switch (ntok) {
    case 1: return gemv_nch<1, EPI>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
    case 2: return gemv_nch<2, EPI>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
    case 4: return gemv_nch<4, EPI>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
    case 8: return gemv_nch<8, EPI>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
    case 16: return gemv_nch<16, EPI>(w, w2, act, y, ldy, err, ymax, amax, st, grid_limit);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------------------ token-batch GEMM
// 16..64 token rows at a time on the tensor cores (mma.sync m16n8k32, int8 x int8 -> int32):
// one MMA per 32-column block gives the exact block sums of 16 tokens x 8 weight rows at once.
// The weight operand is the code nibble shifted to the top of its byte (16 c, exact in int8),
// so the block sum comes out times 16 and an exact arithmetic shift recovers it. Each block
// sum is then scaled by its f16 block scale as integer mantissa and shift and accumulated in
// int64 in registers, the same arithmetic as the GEMV, so the results are identical. The
// activation rows are stored in the GEMV's permuted column order (per 8 columns: even, then
// odd); the fragment layout of m16n8k32 maps k positions 0-3 of a thread to one 4-byte group,
// which is exactly one word of low or high nibbles of the code block.
constexpr int GEMM_THREADS = 128;   // per token group: 4 warps x 8 weight rows
constexpr int GEMM_ROWS = 32;       // weight rows per CTA
constexpr int GEMM_KC = 512;        // columns staged per step
constexpr int GEMM_AP = GEMM_KC + 16;   // padded activation row (bank-conflict-free fragment loads)
constexpr int GEMM_WP = GEMM_KC / 2 + 16;   // padded code row

__device__ __forceinline__ void mma_s8(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int32_t (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// f16 block scale as (signed mantissa, 2^shift), value = m * pw * 2^-24
__device__ __forceinline__ void scale_parts(uint32_t h, int32_t &m, int32_t &pw) {
  const uint32_t e = (h >> 10) & 31u;
  m = (int32_t)(e ? ((h & 1023u) | 1024u) : (h & 1023u));
  if (h & 0x8000u) m = -m;
  pw = 1 << (e ? e - 1 : 0);
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
  // src-size 0 zero-fills the 16 destination bytes (rows past the matrix or the token count)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

template <int MT, int NM>
struct GemmSmem {
  static constexpr int A = MT * 16 * GEMM_AP;                 // activation rows
  static constexpr int W = NM * GEMM_ROWS * GEMM_WP;          // code rows
  static constexpr int S = NM * GEMM_ROWS * (GEMM_KC / 32) * 2;   // block scales
  static constexpr int STAGE = A + W + S;
  static constexpr int KS = NM * (GEMM_KC / 32) * GEMM_ROWS * 4;   // decoded scales [m][block][row]
  static constexpr int TOTAL = 2 * STAGE + KS;                // double buffered staging, one table
};

// One block scale decoded for the GEMM's inner loop: SMALL, the integer k = value * 2^24
// (|k| < 2^31); otherwise the signed mantissa in the low 16 bits and the exponent shift above.
template <bool SMALL>
__device__ __forceinline__ int32_t scale_word(uint32_t h) {
  int32_t m, pw;
  scale_parts(h, m, pw);
  if (SMALL) return m * pw;
  const uint32_t e = (h >> 10) & 31u;
  return (int32_t)(((e ? e - 1 : 0) << 16) | ((uint32_t)m & 0xFFFFu));
}

// SMALL: every block scale of w (and w2) is below 128, so k = scale * 2^24 fits in int32 and
// the 16x block sums accumulate as sum(16 isum * k) < 2^59 with one widening multiply-add per
// value; the exact shift by 4 comes once at the end.
// TH token groups of MT 16-token tiles: warp w takes weight rows 8 (w % 4) .. + 8 of the CTA's
// 32 and token tiles MT (w / 4) .. + MT, so the CTA's 128 TH threads cover MT TH tiles.
template <int MT, int TH, int EPI, bool SMALL>
__global__ void __launch_bounds__(GEMM_THREADS * TH, 2)
k_gemm(DevQ4B w, DevQ4B w2, DevAct act, int ntok, float *__restrict__ y, int ldy, uint32_t *err, uint32_t *ymax,
       unsigned long long *amax, int ks) {
  constexpr int NM = epi_pair(EPI) ? 2 : 1;
  constexpr int M = MT * TH * 16;
  constexpr int NTHR = GEMM_THREADS * TH;
  using SM = GemmSmem<MT * TH, NM>;
  extern __shared__ __align__(16) uint8_t gsm[];
  __shared__ float tmax[M];
  __shared__ unsigned long long tkey[M];
  __shared__ double dsc[M];
  const int tid = threadIdx.x, lane = tid & 31, g = lane >> 2, tig = lane & 3;
  const int warp = (tid >> 5) & 3, mt0 = (tid >> 7) * MT;   // weight-row group, first token tile
  // ks > 1 (EPI_I64 only): work item (row block, K part) writes its part's int64 partial sums
  // to y + part * ntok * ldy; K / ks is a multiple of 256
  const int K = w.cols, rows = w.rows, kper = K / ks;
  const int nch = (kper + GEMM_KC - 1) / GEMM_KC;
  const int nrb = (rows + GEMM_ROWS - 1) / GEMM_ROWS;
  int32_t *KS = reinterpret_cast<int32_t *>(gsm + 2 * SM::STAGE);
  pdl_trigger();
  pdl_wait();
  for (int t = tid; t < M; t += NTHR) {
    dsc[t] = t < ntok ? __dmul_rn(__ddiv_rn((double)act.scale[t], 127.0), 0x1p-24) : 0.0;
    tmax[t] = 0.0f;
    tkey[t] = 0ull;
  }
  // stage the chunk at column k0 (ending at kend) of row block row0 into buffer `buf`
  // (asynchronous copies, one commit group)
  auto stage = [&](int buf, int row0, int k0, int kend) {
    uint8_t *base = gsm + buf * SM::STAGE;
    int8_t *A = reinterpret_cast<int8_t *>(base);
    uint8_t *W = base + SM::A;
    uint8_t *S = W + SM::W;
    // chunk widths are powers of two of at least 256 columns (K % 256 == 0), so every split
    // below is a shift
    const int kc = min(GEMM_KC, kend - k0);
    const int l16 = 31 - __clz(kc >> 4);   // log2(kc / 16)
    for (int i = tid; i < (M << l16); i += NTHR) {
      const int t = i >> l16, c = (i & ((1 << l16) - 1)) << 4;
      const bool ok = t < ntok;
      cp_async16(A + t * GEMM_AP + c, act.q + (size_t)(ok ? t : 0) * K + k0 + c, ok);
    }
#pragma unroll
    for (int m = 0; m < NM; m++) {
      const DevQ4B &q = m ? w2 : w;
      for (int i = tid; i < (GEMM_ROWS << (l16 - 1)); i += NTHR) {   // 16 code bytes per block
        const int r = i >> (l16 - 1), b = i & ((1 << (l16 - 1)) - 1);
        const bool ok = row0 + r < rows;
        cp_async16(W + (m * GEMM_ROWS + r) * GEMM_WP + b * 16,
                   q.codes + (size_t)(ok ? row0 + r : 0) * (K >> 1) + (size_t)((k0 >> 5) + b) * 16, ok);
      }
      const uint8_t *sc = reinterpret_cast<const uint8_t *>(q.scales);
      for (int i = tid; i < (GEMM_ROWS << (l16 - 4)); i += NTHR) {   // 8 block scales per 16 bytes
        const int r = i >> (l16 - 4), j = i & ((1 << (l16 - 4)) - 1);
        const bool ok = row0 + r < rows;
        cp_async16(S + ((m * GEMM_ROWS + r) * (GEMM_KC / 32)) * 2 + j * 16,
                   sc + (size_t)(ok ? row0 + r : 0) * (K >> 4) + (k0 >> 4) + j * 16, ok);
      }
    }
    cp_async_commit();
  };
  for (int wi = blockIdx.x; wi < nrb * ks; wi += gridDim.x) {
    const int rb = wi % nrb, part = wi / nrb;
    const int row0 = rb * GEMM_ROWS, kb0 = part * kper, kend = kb0 + kper;
    int64_t acc[NM][MT][4];
#pragma unroll
    for (int m = 0; m < NM; m++)
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[m][mt][i] = 0;
    __syncthreads();   // both buffers are free
    stage(0, row0, kb0, kend);
    for (int ci = 0; ci < nch; ci++) {
      if (ci + 1 < nch) stage((ci + 1) & 1, row0, kb0 + (ci + 1) * GEMM_KC, kend);
      else cp_async_commit();   // an empty group keeps the wait count uniform
      cp_async_wait_prev();
      __syncthreads();
      const uint8_t *base = gsm + (ci & 1) * SM::STAGE;
      const int8_t *A = reinterpret_cast<const int8_t *>(base);
      const uint8_t *W = base + SM::A;
      const int kc = min(GEMM_KC, kend - (kb0 + ci * GEMM_KC));
      {   // decode the chunk's block scales once: KS[m][block][row]
        const uint16_t *S = reinterpret_cast<const uint16_t *>(W + SM::W);
        for (int i = tid; i < NM * GEMM_ROWS * (GEMM_KC / 32); i += NTHR) {
          const int r = i & (GEMM_ROWS - 1), kb = (i / GEMM_ROWS) % (GEMM_KC / 32), m = i / (GEMM_ROWS * (GEMM_KC / 32));
          KS[i] = scale_word<SMALL>(S[(m * GEMM_ROWS + r) * (GEMM_KC / 32) + kb]);
        }
        __syncthreads();
      }
#pragma unroll 4
      for (int kb = 0; kb < (kc >> 5); kb++) {
        // A fragments: one ldmatrix.x4 per 16-token tile; lane l addresses row l % 8 of
        // matrix l / 8 (rows +8 for matrices 1 and 3, columns +16 for matrices 2 and 3)
        uint32_t af[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
          const int8_t *ab = A + ((mt0 + mt) * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * GEMM_AP + kb * 32 + (lane >> 4) * 16;
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                       : "=r"(af[mt][0]), "=r"(af[mt][1]), "=r"(af[mt][2]), "=r"(af[mt][3])
                       : "r"((uint32_t)__cvta_generic_to_shared(ab)));
        }
#pragma unroll
        for (int m = 0; m < NM; m++) {
          const uint32_t *wr = reinterpret_cast<const uint32_t *>(W + (m * GEMM_ROWS + warp * 8 + g) * GEMM_WP + kb * 16);
          const uint32_t w0 = wr[tig >> 1], w1 = wr[2 + (tig >> 1)];
          const uint32_t b0 = (tig & 1) ? (w0 & 0xF0F0F0F0u) : ((w0 << 4) & 0xF0F0F0F0u);
          const uint32_t b1 = (tig & 1) ? (w1 & 0xF0F0F0F0u) : ((w1 << 4) & 0xF0F0F0F0u);
          const int2 kw = *reinterpret_cast<const int2 *>(KS + (m * (GEMM_KC / 32) + kb) * GEMM_ROWS + warp * 8 + tig * 2);
          if (SMALL) {
            const int32_t k0 = kw.x, k1 = kw.y;   // |k| < 2^31
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
              int32_t c[4];
              mma_s8(af[mt], b0, b1, c);
              acc[m][mt][0] += (int64_t)c[0] * (int64_t)k0;   // 16 x (token g,   row 2 tig)
              acc[m][mt][1] += (int64_t)c[1] * (int64_t)k1;   // 16 x (token g,   row 2 tig + 1)
              acc[m][mt][2] += (int64_t)c[2] * (int64_t)k0;   // 16 x (token g+8, row 2 tig)
              acc[m][mt][3] += (int64_t)c[3] * (int64_t)k1;   // 16 x (token g+8, row 2 tig + 1)
            }
          } else {
            const int32_t m0 = (int16_t)kw.x, p0 = 1 << (kw.x >> 16);
            const int32_t m1 = (int16_t)kw.y, p1 = 1 << (kw.y >> 16);
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
              int32_t c[4];
              mma_s8(af[mt], b0, b1, c);
              acc[m][mt][0] += (int64_t)((c[0] >> 4) * m0) * (int64_t)p0;   // token g,   row 2 tig
              acc[m][mt][1] += (int64_t)((c[1] >> 4) * m1) * (int64_t)p1;   // token g,   row 2 tig + 1
              acc[m][mt][2] += (int64_t)((c[2] >> 4) * m0) * (int64_t)p0;   // token g+8, row 2 tig
              acc[m][mt][3] += (int64_t)((c[3] >> 4) * m1) * (int64_t)p1;   // token g+8, row 2 tig + 1
            }
          }
        }
      }
      __syncthreads();   // buffer ci & 1 may be refilled by the next stage
    }
    if (SMALL) {   // the sums were accumulated 16x: every term is a multiple of 16
#pragma unroll
      for (int m = 0; m < NM; m++)
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int i = 0; i < 4; i++) acc[m][mt][i] >>= 4;
    }
    // epilogue: (token, row) of each accumulator
#pragma unroll
    for (int mt = 0; mt < MT; mt++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int t = (mt0 + mt) * 16 + g + (i >= 2 ? 8 : 0);
        const int row = row0 + warp * 8 + tig * 2 + (i & 1);
        if (t >= ntok || row >= rows) continue;
        if (EPI == EPI_I64) {
          reinterpret_cast<int64_t *>(y)[((size_t)part * ntok + t) * ldy + row] = acc[0][mt][i];
          continue;
        }
        float v = __double2float_rn(__dmul_rn(__ll2double_rn(acc[0][mt][i]), dsc[t]));
        if (epi_pair(EPI)) {
          const float u = __double2float_rn(__dmul_rn(__ll2double_rn(acc[NM - 1][mt][i]), dsc[t]));
          if (!(fabsf(v) < 2048.0f)) { raise_err(err, ERR_ACT_RANGE); v = 0.0f; }
          v = __fmul_rn(EPI == EPI_GELU_MUL ? gelu_exact(v) : silu_exact(v), u);
        }
        y[(size_t)t * ldy + row] = v;
        if (ymax) atomicMax(reinterpret_cast<unsigned int *>(&tmax[t]), __float_as_uint(fabsf(v)));
        if (amax) atomicMax(&tkey[t], argmax_key(v, row));
      }
    }
  }
  __syncthreads();
  for (int t = tid; t < ntok; t += NTHR) {
    if (ymax) {
      const float m = tmax[t];
      if (!(m <= 3.402823466e38f)) raise_err(err, ERR_ACT_RANGE);
      else if (m > 0.0f) atomicMax(ymax + t, __float_as_uint(m));
    }
    if (amax && tkey[t]) atomicMax(amax + t, tkey[t]);
  }
}

template <int MT, int TH, int EPI, bool SMALL>
static cudaError_t gemm_launch(const DevQ4B &w, const DevQ4B &w2, const DevAct &act, int ntok, float *y, int ldy,
                               uint32_t *err, uint32_t *ymax, unsigned long long *amax, cudaStream_t st, int ks) {
  constexpr int NM = epi_pair(EPI) ? 2 : 1;
  const size_t smem = GemmSmem<MT * TH, NM>::TOTAL;
  auto kern = k_gemm<MT, TH, EPI, SMALL>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  int dev = 0, nsm = 148, occ = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, GEMM_THREADS * TH, smem);
  const int nrb = (w.rows + GEMM_ROWS - 1) / GEMM_ROWS;
  const int grid = std::min(nrb * ks, nsm * std::max(occ, 1));
  return launch_k(kern, dim3(grid), dim3(GEMM_THREADS * TH), smem, st, 1, w, w2, act, ntok, y, ldy, err, ymax,
                  amax, ks);
}

// 16-token tiles per warp for full 64-token pieces: 2 (two token groups, 8 warps; the default)
// or 4 (one group of 4 warps, SPB_GEMM_SPLIT=0)
static bool gemm_split() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_GEMM_SPLIT");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}

template <int EPI>
static cudaError_t gemm_mt(const DevQ4B &w, const DevQ4B &w2, const DevAct &act, int ntok, float *y, int ldy,
                           uint32_t *err, uint32_t *ymax, unsigned long long *amax, cudaStream_t st, int ks = 1) {
  const bool small = w.small && (!epi_pair(EPI) || w2.small);
#define SPB_GEMM_MT(MTV, THV)                                                                            \
  return small ? gemm_launch<MTV, THV, EPI, true>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks) \
               : gemm_launch<MTV, THV, EPI, false>(w, w2, act, ntok, y, ldy, err, ymax, amax, st, ks)
  switch ((ntok + 15) / 16) {   // 16-token tiles: split across two warp groups when even
    case 1: SPB_GEMM_MT(1, 1);
    case 2: SPB_GEMM_MT(1, 2);
    case 3: SPB_GEMM_MT(3, 1);
    default:
      if (gemm_split()) SPB_GEMM_MT(2, 2);
      SPB_GEMM_MT(4, 1);
  }
#undef SPB_GEMM_MT
}

// SPB_SPLITK=0 keeps every GEMM whole (comparisons; results are identical)
static bool splitk_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_SPLITK");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}

// token rows from which a batch runs the tcgen05 GEMM (SPB_TC_MIN; SPB_TC=0 never): 16, where its
// 64-token tile already beats the mma.sync GEMM (64-session batch 3367 -> 3724 tok/s)
static int tc_min_tokens() {
  static int n = -1;
  if (n < 0) {
    const char *e = getenv("SPB_TC_MIN");
    n = e ? atoi(e) : 16;
    if (n < 1) n = 1;
  }
  return n;
}

// SPB_GEMM=0 keeps token batches on the dp4a k_gemv (comparisons; results are identical)
static bool gemm_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_GEMM");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}

cudaError_t launch_gemv(const DevQ4B &w, const DevQ4B *w2, const DevAct &act, int ntok, float *y, int ldy,
                        int epi, uint32_t *err, cudaStream_t st, int grid_limit, uint32_t *ymax,
                        unsigned long long *amax, int64_t *ws, size_t ws_elems) {
  if ((w.cols & 31) || w.cols <= 0 || w.rows <= 0 || w.cols > 16384) return cudaErrorInvalidValue;
  if (epi < EPI_STORE || epi > EPI_I64) return cudaErrorInvalidValue;
  if (epi_pair(epi) && (!w2 || w2->rows != w.rows || w2->cols != w.cols)) return cudaErrorInvalidValue;
  if (epi == EPI_I64 && (ymax || amax)) return cudaErrorInvalidValue;
  const size_t yb = (size_t)epi_bytes(epi);   // y row offsets below are in elements of this size
  // large token batches: the tcgen05 GEMM over digit planes, K split into parts when the
  // (row tile x token tile) grid would leave most SMs idle
  if (ntok >= tc_min_tokens() && grid_limit == 0 && gemm_enabled() && gemm_tc_covers(w, w2, epi, ntok)) {
    const int P = gemm_tc_covers(w, w2, epi, ntok);
    const int PM = P * (epi_pair(epi) ? 2 : 1);   // token tile of the GEMM's launch (TcShape::N)
    const int N = ntok <= 64 ? 64 : PM == 2 ? 256 : PM == 3 ? 160 : PM == 4 ? 128 : 80;
    const long tiles = (long)((ntok + N - 1) / N) * ((w.rows + 127) / 128);
    const int nk = w.cols / 128;
    int ks = 1;
    if (epi == EPI_STORE && !ymax && !amax && ws && splitk_enabled())
      while (ks < 4 && tiles * ks * 2 <= 148 && nk % (ks * 2) == 0 && nk / (ks * 2) >= 8 &&
             (size_t)(ks * 2) * ntok * w.rows <= ws_elems)
        ks *= 2;
    if (ks > 1) {
      cudaError_t e = launch_gemm_tc(w, w2, act, ntok, reinterpret_cast<float *>(ws), w.rows, EPI_I64, err, st, nullptr,
                                     nullptr, ks, pdl_enabled() != 0);
      if (e == cudaSuccess)
        e = launch_scale_i64(ws, act.scale, ntok, w.rows, y, ldy, st, ks, (size_t)ntok * w.rows);
      return e;
    }
    return launch_gemm_tc(w, w2, act, ntok, y, ldy, epi, err, st, ymax, amax, 1, pdl_enabled() != 0);
  }
  // token batches (and row counts the k_gemv templates do not cover): the tensor-core GEMM
  const bool odd = ntok > 1 && (ntok & (ntok - 1)) != 0;
  if ((ntok >= 16 || odd) && grid_limit == 0 && (w.cols & 255) == 0 && (gemm_enabled() || odd)) {
    const DevQ4B ww2 = w2 ? *w2 : w;
    // split-K: matrices with fewer 32-row blocks than SMs run their two K halves as separate
    // CTAs into the workspace; the exact int64 halves are summed and scaled afterwards
    const int nrb = (w.rows + GEMM_ROWS - 1) / GEMM_ROWS;
    const bool split = epi == EPI_STORE && !ymax && !amax && ws && splitk_enabled() && nrb < 148 &&
                       (w.cols % 512) == 0 && (size_t)2 * 64 * w.rows <= ws_elems;
    for (int t0 = 0; t0 < ntok; t0 += 64) {
      const int n = std::min(64, ntok - t0);
      const DevAct a2{act.q + (size_t)t0 * w.cols, act.bsum + (size_t)t0 * (w.cols >> 5), act.scale + t0};
      float *y2 = reinterpret_cast<float *>(reinterpret_cast<char *>(y) + (size_t)t0 * ldy * yb);
      uint32_t *ym = ymax ? ymax + t0 : nullptr;
      unsigned long long *am = amax ? amax + t0 : nullptr;
      cudaError_t e;
      if (split) {
        e = gemm_mt<EPI_I64>(w, ww2, a2, n, reinterpret_cast<float *>(ws), w.rows, err, nullptr, nullptr, st, 2);
        if (e == cudaSuccess) e = launch_scale_i64(ws, a2.scale, n, w.rows, y2, ldy, st, 2, (size_t)n * w.rows);
        if (e != cudaSuccess) return e;
        continue;
      }
      switch (epi) {
        case EPI_STORE: e = gemm_mt<EPI_STORE>(w, ww2, a2, n, y2, ldy, err, ym, am, st); break;
        case EPI_GELU_MUL: e = gemm_mt<EPI_GELU_MUL>(w, ww2, a2, n, y2, ldy, err, ym, am, st); break;
        case EPI_SILU_MUL: e = gemm_mt<EPI_SILU_MUL>(w, ww2, a2, n, y2, ldy, err, ym, am, st); break;
        default: e = gemm_mt<EPI_I64>(w, ww2, a2, n, y2, ldy, err, ym, am, st); break;
      }
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  // the staged activations of all rows must fit shared memory: split the token rows
  const size_t per_tok = (size_t)w.cols + (size_t)(w.cols >> 5) * 4 + 8;
  if (ntok > 1 && per_tok * ntok > 160 * 1024) {
    const int h = ntok / 2;
    const DevAct a2{act.q + (size_t)h * w.cols, act.bsum + (size_t)h * (w.cols >> 5), act.scale + h};
    cudaError_t e = launch_gemv(w, w2, act, h, y, ldy, epi, err, st, grid_limit, ymax, amax, ws, ws_elems);
    if (e != cudaSuccess) return e;
    return launch_gemv(w, w2, a2, ntok - h,
                       reinterpret_cast<float *>(reinterpret_cast<char *>(y) + (size_t)h * ldy * yb), ldy, epi, err,
                       st, grid_limit, ymax ? ymax + h : nullptr, amax ? amax + h : nullptr, ws, ws_elems);
  }
  // row counts the k_gemv templates do not cover (K not a multiple of 256, so no GEMM: e.g. a
  // tensor-parallel rank's slice of the attention output or FFN down projection): pieces of
  // 16, 8, 4, 2, 1 rows
  if (ntok > 16 || (ntok & (ntok - 1))) {
    for (int t0 = 0; t0 < ntok;) {
      int n = 16;
      while (n > ntok - t0) n >>= 1;
      const DevAct a2{act.q + (size_t)t0 * w.cols, act.bsum + (size_t)t0 * (w.cols >> 5), act.scale + t0};
      cudaError_t e = launch_gemv(w, w2, a2, n, reinterpret_cast<float *>(reinterpret_cast<char *>(y) + (size_t)t0 * ldy * yb),
                                  ldy, epi, err, st, grid_limit, ymax ? ymax + t0 : nullptr, amax ? amax + t0 : nullptr,
                                  ws, ws_elems);
      if (e != cudaSuccess) return e;
      t0 += n;
    }
    return cudaSuccess;
  }
  const DevQ4B ww2 = w2 ? *w2 : w;
  switch (epi) {
    case EPI_STORE: return gemv_nt<EPI_STORE>(w, ww2, act, ntok, y, ldy, err, ymax, amax, st, grid_limit);
    case EPI_GELU_MUL: return gemv_nt<EPI_GELU_MUL>(w, ww2, act, ntok, y, ldy, err, ymax, amax, st, grid_limit);
    case EPI_SILU_MUL: return gemv_nt<EPI_SILU_MUL>(w, ww2, act, ntok, y, ldy, err, ymax, amax, st, grid_limit);
    case EPI_I64: return gemv_nt<EPI_I64>(w, ww2, act, ntok, y, ldy, err, ymax, amax, st, grid_limit);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------------------ quantizer
constexpr int QUANT_THREADS = 256;

__device__ float block_max(float v, float *red) {
  v = warp_max_f(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float m = lane < nw ? red[lane] : 0.0f;
    m = warp_max_f(m);
    if (lane == 0) red[32] = m;
  }
  __syncthreads();
  return red[32];
}

// quantize one row of K (multiple of 32) values with a known scale s, one warp per block
__device__ __forceinline__ void quant_blocks(const float *src, int K, float s, int8_t *q, int32_t *bsum,
                                             int b0, int bstride) {
  const int lane = threadIdx.x & 31;
  for (int b = b0; b < (K >> 5); b += bstride) {
    const int32_t v = quant1(src[(b << 5) + lane], s);
    q[(b << 5) + perm_pos(lane)] = (int8_t)v;
    const int32_t sum = warp_sum_i32(v);
    if (lane == 0) bsum[b] = sum;
  }
}

// a whole row in one CTA: max, then quantize (used inside k_norm)
__device__ void quant_row(const float *src, int K, int8_t *q, int32_t *bsum, float *scale_out, float *red,
                          uint32_t *err) {
  float m = 0.0f;
  bool bad = false;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    const float a = fabsf(src[i]);
    if (!(a <= 3.402823466e38f)) bad = true;
    else m = fmaxf(m, a);
  }
  if (bad) raise_err(err, ERR_ACT_RANGE);
  const float s = block_max(m, red);
  quant_blocks(src, K, s, q, bsum, threadIdx.x >> 5, blockDim.x >> 5);
  if (threadIdx.x == 0) *scale_out = s;
}

// per-row max |u| into slot[t] (f32 bits), for callers without a producing kernel
__global__ void __launch_bounds__(1024) k_rowmax(const float *u, int ldu, int K, uint32_t *slot, uint32_t *err) {
  __shared__ float red[33];
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  float m = 0.0f;
  bool bad = false;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    const float a = fabsf(u[(size_t)t * ldu + i]);
    if (!(a <= 3.402823466e38f)) bad = true;
    else m = fmaxf(m, a);
  }
  if (bad) raise_err(err, ERR_ACT_RANGE);
  m = block_max(m, red);
  if (threadIdx.x == 0) slot[t] = __float_as_uint(m);
}

// grid (ceil(nblk/8), ntok): warp w of CTA x quantizes block 8x+w with the row's max
__global__ void __launch_bounds__(QUANT_THREADS)
k_quant_blocks(const float *u, int ldu, int K, const uint32_t *maxslot, DevAct act) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.y;
  const float s = __uint_as_float(maxslot[t]);
  const int b = blockIdx.x * (QUANT_THREADS / 32) + (threadIdx.x >> 5);
  if (b < (K >> 5))
    quant_blocks(u + (size_t)t * ldu, K, s, act.q + (size_t)t * K, act.bsum + (size_t)t * (K >> 5), b, 1 << 30);
  if (blockIdx.x == 0 && threadIdx.x == 0) act.scale[t] = s;
}

cudaError_t launch_quant(const float *u, int ldu, int K, int ntok, const DevAct &act, const uint32_t *maxslot,
                         uint32_t *err, cudaStream_t st) {
  if (K & 31) return cudaErrorInvalidValue;
  if (!maxslot) {   // no producer max: compute it into act.scale (as f32 bits) first
    uint32_t *slot = reinterpret_cast<uint32_t *>(act.scale);
    cudaError_t e = launch_k(k_rowmax, dim3(ntok), dim3(1024), 0, st, 1, u, ldu, K, slot, err);
    if (e != cudaSuccess) return e;
    maxslot = slot;
  }
  dim3 grid(((K >> 5) + QUANT_THREADS / 32 - 1) / (QUANT_THREADS / 32), ntok);
  return launch_k(k_quant_blocks, grid, dim3(QUANT_THREADS), 0, st, 1, u, ldu, K, maxslot, act);
}

// ------------------------------------------------------------------------------ RMSNorm
// block-wide 128-bit sum of non-negative int64 terms
__device__ acc128 block_sum128(acc128 v, acc128 *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc128 r;
    r.lo = __shfl_xor_sync(0xffffffffu, v.lo, o);
    r.hi = __shfl_xor_sync(0xffffffffu, v.hi, o);
    acc128_add(v, r);
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    acc128 s = lane < nw ? red[lane] : acc128{0ull, 0ll};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc128 r;
      r.lo = __shfl_xor_sync(0xffffffffu, s.lo, o);
      r.hi = __shfl_xor_sync(0xffffffffu, s.hi, o);
      acc128_add(s, r);
    }
    if (lane == 0) red[32] = s;
  }
  __syncthreads();
  return red[32];
}

// island pieces: per-thread partial sum of (q16(x))^2, the inverse rms from the exact total,
// and one output y = (float)((double)(int64)(xi * inv * wi) * 2^-52) (exact_islands.c:60-79)
__device__ __forceinline__ acc128 rms_partial(const float *src, int n, uint32_t *err) {
  acc128 ss{0ull, 0ll};
  bool bad = false;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float x = src[i];
    if (!(fabsf(x) < 32768.0f)) { bad = true; continue; }
    const int64_t xi = q16_round(x);
    acc128_add(ss, xi * xi);
  }
  if (bad) raise_err(err, ERR_NORM_RANGE);
  return ss;
}

// Exact RMSNorm island over n values in one CTA (any thread count); dst must not alias src.
__device__ void block_rmsnorm(const float *src, const float *w, int n, float *dst, acc128 *red,
                              uint64_t *inv_sh, uint32_t *err) {
  const acc128 tot = block_sum128(rms_partial(src, n, err), red);
  if (threadIdx.x == 0) *inv_sh = rms_inv(tot, n, err);
  __syncthreads();
  const uint64_t inv = *inv_sh;
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = rms_apply(src[i], w[i], inv, err);
  __syncthreads();
}

// ---- norm block as one NORM_CL-CTA cluster of 1024 threads per token row: rank r owns
// columns [r E/NCL, (r+1) E/NCL), one or two per thread. Each reduction (sums of squares, the
// quantizer's max) is finished by warp 0 and pushed into every rank's shared memory, so one
// cluster barrier per reduction and no remote loads.
constexpr int NORM_CL = 4;
constexpr int NORM_CL_THREADS = 1024;
constexpr int NORM_REG_THREADS = 1024;   // the one-CTA form below

// per-thread sum of q16(v)^2 over the thread's columns j * 1024 + tid < E (1024-thread blocks)
template <int EPT>
__device__ __forceinline__ acc128 sq_partial(const float (&v)[EPT], int E, uint32_t *err) {
  acc128 ss{0ull, 0ll};
  bool bad = false;
#pragma unroll
  for (int j = 0; j < EPT; j++) {
    if (j * 1024 + (int)threadIdx.x >= E) continue;
    if (!(fabsf(v[j]) < 32768.0f)) { bad = true; continue; }
    const int64_t xi = q16_round(v[j]);
    acc128_add(ss, xi * xi);
  }
  if (bad) raise_err(err, ERR_NORM_RANGE);
  return ss;
}

__device__ __forceinline__ void cluster_wait_started() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// this CTA's 128-bit partial (warp 0, lane 0 holds it on return; the others hold garbage)
__device__ __forceinline__ acc128 block_partial128(acc128 v, acc128 *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc128 r;
    r.lo = __shfl_xor_sync(0xffffffffu, v.lo, o);
    r.hi = __shfl_xor_sync(0xffffffffu, v.hi, o);
    acc128_add(v, r);
  }
  if (lane == 0) red[warp] = v;
  __syncthreads();
  acc128 s{0ull, 0ll};
  if (warp == 0) {
    s = lane < nw ? red[lane] : acc128{0ull, 0ll};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc128 r;
      r.lo = __shfl_xor_sync(0xffffffffu, s.lo, o);
      r.hi = __shfl_xor_sync(0xffffffffu, s.hi, o);
      acc128_add(s, r);
    }
  }
  return s;
}

template <int EPT>
__global__ void __launch_bounds__(NORM_CL_THREADS)
k_norm_cl(float *x, const float *add, const float *add_w, const float *out_w, int E, DevAct act, float *nx_out,
          uint32_t *err, uint32_t *zero_slot) {
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ acc128 red[32];
  __shared__ acc128 sq_in[2][NORM_CL];   // [reduction][source rank]
  __shared__ float mx_in[NORM_CL];
  __shared__ float fred[33];
  __shared__ uint64_t inv_sh[2];
  const int rank = (int)cluster.block_rank();
  const int t = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ns = E / NORM_CL, off = rank * ns;
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");   // waited on before the first push
  float aw[EPT], ow[EPT];
#pragma unroll
  for (int j = 0; j < EPT; j++) {
    const int c = j * NORM_CL_THREADS + tid;
    aw[j] = (add_w && c < ns) ? add_w[off + c] : 0.0f;
    ow[j] = c < ns ? out_w[off + c] : 0.0f;
  }
  pdl_trigger();
  pdl_wait();
  if (zero_slot && rank == 0 && tid == 0) zero_slot[t] = 0u;
  float *xr = x + (size_t)t * E + off;
  float v[EPT];
#pragma unroll
  for (int j = 0; j < EPT; j++) {
    const int c = j * NORM_CL_THREADS + tid;
    v[j] = c < ns ? xr[c] : 0.0f;
  }
  bool started = false;
  // the cluster-wide inverse rms of the sum of squares over this rank's values
  auto cluster_inv = [&](const float(&vals)[EPT], int k) -> uint64_t {
    const acc128 p = block_partial128(sq_partial<EPT>(vals, ns, err), red);
    if (!started) { cluster_wait_started(); started = true; }
    if (warp == 0) {   // lane r pushes the partial into rank r
      acc128 b;
      b.lo = __shfl_sync(0xffffffffu, p.lo, 0);
      b.hi = __shfl_sync(0xffffffffu, p.hi, 0);
      if (lane < NORM_CL) *cluster.map_shared_rank(&sq_in[k][rank], lane) = b;
    }
    cluster.sync();
    if (warp == 0 && lane == 0) {
      acc128 tot = sq_in[k][0];
      for (int r = 1; r < NORM_CL; r++) acc128_add(tot, sq_in[k][r]);
      inv_sh[k] = rms_inv(tot, E, err);
    }
    __syncthreads();
    return inv_sh[k];
  };
  if (add) {
    const float *ar = add + (size_t)t * E + off;
    float u[EPT];
#pragma unroll
    for (int j = 0; j < EPT; j++) {
      const int c = j * NORM_CL_THREADS + tid;
      u[j] = c < ns ? ar[c] : 0.0f;
    }
    if (add_w) {   // sandwich post-norm of `add`, then the residual add
      const uint64_t inv = cluster_inv(u, 0);
#pragma unroll
      for (int j = 0; j < EPT; j++)
        if (j * NORM_CL_THREADS + tid < ns) u[j] = rms_apply(u[j], aw[j], inv, err);
    }
#pragma unroll
    for (int j = 0; j < EPT; j++) {
      const int c = j * NORM_CL_THREADS + tid;
      if (c < ns) {
        v[j] = __fadd_rn(v[j], u[j]);
        xr[c] = v[j];
      }
    }
  }
  const uint64_t inv = cluster_inv(v, 1);
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < EPT; j++) {
    const int c = j * NORM_CL_THREADS + tid;
    if (c < ns) {
      v[j] = rms_apply(v[j], ow[j], inv, err);
      m = fmaxf(m, fabsf(v[j]));
      if (nx_out) nx_out[(size_t)t * E + off + c] = v[j];
    }
  }
  m = block_max(m, fred);   // every thread holds this CTA's max
  if (tid < NORM_CL) *cluster.map_shared_rank(&mx_in[rank], tid) = m;
  cluster.sync();   // the last cluster access: no rank touches another's memory after it
  float s = mx_in[0];
#pragma unroll
  for (int r = 1; r < NORM_CL; r++) s = fmaxf(s, mx_in[r]);
  if (rank == 0 && tid == 0) act.scale[t] = s;
  int8_t *q = act.q + (size_t)t * E + off;
  int32_t *bs = act.bsum + (size_t)t * (E >> 5) + (off >> 5);
#pragma unroll
  for (int j = 0; j < EPT; j++) {
    const int c = j * NORM_CL_THREADS + tid;
    if (c < ns) {   // ns % 32 == 0: a warp's 32 columns are all in or all out
      const int32_t qv = quant1(v[j], s);
      q[(c & ~31) + perm_pos(lane)] = (int8_t)qv;
      const int32_t sum = warp_sum_i32(qv);
      if (lane == 0) bs[c >> 5] = sum;
    }
  }
}

// single-CTA fallback for any width (rows past the register-resident forms)
constexpr int NORM_THREADS = 1024;

__global__ void __launch_bounds__(NORM_THREADS)
k_norm(float *x, const float *add, const float *add_w, const float *out_w, int E, DevAct act, float *nx_out,
       uint32_t *err, uint32_t *zero_slot) {
  extern __shared__ __align__(16) float nsm[];
  float *tbuf = nsm;          // [E]
  float *nbuf = nsm + E;      // [E]
  __shared__ acc128 red[33];
  __shared__ uint64_t inv_sh;
  __shared__ float fred[33];
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  if (zero_slot && threadIdx.x == 0) zero_slot[t] = 0u;
  float *xr = x + (size_t)t * E;
  if (add) {
    const float *ar = add + (size_t)t * E;
    if (add_w) {
      block_rmsnorm(ar, add_w, E, tbuf, red, &inv_sh, err);
      for (int i = threadIdx.x; i < E; i += blockDim.x) xr[i] = __fadd_rn(xr[i], tbuf[i]);
    } else {
      for (int i = threadIdx.x; i < E; i += blockDim.x) xr[i] = __fadd_rn(xr[i], ar[i]);
    }
    __syncthreads();
  }
  block_rmsnorm(xr, out_w, E, nbuf, red, &inv_sh, err);
  if (nx_out)
    for (int i = threadIdx.x; i < E; i += blockDim.x) nx_out[(size_t)t * E + i] = nbuf[i];
  quant_row(nbuf, E, act.q + (size_t)t * E, act.bsum + (size_t)t * (E >> 5), act.scale + t, fred, err);
}

// ---- norm block as one CTA per token row with the row in registers (E <= 1024 EPT): thread i
// owns columns i + 1024 j, so warp w's 32 columns of slot j are quantizer block 32 j + w. Every
// thread takes the inverse rms from the broadcast 128-bit total itself; the norm weights are
// read before the dependency wait.

// inverse rms of a block's 128-bit sum of squares: warp 0 finishes the sum and lane 0
// computes the island's quotient and square root once, broadcast through shared memory
__device__ __forceinline__ uint64_t block_rms_inv(acc128 v, int n, acc128 *red, uint64_t *inv_sh, uint32_t *err) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc128 r;
    r.lo = __shfl_xor_sync(0xffffffffu, v.lo, o);
    r.hi = __shfl_xor_sync(0xffffffffu, v.hi, o);
    acc128_add(v, r);
  }
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    acc128 s = lane < nw ? red[lane] : acc128{0ull, 0ll};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc128 r;
      r.lo = __shfl_xor_sync(0xffffffffu, s.lo, o);
      r.hi = __shfl_xor_sync(0xffffffffu, s.hi, o);
      acc128_add(s, r);
    }
    if (lane == 0) *inv_sh = rms_inv(s, n, err);
  }
  __syncthreads();
  return *inv_sh;
}

template <int EPT>
__global__ void __launch_bounds__(NORM_REG_THREADS)
k_norm_reg(float *x, const float *add, const float *add_w, const float *out_w, int E, DevAct act, float *nx_out,
           uint32_t *err, uint32_t *zero_slot) {
  __shared__ acc128 red[32];
  __shared__ float fred[33];
  __shared__ uint64_t inv_sh[2];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  float aw[EPT], ow[EPT];
#pragma unroll
  for (int j = 0; j < EPT; j++) {
    const int c = j * NORM_REG_THREADS + tid;
    aw[j] = (add_w && c < E) ? add_w[c] : 0.0f;
    ow[j] = c < E ? out_w[c] : 0.0f;
  }
  pdl_trigger();
  pdl_wait();
  if (zero_slot && tid == 0) zero_slot[t] = 0u;
  float *xr = x + (size_t)t * E;
  float v[EPT];
#pragma unroll
  for (int j = 0; j < EPT; j++) {
    const int c = j * NORM_REG_THREADS + tid;
    v[j] = c < E ? xr[c] : 0.0f;
  }
  if (add) {
    const float *ar = add + (size_t)t * E;
    float u[EPT];
#pragma unroll
    for (int j = 0; j < EPT; j++) {
      const int c = j * NORM_REG_THREADS + tid;
      u[j] = c < E ? ar[c] : 0.0f;
    }
    if (add_w) {   // sandwich post-norm of `add`, then the residual add
      const uint64_t inv = block_rms_inv(sq_partial<EPT>(u, E, err), E, red, &inv_sh[0], err);
#pragma unroll
      for (int j = 0; j < EPT; j++)
        if (j * NORM_REG_THREADS + tid < E) u[j] = rms_apply(u[j], aw[j], inv, err);
    }
#pragma unroll
    for (int j = 0; j < EPT; j++) {
      const int c = j * NORM_REG_THREADS + tid;
      if (c < E) {
        v[j] = __fadd_rn(v[j], u[j]);
        xr[c] = v[j];
      }
    }
  }
  const uint64_t inv = block_rms_inv(sq_partial<EPT>(v, E, err), E, red, &inv_sh[1], err);
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < EPT; j++) {
    const int c = j * NORM_REG_THREADS + tid;
    if (c < E) {
      v[j] = rms_apply(v[j], ow[j], inv, err);
      m = fmaxf(m, fabsf(v[j]));
      if (nx_out) nx_out[(size_t)t * E + c] = v[j];
    }
  }
  const float s = block_max(m, fred);
  if (tid == 0) act.scale[t] = s;
  int8_t *q = act.q + (size_t)t * E;
  int32_t *bs = act.bsum + (size_t)t * (E >> 5);
#pragma unroll
  for (int j = 0; j < EPT; j++) {
    const int c = j * NORM_REG_THREADS + tid;
    if (c < E) {   // E % 32 == 0: a warp's 32 columns are all in or all out
      const int32_t qv = quant1(v[j], s);
      q[(c & ~31) + perm_pos(lane)] = (int8_t)qv;
      const int32_t sum = warp_sum_i32(qv);
      if (lane == 0) bs[c >> 5] = sum;
    }
  }
}

// SPB_NORM_1CTA=1 keeps every row on one CTA (k_norm_reg) instead of a 4-CTA cluster
static bool norm_one_cta() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_NORM_1CTA");
    on = (e && e[0] == '1') ? 1 : 0;
  }
  return on != 0;
}

cudaError_t launch_norm(float *x, const float *add, const float *add_w, const float *out_w, int E, int ntok,
                        const DevAct &act, float *nx_out, uint32_t *err, cudaStream_t st, uint32_t *zero_slot) {
  if (E & 31) return cudaErrorInvalidValue;
  if (E % (NORM_CL * 32) == 0 && E <= NORM_CL * 2 * NORM_CL_THREADS && !norm_one_cta()) {
    if (E <= NORM_CL * NORM_CL_THREADS)
      return launch_k(k_norm_cl<1>, dim3(NORM_CL, ntok), dim3(NORM_CL_THREADS), 0, st, NORM_CL, x, add, add_w,
                      out_w, E, act, nx_out, err, zero_slot);
    return launch_k(k_norm_cl<2>, dim3(NORM_CL, ntok), dim3(NORM_CL_THREADS), 0, st, NORM_CL, x, add, add_w, out_w,
                    E, act, nx_out, err, zero_slot);
  }
  if (E <= 8 * NORM_REG_THREADS) {
#define SPB_NORM_REG(EPTV)                                                                                     \
  return launch_k(k_norm_reg<EPTV>, dim3(ntok), dim3(NORM_REG_THREADS), 0, st, 1, x, add, add_w, out_w, E, act, \
                  nx_out, err, zero_slot)
    if (E <= NORM_REG_THREADS) SPB_NORM_REG(1);
    if (E <= 2 * NORM_REG_THREADS) SPB_NORM_REG(2);
    if (E <= 4 * NORM_REG_THREADS) SPB_NORM_REG(4);
    SPB_NORM_REG(8);
#undef SPB_NORM_REG
  }
  const size_t smem = (size_t)2 * E * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_norm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_k(k_norm, dim3(ntok), dim3(NORM_THREADS), smem, st, 1, x, add, add_w, out_w, E, act, nx_out, err,
                  zero_slot);
}

// ------------------------------------------------------------------------------ RoPE + KV
__global__ void k_rope_kv(RopeArgs a) {
  extern __shared__ __align__(16) float rsm[];
  float *vbuf = rsm;            // [HD] head values
  float *nbuf = rsm + a.HD;     // [HD] normed
  __shared__ acc128 red[33];
  __shared__ uint64_t inv_sh;
  pdl_trigger();
  pdl_wait();
  const int head = blockIdx.x, t = blockIdx.y;
  const int HD = a.HD, half = HD >> 1, QD = a.NH * HD, KVD = a.NKV * HD;
  const float *row = a.qkv + (size_t)t * (QD + 2 * KVD);
  int p;
  KvPages kv;
  if (a.rows) {   // row t of a multi-session batch: its own session's position and cache
    const BatchRow br = a.rows[t];
    p = br.pos;
    kv = br.kv;
  } else {
    p = a.pos_dev[0] + t;
    kv = a.kv;
  }
  const int i = threadIdx.x;   // pair index, blockDim.x == half
  if (a.zero_slot && head == 0 && i == 0) a.zero_slot[t] = 0u;
  // Spinor-block cache: K and V rows are stored as 63-byte blocks (CRC tables, per-warp block
  // images and the rotated K row after the two f32 rows in shared memory)
  const bool spin = kv.rb > 0 && head >= a.NH;
  uint8_t *tab = reinterpret_cast<uint8_t *>(rsm + 2 * HD);
  uint8_t *imgs = tab + 1024;
  int32_t *krow = reinterpret_cast<int32_t *>(imgs + 64 * ((half + 31) / 32));
  if (spin) {
    crc8_tables_build(tab, threadIdx.x, blockDim.x);
    __syncthreads();
  }
  if (head >= a.NH + a.NKV && spin) {   // V head: Spinor blocks of the float projections
    const int g = head - a.NH - a.NKV;
    spin_encode_row(row + QD + KVD + g * HD, false, HD,
                    reinterpret_cast<uint8_t *>(kv.v) + kv_spin_off(kv, a.NKV, a.layer, g, p), nullptr, imgs, tab,
                    a.err);
    return;
  }
  if (head >= a.NH + a.NKV) {  // V head: quantize to the 2^16 grid
    const int g = head - a.NH - a.NKV;
    const float *src = row + QD + KVD + g * HD;
    int32_t *dst = kv.v + kv_elem(kv, a.NL, a.NKV, HD, a.layer, g, p);
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const float v = src[i + r * half];
      int32_t q = 0;
      if (!(fabsf(v) < 16384.0f)) raise_err(a.err, ERR_V_RANGE);
      else q = __float2int_rn(__fmul_rn(v, 65536.0f));
      dst[i + r * half] = q;
    }
    return;
  }
  const bool is_q = head < a.NH;
  const int hh = is_q ? head : head - a.NH;
  const float *src = row + (is_q ? hh * HD : QD + hh * HD);
  vbuf[i] = src[i];
  vbuf[i + half] = src[i + half];
  __syncthreads();
  const float *nw = is_q ? a.q_norm : a.k_norm;
  const float *vals = vbuf;
  if (nw) {
    block_rmsnorm(vbuf, nw, HD, nbuf, red, &inv_sh, a.err);
    vals = nbuf;
  }
  const uint64_t phase = (uint64_t)(int64_t)p * a.W[i];
  int32_t oa, ob;
  cordic_rotate(vals[i], vals[i + half], phase, a.T, a.gain, oa, ob, a.err);
  if (spin) {   // K head: Spinor blocks of the rotated grid row
    krow[i] = oa;
    krow[i + half] = ob;
    __syncthreads();
    spin_encode_row(krow, true, HD, reinterpret_cast<uint8_t *>(kv.k) + kv_spin_off(kv, a.NKV, a.layer, hh, p),
                    nullptr, imgs, tab, a.err);
    return;
  }
  int32_t *dst = is_q ? a.qi + (size_t)t * QD + hh * HD : kv.k + kv_elem(kv, a.NL, a.NKV, HD, a.layer, hh, p);
  dst[i] = oa;
  dst[i + half] = ob;
}

cudaError_t launch_rope_kv(const RopeArgs &a, cudaStream_t st) {
  if (a.HD & 1 || a.HD / 2 > 1024) return cudaErrorInvalidValue;
  if (a.kv.rb > 0 && (a.kv.ptab || a.HD < 64 || a.kv.rb != spin_row_bytes(a.HD))) return cudaErrorInvalidValue;
  dim3 grid(a.NH + 2 * a.NKV, a.ntok);
  // Spinor caches (or batch rows with one among them): + CRC tables, a 64-byte block image per
  // warp, the rotated K row
  const size_t smem = 2 * a.HD * sizeof(float) +
                      (a.kv.rb > 0 || (a.rows && a.rows_spin) ? 1024 + 64 * (size_t)((a.HD / 2 + 31) / 32) + (size_t)a.HD * 4 : 0);
  return launch_k(k_rope_kv, grid, dim3(a.HD / 2), smem, st, 1, a);
}

// ------------------------------------------------------------------------------ attention
constexpr int ATTN_THREADS = 256;
constexpr int ATTN_STAGES = 3;
constexpr int ATTN_SPAN = 1024;   // positions one CTA takes before the row is split further

// positions per ring stage (32 KB of int32 K or V per stage)
template <int HD>
struct AttnSub {
  static constexpr int SUB = 8192 / HD;
};

// CL CTAs (a cluster when CL > 1) split the positions of one (token row, KV head): CL = 16 for
// one long context, 1 when the rows and heads alone fill the GPU.
template <int HD, int G>
__global__ void __launch_bounds__(ATTN_THREADS, 2) k_attn(AttnArgs a, int cmax, int CL) {
  cg::cluster_group cluster = cg::this_cluster();
  constexpr int SUB = AttnSub<HD>::SUB;
  constexpr int V4 = HD / 32;                  // int4 columns per lane in the score dot
  constexpr bool QREG = G * V4 <= 16;          // q slices held in registers (<= 64 words)
  constexpr int GROUPS = ATTN_THREADS / HD;    // position groups in the V-sum
  const int DPR = HD / CL;                     // head dims each rank finalizes
  extern __shared__ __align__(128) uint8_t asm_raw[];
  int32_t *ring = reinterpret_cast<int32_t *>(asm_raw);            // [STAGES][SUB*HD]
  int32_t *qs = ring + ATTN_STAGES * SUB * HD;                       // [G][HD]
  const bool fused = a.qkv != nullptr;
  int32_t *kvn = qs + G * HD;                                        // fused: [2][HD] new K, V rows
  int32_t *sc = kvn + (fused ? 2 * HD : 0);                          // [G][cmax] scores, then e
  // [GROUPS][G][HD] this CTA's V-sums (absent when one thread per head dim pushes them
  // straight from registers), then with CL > 1 the [CL][G][HD/CL] V-sums pushed by each rank
  const bool direct = GROUPS == 1 && CL > 1;
  acc128 *nacc = reinterpret_cast<acc128 *>(sc + ((G * cmax + 3) & ~3));
  acc128 *gat = nacc + (direct ? 0 : GROUPS * G * HD);
  __shared__ __align__(8) uint64_t full[ATTN_STAGES];
  __shared__ int32_t mx_loc[G];
  __shared__ int64_t s_loc[G];
  __shared__ int32_t mx_all[G];
  __shared__ int32_t mx_in[16][G];        // CL > 1: each rank's score maximum, pushed by that rank
  __shared__ int64_t s_in[16][G];         // CL > 1: each rank's exponential sum
  __shared__ float fred[33];
  __shared__ uint64_t ginv[9];                  // fused: inverse rms of each rotated head (G + 1 <= 9)

  const int rank = CL > 1 ? (int)cluster.block_rank() : 0;
  // the partials are pushed into the owning rank's shared memory (no remote loads): this
  // arrival, waited on before the first push, guarantees every rank of the cluster has started
  if (CL > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  const int g = blockIdx.y, t = blockIdx.z;
  const int QD = a.NH * HD;
  int p;
  KvPages kv;
  if (a.rows) {   // row t of a multi-session batch: its own session's position and cache
    const BatchRow br = a.rows[t];
    p = br.pos;
    kv = br.kv;
  } else {
    p = a.pos_dev[0] + t;
    kv = a.kv;
  }
  const int s0 = (a.win >= 0 && p - a.win + 1 > 0) ? p - a.win + 1 : 0;
  const int n = p - s0 + 1;
  // positions [c0, c1) of this rank: an equal split, except that with the fused QK-norm + RoPE
  // the last rank (which also normalises, rotates and stores the new K and V rows) takes own_pct
  // percent of an equal share and the others split the rest
  int c0, c1;
  if (a.qkv && CL > 1 && a.own_pct < 100) {
    const int c = (n + CL - 1) / CL;
    const int own = max(1, min(n, c * a.own_pct / 100));
    const int rest = n - own, cr = (rest + CL - 2) / (CL - 1);
    if (rank < CL - 1) {
      c0 = s0 + rank * cr;
      c1 = min(c0 + cr, s0 + rest);
    } else {
      c0 = s0 + rest;
      c1 = p + 1;
    }
  } else {
    const int c = (n + CL - 1) / CL;
    c0 = s0 + rank * c;
    c1 = min(c0 + c, p + 1);
  }
  const int cn = max(c1 - c0, 0);
  const int nsub = (cn + SUB - 1) / SUB;
  const int total = 2 * nsub;                 // K slices, then V slices
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // this (layer, KV head)'s K or V row of position q
  auto kv_at = [&](bool isv, int q) -> int32_t * {
    return (isv ? kv.v : kv.k) + kv_elem(kv, a.NL, a.NKV, HD, a.layer, g, q);
  };
  // Spinor-block cache (kv.rb > 0): a slice's blocks are copied (16-byte aligned around them)
  // into the tail of its ring stage, SOFF bytes in, and decoded into the stage's int32 rows;
  // the first half of the rows lands below SOFF, so only the second half waits on a barrier
  const bool spin = kv.rb > 0;
  using SG = SpinGeom<HD>;
  constexpr int SOFF = SUB * HD * 4 - ((SUB * SG::RB + 32 + 15) & ~15);
  static_assert(SOFF >= SUB / 2 * HD * 4, "the decoded first half stays below the copied blocks");
  auto spin_src = [&](bool isv, int q) -> const uint8_t * {
    return reinterpret_cast<const uint8_t *>(isv ? kv.v : kv.k) + kv_spin_off(kv, a.NKV, a.layer, g, q);
  };
  // CRC tables and per-(row, chunk) decode multipliers after the exchange buffers
  uint8_t *spin_tab = reinterpret_cast<uint8_t *>(gat + (CL > 1 ? G * HD : 0));
  float *smul = reinterpret_cast<float *>(spin_tab + 1024);

  // slice i -> ring stage i % STAGES: one bulk copy, or two where the slice crosses a page
  // boundary (a slice of SUB <= 128 positions spans at most two pages of >= 128)
  auto issue = [&](int i) {
    const bool isv = i >= nsub;
    const int j = isv ? i - nsub : i;
    const int pos = c0 + j * SUB;
    const int len = min(SUB, c1 - pos);
    const uint32_t bytes = (uint32_t)len * HD * 4;
    uint64_t *bar = &full[i % ATTN_STAGES];
    int32_t *dst = ring + (i % ATTN_STAGES) * SUB * HD;
    if (spin) {
      const uintptr_t A = (uintptr_t)spin_src(isv, pos), A0 = A & ~(uintptr_t)15;
      const uintptr_t A1 = (A + (uintptr_t)len * SG::RB + 15) & ~(uintptr_t)15;
      mbar_arrive_expect_tx(bar, (uint32_t)(A1 - A0));
      bulk_g2s(reinterpret_cast<uint8_t *>(dst) + SOFF, reinterpret_cast<const void *>(A0), (uint32_t)(A1 - A0), bar);
      return;
    }
    mbar_arrive_expect_tx(bar, bytes);
    const int first = min(len, kv.pg - pos % kv.pg);
    bulk_g2s(dst, kv_at(isv, pos), (uint32_t)first * HD * 4, bar);
    if (first < len) bulk_g2s(dst + (size_t)first * HD, kv_at(isv, pos + first), (uint32_t)(len - first) * HD * 4, bar);
  };

  // decode slice i's blocks (landed in its stage) into the stage's int32 rows [0, len)
  auto spin_decode = [&](int i, int32_t *buf, int len) {
    const bool isv = i >= nsub;
    const int pos = c0 + (isv ? i - nsub : i) * SUB;
    const uint8_t *src = reinterpret_cast<const uint8_t *>(buf) + SOFF + ((uintptr_t)spin_src(isv, pos) & 15);
    for (int x = threadIdx.x; x < len * SG::NB; x += ATTN_THREADS)
      smul[x] = spin_block_mul(src + (x / SG::NB) * SG::RB + (x % SG::NB) * SPIN_BYTES);
    __syncthreads();
    constexpr int NV = SUB / 2 * HD / ATTN_THREADS, RSTEP = ATTN_THREADS / HD;
    const int d = threadIdx.x % HD, r0 = threadIdx.x / HD;
    int cb, ci;
    SG::locate(d, cb, ci);
    const int bo = cb * SPIN_BYTES + 7 + (17 * ci) % SPIN_BODY;
#pragma unroll
    for (int k = 0; k < NV; k++) {
      const int r = r0 + k * RSTEP;
      if (r < len) buf[r * HD + d] = spin_grid(src[r * SG::RB + bo], smul[r * SG::NB + cb]);
    }
    int32_t hv[NV];
#pragma unroll
    for (int k = 0; k < NV; k++) {
      const int r = SUB / 2 + r0 + k * RSTEP;
      hv[k] = r < len ? spin_grid(src[r * SG::RB + bo], smul[r * SG::NB + cb]) : 0;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NV; k++) {
      const int r = SUB / 2 + r0 + k * RSTEP;
      if (r < len) buf[r * HD + d] = hv[k];
    }
    __syncthreads();
  };

  // K/V rows before this launch's first new position were written by earlier steps, so a
  // CTA whose slice ends before it can start its copies before the predecessor finishes; fused,
  // the new position's rows are patched into shared memory, so every CTA starts early
  const bool own = fused && cn > 0 && c1 == p + 1;   // this CTA's slice ends at the new position
  const bool early = fused || c1 <= (a.rows ? p : a.pos_dev[0]);
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < ATTN_STAGES; s++) mbar_init(&full[s], 1);
    mbar_init_fence();
    if (early)
      for (int i = 0; i < min(ATTN_STAGES, total); i++) issue(i);
  }
  pdl_wait();
  if (!fused) {
    for (int i = threadIdx.x; i < G * HD; i += ATTN_THREADS) qs[i] = a.qi[(size_t)t * QD + (size_t)g * G * HD + i];
  } else {
    // QK-norm + CORDIC-RoPE of the G query heads (and, for the owner, the new K row): item x =
    // pair x % HALF of rotated head x / HALF, thread tid takes items tid, tid + 256, ...; every
    // head's sum of squares is reduced in the same pass (a warp's items share one head), the
    // inverse rms of the heads is found by one thread each, then every item is normalised and
    // rotated -- the same island steps as k_rope_kv, in one pass however many heads rotate
    constexpr int HALF = HD / 2, WPH = HALF / 32;   // warps per head in one item round
    constexpr int NIT = ((G + 1) * HALF + ATTN_THREADS - 1) / ATTN_THREADS;
    constexpr int NW = ATTN_THREADS / 32;
    static_assert(NIT * NW * (int)sizeof(acc128) <= G * HD * 4, "norm partials fit the q staging");
    acc128 *part = reinterpret_cast<acc128 *>(qs);   // [NIT][NW] per-warp sums, before qs is written
    const int KVD = a.NKV * HD;
    const float *row = a.qkv + (size_t)t * (QD + 2 * KVD);
    const int nrot = G + (own ? 1 : 0), nitems = nrot * HALF;
    float x0[NIT], x1[NIT];
#pragma unroll
    for (int k = 0; k < NIT; k++) {
      const int item = threadIdx.x + k * ATTN_THREADS, j = item / HALF, i = item % HALF;
      const bool act = item < nitems;
      const float *src = row + (j == G ? QD + g * HD : (g * G + j) * HD);
      x0[k] = act ? src[i] : 0.0f;
      x1[k] = act ? src[i + HALF] : 0.0f;
      if (a.q_norm && k * ATTN_THREADS < nitems) {   // (warp-uniform: whole rounds of items)
        acc128 ss{0ull, 0ll};
        bool bad = false;
        if (act) {
          if (!(fabsf(x0[k]) < 32768.0f)) bad = true;
          else { const int64_t xi = q16_round(x0[k]); acc128_add(ss, xi * xi); }
          if (!(fabsf(x1[k]) < 32768.0f)) bad = true;
          else { const int64_t xi = q16_round(x1[k]); acc128_add(ss, xi * xi); }
        }
        if (bad) raise_err(a.err, ERR_NORM_RANGE);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          acc128 r;
          r.lo = __shfl_xor_sync(0xffffffffu, ss.lo, o);
          r.hi = __shfl_xor_sync(0xffffffffu, ss.hi, o);
          acc128_add(ss, r);
        }
        if (lane == 0) part[k * NW + warp] = ss;
      }
    }
    if (a.q_norm) {
      __syncthreads();
      if (threadIdx.x < nrot) {   // head h's items h HALF .. + HALF: round (h HALF) / 256, WPH warps
        const int h = threadIdx.x, k = (h * HALF) / ATTN_THREADS, w0 = ((h * HALF) % ATTN_THREADS) / 32;
        acc128 tot = part[k * NW + w0];
        for (int w = 1; w < WPH; w++) acc128_add(tot, part[k * NW + w0 + w]);
        ginv[h] = rms_inv(tot, HD, a.err);
      }
      __syncthreads();   // (the partials in qs are read: qs may be written from here)
    }
#pragma unroll
    for (int k = 0; k < NIT; k++) {
      const int item = threadIdx.x + k * ATTN_THREADS, j = item / HALF, i = item % HALF;
      if (item >= nitems) continue;
      const bool is_k = j == G;
      float v0 = x0[k], v1 = x1[k];
      if (a.q_norm) {
        const float *nw = is_k ? a.k_norm : a.q_norm;
        const uint64_t inv = ginv[j];
        v0 = rms_apply(v0, nw[i], inv, a.err);
        v1 = rms_apply(v1, nw[i + HALF], inv, a.err);
      }
      int32_t oa, ob;
      cordic_rotate(v0, v1, (uint64_t)(int64_t)p * a.W[i], a.T, a.gain, oa, ob, a.err);
      int32_t *dst = is_k ? kvn : qs + j * HD;
      dst[i] = oa;
      dst[i + HALF] = ob;
      if (is_k && !spin) {
        int32_t *kr = kv_at(false, p);
        kr[i] = oa;
        kr[i + HALF] = ob;
      }
    }
    if (own && spin) {   // the new K and V rows as Spinor blocks; kvn takes their decoded grids
      __syncthreads();
      crc8_tables_build(spin_tab, threadIdx.x, ATTN_THREADS);
      __syncthreads();
      uint8_t *imgs = reinterpret_cast<uint8_t *>(smul);
      spin_encode_row(kvn, true, HD, const_cast<uint8_t *>(spin_src(false, p)), kvn, imgs, spin_tab, a.err);
      spin_encode_row(row + QD + KVD + g * HD, false, HD, const_cast<uint8_t *>(spin_src(true, p)), kvn + HD, imgs,
                      spin_tab, a.err);
    } else if (own) {   // the new V row on the 2^16 grid
      const float *src = row + QD + KVD + g * HD;
      int32_t *vr = kv_at(true, p);
      for (int d = threadIdx.x; d < HD; d += ATTN_THREADS) {
        const float v = src[d];
        int32_t q = 0;
        if (!(fabsf(v) < 16384.0f)) raise_err(a.err, ERR_V_RANGE);
        else q = __float2int_rn(__fmul_rn(v, 65536.0f));
        kvn[HD + d] = q;
        vr[d] = q;
      }
    }
  }
  if (threadIdx.x < G) { mx_loc[threadIdx.x] = INT32_MIN; s_loc[threadIdx.x] = 0; }
  __syncthreads();
  if (threadIdx.x == 0 && !early)
    for (int i = 0; i < min(ATTN_STAGES, total); i++) issue(i);

  // ---- phase 1: exact scores of this CTA's positions -> the 2^14 grid. Eight lanes share a
  // position (lane j takes the int4 columns 4j + 32v), so a warp scores four positions per pass
  // with a three-level butterfly, and lane h of each group finishes head h. |q|, |k| < 2^24
  // keep every partial sum below 2^56.
  const int gq = lane >> 3, gj = lane & 7;
  int4 qr[QREG ? G * V4 : 1];
  if (QREG) {
#pragma unroll
    for (int h = 0; h < G; h++)
#pragma unroll
      for (int v = 0; v < V4; v++) qr[h * V4 + v] = *reinterpret_cast<const int4 *>(qs + h * HD + 32 * v + 4 * gj);
  }
  int32_t lmax = INT32_MIN;   // lanes gj < G: running maximum of head gj
  for (int i = 0; i < nsub; i++) {
    const int stage = i % ATTN_STAGES;
    mbar_wait(&full[stage], (uint32_t)(i / ATTN_STAGES) & 1u, a.err);
    const int32_t *buf = ring + stage * SUB * HD;
    const int len = min(SUB, cn - i * SUB);
    if (spin) spin_decode(i, ring + stage * SUB * HD, len);
    if (own && i == nsub - 1) {   // the new position (the slice's last) from this kernel's K row
      for (int d = threadIdx.x; d < HD; d += ATTN_THREADS) ring[stage * SUB * HD + (len - 1) * HD + d] = kvn[d];
      __syncthreads();
    }
    for (int p4 = warp * 4; p4 < len; p4 += ATTN_THREADS / 8) {   // warp-uniform bound
      const int pp = p4 + gq;
      const bool ok = pp < len;
      const int32_t *kr = buf + (ok ? pp : p4) * HD + 4 * gj;
      int4 kv[V4];
#pragma unroll
      for (int v = 0; v < V4; v++) kv[v] = *reinterpret_cast<const int4 *>(kr + 32 * v);
      int64_t sv = 0;
#pragma unroll
      for (int h = 0; h < G; h++) {
        int64_t acc = 0;
#pragma unroll
        for (int v = 0; v < V4; v++) {
          const int4 q = QREG ? qr[h * V4 + v] : *reinterpret_cast<const int4 *>(qs + h * HD + 32 * v + 4 * gj);
          acc += (int64_t)q.x * kv[v].x;
          acc += (int64_t)q.y * kv[v].y;
          acc += (int64_t)q.z * kv[v].z;
          acc += (int64_t)q.w * kv[v].w;
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 4);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        if (gj == h) sv = acc;
      }
      if (ok && gj < G) {
        float z = __fmul_rn(__double2float_rn(__dmul_rn(__ll2double_rn(sv), 0x1p-32)), a.ascale);
        if (!(fabsf(z) < 131072.0f)) { raise_err(a.err, ERR_SCORE_RANGE); z = 0.0f; }
        const int32_t zi = (int32_t)llround_d((double)z * 16384.0);
        sc[gj * cmax + i * SUB + pp] = zi;
        lmax = max(lmax, zi);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && i + ATTN_STAGES < total) {
      fence_proxy_async_smem();
      issue(i + ATTN_STAGES);
    }
  }
  lmax = max(lmax, __shfl_xor_sync(0xffffffffu, lmax, 8));
  lmax = max(lmax, __shfl_xor_sync(0xffffffffu, lmax, 16));
  if (lane < G && lmax != INT32_MIN) atomicMax(&mx_loc[lane], lmax);
  __syncthreads();
  if (CL > 1) {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    if (threadIdx.x < CL * G) {
      const int r = threadIdx.x / G, h = threadIdx.x % G;
      *cluster.map_shared_rank(&mx_in[rank][h], r) = mx_loc[h];
    }
    cluster.sync();
  }
  if (threadIdx.x < G) {
    int32_t m = mx_loc[threadIdx.x];
    for (int r = 0; r < (CL > 1 ? CL : 0); r++) m = max(m, mx_in[r][threadIdx.x]);
    mx_all[threadIdx.x] = m;
  }
  __syncthreads();
  // ---- phase 2: integer exponentials and their exact sum, one (head, position) per thread
  // (a warp's items may span several heads: one warp sum per head it covers)
  for (int i0 = 0; i0 < G * cn; i0 += ATTN_THREADS) {
    const int i = i0 + threadIdx.x;
    const int h = i < G * cn ? i / cn : G - 1, j = i - h * cn;
    int64_t e = 0;
    if (i < G * cn) {
      const int64_t dz = (((int64_t)sc[h * cmax + j] - (int64_t)mx_all[h]) * ONE) >> 14;
      e = exp_fixed(dz);
      sc[h * cmax + j] = (int32_t)e;
    }
    const int h0 = __shfl_sync(0xffffffffu, h, 0);
#pragma unroll 1
    for (int hh = h0; hh <= __shfl_sync(0xffffffffu, h, 31); hh++) {
      const int64_t part = warp_sum_i64(h == hh ? e : 0);
      if (lane == 0 && part) atomicAdd(reinterpret_cast<unsigned long long *>(&s_loc[hh]), (unsigned long long)part);
    }
  }
  __syncthreads();
  // ---- phase 3: exact 128-bit V-sum, V slices streamed through the same ring
  const int d = threadIdx.x % HD, grp = threadIdx.x / HD;
  acc128 acc[G];
#pragma unroll
  for (int h = 0; h < G; h++) acc[h] = acc128{0ull, 0ll};
  for (int i = nsub; i < total; i++) {
    const int stage = i % ATTN_STAGES;
    mbar_wait(&full[stage], (uint32_t)(i / ATTN_STAGES) & 1u, a.err);
    const int32_t *buf = ring + stage * SUB * HD;
    const int j0 = (i - nsub) * SUB;
    const int len = min(SUB, cn - j0);
    if (spin) spin_decode(i, ring + stage * SUB * HD, len);
    if (own && i == total - 1) {   // ... and its V row
      for (int d = threadIdx.x; d < HD; d += ATTN_THREADS) ring[stage * SUB * HD + (len - 1) * HD + d] = kvn[HD + d];
      __syncthreads();
    }
    // eight positions per fold into 128 bits: e <= 2^30 and |v| < 2^30, so 8 |e v| < 2^63
    // (positions pp < SUB always stay inside the stage; those past len weigh 0)
    for (int p8 = grp; p8 < len; p8 += 8 * GROUPS) {
      int64_t part[G];
#pragma unroll
      for (int h = 0; h < G; h++) part[h] = 0;
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int pp = p8 + u * GROUPS;
        const bool ok = pp < len;
        const int64_t v = buf[pp * HD + d];
#pragma unroll
        for (int h = 0; h < G; h++) part[h] += (int64_t)(ok ? sc[h * cmax + j0 + pp] : 0) * v;
      }
#pragma unroll
      for (int h = 0; h < G; h++) acc128_add(acc[h], part[h]);
    }
    __syncthreads();
    if (threadIdx.x == 0 && i + ATTN_STAGES < total) {
      fence_proxy_async_smem();
      issue(i + ATTN_STAGES);
    }
  }
  // push: head dim dd goes to rank dd / DPR, slot [this rank][h][dd % DPR]
  if (direct) {
    const int o = d / DPR;
#pragma unroll
    for (int h = 0; h < G; h++) *cluster.map_shared_rank(&gat[(rank * G + h) * DPR + (d - o * DPR)], o) = acc[h];
  } else {
#pragma unroll
    for (int h = 0; h < G; h++) nacc[(grp * G + h) * HD + d] = acc[h];
    __syncthreads();
    if (GROUPS > 1) {
      for (int i = threadIdx.x; i < G * HD; i += ATTN_THREADS) {
        acc128 s = nacc[i];
        for (int r = 1; r < GROUPS; r++) acc128_add(s, nacc[r * G * HD + i]);
        nacc[i] = s;
      }
    }
    __syncthreads();
    if (CL > 1)
      for (int i = threadIdx.x; i < G * HD; i += ATTN_THREADS) {
        const int h = i / HD, dd = i % HD, o = dd / DPR;
        *cluster.map_shared_rank(&gat[(rank * G + h) * DPR + (dd - o * DPR)], o) = nacc[i];
      }
  }
  if (CL > 1) {
    if (threadIdx.x < CL * G) {
      const int r = threadIdx.x / G, h = threadIdx.x % G;
      *cluster.map_shared_rank(&s_in[rank][h], r) = s_loc[h];
    }
    cluster.sync();   // the last cluster access: after it no rank touches another's memory
  }
  // ---- phase 4: combine the cluster's partials; rank r finalizes HD/CL dims per head
  float omax = 0.0f;
  for (int i = threadIdx.x; i < G * DPR; i += ATTN_THREADS) {
    const int h = i / DPR, j = i % DPR, dd = rank * DPR + j;
    acc128 N;
    int64_t S;
    if (CL > 1) {
      N = gat[h * DPR + j];
      S = s_in[0][h];
      for (int r = 1; r < CL; r++) {
        acc128_add(N, gat[(r * G + h) * DPR + j]);
        S += s_in[r][h];
      }
    } else {
      N = nacc[h * HD + dd];
      S = s_loc[h];
    }
    const int64_t hi = (int64_t)(((uint64_t)N.hi << 16) | (N.lo >> 48));   // N * 2^16, |N| < 2^78
    const uint64_t lo = N.lo << 16;
    const int64_t qd = floordiv_s128(hi, lo, (uint64_t)S);
    const float o = __double2float_rn(__dmul_rn(__ll2double_rn(qd), 0x1p-32));
    a.ao[(size_t)t * QD + ((size_t)g * G + h) * HD + dd] = o;
    omax = fmaxf(omax, fabsf(o));
  }
  if (a.ao_max) {
    omax = block_max(omax, fred);
    if (threadIdx.x == 0) atomicMax(a.ao_max + t, __float_as_uint(omax));
  }
}


// ---- prefill rows in tiles: the rows of one prefill chunk are consecutive positions of one
// session and read the same K/V rows, so one CTA takes ATILE_QV query vectors of one KV head
// (TQ = ATILE_QV / G consecutive rows x the G query heads that share it) and every staged K/V
// slice serves all of them, where the per-row kernel streams it once per row. Scores of the
// union of the rows' windows, each query's maximum, the island's exponentials with their exact
// int64 sums, then the 128-bit V-sums. ST (stored): the scores stay in shared memory between the
// K pass and the V pass; otherwise (a union too long for shared memory) a second K pass
// recomputes them slice by slice, K and V slices alternating through the ring. A position
// outside a row's own window (a later position of the chunk, or one before the row's sliding
// window) weighs exactly 0, so every integer is the per-row kernel's.
constexpr int ATILE_QV = 16;
constexpr int ATILE_STAGES = 3;

template <int HD>
struct AttnTile {
  static constexpr int SUB = 4096 / HD;                       // positions per ring stage (16 KB)
  static constexpr int V4 = HD / 32;                          // int4 columns per lane of an 8-lane group
  static constexpr int QG = SUB >= 32 ? 1 : 32 / SUB;         // query subsets over the 32 groups
  static constexpr int NPG = 32 / QG;                         // position slots per subset
  static constexpr int PPG = SUB > NPG ? SUB / NPG : 1;       // positions per group per slice
  static constexpr int QPG = ATILE_QV / QG;                   // query vectors per group
  static constexpr int KEEP = QPG / 8;                        // scores each lane keeps per position
  static constexpr int GROUPS = ATTN_THREADS / HD;            // position groups of the V-sum
  static constexpr size_t RING = (size_t)ATILE_STAGES * SUB * HD * 4;
  // + the scores of the whole union when stored, else the exponentials of one slice
  static constexpr size_t BASE = RING + (size_t)ATILE_QV * HD * 4;
  static size_t smem(bool st, int cmax) { return BASE + (size_t)ATILE_QV * (st ? cmax : SUB) * 4; }
  static_assert(NPG * PPG == SUB && QPG % 8 == 0, "every (query, position) of a slice has one group");
  static_assert(16 * GROUPS == SUB, "each V-sum thread folds two runs of 8 positions per slice");
  static_assert((size_t)(GROUPS - 1) * ATILE_QV * HD * sizeof(acc128) <= RING, "V-sum partials fit the ring");
};

template <int HD, int G, bool ST>
__global__ void __launch_bounds__(ATTN_THREADS, ST ? 1 : 2) k_attn_tile(AttnArgs a, int cmax) {
  using AT = AttnTile<HD>;
  constexpr int SUB = AT::SUB, V4 = AT::V4, NPG = AT::NPG, PPG = AT::PPG, QPG = AT::QPG, KEEP = AT::KEEP;
  constexpr int GROUPS = AT::GROUPS, QV = ATILE_QV, TQ = ATILE_QV / G, S = ATILE_STAGES;
  extern __shared__ __align__(128) uint8_t at_raw[];
  int32_t *ring = reinterpret_cast<int32_t *>(at_raw);   // [S][SUB][HD]
  int32_t *qs = ring + S * SUB * HD;                       // [QV][HD] rotated queries
  int32_t *es = qs + QV * HD;                              // [QV][ST ? cmax : SUB] scores -> exponentials
  const int estride = ST ? cmax : SUB;
  __shared__ __align__(8) uint64_t full[S];
  __shared__ int32_t mx[QV];
  __shared__ unsigned long long ssum[QV];
  __shared__ uint32_t omx[TQ];

  const int g = blockIdx.y, t0 = blockIdx.x * TQ, tid = threadIdx.x, lane = tid & 31;
  const int QD = a.NH * HD;
  const int nrow = min(TQ, a.ntok - t0);
  pdl_trigger();
  if (tid == 0) {
    for (int s = 0; s < S; s++) mbar_init(&full[s], 1);
    mbar_init_fence();
  }
  if (tid < QV) { mx[tid] = INT32_MIN; ssum[tid] = 0ull; }
  if (tid < TQ) omx[tid] = 0u;
  pdl_wait();
  const int pbase = a.pos_dev[0] + t0;   // position of the tile's first row
  auto wstart = [&](int p) { return (a.win >= 0 && p - a.win + 1 > 0) ? p - a.win + 1 : 0; };
  const int u0 = wstart(pbase), u1 = pbase + nrow;   // the union of the rows' windows: [u0, u1)
  const int ulen = u1 - u0;
  if (ST && ulen > cmax) {   // (the launch sized cmax for every tile; never taken)
    if (tid == 0) raise_err(a.err, ERR_SCORE_RANGE);
    return;
  }
  const int nsl = (ulen + SUB - 1) / SUB;
  const int total = (ST ? 2 : 3) * nsl;
  auto kv_at = [&](bool isv, int q) -> int32_t * {
    return (isv ? a.kv.v : a.kv.k) + kv_elem(a.kv, a.NL, a.NKV, HD, a.layer, g, q);
  };
  // item i -> (slice, K or V): ST: the K slices, then the V slices; otherwise pass A's K slices,
  // then pass B's K and V slices alternating
  auto item = [&](int i, int &sl) -> bool {
    if (i < nsl) { sl = i; return false; }
    if (ST) { sl = i - nsl; return true; }
    sl = (i - nsl) >> 1;
    return ((i - nsl) & 1) != 0;
  };
  // a slice of SUB <= 64 positions spans at most two pages of >= 128
  auto issue = [&](int i) {
    int sl;
    const bool isv = item(i, sl);
    const int pos = u0 + sl * SUB;
    const int len = min(SUB, u1 - pos);
    uint64_t *bar = &full[i % S];
    mbar_arrive_expect_tx(bar, (uint32_t)len * HD * 4);
    int32_t *dst = ring + (i % S) * SUB * HD;
    const int first = min(len, a.kv.pg - pos % a.kv.pg);
    bulk_g2s(dst, kv_at(isv, pos), (uint32_t)first * HD * 4, bar);
    if (first < len) bulk_g2s(dst + (size_t)first * HD, kv_at(isv, pos + first), (uint32_t)(len - first) * HD * 4, bar);
  };
  for (int i = tid; i < QV * HD; i += ATTN_THREADS) {
    const int qv = i / HD, d = i - qv * HD, r = qv / G, h = qv - r * G;
    qs[i] = r < nrow ? a.qi[(size_t)(t0 + r) * QD + (size_t)(g * G + h) * HD + d] : 0;
  }
  __syncthreads();   // barriers initialised, queries staged
  if (tid == 0)
    for (int i = 0; i < min(S, total); i++) issue(i);
  auto next = [&](int i) {   // after the __syncthreads that freed item i's stage
    if (tid == 0 && i + S < total) {
      fence_proxy_async_smem();
      issue(i + S);
    }
  };

  // scores: 8-lane group gi takes slot gi % NPG of query subset gi / NPG; lane j of the group
  // holds the int4 columns 4j + 32v of the position's K row; after the three-level butterfly
  // lane (l % 8) keeps the raw score of the group's query l, and the conversions run once all
  // queries are reduced, every lane busy
  const int gi = tid >> 3, gj = tid & 7, qsub = gi / NPG, pslot = gi % NPG;
  auto valid_at = [&](int qv, int jpos) {
    const int r = qv / G;
    const int p = pbase + r;
    return r < nrow && jpos <= p && jpos >= wstart(p);
  };
  auto to_grid = [&](int64_t sv, bool ok) -> int32_t {
    float z = __fmul_rn(__double2float_rn(__dmul_rn(__ll2double_rn(sv), 0x1p-32)), a.ascale);
    if (!(fabsf(z) < 131072.0f)) {
      if (ok) raise_err(a.err, ERR_SCORE_RANGE);
      z = 0.0f;
    }
    return (int32_t)llround_d((double)z * 16384.0);
  };
  auto score = [&](const int32_t *buf, int sl, int len, auto &&use) {
#pragma unroll 1
    for (int r = 0; r < PPG; r++) {
      const int pp = pslot + r * NPG;
      const bool inb = pp < len;
      const int32_t *kr = buf + (inb ? pp : 0) * HD + 4 * gj;
      int4 kv[V4];
#pragma unroll
      for (int v = 0; v < V4; v++) kv[v] = *reinterpret_cast<const int4 *>(kr + 32 * v);
      int64_t kept[KEEP];
#pragma unroll
      for (int l = 0; l < QPG; l++) {
        const int32_t *qr = qs + (qsub * QPG + l) * HD + 4 * gj;
        int64_t acc = 0;
#pragma unroll
        for (int v = 0; v < V4; v++) {
          const int4 q = *reinterpret_cast<const int4 *>(qr + 32 * v);
          acc += (int64_t)q.x * kv[v].x;
          acc += (int64_t)q.y * kv[v].y;
          acc += (int64_t)q.z * kv[v].z;
          acc += (int64_t)q.w * kv[v].w;
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 4);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        if ((l & 7) == gj) kept[l >> 3] = acc;
      }
#pragma unroll
      for (int k = 0; k < KEEP; k++) {
        const int qv = qsub * QPG + gj + 8 * k;
        use(k, qv, pp, kept[k], inb && valid_at(qv, u0 + sl * SUB + pp));
      }
    }
  };
  int64_t lsum[KEEP];
#pragma unroll
  for (int k = 0; k < KEEP; k++) lsum[k] = 0;
  auto exps_into = [&](int k, int qv, int idx, int32_t zi, bool ok) {
    int64_t e = 0;
    if (ok) e = exp_fixed((((int64_t)zi - (int64_t)mx[qv]) * ONE) >> 14);
    es[qv * estride + idx] = (int32_t)e;
    lsum[k] += e;
  };

  // ---- K pass: each query's maximum over its own window (ST: and its scores)
  int32_t lmax[KEEP];
#pragma unroll
  for (int k = 0; k < KEEP; k++) lmax[k] = INT32_MIN;
  for (int i = 0; i < nsl; i++) {
    const int stage = i % S;
    mbar_wait(&full[stage], (uint32_t)(i / S) & 1u, a.err);
    score(ring + stage * SUB * HD, i, min(SUB, u1 - (u0 + i * SUB)), [&](int k, int qv, int pp, int64_t sv, bool ok) {
      if (ok) {
        const int32_t zi = to_grid(sv, true);
        lmax[k] = max(lmax[k], zi);
        if (ST) es[qv * estride + i * SUB + pp] = zi;
      }
    });
    __syncthreads();
    next(i);
  }
#pragma unroll
  for (int k = 0; k < KEEP; k++) {   // the warp's four groups hold the same queries
    int32_t m = lmax[k];
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 8));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 16));
    if (lane < 8 && m != INT32_MIN) atomicMax(&mx[qsub * QPG + gj + 8 * k], m);
  }
  __syncthreads();
  if (ST) {   // exponentials of the stored scores: thread tid takes positions tid, tid + 256, ...
    for (int q = 0; q < QV; q++) {
      int64_t sm = 0;
      for (int j = tid; j < ulen; j += ATTN_THREADS) {
        int64_t e = 0;
        if (valid_at(q, u0 + j)) e = exp_fixed((((int64_t)es[q * estride + j] - (int64_t)mx[q]) * ONE) >> 14);
        es[q * estride + j] = (int32_t)e;
        sm += e;
      }
      sm = warp_sum_i64(sm);
      if (lane == 0 && sm) atomicAdd(&ssum[q], (unsigned long long)sm);
    }
    __syncthreads();
  }

  // ---- V pass (not ST: K slices again for the exponentials, alternating with the V slices):
  // thread (d, grp) folds the run of 16 positions grp * 16 .. of each slice, eight per fold
  // into 128 bits (e <= 2^30 and |v| < 2^30, so 8 |e v| < 2^63); positions past len weigh 0
  const int d = tid % HD, grp = tid / HD;
  acc128 acc[QV];
#pragma unroll
  for (int q = 0; q < QV; q++) acc[q] = acc128{0ull, 0ll};
  for (int i = nsl; i < total; i++) {
    const int stage = i % S;
    mbar_wait(&full[stage], (uint32_t)(i / S) & 1u, a.err);
    const int32_t *buf = ring + stage * SUB * HD;
    int sl;
    const bool isv = item(i, sl);
    const int len = min(SUB, u1 - (u0 + sl * SUB));
    if (!isv) {
      score(buf, sl, len, [&](int k, int qv, int pp, int64_t sv, bool ok) {
        exps_into(k, qv, pp, ok ? to_grid(sv, false) : 0, ok);
      });
    } else {
      const int32_t *eb = es + (ST ? sl * SUB : 0);
#pragma unroll
      for (int f = 0; f < 2; f++) {
        const int pb = grp * 16 + f * 8;
        if (pb < len) {
          int64_t v[8];
#pragma unroll
          for (int u = 0; u < 8; u++) v[u] = pb + u < len ? (int64_t)buf[(pb + u) * HD + d] : 0;
#pragma unroll
          for (int q = 0; q < QV; q++) {
            const int4 e0 = *reinterpret_cast<const int4 *>(eb + q * estride + pb);
            const int4 e1 = *reinterpret_cast<const int4 *>(eb + q * estride + pb + 4);
            int64_t part = (int64_t)e0.x * v[0] + (int64_t)e0.y * v[1] + (int64_t)e0.z * v[2] +
                           (int64_t)e0.w * v[3] + (int64_t)e1.x * v[4] + (int64_t)e1.y * v[5] +
                           (int64_t)e1.z * v[6] + (int64_t)e1.w * v[7];
            acc128_add(acc[q], part);
          }
        }
      }
    }
    __syncthreads();
    next(i);
  }
  if (!ST) {
#pragma unroll
    for (int k = 0; k < KEEP; k++) {
      int64_t sm = lsum[k];
      sm += __shfl_xor_sync(0xffffffffu, sm, 8);
      sm += __shfl_xor_sync(0xffffffffu, sm, 16);
      if (lane < 8 && sm) atomicAdd(&ssum[qsub * QPG + gj + 8 * k], (unsigned long long)sm);
    }
  }
  if (GROUPS > 1) {   // the ring is idle now: it holds the other position groups' partials
    acc128 *red = reinterpret_cast<acc128 *>(ring);
    if (grp > 0)
#pragma unroll
      for (int q = 0; q < QV; q++) red[((grp - 1) * QV + q) * HD + d] = acc[q];
    __syncthreads();
    if (grp == 0)
      for (int r = 1; r < GROUPS; r++)
#pragma unroll
        for (int q = 0; q < QV; q++) acc128_add(acc[q], red[((r - 1) * QV + q) * HD + d]);
  }
  __syncthreads();   // the exponential sums are complete

  // ---- finalize: thread d of group 0 writes head dim d of every query
  if (grp == 0) {
    float rm[TQ];
#pragma unroll
    for (int r = 0; r < TQ; r++) rm[r] = 0.0f;
#pragma unroll
    for (int q = 0; q < QV; q++) {
      const int r = q / G, h = q % G;
      if (r < nrow) {
        const acc128 N = acc[q];
        const int64_t hi = (int64_t)(((uint64_t)N.hi << 16) | (N.lo >> 48));   // N * 2^16, |N| < 2^78
        const uint64_t lo = N.lo << 16;
        const int64_t qd = floordiv_s128(hi, lo, (uint64_t)ssum[q]);
        const float o = __double2float_rn(__dmul_rn(__ll2double_rn(qd), 0x1p-32));
        a.ao[(size_t)(t0 + r) * QD + ((size_t)g * G + h) * HD + d] = o;
        rm[r] = fmaxf(rm[r], fabsf(o));
      }
    }
    if (a.ao_max) {
#pragma unroll
      for (int r = 0; r < TQ; r++) {
        const float m = warp_max_f(rm[r]);
        if (lane == 0 && r < nrow) atomicMax(&omx[r], __float_as_uint(m));
      }
    }
  }
  if (a.ao_max) {
    __syncthreads();
    if (tid < nrow) atomicMax(a.ao_max + t0 + tid, omx[tid]);
  }
}

constexpr size_t ATILE_SMEM_MAX = 220 * 1024;

// SPB_ATTN_TILE_STORE=0 always recomputes the scores in a second K pass (comparisons)
static bool attn_tile_store_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_ATTN_TILE_STORE");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}

template <int HD, int G>
static cudaError_t attn_tile(const AttnArgs &a, cudaStream_t st) {
  using AT = AttnTile<HD>;
  constexpr int TQ = ATILE_QV / G;
  // the longest union of a tile's windows: the window plus TQ - 1 rows, at most the capacity
  const int span = a.win >= 0 ? std::min(a.P, a.win + TQ - 1) : a.P;
  const int cmax = (span + AT::SUB - 1) / AT::SUB * AT::SUB;   // the V pass reads whole slices of it
  const dim3 grid((a.ntok + TQ - 1) / TQ, a.NKV);
  if (attn_tile_store_enabled() && AT::smem(true, cmax) <= ATILE_SMEM_MAX) {
    auto kern = k_attn_tile<HD, G, true>;
    static bool set = false;
    if (!set) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATILE_SMEM_MAX);
      if (e != cudaSuccess) return e;
      set = true;
    }
    return launch_k(kern, grid, dim3(ATTN_THREADS), AT::smem(true, cmax), st, 1, a, cmax);
  }
  auto kern = k_attn_tile<HD, G, false>;
  static bool set = false;
  if (!set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AT::smem(false, 0));
    if (e != cudaSuccess) return e;
    set = true;
  }
  return launch_k(kern, grid, dim3(ATTN_THREADS), AT::smem(false, 0), st, 1, a, 0);
}

// token rows of one session from which attention runs in row tiles (SPB_ATTN_TILE; 0 never)
static int attn_tile_min() {
  static int n = -1;
  if (n < 0) {
    const char *e = getenv("SPB_ATTN_TILE");
    n = e ? atoi(e) : 16;
    if (n < 0) n = 0;
  }
  return n;
}

template <int HD, int G>
static size_t attn_smem(int cmax, int cl, bool fused, bool spin = false) {
  constexpr int SUB = AttnSub<HD>::SUB, GROUPS = ATTN_THREADS / HD;
  const bool direct = GROUPS == 1 && cl > 1;
  return (size_t)ATTN_STAGES * SUB * HD * 4 + (size_t)G * HD * 4 + (fused ? (size_t)2 * HD * 4 : 0) +
         (size_t)((G * cmax + 3) & ~3) * 4 +
         (direct ? 0 : (size_t)GROUPS * G * HD * sizeof(acc128)) + (cl > 1 ? (size_t)G * HD * sizeof(acc128) : 0) +
         (spin ? 2048 : 0);   // Spinor caches: CRC tables, decode multipliers
}

// SPB_ATTN_OWN: the share of positions (percent of an equal split) the owning rank of a fused
// decode row takes (100: an equal split; default 50, measured 3.79 against 3.83-3.86 ms per
// 12B decode step)
static int attn_own_pct() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("SPB_ATTN_OWN");
    v = e ? atoi(e) : 50;
    if (v < 0) v = 0;
    if (v > 100) v = 100;
  }
  return v;
}

template <int HD, int G>
static cudaError_t attn_cl(const AttnArgs &a, cudaStream_t st) {
  // Largest cluster: 16 CTAs where the device can co-schedule them (asked once, before any
  // launch, so a graph capture never sees a failed launch), else the portable 8.
  static int clmax = 0, nsm = 148;
  auto kern = k_attn<HD, G>;
  if (clmax == 0) {
    clmax = 8;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) {
      clmax = 0;
      return e;
    }
    auto k16 = kern;
    if (cudaFuncSetAttribute(k16, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(16, 1, 1);
      cfg.blockDim = dim3(ATTN_THREADS);
      cfg.dynamicSmemBytes = attn_smem<HD, G>((a.P + 15) / 16, 16, a.qkv != nullptr);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 16;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int nclusters = 0;
      if (cudaOccupancyMaxActiveClusters(&nclusters, k16, &cfg) == cudaSuccess && nclusters >= 4) clmax = 16;
    }
    (void)cudaGetLastError();
  }
  // Split a row's positions over more CTAs only while (rows x KV heads) CTAs leave SMs idle or
  // a CTA would cover more than ATTN_SPAN positions; the score buffer bounds it from below.
  const int span = a.win >= 0 ? std::min(a.P, a.win) : a.P;
  int cl = 1;
  while (cl < clmax && ((long)a.ntok * a.NKV * cl < 2L * nsm || span > cl * ATTN_SPAN)) cl *= 2;
  // (batch rows with a Spinor row among them carry the Spinor scratch: 2 KB that would otherwise
  // cost the 64-session attention its second CTA per SM)
  const bool fused = a.qkv != nullptr, spin = a.kv.rb > 0 || (a.rows != nullptr && a.rows_spin);
  while (cl < clmax && attn_smem<HD, G>((a.P + cl - 1) / cl, cl, fused, spin) > 200 * 1024) cl *= 2;
  // a rank's positions at most (the other ranks' share grows when the owner's shrinks)
  AttnArgs b = a;
  b.own_pct = attn_own_pct();
  const int cmax = (fused && cl > 1 && b.own_pct < 100) ? (a.P + cl - 2) / (cl - 1) : (a.P + cl - 1) / cl;
  const size_t smem = attn_smem<HD, G>(cmax, cl, fused, spin);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  return launch_k(kern, dim3(cl, a.NKV, a.ntok), dim3(ATTN_THREADS), smem, st, cl, b, cmax, cl);
}

cudaError_t launch_attn(const AttnArgs &a, cudaStream_t st) {
  const int G = a.NH / a.NKV;
  if (a.NH % a.NKV || a.P <= 0) return cudaErrorInvalidValue;
  // Spinor-block caches: unpaged caches (a session's own, or each batch row's), head_dim 64 / 128 / 256
  if (a.kv.rb > 0 && (a.kv.ptab || a.HD < 64 || a.kv.rb != spin_row_bytes(a.HD))) return cudaErrorInvalidValue;
  // prefill chunks (rows of one session, K/V already stored by k_rope_kv): row tiles
  const bool tile = !a.rows && !a.qkv && a.kv.rb == 0 && attn_tile_min() > 0 && a.ntok >= attn_tile_min();
#define SPB_ATTN_CASE(HDV, GV) \
  if (a.HD == HDV && G == GV) return tile ? attn_tile<HDV, GV>(a, st) : attn_cl<HDV, GV>(a, st);
  SPB_ATTN_CASE(64, 1) SPB_ATTN_CASE(64, 2) SPB_ATTN_CASE(64, 4) SPB_ATTN_CASE(64, 8)
  SPB_ATTN_CASE(128, 1) SPB_ATTN_CASE(128, 2) SPB_ATTN_CASE(128, 4) SPB_ATTN_CASE(128, 8)
  SPB_ATTN_CASE(256, 1) SPB_ATTN_CASE(256, 2) SPB_ATTN_CASE(256, 4) SPB_ATTN_CASE(256, 8)
#undef SPB_ATTN_CASE
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------------------ misc
__global__ void k_embed(DevQ4B emb, const int32_t *tok_dev, float scale, int use_scale, float *x, int vocab,
                        uint32_t *err) {
  pdl_trigger();
  const int t = blockIdx.x;
  int tok = tok_dev[t];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) raise_err(err, ERR_TOKEN);
    tok = 0;
  }
  const int E = emb.cols;
  const uint8_t *cr = emb.codes + (size_t)tok * (E >> 1);
  const uint16_t *sr = emb.scales + (size_t)tok * (E >> 5);
  for (int i = threadIdx.x; i < E; i += blockDim.x) {
    const uint32_t b = (i & 1) ? (cr[i >> 1] >> 4) : (cr[i >> 1] & 0xF);
    const int c = b >= 8 ? (int)b - 16 : (int)b;
    float v = __fmul_rn((float)c, f16_value(sr[i >> 5]));
    if (use_scale) v = __fmul_rn(v, scale);
    x[(size_t)t * E + i] = v;
  }
}

cudaError_t launch_embed(const DevQ4B &emb, const int32_t *tok_dev, int ntok, float scale, int use_scale,
                         float *x, int vocab, uint32_t *err, cudaStream_t st) {
  k_embed<<<ntok, 256, 0, st>>>(emb, tok_dev, scale, use_scale, x, vocab, err);
  return cudaGetLastError();
}

// one warp per row (8 rows per CTA); the int64 bound restates xref_q4b_check (the checker's
// upload test): a lane saturates its partial sum at the limit, so the warp sum cannot wrap
__global__ void __launch_bounds__(256) k_q4b_rowinfo(const uint16_t *scales, int rows, int nblk, uint8_t *shift,
                                                     int *info) {
  const int lane = threadIdx.x & 31, r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const uint64_t lim = (1ull << 63) / (32u * 8u * 127u);
  const uint16_t *row = scales + (size_t)r * nblk;
  uint64_t sum = 0;
  int bad = 0, emax = 0, smin = 64, smax = -1;
  for (int b = lane; b < nblk; b += 32) {
    const uint32_t h = row[b], e = (h >> 10) & 31u, mant = h & 1023u;
    if (e == 31) { bad = 1; continue; }
    const uint32_t m = e ? (mant | 1024u) : mant;
    const int sh = e ? (int)e - 1 : 0;
    sum += (uint64_t)m << sh;
    if (sum >= lim) sum = lim;
    emax = max(emax, (int)e);
    if (m) { smin = min(smin, sh); smax = max(smax, sh); }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, o));
    smin = min(smin, __shfl_xor_sync(0xffffffffu, smin, o));
    smax = max(smax, __shfl_xor_sync(0xffffffffu, smax, o));
  }
  if (lane == 0) {
    if (bad || sum >= lim) atomicOr(info, 1);
    atomicMax(info + 1, emax);
    const int s0 = smax < 0 ? 0 : smin;
    if (shift) shift[r] = (uint8_t)s0;
    atomicMax(info + 2, smax < 0 ? 0 : smax - s0);
  }
}

cudaError_t launch_q4b_rowinfo(const uint16_t *scales, int rows, int nblk, uint8_t *shift, int *info,
                               cudaStream_t st) {
  if (rows <= 0 || nblk <= 0) return cudaErrorInvalidValue;
  k_q4b_rowinfo<<<(rows + 7) / 8, 256, 0, st>>>(scales, rows, nblk, shift, info);
  return cudaGetLastError();
}

// decode the keys left by the LM-head GEMV into token ids and clear them for the next step
__global__ void k_argmax_take(unsigned long long *keys, int ntok, int32_t *out) {
  pdl_trigger();
  pdl_wait();
  for (int t = threadIdx.x; t < ntok; t += blockDim.x) {
    const unsigned long long k = keys[t];
    out[t] = (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    keys[t] = 0ull;
  }
}

cudaError_t launch_argmax_take(unsigned long long *keys, int ntok, int32_t *out, cudaStream_t st) {
  return launch_k(k_argmax_take, dim3(1), dim3(128), 0, st, 1, keys, ntok, out);
}

__global__ void k_scale_i64(const int64_t *acc, const float *scale, int n, float *y, int ldy, int parts,
                            size_t pstride) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.y;
  const double d = __dmul_rn(__ddiv_rn((double)scale[t], 127.0), 0x1p-24);
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
    int64_t a = acc[(size_t)t * n + j];
    for (int p = 1; p < parts; p++) a += acc[p * pstride + (size_t)t * n + j];
    y[(size_t)t * ldy + j] = __double2float_rn(__dmul_rn(__ll2double_rn(a), d));
  }
}

cudaError_t launch_scale_i64(const int64_t *acc, const float *scale, int ntok, int n, float *y, int ldy,
                             cudaStream_t st, int parts, size_t part_stride) {
  return launch_k(k_scale_i64, dim3((n + 255) / 256, ntok), dim3(256), 0, st, 1, acc, scale, n, y, ldy, parts,
                  part_stride);
}

// the key's low word is 0xFFFFFFFF - row: a row offset subtracts from it
__global__ void k_keys_rebase(unsigned long long *keys, int ntok, int base) {
  pdl_trigger();
  pdl_wait();
  for (int t = threadIdx.x; t < ntok; t += blockDim.x)
    if (keys[t]) keys[t] -= (unsigned long long)(uint32_t)base;
}

cudaError_t launch_keys_rebase(unsigned long long *keys, int ntok, int base, cudaStream_t st) {
  return launch_k(k_keys_rebase, dim3(1), dim3(128), 0, st, 1, keys, ntok, base);
}

__global__ void k_advance(int32_t *pos_dev, int n, const int32_t *src_tok, int32_t *dst_tok) {
  pdl_trigger();
  pdl_wait();
  pos_dev[0] += n;
  if (src_tok && dst_tok) dst_tok[0] = src_tok[0];
}

cudaError_t launch_advance(int32_t *pos_dev, int n, const int32_t *src_tok, int32_t *dst_tok, cudaStream_t st) {
  return launch_k(k_advance, dim3(1), dim3(1), 0, st, 1, pos_dev, n, src_tok, dst_tok);
}

// ------------------------------------------------------------------------------ synthetic weights
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void k_synth_codes(uint64_t *dst, size_t nwords, uint64_t key) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nwords; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = splitmix64(i + key);
}

// one generated block scale: the matrix's exponent field, the word's low 10 bits as mantissa and
// its bit 10 as sign (the host generator's rule, spmodel.gen_bscale)
__device__ __forceinline__ uint16_t synth_scale_bits(uint64_t w, int exp_field) {
  return (uint16_t)(((uint32_t)exp_field << 10) | (uint32_t)(w & 0x3FFull) | ((uint32_t)((w >> 10) & 1ull) << 15));
}

__global__ void k_synth_scales(uint16_t *dst, int rows, int nblk, int exp_field, uint64_t key) {
  const size_t n = (size_t)rows * nblk;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = synth_scale_bits(splitmix64(i + key), exp_field);
}

__global__ void k_synth_norm(float *dst, int n, uint64_t key) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint64_t w = splitmix64((uint64_t)i + key);
    const uint64_t k = 7549747ull + (w >> 40) % 1677722ull;
    dst[i] = __double2float_rn(__dmul_rn((double)k, 0x1p-23));
  }
}

cudaError_t launch_synth_codes(uint8_t *dst, size_t nbytes, uint64_t key, cudaStream_t st) {
  if (nbytes % 8 || ((uintptr_t)dst & 7)) return cudaErrorInvalidValue;
  k_synth_codes<<<148 * 8, 256, 0, st>>>(reinterpret_cast<uint64_t *>(dst), nbytes / 8, key);
  return cudaGetLastError();
}

cudaError_t launch_synth_scales(uint16_t *dst, int rows, int nblk_src, int nblk_dst, int exp_field, uint64_t key,
                                cudaStream_t st) {
  if (nblk_src != nblk_dst) return cudaErrorInvalidValue;
  k_synth_scales<<<148 * 8, 256, 0, st>>>(dst, rows, nblk_src, exp_field, key);
  return cudaGetLastError();
}

__global__ void k_synth_codes_cols(uint64_t *dst, int rows, size_t dst_words, size_t src_words, size_t off_words,
                                   uint64_t key) {
  const size_t n = (size_t)rows * dst_words;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / dst_words, j = i - r * dst_words;
    dst[i] = splitmix64(r * src_words + off_words + j + key);
  }
}

__global__ void k_synth_scales_cols(uint16_t *dst, int rows, int nblk_dst, int nblk_src, int blk_off, int exp_field,
                                    uint64_t key) {
  const size_t n = (size_t)rows * nblk_dst;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / nblk_dst, j = i - r * nblk_dst;
    const uint64_t w = splitmix64(r * (size_t)nblk_src + (size_t)blk_off + j + key);
    dst[i] = synth_scale_bits(w, exp_field);
  }
}

cudaError_t launch_synth_codes_cols(uint8_t *dst, int rows, size_t dst_row_bytes, size_t src_row_bytes,
                                   size_t src_off, uint64_t key, cudaStream_t st) {
  if ((dst_row_bytes | src_row_bytes | src_off) % 8 || ((uintptr_t)dst & 7)) return cudaErrorInvalidValue;
  k_synth_codes_cols<<<148 * 8, 256, 0, st>>>(reinterpret_cast<uint64_t *>(dst), rows, dst_row_bytes / 8,
                                              src_row_bytes / 8, src_off / 8, key);
  return cudaGetLastError();
}

cudaError_t launch_synth_scales_cols(uint16_t *dst, int rows, int nblk_dst, int nblk_src, int blk_off,
                                    int exp_field, uint64_t key, cudaStream_t st) {
  k_synth_scales_cols<<<148 * 8, 256, 0, st>>>(dst, rows, nblk_dst, nblk_src, blk_off, exp_field, key);
  return cudaGetLastError();
}

cudaError_t launch_synth_norm(float *dst, int n, uint64_t key, cudaStream_t st) {
  k_synth_norm<<<(n + 255) / 256, 256, 0, st>>>(dst, n, key);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ isolated islands
__global__ void k_rmsnorm_rows(const float *x, const float *w, int n, float *out, uint32_t *err) {
  __shared__ acc128 red[33];
  __shared__ uint64_t inv_sh;
  const size_t r = blockIdx.x;
  block_rmsnorm(x + r * n, w, n, out + r * n, red, &inv_sh, err);
}

__global__ void k_eltwise(const float *x, int n, float *out, int op, uint32_t *err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = x[i];
  if (!(fabsf(v) < 2048.0f)) raise_err(err, ERR_ACT_RANGE);
  out[i] = op == 0 ? gelu_exact(v) : silu_exact(v);
}

__global__ void k_rope_rows(const float *v, int d, const int32_t *pos, const uint64_t *W, const uint64_t *T,
                            uint64_t gain, int32_t *out, uint32_t *err) {
  const int r = blockIdx.x, i = threadIdx.x, half = d >> 1;
  const float *row = v + (size_t)r * d;
  const uint64_t phase = (uint64_t)(int64_t)pos[r] * W[i];
  int32_t oa, ob;
  cordic_rotate(row[i], row[i + half], phase, T, gain, oa, ob, err);
  out[(size_t)r * d + i] = oa;
  out[(size_t)r * d + i + half] = ob;
}

cudaError_t launch_rmsnorm_rows(const float *x, const float *w, int n, int rows, float *out, uint32_t *err,
                                cudaStream_t st) {
  k_rmsnorm_rows<<<rows, 256, 0, st>>>(x, w, n, out, err);
  return cudaGetLastError();
}

cudaError_t launch_eltwise(const float *x, int n, float *out, int op, uint32_t *err, cudaStream_t st) {
  k_eltwise<<<(n + 255) / 256, 256, 0, st>>>(x, n, out, op, err);
  return cudaGetLastError();
}

cudaError_t launch_rope_rows(const float *v, int d, int rows, const int32_t *pos, const uint64_t *W,
                             const uint64_t *T, uint64_t gain, int32_t *out, uint32_t *err, cudaStream_t st) {
  k_rope_rows<<<rows, d / 2, 0, st>>>(v, d, pos, W, T, gain, out, err);
  return cudaGetLastError();
}

}  // namespace spb
