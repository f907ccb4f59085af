// spb_kernels.cuh -- launch interface of the sm_100a kernels (host side of spb_kernels.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace spb {

// error bits raised by kernels (host maps any to a range error)
enum : uint32_t {
  ERR_NORM_RANGE = 1u << 0,   // RMSNorm input outside the int64 sum-of-squares range
  ERR_ACT_RANGE = 1u << 1,    // GELU / SiLU input |x| >= 2048, or non-finite activation
  ERR_ROPE_RANGE = 1u << 2,   // q/k outside |x| < 256 or rotated value outside 2^24 grid units
  ERR_V_RANGE = 1u << 3,      // |v| >= 16384
  ERR_SCORE_RANGE = 1u << 4,  // |score| >= 2^17
  ERR_TOKEN = 1u << 5,        // token id outside [0, vocab)
  ERR_TIMEOUT = 1u << 6,      // a bounded wait on an asynchronous copy gave up
};


// One OK_Q4B matrix resident in HBM: codes [rows][cols/2] (low nibble = even column),
// f16 block scales [rows][cols/32]; cols is padded to a multiple of 32 at upload.
struct DevQ4B {
  const uint8_t *codes;
  const uint16_t *scales;
  int rows, cols;
  int small;   // 1 when every block scale is below 128 in magnitude (f16 exponent field <= 21),
               // so each scale as the integer k = value * 2^24 fits in int32 (set after upload)
  // Row facts for the tensor-core GEMM (set after upload with launch_q4b_rowinfo): shift[r] =
  // the smallest exponent shift s = max(e - 1, 0) among row r's nonzero block scales, and
  // planes = the 8-bit digit planes (2..4) that hold every weight code * mantissa *
  // 2^(s_block - shift[r]) of the matrix as a two's-complement integer; 0 = not described.
  const uint8_t *shift;
  int planes;
  // optional (unless SPB_TC_PLANES=0): the `planes` digit planes precomputed once,
  // [planes][rows][cols] bytes in the activation column order, for the token-batch GEMM's TMA
  const uint8_t *pl;
};

// Fill w.pl (planes x rows x cols bytes) with the digit planes of w (described: shift, planes)
cudaError_t launch_q4b_planes(const DevQ4B &w, uint8_t *pl, cudaStream_t st);

// Per-row facts of an OK_Q4B matrix's block scales, one warp per row:
//   shift[r]  as DevQ4B::shift (0 for a row without a nonzero block)
//   info[0]  |= 1 when a row breaks the exact int64 accumulation bound (sum_b |k_b| * 32 * 8 * 127
//               must stay below 2^63, k_b the scale as an integer times 2^24) or holds an inf/NaN
//   info[1]   max= the largest f16 exponent field (DevQ4B::small iff <= 21)
//   info[2]   max= the largest spread max_b s_b - shift[r] over nonzero blocks
// info must be zero on entry.
cudaError_t launch_q4b_rowinfo(const uint16_t *scales, int rows, int nblk, uint8_t *shift, int *info,
                               cudaStream_t st);
// digit planes for a spread (2, 3, 4), or 0 beyond what the tensor-core GEMM covers
inline int q4b_planes_for_spread(int spread) { return spread <= 1 ? 2 : spread <= 9 ? 3 : spread <= 17 ? 4 : 0; }

// A quantized activation set: NTOK rows of K int8 codes in the GEMV's interleaved
// order (per 8-column group: even columns then odd columns), the per-32-block code
// sums, and each row's f32 scale (max |u|).
struct DevAct {
  int8_t *q;       // [ntok][K]
  int32_t *bsum;   // [ntok][K/32]
  float *scale;    // [ntok]
};

enum GemvEpi : int {
  EPI_STORE = 0,      // y[t][j] = acc -> f32
  EPI_GELU_MUL = 1,   // y[t][j] = gelu_exact(gate_j) * up_j   (two matrices)
  EPI_SILU_MUL = 2,   // y[t][j] = silu_exact(gate_j) * up_j
  EPI_I64 = 3,        // y viewed as int64: y[t][j] = the exact accumulator, unscaled (the partial
                      // sums of a K-split matrix, all-reduced before launch_scale_i64)
};
__host__ __device__ constexpr bool epi_pair(int epi) { return epi == EPI_GELU_MUL || epi == EPI_SILU_MUL; }
// bytes of one y element
__host__ __device__ constexpr int epi_bytes(int epi) { return epi == EPI_I64 ? 8 : 4; }

// y[t][j] for t < ntok over `w` (and `w2` for the gated epilogues). ymax (nullable):
// per-token slots receiving atomicMax of the f32 bits of max |y| (the next quantizer's scale).
// amax (nullable, zero on entry): per-token 64-bit greedy-argmax keys (first maximum).
// ws (nullable): int64 workspace of ws_elems for split-K token batches (2 * 64 * rows values
// for a K-halved matrix; without it every GEMM stays whole)
cudaError_t launch_gemv(const DevQ4B &w, const DevQ4B *w2, const DevAct &act, int ntok, float *y,
                        int ldy, int epi, uint32_t *err, cudaStream_t st, int grid_limit = 0,
                        uint32_t *ymax = nullptr, unsigned long long *amax = nullptr, int64_t *ws = nullptr,
                        size_t ws_elems = 0);

// The token-batch GEMM on the tcgen05 tensor cores (spb_gemm_tc.cu), from the digit planes of
// the described block scales (DevQ4B::shift / planes). covers: the planes it would run with, 0
// when it does not take this matrix (or pair). ks > 1 (EPI_I64 only) splits K into ks parts,
// part p writing its exact partial sums to y + p * ntok * ldy (int64 elements).
int gemm_tc_covers(const DevQ4B &w, const DevQ4B *w2, int epi, int ntok);
cudaError_t launch_gemm_tc(const DevQ4B &w, const DevQ4B *w2, const DevAct &act, int ntok, float *y, int ldy, int epi,
                           uint32_t *err, cudaStream_t st, uint32_t *ymax, unsigned long long *amax, int ks, bool pdl);

// y[t][j] = (float)(acc[t][j] * (scale[t] / 127 * 2^-24)), the GEMV epilogue's rounding, for
// n outputs of ntok rows (acc row stride n, y row stride ldy); with parts > 1, acc is the exact
// sum of the parts at acc + p * part_stride
cudaError_t launch_scale_i64(const int64_t *acc, const float *scale, int ntok, int n, float *y, int ldy,
                             cudaStream_t st, int parts = 1, size_t part_stride = 0);
// greedy-argmax keys of a row slice starting at global row `base` -> keys over global rows
cudaError_t launch_keys_rebase(unsigned long long *keys, int ntok, int base, cudaStream_t st);

// Quantize ntok rows of K floats (row stride ldu) into `act`. maxslot: per-row max |u| as
// f32 bits already produced upstream; NULL computes it first.
cudaError_t launch_quant(const float *u, int ldu, int K, int ntok, const DevAct &act,
                         const uint32_t *maxslot, uint32_t *err, cudaStream_t st);

// Residual + RMSNorm + quantization block (one CTA per token row):
//   if add:    t = add_w ? rmsnorm_exact(add, add_w) : add;  x += t
//   nx = rmsnorm_exact(x, out_w);  act <- quant(nx);  (nx also stored when nx_out)
// zero_slot (nullable): per-row max slots cleared for the next producing kernel.
cudaError_t launch_norm(float *x, const float *add, const float *add_w, const float *out_w, int E,
                        int ntok, const DevAct &act, float *nx_out, uint32_t *err, cudaStream_t st,
                        uint32_t *zero_slot = nullptr);

// Where one session's cached K/V rows live: pages of `pg` positions, the session's page j at
// physical page ptab[j] of a pool whose pages are laid out [NL][NKV][pg][HD] int32 (K and V in
// separate pools, the same page index in both). ptab == nullptr: the session's own single page,
// pg = its capacity, i.e. the contiguous [NL][NKV][P][HD] cache.
struct KvPages {
  int32_t *k, *v;
  const int32_t *ptab;
  int pg;
  // rb > 0: the rows are Spinor blocks (rb = ceil(HD / 55) * 63 bytes per position and KV head),
  // k and v then point at bytes laid out [NL][NKV][pg][rb]; single page only (ptab == nullptr)
  int rb = 0;
};

// byte offset of (layer L, KV head g, position p) in a Spinor-block cache (kv.rb > 0)
__host__ __device__ inline size_t kv_spin_off(const KvPages &kv, int NKV, int L, int g, int p) {
  return (((size_t)L * NKV + g) * (size_t)kv.pg + (size_t)p) * (size_t)kv.rb;
}

// element offset of (layer L, KV head g, position p) in k or v; the page table is read where it
// lives (device code: device tables; host code: a host copy)
__host__ __device__ inline size_t kv_elem(const KvPages &kv, int NL, int NKV, int HD, int L, int g, int p) {
  const int j = p / kv.pg;
  const size_t page = kv.ptab ? (size_t)kv.ptab[j] : 0;
  return ((page * NL + L) * NKV + g) * (size_t)kv.pg * HD + (size_t)(p - j * kv.pg) * HD;
}

// One token row of a multi-session batch: its session's K/V pages, the row's position and the
// session's capacity P.
struct BatchRow {
  KvPages kv;
  int32_t pos, P;
};

struct RopeArgs {
  const float *qkv;        // [ntok][QD + 2*KVD] projections
  int32_t *qi;             // [ntok][QD] rotated q on the 2^16 grid
  KvPages kv;              // the session's K/V pages (unused with rows)
  int NL;                  // layers (the page layout's stride)
  const float *q_norm, *k_norm;  // nullable when the model has no QK-norm
  const uint64_t *W;       // turn table [HD/2]
  const uint64_t *T;       // CORDIC arctangent table [30]
  uint64_t gain;           // CORDIC gain compensation, Q62
  const int32_t *pos_dev;  // device position of token row 0 (rows t use pos+t)
  int NH, NKV, HD, P, ntok;
  uint32_t *err;
  uint32_t *zero_slot;     // nullable: per-row max slots cleared for the attention output
  const BatchRow *rows;    // nullable: rows of different sessions (kv, P, pos_dev unused)
  int layer;               // the layer whose cache rows are written
  int rows_spin;           // with rows: 1 when any row keeps Spinor blocks (sizes the shared memory)
};
cudaError_t launch_rope_kv(const RopeArgs &a, cudaStream_t st);

struct AttnArgs {
  const int32_t *qi;       // [ntok][NH*HD]
  KvPages kv;              // the session's K/V pages (unused with rows)
  int NL;                  // layers (the page layout's stride)
  float *ao;               // [ntok][NH*HD]
  const int32_t *pos_dev;  // position of token row 0
  int NH, NKV, HD, P, win, ntok;
  float ascale;
  uint32_t *err;
  uint32_t *ao_max;        // nullable: per-row atomicMax of the f32 bits of max |ao|
  const BatchRow *rows;    // nullable: rows of different sessions (kv, pos_dev unused;
                           // P = the largest capacity, sizes the shared memory)
  int layer;               // the layer whose cache rows are read
  // fused QK-norm + RoPE + K/V store, for rows whose only new position is their own (decode
  // rows, batch rows): with qkv set, every CTA normalises and rotates its query heads itself
  // (qi unused) and the CTA whose position slice ends at the new position stores that
  // position's rotated K row and quantized V row (as k_rope_kv does)
  const float *qkv;        // nullable: [ntok][QD + 2*KVD] projections
  const float *q_norm, *k_norm;
  const uint64_t *W, *T;
  uint64_t gain;
  int own_pct;             // set by launch_attn: the owning rank's share of positions (percent)
  int rows_spin;           // with rows: 1 when any row keeps Spinor blocks (sizes the shared memory)
};
cudaError_t launch_attn(const AttnArgs &a, cudaStream_t st);

cudaError_t launch_embed(const DevQ4B &emb, const int32_t *tok_dev, int ntok, float scale, int use_scale,
                         float *x, int vocab, uint32_t *err, cudaStream_t st);
// token ids from the LM-head GEMV's argmax keys (and clear the keys)
cudaError_t launch_argmax_take(unsigned long long *keys, int ntok, int32_t *out, cudaStream_t st);
cudaError_t launch_advance(int32_t *pos_dev, int n, const int32_t *src_tok, int32_t *dst_tok,
                           cudaStream_t st);

// counter-based synthetic weights (same generator as spmodel.py)
cudaError_t launch_synth_codes(uint8_t *dst, size_t nbytes, uint64_t key, cudaStream_t st);
cudaError_t launch_synth_scales(uint16_t *dst, int rows, int nblk_src, int nblk_dst, int exp_field,
                                uint64_t key, cudaStream_t st);
// column slices of a generated matrix: rows of dst_row_bytes (scales: nblk_dst) taken at byte
// (block) offset src_off of source rows src_row_bytes (nblk_src) long; keys as above
cudaError_t launch_synth_codes_cols(uint8_t *dst, int rows, size_t dst_row_bytes, size_t src_row_bytes,
                                   size_t src_off, uint64_t key, cudaStream_t st);
cudaError_t launch_synth_scales_cols(uint16_t *dst, int rows, int nblk_dst, int nblk_src, int blk_off,
                                    int exp_field, uint64_t key, cudaStream_t st);
cudaError_t launch_synth_norm(float *dst, int n, uint64_t key, cudaStream_t st);

// store `msg` as this thread's spb_last_error() text and return `code` (host runtime)
int record_error(int code, const char *msg);

// isolated islands (parity tests)
cudaError_t launch_rmsnorm_rows(const float *x, const float *w, int n, int rows, float *out, uint32_t *err,
                                cudaStream_t st);
cudaError_t launch_eltwise(const float *x, int n, float *out, int op, uint32_t *err, cudaStream_t st);
cudaError_t launch_rope_rows(const float *v, int d, int rows, const int32_t *pos, const uint64_t *W,
                             const uint64_t *T, uint64_t gain, int32_t *out, uint32_t *err, cudaStream_t st);

}  // namespace spb
