// spb_runtime.cu -- host runtime of libspb200.so: model residency in HBM, resident
// exact KV sessions, the per-token kernel schedule (captured once as a CUDA graph),
// integer RoPE/CORDIC tables, and the C ABI declared in include/spb200.h.
//
// Schedule of one token row (decode; prefill runs the same schedule on chunks of up to 64
// rows, whose GEMVs become the tensor-core token-batch GEMM from 16 rows on):
//   embed -> per layer { norm(+residual)+quant -> GEMV Q|K|V -> QK-norm+CORDIC-RoPE+KV
//   store -> cluster attention -> quant -> GEMV O -> norm(+sandwich)+quant -> GEMV
//   gate|up with the exact GELU/SiLU * up epilogue -> quant -> GEMV down }
//   -> final norm+quant -> GEMV LM head -> argmax -> position advance.
// This mirrors kv_step_gemma3 (sp_session.c:380-464) and kv_step (sp_session.c:274-363).
#include "../../include/spb200.h"
#include "spb_kernels.cuh"
#include "spb_spinor.cuh"
#include "spb_tp.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

using namespace spb;

// ------------------------------------------------------------------------------ errors
static thread_local char g_err[512];

static int set_err(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

#define CU(call)                                                                              \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess)                                                                    \
      return set_err(e_ == cudaErrorMemoryAllocation ? SPB_EOOM : SPB_ECUDA, "%s: %s (%s:%d)", \
                     #call, cudaGetErrorString(e_), __FILE__, __LINE__);                      \
  } while (0)

extern "C" const char *spb_last_error(void) { return g_err; }

int spb::record_error(int code, const char *msg) { return set_err(code, "%s", msg); }

extern "C" int spb_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

static const char *err_bits_text(uint32_t b) {
  if (b & ERR_TOKEN) return "token id outside [0, vocab)";
  if (b & ERR_NORM_RANGE) return "RMSNorm input outside the exact range (|x| < 32768, sum x^2 < 2^31)";
  if (b & ERR_ACT_RANGE) return "activation outside the exact range (non-finite, or GELU/SiLU |x| >= 2048)";
  if (b & ERR_ROPE_RANGE) return "q/k outside the exact RoPE range (|x| < 256)";
  if (b & ERR_V_RANGE) return "v outside the exact range (|v| < 16384)";
  if (b & ERR_SCORE_RANGE) return "attention score outside the exact range (|z| < 2^17)";
  if (b & ERR_TIMEOUT) return "a bounded wait gave up (timeout)";
  return "unknown";
}

// ------------------------------------------------------------------------------ tables
// Integer-only tables of the CORDIC-RoPE (builder-defined: turns as Q64, Volder's
// micro-rotations, pi from Machin's formula with an integer arctangent series).
typedef unsigned __int128 u128;

static u128 atan_inv_q124(uint32_t m) {   // atan(1/m) * 2^124
  u128 p = ((u128)1 << 124) / m, m2 = (u128)m * m, sum = 0;
  bool add = true;
  for (uint32_t k = 1; p != 0; k += 2) {
    const u128 t = p / k;
    sum = add ? sum + t : sum - t;
    add = !add;
    p /= m2;
  }
  return sum;
}

static u128 two_pi_q124() { return 2 * (16 * atan_inv_q124(5) - 4 * atan_inv_q124(239)); }

static u128 atan_pow2_q124(int k) {       // atan(2^-k) * 2^124, k >= 1
  u128 p = (u128)1 << (124 - k), sum = 0;
  bool add = true;
  for (uint32_t n = 1; p != 0; n += 2) {
    const u128 t = p / n;
    sum = add ? sum + t : sum - t;
    add = !add;
    p >>= 2 * k;
  }
  return sum;
}

static u128 ratio_shift(u128 num, u128 den, int shift) {   // round(num * 2^shift / den), num < den
  u128 r = num, q = 0;
  for (int i = 0; i < shift; i++) {
    r <<= 1;
    q <<= 1;
    if (r >= den) { r -= den; q |= 1; }
  }
  if ((r << 1) >= den) q++;
  return q;
}

static u128 isqrt128(u128 v) {
  u128 res = 0, bit = (u128)1 << 126;
  while (bit > v) bit >>= 2;
  while (bit) {
    if (v >= res + bit) { v -= res + bit; res = (res >> 1) + bit; }
    else res >>= 1;
    bit >>= 2;
  }
  return res;
}

extern "C" void spb_cordic_tables(uint64_t T[30], uint64_t *gain_q62) {
  const u128 P = two_pi_q124();
  T[0] = 1ull << 61;
  for (int k = 1; k < 30; k++) T[k] = (uint64_t)ratio_shift(atan_pow2_q124(k), P, 64);
  u128 g = (u128)1 << 62;
  for (int k = 0; k < 30; k++) g = (g << 62) / isqrt128(((u128)1 << 124) + ((u128)1 << (124 - 2 * k)));
  if (gain_q62) *gain_q62 = (uint64_t)g;
}

extern "C" int spb_rope_freq_table(float base, int d, uint64_t *W) {
  uint32_t bits;
  memcpy(&bits, &base, 4);
  const uint32_t e8 = (bits >> 23) & 0xFFu, mant = bits & 0x7FFFFFu;
  if ((bits >> 31) || e8 < 127u || e8 == 255u || d <= 0 || (d & 1) || !W)
    return set_err(SPB_EBADARG, "spb_rope_freq_table: base must be finite and >= 1, d even");
  u128 y = (u128)(mant | 0x800000u) << 39, L = 0;   // log2(mantissa), Q62, bit by bit
  for (int j = 1; j <= 62; j++) {
    y = (y * y) >> 62;
    if (y >= ((u128)1 << 63)) { y >>= 1; L |= (u128)1 << (62 - j); }
  }
  L += (u128)(e8 - 127u) << 62;
  u128 c[63];                                        // c_j = 2^(-2^-j), Q62
  c[1] = isqrt128((u128)1 << 123);
  for (int j = 2; j <= 62; j++) c[j] = isqrt128(c[j - 1] << 62);
  const u128 P = two_pi_q124();
  for (int i = 0; i < d / 2; i++) {
    const u128 t = ((u128)(2 * i) * L) / (u128)d;
    const u128 n = t >> 62, f = t & (((u128)1 << 62) - 1);
    u128 r = (u128)1 << 62;
    for (int j = 1; j <= 62; j++)
      if ((f >> (62 - j)) & 1) r = (r * c[j]) >> 62;
    W[i] = n > 126 ? 0 : (uint64_t)ratio_shift(r, P, 126 - (int)n);
  }
  return SPB_OK;
}

// ------------------------------------------------------------------------------ model
struct DevLayer {
  DevQ4B qkv, o, g, u, d;
  const float *attn_norm, *q_norm, *k_norm, *post_attn, *ffn_norm, *post_ffw;
  bool global;
  int win;
};

struct spb_model {
  int device;
  spb_config cfg;
  int E, FF, NH, NKV, HD, QD, KVD, V, NL;
  bool gemma;
  uint8_t *wbuf = nullptr;
  size_t wbytes = 0;
  std::vector<DevLayer> layers;
  DevQ4B embd{}, out{};
  const float *out_norm = nullptr;
  uint64_t *tabs = nullptr;   // [0,30) CORDIC atan, [32, 32+HD/2) global W, then local W
  uint64_t gain = 0;
  float es = 1.0f;
  int64_t stream_bytes = 0;
  // tensor parallel: this rank's shard (NH, NKV, FF local; V = its LM-head rows [vbase, vbase+V)
  // of Vfull); without a group Vfull == V and vbase == 0
  spb_tp *tp = nullptr;
  int Vfull = 0, vbase = 0;
  bool out_sep = false;   // the LM head has its own storage (untied, or a vocabulary slice)
  uint8_t *shifts = nullptr;   // every matrix's DevQ4B::shift rows (one allocation)
  uint8_t *pbuf = nullptr;     // the layer matrices' precomputed digit planes (tc_planes_enabled)
  // closed sessions' device buffers, streams and pinned staging, handed to the next open that
  // fits (a clone-and-close loop then neither allocates nor synchronises the device)
  struct Spare { uint8_t *buf; size_t bytes; cudaStream_t st; void *h_pinned, *h_rows, *h_argmax; };
  std::mutex spare_mu;
  std::vector<Spare> spares;
};

static int describe_matrices(spb_model *m);

static size_t q4b_bytes(int rows, int cols) { return (size_t)rows * (cols / 2) + (size_t)rows * (cols / 32) * 2; }

static int check_cfg(const spb_config &c) {
  if (c.n_layers <= 0 || c.n_embd <= 0 || c.n_ff <= 0 || c.n_head <= 0 || c.n_head_kv <= 0 || c.n_vocab <= 0)
    return set_err(SPB_EBADARG, "spb: non-positive model dimension");
  if (c.arch != SPB_ARCH_QWEN3 && c.arch != SPB_ARCH_GEMMA3) return set_err(SPB_EUNSUPPORTED, "spb: arch %d", c.arch);
  if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256)
    return set_err(SPB_EUNSUPPORTED, "spb: head_dim %d not in {64,128,256}", c.head_dim);
  if (c.n_head % c.n_head_kv || c.n_head / c.n_head_kv > 8)
    return set_err(SPB_EUNSUPPORTED, "spb: n_head/n_head_kv must be an integer <= 8");
  if ((c.n_embd & 31) || ((c.n_head * c.head_dim) & 31) || (c.n_ff & 31))
    return set_err(SPB_EUNSUPPORTED, "spb: n_embd, n_head*head_dim and n_ff must be multiples of 32");
  if (c.n_embd > 16384) return set_err(SPB_EUNSUPPORTED, "spb: n_embd > 16384");
  return SPB_OK;
}

// nv_out > 0: a vocabulary slice of nv_out LM-head rows (tensor parallel), stored apart from
// the whole embedding table
static int model_alloc(const spb_config &c, int device, spb_model **out, int nv_out = 0) {
  int rc = check_cfg(c);
  if (rc) return rc;
  CU(cudaSetDevice(device));
  spb_model *m = new spb_model();
  m->device = device;
  m->cfg = c;
  m->E = c.n_embd; m->FF = c.n_ff; m->NH = c.n_head; m->NKV = c.n_head_kv; m->HD = c.head_dim;
  m->QD = c.n_head * c.head_dim; m->KVD = c.n_head_kv * c.head_dim; m->NL = c.n_layers;
  m->Vfull = c.n_vocab;
  m->V = nv_out > 0 ? nv_out : c.n_vocab;
  m->gemma = c.arch == SPB_ARCH_GEMMA3;
  m->out_sep = !m->gemma || nv_out > 0;
  m->es = sqrtf((float)m->E);
  // layout: per layer qkv, o, gate, up, down, then norms; embedding; LM head (if untied)
  size_t off = 0;
  auto take = [&](size_t n) { size_t o = off; off = (off + n + 255) & ~(size_t)255; return o; };
  struct Off { size_t qkv_c, qkv_s, o_c, o_s, g_c, g_s, u_c, u_s, d_c, d_s, norms; };
  std::vector<Off> lo(m->NL);
  const int QKV = m->QD + 2 * m->KVD;
  const int nnorm = 4 * m->E + 2 * m->HD;   // attn, post_attn, ffn, post_ffw, q, k
  for (int L = 0; L < m->NL; L++) {
    Off &o = lo[L];
    o.qkv_c = take((size_t)QKV * m->E / 2); o.qkv_s = take((size_t)QKV * (m->E / 32) * 2);
    o.o_c = take((size_t)m->E * m->QD / 2); o.o_s = take((size_t)m->E * (m->QD / 32) * 2);
    o.g_c = take((size_t)m->FF * m->E / 2); o.g_s = take((size_t)m->FF * (m->E / 32) * 2);
    o.u_c = take((size_t)m->FF * m->E / 2); o.u_s = take((size_t)m->FF * (m->E / 32) * 2);
    o.d_c = take((size_t)m->E * m->FF / 2); o.d_s = take((size_t)m->E * (m->FF / 32) * 2);
    o.norms = take((size_t)nnorm * 4);
  }
  const size_t emb_c = take((size_t)m->Vfull * m->E / 2), emb_s = take((size_t)m->Vfull * (m->E / 32) * 2);
  const bool untied = m->out_sep;
  size_t out_c = 0, out_s = 0;
  if (untied) { out_c = take((size_t)m->V * m->E / 2); out_s = take((size_t)m->V * (m->E / 32) * 2); }
  const size_t onorm = take((size_t)m->E * 4);
  const size_t tabs = take((size_t)(32 + m->HD) * 8);
  m->wbytes = off;
  cudaError_t e = cudaMalloc(&m->wbuf, off);
  if (e != cudaSuccess) {
    delete m;
    return set_err(SPB_EOOM, "spb_model: cudaMalloc(%zu): %s", off, cudaGetErrorString(e));
  }
  uint8_t *B = m->wbuf;
  m->layers.resize(m->NL);
  const int period = c.swa_period > 0 ? c.swa_period : 6;
  for (int L = 0; L < m->NL; L++) {
    const Off &o = lo[L];
    DevLayer &d = m->layers[L];
    d.qkv = {B + o.qkv_c, (const uint16_t *)(B + o.qkv_s), QKV, m->E};
    d.o = {B + o.o_c, (const uint16_t *)(B + o.o_s), m->E, m->QD};
    d.g = {B + o.g_c, (const uint16_t *)(B + o.g_s), m->FF, m->E};
    d.u = {B + o.u_c, (const uint16_t *)(B + o.u_s), m->FF, m->E};
    d.d = {B + o.d_c, (const uint16_t *)(B + o.d_s), m->E, m->FF};
    const float *nb = (const float *)(B + o.norms);
    d.attn_norm = nb; d.post_attn = nb + m->E; d.ffn_norm = nb + 2 * m->E; d.post_ffw = nb + 3 * m->E;
    d.q_norm = c.has_qk_norm ? nb + 4 * m->E : nullptr;
    d.k_norm = c.has_qk_norm ? nb + 4 * m->E + m->HD : nullptr;
    d.global = !m->gemma || (L % period) == period - 1;
    d.win = (m->gemma && !d.global && c.sliding_window > 0) ? c.sliding_window : -1;
  }
  m->embd = {B + emb_c, (const uint16_t *)(B + emb_s), m->Vfull, m->E};
  m->out = untied ? DevQ4B{B + out_c, (const uint16_t *)(B + out_s), m->V, m->E} : m->embd;
  m->out_norm = (const float *)(B + onorm);
  m->tabs = (uint64_t *)(B + tabs);
  // tables
  std::vector<uint64_t> ht(32 + m->HD, 0);
  spb_cordic_tables(ht.data(), &m->gain);
  rc = spb_rope_freq_table(c.rope_base, m->HD, ht.data() + 32);
  if (!rc) rc = spb_rope_freq_table(m->gemma ? c.rope_base_local : c.rope_base, m->HD, ht.data() + 32 + m->HD / 2);
  if (rc) { cudaFree(m->wbuf); delete m; return rc; }
  e = cudaMemcpy(m->tabs, ht.data(), ht.size() * 8, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) { cudaFree(m->wbuf); delete m; return set_err(SPB_ECUDA, "spb_model: tables: %s", cudaGetErrorString(e)); }
  m->stream_bytes = (int64_t)m->NL * (int64_t)(q4b_bytes(QKV, m->E) + q4b_bytes(m->E, m->QD) +
                                              2 * q4b_bytes(m->FF, m->E) + q4b_bytes(m->E, m->FF)) +
                    (int64_t)q4b_bytes(m->V, m->E);
  *out = m;
  return SPB_OK;
}

// |acc| bound of the int64 block accumulation: sum_b |k_b| * 32 * 8 * 127 < 2^63
static bool q4b_bound_ok(const spb_q4b &w) {
  const int nblk = (w.cols + 31) / 32;
  const uint64_t lim = (1ull << 63) / (32u * 8u * 127u);
  for (int r = 0; r < w.rows; r++) {
    uint64_t s = 0;
    const uint16_t *bs = w.bscale + (size_t)r * nblk;
    for (int b = 0; b < nblk; b++) {
      const uint32_t h = bs[b], e = (h >> 10) & 31u, mant = h & 1023u;
      if (e == 31) return false;
      s += e ? (uint64_t)(mant | 1024u) << (e - 1) : mant;
      if (s >= lim) return false;
    }
  }
  return true;
}

// rows [r0, r0 + nr) x columns [c0, c0 + nc) of a host matrix of rows x cols into rows
// [row0, row0 + nr) of dst (nc columns wide); c0 and nc are multiples of 32
static int put_q4b_part(const spb_q4b &w, int rows, int cols, int r0, int nr, int c0, int nc, const DevQ4B &dst,
                        int row0, const char *what) {
  if (!w.codes || !w.bscale || w.rows != rows || w.cols != cols)
    return set_err(SPB_EBADARG, "spb_model_upload: %s shape [%d x %d], expected [%d x %d]", what, w.rows, w.cols,
                   rows, cols);
  if (!q4b_bound_ok(w))
    return set_err(SPB_ERANGE, "spb_model_upload: %s block scales exceed the exact int64 accumulation bound", what);
  CU(cudaMemcpy2D((void *)(dst.codes + (size_t)row0 * (nc / 2)), (size_t)nc / 2,
                  w.codes + (size_t)r0 * (cols / 2) + c0 / 2, (size_t)cols / 2, (size_t)nc / 2, nr,
                  cudaMemcpyHostToDevice));
  CU(cudaMemcpy2D((void *)(dst.scales + (size_t)row0 * (nc / 32)), (size_t)nc / 32 * 2,
                  w.bscale + (size_t)r0 * (cols / 32) + c0 / 32, (size_t)cols / 32 * 2, (size_t)nc / 32 * 2, nr,
                  cudaMemcpyHostToDevice));
  return SPB_OK;
}

static int put_q4b(const spb_q4b &w, int rows, int cols, const DevQ4B &dst, int row0, const char *what) {
  return put_q4b_part(w, rows, cols, 0, rows, 0, cols, dst, row0, what);
}

static int put_f32(const float *src, const float *dst, int n, const char *what) {
  if (!src) return set_err(SPB_EBADARG, "spb_model_upload: missing %s", what);
  CU(cudaMemcpy((void *)dst, src, (size_t)n * 4, cudaMemcpyHostToDevice));
  return SPB_OK;
}

// Copy a whole host model, or with sh (spb_tp_shard's ranges) the rank's slices of it, into m.
static int upload_fill(spb_model *m, const spb_model_desc *desc, const int32_t *sh) {
  const spb_config &full = desc->cfg;
  const int E = m->E, HD = m->HD, QDf = full.n_head * HD, KVDf = full.n_head_kv * HD, FFf = full.n_ff;
  const int q0 = sh ? sh[0] * HD : 0, kv0 = sh ? sh[2] * HD : 0, f0 = sh ? sh[4] : 0, v0 = sh ? sh[6] : 0;
  int rc = SPB_OK;
#define PUT(x)          \
  do {                  \
    rc = (x);           \
    if (rc) return rc;  \
  } while (0)
  for (int L = 0; L < m->NL; L++) {
    const spb_layer_desc &s = desc->layers[L];
    DevLayer &d = m->layers[L];
    PUT(put_q4b_part(s.wq, QDf, E, q0, m->QD, 0, E, d.qkv, 0, "attn_q"));
    PUT(put_q4b_part(s.wk, KVDf, E, kv0, m->KVD, 0, E, d.qkv, m->QD, "attn_k"));
    PUT(put_q4b_part(s.wv, KVDf, E, kv0, m->KVD, 0, E, d.qkv, m->QD + m->KVD, "attn_v"));
    PUT(put_q4b_part(s.wo, E, QDf, 0, E, q0, m->QD, d.o, 0, "attn_output"));
    PUT(put_q4b_part(s.wg, FFf, E, f0, m->FF, 0, E, d.g, 0, "ffn_gate"));
    PUT(put_q4b_part(s.wu, FFf, E, f0, m->FF, 0, E, d.u, 0, "ffn_up"));
    PUT(put_q4b_part(s.wd, E, FFf, 0, E, f0, m->FF, d.d, 0, "ffn_down"));
    PUT(put_f32(s.attn_norm, d.attn_norm, m->E, "attn_norm"));
    PUT(put_f32(s.ffn_norm, d.ffn_norm, m->E, "ffn_norm"));
    if (m->gemma) {
      PUT(put_f32(s.post_attn_norm, d.post_attn, m->E, "post_attention_norm"));
      PUT(put_f32(s.post_ffw_norm, d.post_ffw, m->E, "post_ffw_norm"));
    }
    if (desc->cfg.has_qk_norm) {
      PUT(put_f32(s.q_norm, d.q_norm, m->HD, "attn_q_norm"));
      PUT(put_f32(s.k_norm, d.k_norm, m->HD, "attn_k_norm"));
    }
  }
  PUT(put_q4b(desc->token_embd, m->Vfull, m->E, m->embd, 0, "token_embd"));
  if (m->out_sep)
    PUT(put_q4b_part(m->gemma ? desc->token_embd : desc->output, m->Vfull, E, v0, m->V, 0, E, m->out, 0, "output"));
  PUT(put_f32(desc->output_norm, m->out_norm, m->E, "output_norm"));
  PUT(describe_matrices(m));
#undef PUT
  return SPB_OK;
}

extern "C" int spb_model_upload(const spb_model_desc *desc, int device, spb_model **out) {
  if (!desc || !out || !desc->layers) return set_err(SPB_EBADARG, "spb_model_upload: null arg");
  *out = nullptr;
  spb_model *m = nullptr;
  int rc = model_alloc(desc->cfg, device, &m);
  if (!rc) rc = upload_fill(m, desc, nullptr);
  if (rc) { spb_model_free(m); return rc; }
  *out = m;
  return SPB_OK;
}

// the rank's local geometry: its heads and FFN columns, the whole vocabulary for the embedding
static spb_config local_cfg(const spb_config &full, const int32_t sh[8]) {
  spb_config c = full;
  c.n_head = sh[1];
  c.n_head_kv = sh[3];
  c.n_ff = sh[5];
  return c;
}

extern "C" int spb_model_upload_tp(const spb_model_desc *desc, spb_tp *tp, spb_model **out) {
  if (!desc || !out || !desc->layers || !tp) return set_err(SPB_EBADARG, "spb_model_upload_tp: null arg");
  *out = nullptr;
  int32_t sh[8];
  int rc = spb_tp_shard(&desc->cfg, spb_tp_rank(tp), spb_tp_world(tp), sh);
  if (rc) return rc;
  spb_model *m = nullptr;
  rc = model_alloc(local_cfg(desc->cfg, sh), tp_device(tp), &m, sh[7]);
  if (rc) return rc;
  m->tp = tp;
  m->vbase = sh[6];
  rc = upload_fill(m, desc, sh);
  if (rc) { spb_model_free(m); return rc; }
  *out = m;
  return SPB_OK;
}

// SPB_TC_PLANES=0: the token-batch GEMM converts OK_Q4B codes into digit planes inside every CTA
// instead of loading planes precomputed once per matrix (comparisons; the same bytes). The
// planes cost planes x rows x cols bytes (about 2 bytes per weight); without room for them the
// converters stay.
static bool tc_planes_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_TC_PLANES");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}

// Describe every matrix's block scales once (launch_q4b_rowinfo): the exact-range check, the
// small-scale flag of the token-batch GEMM and the per-row shifts and digit planes of the
// tensor-core GEMM. A matrix outside the exact int64 bound is refused with SPB_ERANGE.
static int describe_matrices(spb_model *m) {
  std::vector<DevQ4B *> ws;
  for (DevLayer &d : m->layers) {
    ws.push_back(&d.qkv); ws.push_back(&d.o); ws.push_back(&d.g); ws.push_back(&d.u); ws.push_back(&d.d);
  }
  ws.push_back(&m->embd);
  if (m->out_sep) ws.push_back(&m->out);
  size_t nrows = 0;
  for (DevQ4B *w : ws) nrows += ((size_t)w->rows + 255) & ~(size_t)255;
  cudaFree(m->shifts);
  m->shifts = nullptr;
  int *dev = nullptr;
  CU(cudaMalloc(&m->shifts, nrows));
  CU(cudaMalloc(&dev, ws.size() * 4 * sizeof(int)));
  cudaError_t e = cudaMemset(dev, 0, ws.size() * 4 * sizeof(int));
  size_t off = 0;
  for (size_t i = 0; i < ws.size() && e == cudaSuccess; i++) {
    ws[i]->shift = m->shifts + off;
    e = launch_q4b_rowinfo(ws[i]->scales, ws[i]->rows, ws[i]->cols / 32, m->shifts + off, dev + 4 * i, 0);
    off += ((size_t)ws[i]->rows + 255) & ~(size_t)255;
  }
  std::vector<int> info(ws.size() * 4, 0);
  if (e == cudaSuccess) e = cudaMemcpy(info.data(), dev, info.size() * sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(dev);
  if (e != cudaSuccess) return set_err(SPB_ECUDA, "spb_model: scale check: %s", cudaGetErrorString(e));
  for (size_t i = 0; i < ws.size(); i++) {
    if (info[4 * i]) return set_err(SPB_ERANGE, "spb_model: block scales exceed the exact int64 accumulation bound");
    ws[i]->small = info[4 * i + 1] <= 21 ? 1 : 0;
    ws[i]->planes = q4b_planes_for_spread(info[4 * i + 2]);
  }
  if (!m->out_sep) m->out = m->embd;
  // every layer matrix's digit planes precomputed once (planes x rows x cols bytes, ~2 bytes per
  // weight at two planes) for the prefill GEMM's TMA; the embedding and LM head keep the
  // converters (no prefill logits beyond the last chunk's 64 rows)
  cudaFree(m->pbuf);
  m->pbuf = nullptr;
  if (tc_planes_enabled()) {
    const size_t nlayer = ws.size() - (m->out_sep ? 2 : 1);
    size_t bytes = 0;
    for (size_t i = 0; i < nlayer; i++)
      if (ws[i]->planes >= 2 && ws[i]->cols % 128 == 0)
        bytes += ((size_t)ws[i]->planes * ws[i]->rows * ws[i]->cols + 255) & ~(size_t)255;
    if (bytes && cudaMalloc(&m->pbuf, bytes) == cudaSuccess) {
      size_t o = 0;
      for (size_t i = 0; i < nlayer && e == cudaSuccess; i++) {
        if (ws[i]->planes < 2 || ws[i]->cols % 128) continue;
        ws[i]->pl = m->pbuf + o;
        e = launch_q4b_planes(*ws[i], m->pbuf + o, 0);
        o += ((size_t)ws[i]->planes * ws[i]->rows * ws[i]->cols + 255) & ~(size_t)255;
      }
      if (e == cudaSuccess) e = cudaDeviceSynchronize();
      if (e != cudaSuccess) return set_err(SPB_ECUDA, "spb_model: digit planes: %s", cudaGetErrorString(e));
    } else {
      (void)cudaGetLastError();   // no room for the planes: the converters stay
    }
  }
  return SPB_OK;
}

// splitmix64 key of a generator stream (matches spmodel.stream_key)
static uint64_t splitmix64_h(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static uint64_t stream_key(uint64_t seed, uint64_t stream) { return splitmix64_h(seed * 0x10001ull + stream); }
static int scale_exp_field(int cols) { return (int)std::floor(std::log2(1.0 / (8.0 * std::sqrt((double)cols)))) + 15; }

// rows [src_row0, src_row0 + rows) of generator stream `tid` (a cols-wide matrix) into rows
// [row0, row0 + rows) of d: the generators count words (codes) and blocks (scales) from the
// matrix start, so a row offset is a key offset
static int synth_matrix(const DevQ4B &d, int row0, int rows, int cols, int tid, uint64_t seed, int src_row0 = 0) {
  CU(launch_synth_codes((uint8_t *)d.codes + (size_t)row0 * (cols / 2), (size_t)rows * (cols / 2),
                        stream_key(seed, 2ull * tid) + (uint64_t)src_row0 * (cols / 16), 0));
  CU(launch_synth_scales((uint16_t *)d.scales + (size_t)row0 * (cols / 32), rows, cols / 32, cols / 32,
                         scale_exp_field(cols), stream_key(seed, 2ull * tid + 1) + (uint64_t)src_row0 * (cols / 32),
                         0));
  return SPB_OK;
}

// columns [c0, c0 + d.cols) of generator stream `tid` (a rows x cols_full matrix) into d
static int synth_matrix_cols(const DevQ4B &d, int cols_full, int c0, int tid, uint64_t seed) {
  CU(launch_synth_codes_cols((uint8_t *)d.codes, d.rows, (size_t)d.cols / 2, (size_t)cols_full / 2, (size_t)c0 / 2,
                             stream_key(seed, 2ull * tid), 0));
  CU(launch_synth_scales_cols((uint16_t *)d.scales, d.rows, d.cols / 32, cols_full / 32, c0 / 32,
                              scale_exp_field(cols_full), stream_key(seed, 2ull * tid + 1), 0));
  return SPB_OK;
}

// Generate the whole model, or with sh (spb_tp_shard's ranges) the rank's slices of the model
// `full` describes, into m.
static int synth_fill(spb_model *m, const spb_config &full, uint64_t seed, const int32_t *sh) {
  const int HD = m->HD, QDf = full.n_head * HD, FFf = full.n_ff;
  const int q0 = sh ? sh[0] * HD : 0, kv0 = sh ? sh[2] * HD : 0, f0 = sh ? sh[4] : 0, v0 = sh ? sh[6] : 0;
  int rc = SPB_OK;
  // stream ids: globals 1..3, layer L field f -> 64 + 64 L + f (spmodel.LAYER_FIELDS order)
  enum { F_ATTN_NORM, F_Q, F_K, F_V, F_O, F_QN, F_KN, F_POST_ATTN, F_FFN_NORM, F_GATE, F_UP, F_DOWN, F_POST_FFW };
  auto lid = [](int L, int f) { return 64 + 64 * L + f; };
  for (int L = 0; L < m->NL && !rc; L++) {
    DevLayer &d = m->layers[L];
    rc = synth_matrix(d.qkv, 0, m->QD, m->E, lid(L, F_Q), seed, q0);
    if (!rc) rc = synth_matrix(d.qkv, m->QD, m->KVD, m->E, lid(L, F_K), seed, kv0);
    if (!rc) rc = synth_matrix(d.qkv, m->QD + m->KVD, m->KVD, m->E, lid(L, F_V), seed, kv0);
    if (!rc) rc = synth_matrix_cols(d.o, QDf, q0, lid(L, F_O), seed);
    if (!rc) rc = synth_matrix(d.g, 0, m->FF, m->E, lid(L, F_GATE), seed, f0);
    if (!rc) rc = synth_matrix(d.u, 0, m->FF, m->E, lid(L, F_UP), seed, f0);
    if (!rc) rc = synth_matrix_cols(d.d, FFf, f0, lid(L, F_DOWN), seed);
    struct { const float *p; int n, f; } norms[] = {
        {d.attn_norm, m->E, F_ATTN_NORM}, {d.ffn_norm, m->E, F_FFN_NORM}, {d.post_attn, m->E, F_POST_ATTN},
        {d.post_ffw, m->E, F_POST_FFW}, {d.q_norm, m->HD, F_QN}, {d.k_norm, m->HD, F_KN}};
    for (auto &nz : norms)
      if (!rc && nz.p) {
        cudaError_t e = launch_synth_norm((float *)nz.p, nz.n, stream_key(seed, 2ull * lid(L, nz.f)), 0);
        if (e != cudaSuccess) rc = set_err(SPB_ECUDA, "synth norm: %s", cudaGetErrorString(e));
      }
  }
  if (!rc) rc = synth_matrix(m->embd, 0, m->Vfull, m->E, 1, seed);
  if (!rc && m->out_sep) rc = synth_matrix(m->out, 0, m->V, m->E, m->gemma ? 1 : 2, seed, v0);
  if (!rc) {
    cudaError_t e = launch_synth_norm((float *)m->out_norm, m->E, stream_key(seed, 2ull * 3), 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) rc = set_err(SPB_ECUDA, "synth: %s", cudaGetErrorString(e));
  }
  if (!rc) rc = describe_matrices(m);
  return rc;
}

extern "C" int spb_model_synthetic(const spb_config *cfg, uint64_t seed, int device, spb_model **out) {
  if (!cfg || !out) return set_err(SPB_EBADARG, "spb_model_synthetic: null arg");
  *out = nullptr;
  spb_model *m = nullptr;
  int rc = model_alloc(*cfg, device, &m);
  if (!rc) rc = synth_fill(m, *cfg, seed, nullptr);
  if (rc) { spb_model_free(m); return rc; }
  *out = m;
  return SPB_OK;
}

extern "C" int spb_model_synthetic_tp(const spb_config *cfg, uint64_t seed, spb_tp *tp, spb_model **out) {
  if (!cfg || !out || !tp) return set_err(SPB_EBADARG, "spb_model_synthetic_tp: null arg");
  *out = nullptr;
  int32_t sh[8];
  int rc = spb_tp_shard(cfg, spb_tp_rank(tp), spb_tp_world(tp), sh);
  if (rc) return rc;
  spb_model *m = nullptr;
  rc = model_alloc(local_cfg(*cfg, sh), tp_device(tp), &m, sh[7]);
  if (rc) return rc;
  m->tp = tp;
  m->vbase = sh[6];
  rc = synth_fill(m, *cfg, seed, sh);
  if (rc) { spb_model_free(m); return rc; }
  *out = m;
  return SPB_OK;
}

static void spare_destroy(const spb_model::Spare &p) {
  if (p.st) cudaStreamDestroy(p.st);
  cudaFreeHost(p.h_pinned);
  cudaFreeHost(p.h_rows);
  cudaFreeHost(p.h_argmax);
  cudaFree(p.buf);
}

// free every kept session buffer (model teardown, or an open that found no device memory)
static void spares_drop(spb_model *m) {
  std::vector<spb_model::Spare> v;
  {
    std::lock_guard<std::mutex> lk(m->spare_mu);
    v.swap(m->spares);
  }
  for (const auto &p : v) spare_destroy(p);
}

extern "C" void spb_model_free(spb_model *m) {
  if (!m) return;
  cudaSetDevice(m->device);
  spares_drop(m);
  cudaFree(m->wbuf);
  cudaFree(m->shifts);
  cudaFree(m->pbuf);
  delete m;
}

extern "C" int64_t spb_model_weight_bytes(const spb_model *m) { return m ? m->stream_bytes : 0; }

// ------------------------------------------------------------------------------ session
// A pool of K/V pages for the paged sessions of one model: page i holds `pg` positions of every
// layer and KV head, [NL][NKV][pg][HD] int32 for K at k + i * page_elems and for V likewise. A
// page is shared by the sessions whose page tables name it (refs) and copied before one of them
// writes into it while another still holds it (copy-on-write), so a clone costs its page table.
struct spb_kvpool {
  spb_model *m = nullptr;
  int pg = 0, npages = 0;
  size_t page_elems = 0;
  int32_t *k = nullptr, *v = nullptr;
  std::mutex mu;
  std::vector<int32_t> refs;        // sessions holding each page
  std::vector<int32_t> free_list;
};

constexpr int NT_MAX = 256;   // token rows per schedule pass (a prefill chunk without logits)
constexpr size_t SPARE_MAX_BYTES = (size_t)1 << 30;   // largest closed-session buffer kept for reuse
constexpr size_t SPARE_MAX = 16;                      // closed-session buffers kept per model
constexpr size_t SPARE_TOTAL_BYTES = (size_t)4 << 30; // and their bytes at most, per model

// SPB_SESSION_REUSE=0: every open allocates and every close frees (comparisons)
static bool session_reuse_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_SESSION_REUSE");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}
constexpr int LG_MAX = 64;    // token rows of a pass that produces logits (and of a decode batch)

struct spb_session {
  spb_model *m;
  int pmax;
  int pos;                        // host mirror of pos_dev
  cudaStream_t st = nullptr;
  uint8_t *buf = nullptr;         // one allocation for cache (unpaged) + scratch
  KvPages kv{};                   // where the K/V rows live: its own [NL][NKV][pmax][HD], or pool pages
  spb_kvpool *pool = nullptr;     // paged: the pool its pages come from
  std::vector<int32_t> pages;     // paged: host copy of its page table (-1: no page yet)
  int32_t *ptab_dev = nullptr;    // paged: the device page table [pages.size()]
  float *x, *qkv, *ao, *ap, *gg, *dn, *logits;
  int32_t *qi;
  DevAct act;
  int32_t *pos_dev, *tok_dev, *argmax_dev, *hist_dev;
  uint32_t *err_dev;
  uint32_t *ao_max, *gg_max;      // [NT_MAX] per-row max |y| slots (f32 bits) of the producers
  unsigned long long *amax_keys;  // [NT_MAX] greedy-argmax keys of the LM head (zero between steps)
  int32_t *h_pinned = nullptr;    // pinned staging: [0..NT_MAX) tokens, [NT_MAX] err, [NT_MAX+1] argmax
  BatchRow *rows_dev = nullptr;   // [NT_MAX] rows of a multi-session batch led by this session
  BatchRow *h_rows = nullptr;     // pinned staging for rows_dev
  int32_t *h_argmax = nullptr;    // pinned [NT_MAX] batch argmaxes
  cudaGraphExec_t step_graph = nullptr;
  size_t buf_bytes = 0;
  // tensor parallel: int64 partial sums of the K-split matrices [NT_MAX][E], this rank's LM-head
  // logits [LG_MAX][V] and the all-gathered slices [world][LG_MAX][V]
  int64_t *y64 = nullptr;
  float *logits_l = nullptr, *logits_g = nullptr;
  int64_t *ws = nullptr;          // split-K workspace of the token-batch GEMMs [4][NT_MAX][E]
  size_t ws_elems = 0;
  unsigned flags = 0;             // SPB_KV_SPINOR: K/V rows kept as Spinor blocks (kv.rb bytes each)
};

static size_t kv_layer_elems(const spb_model *m, int pmax) { return (size_t)m->NKV * pmax * m->HD; }

// bytes of one layer's Spinor-block K (or V) cache
static size_t kv_spin_layer_bytes(const spb_model *m, int pmax) {
  return (size_t)m->NKV * pmax * (size_t)spin_row_bytes(m->HD);
}

static int session_open(spb_model *m, int pmax, spb_kvpool *pool, spb_session **out, unsigned flags = 0) {
  if (!m || !out || pmax <= 0) return set_err(SPB_EBADARG, "spb_session_open: bad arg");
  *out = nullptr;
  if (flags & ~(unsigned)SPB_KV_SPINOR) return set_err(SPB_EBADARG, "spb_session_open_ex: unknown flags 0x%x", flags);
  const bool spin = (flags & SPB_KV_SPINOR) != 0;
  if (spin && (pool || m->HD < 64 || m->HD > 256 || (m->HD & (m->HD - 1))))
    return set_err(SPB_EUNSUPPORTED, "spb_session_open_ex: Spinor K/V needs an unpaged session and head_dim 64, 128 or 256");
  CU(cudaSetDevice(m->device));
  spb_session *s = new spb_session();
  s->m = m;
  s->pmax = pmax;
  s->pos = 0;
  s->pool = pool;
  const int npg = pool ? (pmax + pool->pg - 1) / pool->pg : 0;
  if (pool) s->pages.assign((size_t)npg, -1);
  const int E = m->E, QKV = m->QD + 2 * m->KVD, maxK = std::max(std::max(E, m->QD), m->FF);
  size_t off = 0;
  auto take = [&](size_t n) { size_t o = off; off = (off + n + 255) & ~(size_t)255; return o; };
  const size_t kvn = pool ? 0 : (size_t)m->NL * kv_layer_elems(m, pmax);
  // Spinor blocks: + 32 bytes, as the attention's bulk copies read 16-byte-aligned spans around a slice
  const size_t kvb = spin ? (size_t)m->NL * kv_spin_layer_bytes(m, pmax) + 32 : kvn * 4;
  const size_t o_kc = take(kvb), o_vc = take(kvb), o_ptab = take((size_t)npg * 4);
  const size_t o_x = take((size_t)NT_MAX * E * 4), o_qkv = take((size_t)NT_MAX * QKV * 4);
  const size_t o_ao = take((size_t)NT_MAX * m->QD * 4), o_ap = take((size_t)NT_MAX * E * 4);
  const size_t o_gg = take((size_t)NT_MAX * m->FF * 4), o_dn = take((size_t)NT_MAX * E * 4);
  const size_t o_lg = take((size_t)LG_MAX * m->Vfull * 4), o_qi = take((size_t)NT_MAX * m->QD * 4);
  const size_t o_y64 = m->tp ? take((size_t)NT_MAX * E * 8) : 0;
  const size_t o_ws = take((size_t)4 * NT_MAX * E * 8);
  const size_t o_lgl = m->tp ? take((size_t)LG_MAX * m->V * 4) : 0;
  const size_t o_lgg = m->tp ? take((size_t)LG_MAX * m->Vfull * 4) : 0;
  const size_t o_aq = take((size_t)NT_MAX * maxK), o_ab = take((size_t)NT_MAX * (maxK / 32) * 4);
  const size_t o_as = take(NT_MAX * 4), o_pos = take(4), o_tok = take(NT_MAX * 4), o_am = take(NT_MAX * 4);
  const size_t o_hist = take((size_t)pmax * 4), o_err = take(4), o_slots = take(2 * NT_MAX * 4);
  const size_t o_keys = take(NT_MAX * 8);
  const size_t o_rows = take(NT_MAX * sizeof(BatchRow));
  cudaError_t e = cudaSuccess;
  if (session_reuse_enabled()) {
    // the most recently closed buffer of exactly this size, else the smallest within 25 % above it
    std::lock_guard<std::mutex> lk(m->spare_mu);
    int pick = -1;
    for (int i = (int)m->spares.size() - 1; i >= 0; i--) {
      const size_t b = m->spares[i].bytes;
      if (b == off) { pick = i; break; }
      if (b > off && b - off <= off / 4 && (pick < 0 || b < m->spares[pick].bytes)) pick = i;
    }
    if (pick >= 0) {
      const spb_model::Spare p = m->spares[pick];
      s->buf = p.buf; s->buf_bytes = p.bytes; s->st = p.st;
      s->h_pinned = (int32_t *)p.h_pinned; s->h_rows = (BatchRow *)p.h_rows; s->h_argmax = (int32_t *)p.h_argmax;
      m->spares.erase(m->spares.begin() + pick);
    }
  }
  if (!s->buf) {
    e = cudaMalloc(&s->buf, off);
    if (e == cudaErrorMemoryAllocation) {
      cudaGetLastError();
      spares_drop(m);
      e = cudaMalloc(&s->buf, off);
    }
    if (e != cudaSuccess) {
      s->buf = nullptr;
      delete s;
      return set_err(SPB_EOOM, "spb_session_open: cudaMalloc(%zu): %s", off, cudaGetErrorString(e));
    }
    s->buf_bytes = off;
  }
  uint8_t *B = s->buf;
  if (pool) {
    s->ptab_dev = (int32_t *)(B + o_ptab);
    s->kv = KvPages{pool->k, pool->v, s->ptab_dev, pool->pg};
  } else {
    s->kv = KvPages{(int32_t *)(B + o_kc), (int32_t *)(B + o_vc), nullptr, pmax, spin ? spin_row_bytes(m->HD) : 0};
  }
  s->flags = flags;
  s->x = (float *)(B + o_x); s->qkv = (float *)(B + o_qkv); s->ao = (float *)(B + o_ao);
  s->ap = (float *)(B + o_ap); s->gg = (float *)(B + o_gg); s->dn = (float *)(B + o_dn);
  s->logits = (float *)(B + o_lg); s->qi = (int32_t *)(B + o_qi);
  s->act = {(int8_t *)(B + o_aq), (int32_t *)(B + o_ab), (float *)(B + o_as)};
  s->pos_dev = (int32_t *)(B + o_pos); s->tok_dev = (int32_t *)(B + o_tok); s->argmax_dev = (int32_t *)(B + o_am);
  s->hist_dev = (int32_t *)(B + o_hist); s->err_dev = (uint32_t *)(B + o_err);
  s->ao_max = (uint32_t *)(B + o_slots); s->gg_max = s->ao_max + NT_MAX;
  s->amax_keys = (unsigned long long *)(B + o_keys);
  s->rows_dev = (BatchRow *)(B + o_rows);
  s->ws = (int64_t *)(B + o_ws);
  s->ws_elems = (size_t)4 * NT_MAX * E;
  if (m->tp) {
    s->y64 = (int64_t *)(B + o_y64);
    s->logits_l = (float *)(B + o_lgl);
    s->logits_g = (float *)(B + o_lgg);
  }
  if (!s->st) e = cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking);
  if (e == cudaSuccess && !s->h_pinned) e = cudaMallocHost(&s->h_pinned, (NT_MAX + 4) * 4);
  if (e == cudaSuccess && !s->h_rows) e = cudaMallocHost(&s->h_rows, NT_MAX * sizeof(BatchRow));
  if (e == cudaSuccess && !s->h_argmax) e = cudaMallocHost(&s->h_argmax, NT_MAX * 4);
  if (e == cudaSuccess) e = cudaMemsetAsync(s->buf, 0, off, s->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->st);
  if (e != cudaSuccess) { spb_session_close(s); return set_err(SPB_ECUDA, "spb_session_open: %s", cudaGetErrorString(e)); }
  *out = s;
  return SPB_OK;
}

extern "C" int spb_session_open(spb_model *m, int pmax, spb_session **out) { return session_open(m, pmax, nullptr, out); }

extern "C" int spb_session_open_ex(spb_model *m, int pmax, unsigned flags, spb_session **out) {
  return session_open(m, pmax, nullptr, out, flags);
}

extern "C" int spb_session_open_paged(spb_kvpool *pool, int pmax, spb_session **out) {
  if (!pool) return set_err(SPB_EBADARG, "spb_session_open_paged: null pool");
  return session_open(pool->m, pmax, pool, out);
}

// give back this session's pages (after its stream has drained)
static void release_pages(spb_session *s) {
  if (!s->pool) return;
  std::lock_guard<std::mutex> lk(s->pool->mu);
  for (int32_t &pg : s->pages) {
    if (pg >= 0 && --s->pool->refs[pg] == 0) s->pool->free_list.push_back(pg);
    pg = -1;
  }
}

// Make positions [pos, pos + n) writable: every page they touch becomes this session's alone (a
// fresh page, or a copy of a page another session still holds), then the device page table
// follows. A copy is waited for before the other holder may write its page in place again.
static int prepare_write(spb_session *s, int pos, int n) {
  spb_kvpool *pool = s->pool;
  if (!pool || n <= 0) return SPB_OK;
  if (pos < 0 || pos + n > s->pmax) return set_err(SPB_ECONTEXT_FULL, "spb: context full");
  bool changed = false, copied = false;
  {
    std::lock_guard<std::mutex> lk(pool->mu);
    for (int j = pos / pool->pg; j <= (pos + n - 1) / pool->pg; j++) {
      const int cur = s->pages[j];
      if (cur >= 0 && pool->refs[cur] == 1) continue;
      if (pool->free_list.empty()) return set_err(SPB_EOOM, "spb: the KV page pool has no free page");
      const int np = pool->free_list.back();
      pool->free_list.pop_back();
      pool->refs[np] = 1;
      if (cur >= 0) {   // shared: copy before writing
        const size_t bytes = pool->page_elems * 4;
        CU(cudaMemcpyAsync(pool->k + (size_t)np * pool->page_elems, pool->k + (size_t)cur * pool->page_elems, bytes,
                           cudaMemcpyDeviceToDevice, s->st));
        CU(cudaMemcpyAsync(pool->v + (size_t)np * pool->page_elems, pool->v + (size_t)cur * pool->page_elems, bytes,
                           cudaMemcpyDeviceToDevice, s->st));
        pool->refs[cur]--;
        copied = true;
      }
      s->pages[j] = np;
      changed = true;
    }
  }
  if (changed)
    CU(cudaMemcpyAsync(s->ptab_dev, s->pages.data(), s->pages.size() * 4, cudaMemcpyHostToDevice, s->st));
  if (copied) CU(cudaStreamSynchronize(s->st));
  return SPB_OK;
}

extern "C" int spb_kvpool_create(spb_model *m, int page_positions, int n_pages, spb_kvpool **out) {
  if (!m || !out || n_pages <= 0 || page_positions < 128 || (page_positions % 128))
    return set_err(SPB_EBADARG, "spb_kvpool_create: page_positions a positive multiple of 128, n_pages > 0");
  *out = nullptr;
  CU(cudaSetDevice(m->device));
  spb_kvpool *p = new spb_kvpool();
  p->m = m;
  p->pg = page_positions;
  p->npages = n_pages;
  p->page_elems = (size_t)m->NL * m->NKV * page_positions * m->HD;
  const size_t bytes = p->page_elems * 4 * (size_t)n_pages;
  cudaError_t e = cudaMalloc(&p->k, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&p->v, bytes);
  if (e != cudaSuccess) {
    cudaFree(p->k);
    delete p;
    return set_err(SPB_EOOM, "spb_kvpool_create: cudaMalloc(2 x %zu): %s", bytes, cudaGetErrorString(e));
  }
  p->refs.assign((size_t)n_pages, 0);
  for (int i = n_pages - 1; i >= 0; i--) p->free_list.push_back(i);
  *out = p;
  return SPB_OK;
}

extern "C" void spb_kvpool_free(spb_kvpool *p) {
  if (!p) return;
  cudaSetDevice(p->m->device);
  cudaFree(p->k);
  cudaFree(p->v);
  delete p;
}

extern "C" int spb_kvpool_free_pages(spb_kvpool *p) {
  if (!p) return -1;
  std::lock_guard<std::mutex> lk(p->mu);
  return (int)p->free_list.size();
}

extern "C" void spb_session_close(spb_session *s) {
  if (!s) return;
  cudaSetDevice(s->m->device);
  if (s->st) cudaStreamSynchronize(s->st);
  release_pages(s);
  if (s->step_graph) cudaGraphExecDestroy(s->step_graph);
  const spb_model::Spare p{s->buf, s->buf_bytes, s->st, s->h_pinned, s->h_rows, s->h_argmax};
  spb_model *m = s->m;
  delete s;
  // kept for the next open: buffers of at most SPARE_MAX_BYTES (scratch and paged sessions, not
  // large private caches), only after a clean stream; the oldest make room for SPARE_MAX buffers
  // and SPARE_TOTAL_BYTES
  if (p.buf && p.st && p.h_pinned && p.h_rows && p.h_argmax && p.bytes <= SPARE_MAX_BYTES && session_reuse_enabled() &&
      cudaStreamQuery(p.st) == cudaSuccess) {
    std::vector<spb_model::Spare> old;
    {
      std::lock_guard<std::mutex> lk(m->spare_mu);
      m->spares.push_back(p);
      size_t total = 0;
      for (const auto &q : m->spares) total += q.bytes;
      while (m->spares.size() > 1 && (m->spares.size() > SPARE_MAX || total > SPARE_TOTAL_BYTES)) {
        total -= m->spares.front().bytes;
        old.push_back(m->spares.front());
        m->spares.erase(m->spares.begin());
      }
    }
    for (const auto &q : old) spare_destroy(q);
    return;
  }
  spare_destroy(p);
}

extern "C" void *spb_session_stream(spb_session *s) { return s ? (void *)s->st : nullptr; }
extern "C" int spb_session_position(const spb_session *s) { return s ? s->pos : -1; }

// SPB_ROPE_FUSED=0 keeps k_rope_kv as its own launch for decode rows too (comparisons; results
// are identical)
static bool rope_fused_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("SPB_ROPE_FUSED");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on != 0;
}

// Enqueue the schedule for nt rows (tokens already in tok_dev, positions at pos_dev). With
// rows (device, [nt]), row t belongs to its own session: RoPE/KV store and attention use that
// session's cache and position; Pmax is the largest of their capacities.
static cudaError_t enqueue_rows(spb_session *s, int nt, bool want_logits, const BatchRow *rows = nullptr,
                                int Pmax = 0, bool rows_spin = false) {
  spb_model *m = s->m;
  cudaStream_t st = s->st;
  const int E = m->E, QKV = m->QD + 2 * m->KVD;
  const float ascale = 1.0f / sqrtf((float)m->HD);
  cudaError_t e;
#define K(x)                        \
  do {                              \
    e = (x);                        \
    if (e != cudaSuccess) return e; \
  } while (0)
  K(launch_embed(m->embd, s->tok_dev, nt, m->es, m->gemma ? 1 : 0, s->x, m->Vfull, s->err_dev, st));
  // rows whose only new position is their own (a decode row, or rows of distinct sessions) get
  // QK-norm, RoPE and the K/V store inside the attention kernel; prefill chunks, whose rows read
  // each other's new K/V, keep the separate k_rope_kv
  const bool fuse_rope = (nt == 1 || rows != nullptr) && rope_fused_enabled();
  // a K-split matrix (tensor parallel): exact int64 partial sums, summed over the group, then
  // scaled with the GEMV's own rounding
  auto split_gemv = [&](const DevQ4B &w, float *y) -> cudaError_t {
    if (!m->tp) return launch_gemv(w, nullptr, s->act, nt, y, E, EPI_STORE, s->err_dev, st, 0, nullptr, nullptr, s->ws,
                                   s->ws_elems);
    cudaError_t r = launch_gemv(w, nullptr, s->act, nt, reinterpret_cast<float *>(s->y64), E, EPI_I64, s->err_dev, st);
    if (r == cudaSuccess) r = tp_sum_i64(m->tp, s->y64, (size_t)nt * E, st, s->err_dev);
    if (r == cudaSuccess) r = launch_scale_i64(s->y64, s->act.scale, nt, E, y, E, st);
    return r;
  };
  for (int L = 0; L < m->NL; L++) {
    const DevLayer &d = m->layers[L];
    // the attention norm also clears the attention output's max slots (filled by k_attn)
    if (L == 0) {
      K(launch_norm(s->x, nullptr, nullptr, d.attn_norm, E, nt, s->act, nullptr, s->err_dev, st, s->ao_max));
    } else {
      const DevLayer &p = m->layers[L - 1];
      K(launch_norm(s->x, s->dn, m->gemma ? p.post_ffw : nullptr, d.attn_norm, E, nt, s->act, nullptr, s->err_dev, st,
                    s->ao_max));
    }
    K(launch_gemv(d.qkv, nullptr, s->act, nt, s->qkv, QKV, EPI_STORE, s->err_dev, st));
    RopeArgs ra{};
    ra.rows = rows; ra.layer = L;
    ra.qkv = s->qkv; ra.qi = s->qi; ra.kv = s->kv; ra.NL = m->NL;
    ra.q_norm = d.q_norm; ra.k_norm = d.k_norm;
    ra.W = m->tabs + 32 + (d.global ? 0 : m->HD / 2);
    ra.T = m->tabs; ra.gain = m->gain; ra.pos_dev = s->pos_dev;
    ra.NH = m->NH; ra.NKV = m->NKV; ra.HD = m->HD; ra.P = s->pmax; ra.ntok = nt; ra.err = s->err_dev;
    ra.zero_slot = s->ao_max;
    ra.rows_spin = rows_spin ? 1 : 0;
    if (!fuse_rope) K(launch_rope_kv(ra, st));
    AttnArgs aa{};
    aa.rows = rows; aa.layer = L;
    aa.qi = s->qi; aa.kv = s->kv; aa.NL = m->NL; aa.ao = s->ao; aa.pos_dev = s->pos_dev;
    aa.NH = m->NH; aa.NKV = m->NKV; aa.HD = m->HD; aa.P = rows ? Pmax : s->pmax; aa.win = d.win; aa.ntok = nt;
    aa.ascale = ascale; aa.err = s->err_dev; aa.ao_max = s->ao_max;
    aa.rows_spin = rows_spin ? 1 : 0;
    if (fuse_rope) {
      aa.qkv = s->qkv; aa.q_norm = d.q_norm; aa.k_norm = d.k_norm;
      aa.W = ra.W; aa.T = m->tabs; aa.gain = m->gain;
    }
    K(launch_attn(aa, st));
    if (m->tp) K(tp_max_u32(m->tp, s->ao_max, nt, st, s->err_dev));   // the quantizer's max over all heads
    K(launch_quant(s->ao, m->QD, m->QD, nt, s->act, s->ao_max, s->err_dev, st));
    K(split_gemv(d.o, s->ap));
    K(launch_norm(s->x, s->ap, m->gemma ? d.post_attn : nullptr, d.ffn_norm, E, nt, s->act, nullptr, s->err_dev, st,
                  s->gg_max));
    K(launch_gemv(d.g, &d.u, s->act, nt, s->gg, m->FF, m->gemma ? EPI_GELU_MUL : EPI_SILU_MUL, s->err_dev, st, 0,
                  s->gg_max));
    if (m->tp) K(tp_max_u32(m->tp, s->gg_max, nt, st, s->err_dev));   // ... over all FFN columns
    K(launch_quant(s->gg, m->FF, m->FF, nt, s->act, s->gg_max, s->err_dev, st));
    K(split_gemv(d.d, s->dn));
  }
  if (want_logits) {
    const DevLayer &p = m->layers[m->NL - 1];
    K(launch_norm(s->x, s->dn, m->gemma ? p.post_ffw : nullptr, m->out_norm, E, nt, s->act, nullptr, s->err_dev, st));
    if (!m->tp) {
      K(launch_gemv(m->out, nullptr, s->act, nt, s->logits, m->V, EPI_STORE, s->err_dev, st, 0, nullptr,
                    s->amax_keys));
    } else {   // vocabulary rows [vbase, vbase + V): global argmax keys, then every rank's slice
      K(launch_gemv(m->out, nullptr, s->act, nt, s->logits_l, m->V, EPI_STORE, s->err_dev, st, 0, nullptr,
                    s->amax_keys));
      K(launch_keys_rebase(s->amax_keys, nt, m->vbase, st));
      K(tp_max_u64(m->tp, s->amax_keys, nt, st, s->err_dev));
      K(tp_gather_f32(m->tp, s->logits_l, s->logits_g, (size_t)nt * m->V, st));
      const int world = spb_tp_world(m->tp);
      for (int r = 0; r < world; r++)   // [rank][t][V] -> [t][rank * V + j]
        K(cudaMemcpy2DAsync(s->logits + (size_t)r * m->V, (size_t)m->Vfull * 4,
                            s->logits_g + (size_t)r * nt * m->V, (size_t)m->V * 4, (size_t)m->V * 4, nt,
                            cudaMemcpyDeviceToDevice, st));
    }
    K(launch_argmax_take(s->amax_keys, nt, s->argmax_dev, st));
  }
#undef K
  return cudaSuccess;
}

// read and clear the device error word; returns SPB_ERANGE on any raised bit
static int collect_errors(spb_session *s) {
  uint32_t *h = reinterpret_cast<uint32_t *>(s->h_pinned + NT_MAX);
  CU(cudaMemcpyAsync(h, s->err_dev, 4, cudaMemcpyDeviceToHost, s->st));
  CU(cudaMemsetAsync(s->err_dev, 0, 4, s->st));
  CU(cudaStreamSynchronize(s->st));
  // a bounded device wait that gave up is a device failure (SP_ECUDA), every other bit a value
  // that left the exact range
  if (*h & ERR_TIMEOUT) return set_err(SPB_ECUDA, "spb: %s (error bits 0x%x)", err_bits_text(ERR_TIMEOUT), *h);
  if (*h) return set_err(SPB_ERANGE, "spb: %s (error bits 0x%x)", err_bits_text(*h), *h);
  return SPB_OK;
}

static int sync_pos(spb_session *s) {
  CU(cudaMemcpyAsync(s->pos_dev, &s->pos, 4, cudaMemcpyHostToDevice, s->st));
  return SPB_OK;
}

extern "C" int spb_session_prefill(spb_session *s, const int32_t *tokens, int n_tok, float *logits) {
  if (!s || !tokens || n_tok <= 0) return set_err(SPB_EBADARG, "spb_session_prefill: bad arg");
  if (n_tok > s->pmax - s->pos) return set_err(SPB_ECONTEXT_FULL, "spb_session_prefill: context full");
  CU(cudaSetDevice(s->m->device));
  const int pos0 = s->pos;
  int rc = prepare_write(s, s->pos, n_tok);
  if (rc) return rc;
  rc = sync_pos(s);
  if (rc) return rc;
  int done = 0;
  while (done < n_tok) {
    int nt = logits ? LG_MAX : NT_MAX;   // the logits buffer holds LG_MAX rows
    while (nt > n_tok - done) nt >>= 1;
    memcpy(s->h_pinned, tokens + done, (size_t)nt * 4);
    CU(cudaMemcpyAsync(s->tok_dev, s->h_pinned, (size_t)nt * 4, cudaMemcpyHostToDevice, s->st));
    CU(enqueue_rows(s, nt, logits != nullptr));
    CU(launch_advance(s->pos_dev, nt, nullptr, nullptr, s->st));
    if (logits)
      CU(cudaMemcpyAsync(logits + (size_t)done * s->m->Vfull, s->logits, (size_t)nt * s->m->Vfull * 4,
                         cudaMemcpyDeviceToHost, s->st));
    // the pinned token staging is reused next chunk: wait for the H2D copy
    CU(cudaStreamSynchronize(s->st));
    done += nt;
  }
  rc = collect_errors(s);
  if (rc) { s->pos = pos0; sync_pos(s); cudaStreamSynchronize(s->st); return rc; }
  s->pos = pos0 + n_tok;
  return SPB_OK;
}

static int ensure_step_graph(spb_session *s) {
  if (s->step_graph) return SPB_OK;
  cudaGraph_t g = nullptr;
  CU(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
  cudaError_t e = enqueue_rows(s, 1, true);
  if (e == cudaSuccess) e = launch_advance(s->pos_dev, 1, s->argmax_dev, s->tok_dev, s->st);
  cudaError_t e2 = cudaStreamEndCapture(s->st, &g);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return set_err(SPB_ECUDA, "spb: graph capture: %s", cudaGetErrorString(e != cudaSuccess ? e : e2));
  }
  e = cudaGraphInstantiate(&s->step_graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return set_err(SPB_ECUDA, "spb: graph instantiate: %s", cudaGetErrorString(e));
  return SPB_OK;
}

extern "C" int spb_session_decode_step_argmax(spb_session *s, int32_t token, float *logits, int32_t *argmax) {
  if (!s) return set_err(SPB_EBADARG, "spb_session_decode_step: null session");
  if (s->pos >= s->pmax) return set_err(SPB_ECONTEXT_FULL, "spb_session_decode_step: context full");
  CU(cudaSetDevice(s->m->device));
  int rc = prepare_write(s, s->pos, 1);
  if (rc) return rc;
  rc = ensure_step_graph(s);
  if (rc) return rc;
  s->h_pinned[0] = token;
  CU(cudaMemcpyAsync(s->tok_dev, s->h_pinned, 4, cudaMemcpyHostToDevice, s->st));
  CU(cudaGraphLaunch(s->step_graph, s->st));
  if (logits) CU(cudaMemcpyAsync(logits, s->logits, (size_t)s->m->Vfull * 4, cudaMemcpyDeviceToHost, s->st));
  if (argmax) CU(cudaMemcpyAsync(s->h_pinned + NT_MAX + 1, s->argmax_dev, 4, cudaMemcpyDeviceToHost, s->st));
  rc = collect_errors(s);
  if (rc) { sync_pos(s); cudaStreamSynchronize(s->st); return rc; }
  if (argmax) *argmax = s->h_pinned[NT_MAX + 1];
  s->pos += 1;
  return SPB_OK;
}

extern "C" int spb_session_decode_step(spb_session *s, int32_t token, float *logits) {
  return spb_session_decode_step_argmax(s, token, logits, nullptr);
}

// One decode step for B sessions at once (each at its own position): one pass of the schedule
// over B token rows, so every weight matrix is streamed once for all of them and the GEMVs
// become the token-batch GEMM. ss[0] leads: its stream and scratch rows run the step.
extern "C" int spb_batch_decode_step(spb_session *const *ss, int B, const int32_t *tokens, float *logits,
                                     int32_t *argmax) {
  if (!ss || !tokens || B <= 0 || B > LG_MAX) return set_err(SPB_EBADARG, "spb_batch_decode_step: B in [1, %d]", LG_MAX);
  spb_session *lead = ss[0];
  if (!lead) return set_err(SPB_EBADARG, "spb_batch_decode_step: null session");
  int Pmax = 0;
  bool any_spin = false;
  for (int i = 0; i < B; i++) {
    spb_session *s = ss[i];
    if (s && s->kv.rb) any_spin = true;
    if (!s || s->m != lead->m) return set_err(SPB_EBADARG, "spb_batch_decode_step: sessions must share one model");
    if (s->pos >= s->pmax) return set_err(SPB_ECONTEXT_FULL, "spb_batch_decode_step: session %d context full", i);
    for (int j = 0; j < i; j++)
      if (ss[j] == s) return set_err(SPB_EBADARG, "spb_batch_decode_step: session %d repeated", i);
    Pmax = std::max(Pmax, s->pmax);
  }
  CU(cudaSetDevice(lead->m->device));
  for (int i = 0; i < B; i++) {   // every row's new position writable (copy-on-write on its own stream)
    const int rc = prepare_write(ss[i], ss[i]->pos, 1);
    if (rc) return rc;
  }
  for (int i = 1; i < B; i++) CU(cudaStreamSynchronize(ss[i]->st));   // their caches are settled
  for (int i = 0; i < B; i++) {
    lead->h_pinned[i] = tokens[i];
    lead->h_rows[i] = BatchRow{ss[i]->kv, ss[i]->pos, ss[i]->pmax};
  }
  CU(cudaMemcpyAsync(lead->tok_dev, lead->h_pinned, (size_t)B * 4, cudaMemcpyHostToDevice, lead->st));
  CU(cudaMemcpyAsync(lead->rows_dev, lead->h_rows, (size_t)B * sizeof(BatchRow), cudaMemcpyHostToDevice, lead->st));
  CU(enqueue_rows(lead, B, true, lead->rows_dev, Pmax, any_spin));
  if (logits)
    CU(cudaMemcpyAsync(logits, lead->logits, (size_t)B * lead->m->Vfull * 4, cudaMemcpyDeviceToHost, lead->st));
  CU(cudaMemcpyAsync(lead->h_argmax, lead->argmax_dev, (size_t)B * 4, cudaMemcpyDeviceToHost, lead->st));
  int rc = collect_errors(lead);
  if (rc) return rc;   // no position moved
  if (argmax) memcpy(argmax, lead->h_argmax, (size_t)B * 4);
  for (int i = 0; i < B; i++) {
    ss[i]->pos += 1;
    rc = sync_pos(ss[i]);
    if (rc) return rc;
  }
  for (int i = 0; i < B; i++) CU(cudaStreamSynchronize(ss[i]->st));
  return SPB_OK;
}

extern "C" int spb_session_decode_greedy(spb_session *s, int32_t token, int n_steps, int32_t *tokens_out) {
  if (!s || n_steps < 0) return set_err(SPB_EBADARG, "spb_session_decode_greedy: bad arg");
  if (n_steps > s->pmax - s->pos) return set_err(SPB_ECONTEXT_FULL, "spb_session_decode_greedy: context full");
  if (n_steps == 0) return SPB_OK;
  CU(cudaSetDevice(s->m->device));
  int rc = prepare_write(s, s->pos, n_steps);
  if (rc) return rc;
  rc = ensure_step_graph(s);
  if (rc) return rc;
  s->h_pinned[0] = token;
  CU(cudaMemcpyAsync(s->tok_dev, s->h_pinned, 4, cudaMemcpyHostToDevice, s->st));
  for (int i = 0; i < n_steps; i++) {
    CU(cudaGraphLaunch(s->step_graph, s->st));
    // after the step, tok_dev holds this step's argmax (the graph's last node copies it)
    CU(cudaMemcpyAsync(s->hist_dev + s->pos + i, s->tok_dev, 4, cudaMemcpyDeviceToDevice, s->st));
  }
  if (tokens_out)
    CU(cudaMemcpyAsync(tokens_out, s->hist_dev + s->pos, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, s->st));
  rc = collect_errors(s);
  if (rc) { sync_pos(s); cudaStreamSynchronize(s->st); return rc; }
  s->pos += n_steps;
  return SPB_OK;
}

extern "C" int spb_session_rewind(spb_session *s, int n) {
  if (!s) return set_err(SPB_EBADARG, "spb_session_rewind: null session");
  if (n < 0 || n > s->pos) return set_err(SPB_EBADARG, "spb_session_rewind: n > position");
  s->pos -= n;
  CU(cudaSetDevice(s->m->device));
  int rc = sync_pos(s);
  if (rc) return rc;
  CU(cudaStreamSynchronize(s->st));
  return SPB_OK;
}

// sp_session_clone semantics (sp_session.c:773-816): the clone continues from the same
// position with the same history and cache. Paged: the clone takes the same pages (O(pages) on
// the host, no K/V copied; a page is copied later only where one of the two writes into it).
// Unpaged: a deep copy of the cache on the device.
static int clone_state(const spb_session *s, spb_session *c);

extern "C" int spb_session_clone(const spb_session *s, spb_session **out) {
  if (!s || !out) return set_err(SPB_EBADARG, "spb_session_clone: null arg");
  *out = nullptr;
  spb_session *c = nullptr;
  int rc = session_open(s->m, s->pmax, s->pool, &c, s->flags);
  if (rc) return rc;
  rc = clone_state(s, c);
  if (rc) {   // no half-made clone is handed out (its pages, if it took any, go back)
    spb_session_close(c);
    return rc;
  }
  *out = c;
  return SPB_OK;
}

// the cache (or the page references), history and position of s into the new session c
static int clone_state(const spb_session *s, spb_session *c) {
  CU(cudaStreamSynchronize(s->st));
  if (s->pool) {
    {
      std::lock_guard<std::mutex> lk(s->pool->mu);
      for (int32_t pg : s->pages)
        if (pg >= 0) s->pool->refs[pg]++;
      c->pages = s->pages;
    }
    CU(cudaMemcpyAsync(c->ptab_dev, c->pages.data(), c->pages.size() * 4, cudaMemcpyHostToDevice, c->st));
  } else {
    const size_t kvb = s->kv.rb ? (size_t)s->m->NL * kv_spin_layer_bytes(s->m, s->pmax)
                                : (size_t)s->m->NL * kv_layer_elems(s->m, s->pmax) * 4;
    CU(cudaMemcpyAsync(c->kv.k, s->kv.k, kvb, cudaMemcpyDeviceToDevice, c->st));
    CU(cudaMemcpyAsync(c->kv.v, s->kv.v, kvb, cudaMemcpyDeviceToDevice, c->st));
  }
  CU(cudaMemcpyAsync(c->hist_dev, s->hist_dev, (size_t)s->pmax * 4, cudaMemcpyDeviceToDevice, c->st));
  c->pos = s->pos;
  const int rc = sync_pos(c);
  if (rc) return rc;
  CU(cudaStreamSynchronize(c->st));
  return SPB_OK;
}

extern "C" int spb_session_kv_read(const spb_session *s, int layer, int pos, int which, int32_t *out) {
  if (!s || !out || layer < 0 || layer >= s->m->NL || pos < 0 || pos >= s->pmax)
    return set_err(SPB_EBADARG, "spb_session_kv_read: bad arg");
  const spb_model *m = s->m;
  if (s->kv.rb) return set_err(SPB_EUNSUPPORTED, "spb_session_kv_read: a Spinor session's rows are blocks (spb_session_kv_bytes)");
  KvPages hk = s->kv;
  if (s->pool) {
    if (s->pages[pos / s->pool->pg] < 0) return set_err(SPB_EBADARG, "spb_session_kv_read: position never written");
    hk.ptab = s->pages.data();   // the host copy of the page table
  }
  const int32_t *base = which ? s->kv.v : s->kv.k;
  CU(cudaStreamSynchronize(s->st));
  for (int g = 0; g < m->NKV; g++)
    CU(cudaMemcpy(out + (size_t)g * m->HD, base + kv_elem(hk, m->NL, m->NKV, m->HD, layer, g, pos), (size_t)m->HD * 4,
                  cudaMemcpyDeviceToHost));
  return SPB_OK;
}

extern "C" int spb_session_kv_bytes(const spb_session *s, int layer, int pos, int which, uint8_t *out) {
  if (!s || !out || layer < 0 || layer >= s->m->NL || pos < 0 || pos >= s->pmax)
    return set_err(SPB_EBADARG, "spb_session_kv_bytes: bad arg");
  if (!s->kv.rb) return set_err(SPB_EBADARG, "spb_session_kv_bytes: not a Spinor session");
  const spb_model *m = s->m;
  const uint8_t *base = reinterpret_cast<const uint8_t *>(which ? s->kv.v : s->kv.k);
  CU(cudaStreamSynchronize(s->st));
  for (int g = 0; g < m->NKV; g++)
    CU(cudaMemcpy(out + (size_t)g * s->kv.rb, base + kv_spin_off(s->kv, m->NKV, layer, g, pos), (size_t)s->kv.rb,
                  cudaMemcpyDeviceToHost));
  return SPB_OK;
}

extern "C" int spb_forward(spb_model *m, const int32_t *tokens, int n_tok, float *logits) {
  if (!m || !tokens || n_tok <= 0 || !logits) return set_err(SPB_EBADARG, "spb_forward: bad arg");
  spb_session *s = nullptr;
  int rc = spb_session_open(m, n_tok, &s);
  if (rc) return rc;
  rc = spb_session_prefill(s, tokens, n_tok, logits);
  spb_session_close(s);
  return rc;
}

// ------------------------------------------------------------------------------ isolated kernels
struct DevWork {
  int device = -1;
  uint8_t *buf = nullptr;
  size_t cap = 0;
  uint32_t *err = nullptr;
};
static std::mutex g_work_mu;
static DevWork g_work[64];

static int work_get(size_t need, uint8_t **buf, uint32_t **err) {
  int dev = 0;
  CU(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_err(SPB_EBADARG, "spb: device id");
  std::lock_guard<std::mutex> lk(g_work_mu);
  DevWork &w = g_work[dev];
  if (!w.err) CU(cudaMalloc(&w.err, 256));
  if (!w.err) return SPB_EOOM;
  if (w.cap < need) {
    if (w.buf) cudaFree(w.buf);
    w.buf = nullptr;
    w.cap = 0;
    CU(cudaMalloc(&w.buf, need));
    w.cap = need;
    CU(cudaMemset(w.err, 0, 256));
  }
  *buf = w.buf;
  *err = w.err;
  return SPB_OK;
}

extern "C" int spb_gemv_q4b(const uint8_t *codes, const uint16_t *bscale, int rows, int cols, const float *x,
                            int n_tok, float *y, void *stream) {
  if (!codes || !bscale || !x || !y || rows <= 0 || cols <= 0 || (cols & 31))
    return set_err(SPB_EBADARG, "spb_gemv_q4b: bad arg (cols must be a positive multiple of 32)");
  if (n_tok != 1 && n_tok != 2 && n_tok != 4 && n_tok != 8 && n_tok != 16)
    return set_err(SPB_EBADARG, "spb_gemv_q4b: n_tok must be 1, 2, 4, 8 or 16");
  const size_t need = (size_t)n_tok * cols + (size_t)n_tok * (cols / 32) * 4 + 256 + 64;
  uint8_t *wb;
  uint32_t *err;
  int rc = work_get(need, &wb, &err);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  DevAct act{(int8_t *)wb, (int32_t *)(wb + (size_t)n_tok * cols),
             (float *)(wb + (((size_t)n_tok * cols + (size_t)n_tok * (cols / 32) * 4 + 255) & ~(size_t)255))};
  CU(launch_quant(x, cols, cols, n_tok, act, nullptr, err, st));
  DevQ4B w{codes, bscale, rows, cols};
  CU(launch_gemv(w, nullptr, act, n_tok, y, rows, EPI_STORE, err, st));
  return SPB_OK;
}

// ---- a prepared matrix: the block scales described once, then any number of token rows
struct spb_q4b_mat {
  int device;
  DevQ4B w;
  uint8_t *shift;   // device [rows]
  uint8_t *pl = nullptr;   // the precomputed digit planes (tc_planes_enabled)
};

extern "C" int spb_q4b_prepare(const uint8_t *codes, const uint16_t *bscale, int rows, int cols, void *stream,
                               spb_q4b_mat **out) {
  if (!out) return set_err(SPB_EBADARG, "spb_q4b_prepare: null out");
  *out = nullptr;
  if (!codes || !bscale || rows <= 0 || cols <= 0 || (cols & 31) || cols > 16384)
    return set_err(SPB_EBADARG, "spb_q4b_prepare: bad arg (cols a positive multiple of 32, at most 16384)");
  if ((uintptr_t)codes & 15) return set_err(SPB_EBADARG, "spb_q4b_prepare: codes must be 16-byte aligned");
  int dev = 0;
  CU(cudaGetDevice(&dev));
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t *buf = nullptr;
  const size_t sh_bytes = ((size_t)rows + 255) & ~(size_t)255;
  CU(cudaMalloc(&buf, sh_bytes + 16));
  int *info = reinterpret_cast<int *>(buf + sh_bytes);
  int h[4] = {0, 0, 0, 0};
  cudaError_t e = cudaMemsetAsync(info, 0, 16, st);
  if (e == cudaSuccess) e = launch_q4b_rowinfo(bscale, rows, cols / 32, buf, info, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(h, info, 16, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    cudaFree(buf);
    return set_err(SPB_ECUDA, "spb_q4b_prepare: %s", cudaGetErrorString(e));
  }
  if (h[0]) {
    cudaFree(buf);
    return set_err(SPB_ERANGE, "spb_q4b_prepare: block scales exceed the exact int64 accumulation bound "
                               "(or hold inf/NaN)");
  }
  spb_q4b_mat *m = new spb_q4b_mat();
  m->device = dev;
  m->shift = buf;
  m->w = DevQ4B{codes, bscale, rows, cols, h[1] <= 21 ? 1 : 0, buf, q4b_planes_for_spread(h[2])};
  if (tc_planes_enabled() && m->w.planes >= 2 && cols % 128 == 0) {
    const size_t pb = (size_t)m->w.planes * rows * cols;
    if (cudaMalloc(&m->pl, pb) == cudaSuccess) {
      m->w.pl = m->pl;
      e = launch_q4b_planes(m->w, m->pl, st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(st);
      if (e != cudaSuccess) {
        spb_q4b_release(m);
        return set_err(SPB_ECUDA, "spb_q4b_prepare: digit planes: %s", cudaGetErrorString(e));
      }
    } else {
      (void)cudaGetLastError();   // no room: the GEMM converts the codes itself
      m->pl = nullptr;
    }
  }
  *out = m;
  return SPB_OK;
}

extern "C" void spb_q4b_release(spb_q4b_mat *m) {
  if (!m) return;
  cudaFree(m->shift);
  cudaFree(m->pl);
  delete m;
}

extern "C" int spb_q4b_info(const spb_q4b_mat *m, int32_t out[4]) {
  if (!m || !out) return set_err(SPB_EBADARG, "spb_q4b_info: null arg");
  out[0] = m->w.rows;
  out[1] = m->w.cols;
  out[2] = m->w.small;
  out[3] = m->w.planes;
  return SPB_OK;
}

extern "C" int spb_q4b_matmul(const spb_q4b_mat *m, const float *x, int n_tok, float *y, void *stream) {
  if (!m || !x || !y || n_tok <= 0) return set_err(SPB_EBADARG, "spb_q4b_matmul: bad arg");
  const int rows = m->w.rows, cols = m->w.cols;
  // quantized rows, their block sums and scales, then the split-K workspace of the token-batch GEMM
  const size_t qb = ((size_t)n_tok * cols + 255) & ~(size_t)255;
  const size_t bb = ((size_t)n_tok * (cols / 32) * 4 + 255) & ~(size_t)255;
  const size_t sb = ((size_t)n_tok * 4 + 255) & ~(size_t)255;
  const size_t ws_elems = (size_t)2 * 64 * rows;
  uint8_t *wb;
  uint32_t *err;
  int rc = work_get(qb + bb + sb + ws_elems * 8, &wb, &err);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  DevAct act{(int8_t *)wb, (int32_t *)(wb + qb), (float *)(wb + qb + bb)};
  CU(launch_quant(x, cols, cols, n_tok, act, nullptr, err, st));
  CU(launch_gemv(m->w, nullptr, act, n_tok, y, rows, EPI_STORE, err, st, 0, nullptr, nullptr,
                 (int64_t *)(wb + qb + bb + sb), ws_elems));
  return SPB_OK;
}

extern "C" int spb_quantize_rows(const float *x, int cols, int n_tok, int8_t *q, int32_t *bsum, float *scale,
                                 void *stream) {
  if (!x || !q || !bsum || !scale || cols <= 0 || (cols & 31) || n_tok <= 0)
    return set_err(SPB_EBADARG, "spb_quantize_rows: bad arg (cols must be a positive multiple of 32)");
  uint8_t *wb;
  uint32_t *err;
  int rc = work_get(256, &wb, &err);
  if (rc) return rc;
  CU(launch_quant(x, cols, cols, n_tok, DevAct{q, bsum, scale}, nullptr, err, (cudaStream_t)stream));
  return SPB_OK;
}

static int gemv_q_common(const uint8_t *codes, const uint16_t *bscale, const uint8_t *codes2, const uint16_t *bscale2,
                         int rows, int cols, const int8_t *q, const int32_t *bsum, const float *scale, int n_tok,
                         int epi, float *y, void *stream) {
  if (!codes || !bscale || !q || !bsum || !scale || !y || rows <= 0 || cols <= 0 || (cols & 31))
    return set_err(SPB_EBADARG, "spb_gemv_q4b_q: bad arg (cols must be a positive multiple of 32)");
  if (n_tok != 1 && n_tok != 2 && n_tok != 4 && n_tok != 8 && n_tok != 16)
    return set_err(SPB_EBADARG, "spb_gemv_q4b_q: n_tok must be 1, 2, 4, 8 or 16");
  if (epi != EPI_STORE && (!codes2 || !bscale2)) return set_err(SPB_EBADARG, "spb_gemv_q4b_gated_q: null up matrix");
  if (((uintptr_t)q & 15) || ((uintptr_t)codes & 15) || (codes2 && ((uintptr_t)codes2 & 15)))
    return set_err(SPB_EBADARG, "spb_gemv_q4b_q: codes and q must be 16-byte aligned");
  uint8_t *wb;
  uint32_t *err;
  int rc = work_get(256, &wb, &err);
  if (rc) return rc;
  DevQ4B w{codes, bscale, rows, cols}, w2{codes2, bscale2, rows, cols};
  CU(launch_gemv(w, epi != EPI_STORE ? &w2 : nullptr, DevAct{(int8_t *)q, (int32_t *)bsum, (float *)scale}, n_tok,
                 y, rows, epi, err, (cudaStream_t)stream));
  return SPB_OK;
}

extern "C" int spb_gemv_q4b_q(const uint8_t *codes, const uint16_t *bscale, int rows, int cols, const int8_t *q,
                              const int32_t *bsum, const float *scale, int n_tok, float *y, void *stream) {
  return gemv_q_common(codes, bscale, nullptr, nullptr, rows, cols, q, bsum, scale, n_tok, EPI_STORE, y, stream);
}

extern "C" int spb_gemv_q4b_gated_q(const uint8_t *codes_g, const uint16_t *bscale_g, const uint8_t *codes_u,
                                    const uint16_t *bscale_u, int rows, int cols, const int8_t *q,
                                    const int32_t *bsum, const float *scale, int n_tok, int act, float *y,
                                    void *stream) {
  if (act != 0 && act != 1) return set_err(SPB_EBADARG, "spb_gemv_q4b_gated_q: act must be 0 (GELU) or 1 (SiLU)");
  return gemv_q_common(codes_g, bscale_g, codes_u, bscale_u, rows, cols, q, bsum, scale, n_tok,
                       act == 0 ? EPI_GELU_MUL : EPI_SILU_MUL, y, stream);
}

extern "C" int spb_graph_begin(void *stream) {
  CU(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeRelaxed));
  return SPB_OK;
}

extern "C" int spb_graph_end(void *stream, void **graph_exec) {
  if (!graph_exec) return set_err(SPB_EBADARG, "spb_graph_end: null out");
  cudaGraph_t g = nullptr;
  CU(cudaStreamEndCapture((cudaStream_t)stream, &g));
  cudaGraphExec_t ex = nullptr;
  cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return set_err(SPB_ECUDA, "spb_graph_end: %s", cudaGetErrorString(e));
  *graph_exec = ex;
  return SPB_OK;
}

extern "C" int spb_graph_launch(void *graph_exec, void *stream) {
  if (!graph_exec) return set_err(SPB_EBADARG, "spb_graph_launch: null graph");
  CU(cudaGraphLaunch((cudaGraphExec_t)graph_exec, (cudaStream_t)stream));
  return SPB_OK;
}

extern "C" void spb_graph_free(void *graph_exec) {
  if (graph_exec) cudaGraphExecDestroy((cudaGraphExec_t)graph_exec);
}

extern "C" int spb_take_device_errors(void) {
  uint8_t *wb;
  uint32_t *err;
  int rc = work_get(256, &wb, &err);
  if (rc) return rc;
  uint32_t h = 0;
  CU(cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost));
  CU(cudaMemset(err, 0, 4));
  return (int)h;
}

extern "C" int spb_rmsnorm_exact_dev(const float *x, const float *w, int n, int rows, float *out, void *stream) {
  if (!x || !w || !out || n <= 0 || rows <= 0 || n > 16384) return set_err(SPB_EBADARG, "spb_rmsnorm_exact_dev: bad arg");
  uint8_t *wb;
  uint32_t *err;
  int rc = work_get(256, &wb, &err);
  if (rc) return rc;
  CU(launch_rmsnorm_rows(x, w, n, rows, out, err, (cudaStream_t)stream));
  return SPB_OK;
}

static int eltwise(const float *x, int n, float *out, void *stream, int op) {
  if (!x || !out || n <= 0) return set_err(SPB_EBADARG, "spb eltwise: bad arg");
  uint8_t *wb;
  uint32_t *err;
  int rc = work_get(256, &wb, &err);
  if (rc) return rc;
  CU(launch_eltwise(x, n, out, op, err, (cudaStream_t)stream));
  return SPB_OK;
}
extern "C" int spb_gelu_exact_dev(const float *x, int n, float *out, void *stream) { return eltwise(x, n, out, stream, 0); }
extern "C" int spb_silu_exact_dev(const float *x, int n, float *out, void *stream) { return eltwise(x, n, out, stream, 1); }

extern "C" int spb_rope_cordic_dev(const float *v, int d, int rows, const int32_t *pos, float base, int32_t *out,
                                   void *stream) {
  if (!v || !pos || !out || rows <= 0 || d <= 0 || (d & 1) || d > 2048) return set_err(SPB_EBADARG, "spb_rope_cordic_dev: bad arg");
  std::vector<uint64_t> ht(32 + d / 2, 0);
  uint64_t gain = 0;
  spb_cordic_tables(ht.data(), &gain);
  int rc = spb_rope_freq_table(base, d, ht.data() + 32);
  if (rc) return rc;
  const size_t need = ht.size() * 8;
  uint8_t *wb;
  uint32_t *err;
  rc = work_get(need, &wb, &err);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  CU(cudaMemcpyAsync(wb, ht.data(), need, cudaMemcpyHostToDevice, st));
  CU(launch_rope_rows(v, d, rows, pos, (const uint64_t *)wb + 32, (const uint64_t *)wb, gain, out, err, st));
  CU(cudaStreamSynchronize(st));
  return SPB_OK;
}
