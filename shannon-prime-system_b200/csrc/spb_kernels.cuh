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
};

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
};

// y[t][j] for t < ntok over `w` (and `w2` for the gated epilogues). ymax (nullable):
// per-token slots receiving atomicMax of the f32 bits of max |y| (the next quantizer's scale).
// amax (nullable, zero on entry): per-token 64-bit greedy-argmax keys (first maximum).
cudaError_t launch_gemv(const DevQ4B &w, const DevQ4B *w2, const DevAct &act, int ntok, float *y,
                        int ldy, int epi, uint32_t *err, cudaStream_t st, int grid_limit = 0,
                        uint32_t *ymax = nullptr, unsigned long long *amax = nullptr);

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

struct RopeArgs {
  const float *qkv;        // [ntok][QD + 2*KVD] projections
  int32_t *qi;             // [ntok][QD] rotated q on the 2^16 grid
  int32_t *kc, *vc;        // this layer's cache [NKV][P][HD]
  const float *q_norm, *k_norm;  // nullable when the model has no QK-norm
  const uint64_t *W;       // turn table [HD/2]
  const uint64_t *T;       // CORDIC arctangent table [30]
  uint64_t gain;           // CORDIC gain compensation, Q62
  const int32_t *pos_dev;  // device position of token row 0 (rows t use pos+t)
  int NH, NKV, HD, P, ntok;
  uint32_t *err;
  uint32_t *zero_slot;     // nullable: per-row max slots cleared for the attention output
};
cudaError_t launch_rope_kv(const RopeArgs &a, cudaStream_t st);

struct AttnArgs {
  const int32_t *qi;       // [ntok][NH*HD]
  const int32_t *kc, *vc;  // this layer's cache [NKV][P][HD]
  float *ao;               // [ntok][NH*HD]
  const int32_t *pos_dev;  // position of token row 0
  int NH, NKV, HD, P, win, ntok;
  float ascale;
  uint32_t *err;
  uint32_t *ao_max;        // nullable: per-row atomicMax of the f32 bits of max |ao|
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
