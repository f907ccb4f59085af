// spb_decode.cu -- one greedy decode step (one token, batch 1) as ONE persistent kernel.
//
// At batch 1 the multi-kernel schedule of spb_kernels.cu is bound by the fixed cost of its
// ~8 launches per layer (ramp, drain, the latency of each dependent read), not by HBM. Here
// one CTA per SM (a cooperative launch, so all of them are resident) runs the whole step,
// layer after layer, with the same exact numeric rules:
//
//   * warp 16, the producer, streams every weight tile, norm weight vector and KV slice this
//     CTA consumes in the step, in consumption order, into a ring of shared-memory slots
//     with TMA bulk copies (cp.async.bulk, completion on an mbarrier per slot). It runs ahead
//     across phase boundaries: while the compute warps wait at a grid barrier, reduce a norm
//     or run attention, the next matrices are already landing in shared memory.
//   * warps 0-15, the consumers, run the phases. Where a phase needs whole rows written by
//     other CTAs they meet at a grid barrier (a monotonic counter in global memory polled
//     with acquire loads) and then fetch those rows with one bulk copy.
//
// Phases of one layer:
//   norm  every CTA recomputes the residual add and the RMSNorm island (exact_islands.c:60-79)
//         for the whole row in shared memory and quantizes it (sp_frob_quant1,
//         frobenius_lift.c:27-35), so no barrier separates a norm from the GEMV that
//         consumes it; CTA c writes slice c of the new residual.
//   GEMV  CTA c owns a contiguous range of output rows (matmul_arena's Q4B branch,
//         forward_dispatch.c:69-86); a tile is up to 16 rows (4 rows of the 15360-column
//         down matrix, whose rows split into 4 column segments); one warp per (row,
//         segment) and the warp's activation words stay in registers for the whole phase.
//   attn  KV head g is split by position over the CTAs c = g (mod NKV) (sp_attn_head,
//         forward_kernels.c:59-81). Each part applies the QK-norm island and CORDIC-RoPE to
//         its query heads itself; the part holding the new position also rotates and stores
//         the new K/V row. Two per-head barriers exchange the integer score maximum and then
//         the exact partial sums; each part finalizes a slice of the head's outputs.
// The final norm feeds the LM head, whose CTAs fold a greedy-argmax key into one 64-bit
// atomic; CTA 0 publishes the token and advances the position after the last barrier.
//
// The code that runs once per layer is kept small (rolled loops over shared memory, one
// copy of each phase): the whole step re-executes it 48 times with other phases in between,
// and instruction fetches that miss the SM's instruction cache cost an L2 round trip each.
#include "spb_async.cuh"
#include "spb_device.cuh"
#include "spb_exact.cuh"
#include "spb_kernels.cuh"

namespace spb {

namespace {

constexpr int CW = 16;                  // compute warps
constexpr int CT = CW * 32;             // compute threads
constexpr int NTHREADS = CT + 32;       // + the producer warp
constexpr int NSLOT = 4;                // ring slots
constexpr int SLOT = 34816;             // bytes per slot: 16 rows of 3840 or 15 of 4096 columns
constexpr int EMAX = 4096;              // widest residual row
constexpr int KMAX = 16384;             // widest GEMV input
constexpr int RACC = 256;               // rows per CTA of a GEMV with a phase epilogue
constexpr int SCMAX = 1024;             // attention scores per CTA (query heads x positions)
constexpr int GHMAX = 512;              // query heads per KV head x head_dim
constexpr int HDMAX = 256;
constexpr int MINP = 16;                // fewest positions per attention part
constexpr int VBUF = 4096;              // floats per vector buffer
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;   // every wait gives up after 2 s
constexpr uint32_t SLEEP_NS = 2000;                  // hardware sleep per mbarrier poll

// dynamic shared memory
constexpr int OFF_XA = NSLOT * SLOT;                 // activation codes, two planes of [KMAX/32][16]
constexpr int PLANE = KMAX / 2;
constexpr int OFF_XS = OFF_XA + KMAX;                // [KMAX/32] per-block code sums
constexpr int OFF_RACC = OFF_XS + (KMAX / 32) * 4;   // [2][RACC] int64 row accumulators
constexpr int OFF_SC = OFF_RACC + 2 * RACC * 8;      // [SCMAX] scores, then exponentials
constexpr int OFF_QS = OFF_SC + SCMAX * 4;           // [GHMAX] rotated queries
constexpr int OFF_KN = OFF_QS + GHMAX * 4;           // [HDMAX] rotated new key
constexpr int OFF_VN = OFF_KN + HDMAX * 4;           // [HDMAX] new value on the 2^16 grid
constexpr int OFF_VB = OFF_VN + HDMAX * 4;           // [2][VBUF] f32 vectors fetched by bulk copy
constexpr int SMEM = OFF_VB + 2 * VBUF * 4;
static_assert(2 * EMAX * 4 <= SLOT, "two norm weight vectors per slot");
static_assert(EMAX <= VBUF, "a residual row per vector buffer");

constexpr int SYNC_GRID = 0, SYNC_EXIT = 32, SYNC_ABORT = 64, SYNC_HEAD = 96;

struct Sh {
  uint64_t full[NSLOT], empty[NSLOT], vbar[2];
  acc128 red128[CW];
  float redf[CW];
  uint64_t inv[9];
  uint64_t T[CORDIC_ITERS];   // CORDIC arctangent table
  DecLayer ly[3];             // layer descriptors L-1, L, L+1 (index L % 3)
  int32_t mx[8], mg[8];
  unsigned long long ssum[8];
  unsigned long long key;
  uint32_t issued;
  int abort;
};

__shared__ Sh g_sh;
extern __shared__ __align__(1024) uint8_t dsm[];

__device__ __forceinline__ uint8_t *ring_slot(int s) { return dsm + (size_t)s * SLOT; }
__device__ __forceinline__ int8_t *xa() { return reinterpret_cast<int8_t *>(dsm + OFF_XA); }
__device__ __forceinline__ int32_t *xs() { return reinterpret_cast<int32_t *>(dsm + OFF_XS); }
__device__ __forceinline__ unsigned long long *racc() { return reinterpret_cast<unsigned long long *>(dsm + OFF_RACC); }
__device__ __forceinline__ int32_t *sc() { return reinterpret_cast<int32_t *>(dsm + OFF_SC); }
__device__ __forceinline__ int32_t *qs() { return reinterpret_cast<int32_t *>(dsm + OFF_QS); }
__device__ __forceinline__ int32_t *kn() { return reinterpret_cast<int32_t *>(dsm + OFF_KN); }
__device__ __forceinline__ int32_t *vn() { return reinterpret_cast<int32_t *>(dsm + OFF_VN); }
__device__ __forceinline__ float *vb(int b) { return reinterpret_cast<float *>(dsm + OFF_VB) + b * VBUF; }

__device__ __forceinline__ int tid_() { return threadIdx.x; }
__device__ __forceinline__ int warp_() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_() { return threadIdx.x & 31; }

// thread-uniform progress of the consumers: tiles consumed, vector-buffer phases, barriers
struct Cnt {
  uint32_t T, vp0, vp1, gep, hep;
};

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory"); }

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool aborted() { return *(volatile int *)&g_sh.abort != 0; }

__device__ __noinline__ void set_abort(const DecodeArgs &a) {
  *(volatile int *)&g_sh.abort = 1;
  if (a.sync) atomicExch(a.sync + SYNC_ABORT, 1u);
  raise_err(a.err, ERR_TIMEOUT);
}

// wait for phase `parity` of a shared-memory mbarrier; false on abort or after the limit
__device__ __noinline__ bool wait_bar_slow(const DecodeArgs &a, uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = now_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, SLEEP_NS)) return true;
    if (aborted()) return false;
    if (now_ns() - t0 > WAIT_LIMIT_NS) break;
  }
  set_abort(a);
  return false;
}
__device__ __forceinline__ bool wait_bar(const DecodeArgs &a, uint64_t *bar, uint32_t parity) {
  return mbar_try_wait(bar, parity) || wait_bar_slow(a, bar, parity);
}

// all compute threads: arrive on a global counter and wait until it reaches `target`
__device__ __noinline__ bool counter_sync(const DecodeArgs &a, uint32_t *ctr, uint32_t target) {
  cbar();
  if (tid_() == 0 && !aborted()) {
    __threadfence();
    atomicAdd(ctr, 1u);
    const uint64_t t0 = now_ns();
    for (uint32_t it = 1;; it++) {
      if (ld_acquire(ctr) >= target) break;
      if ((it & 63u) == 0) {
        if (*(volatile uint32_t *)(a.sync + SYNC_ABORT)) { *(volatile int *)&g_sh.abort = 1; break; }
        if (now_ns() - t0 > WAIT_LIMIT_NS) { set_abort(a); break; }
      }
    }
    __threadfence();
  }
  cbar();
  return !aborted();
}

__device__ __forceinline__ bool grid_sync(const DecodeArgs &a, Cnt &c) {
  c.gep++;
  return counter_sync(a, a.sync + SYNC_GRID, c.gep * gridDim.x);
}

// Bulk copy of `bytes` of global memory written earlier in this step (possibly by other
// CTAs, ordered by the barrier just passed) into vector buffer b; issued by thread 0.
__device__ __forceinline__ void vload(int b, const void *src, uint32_t bytes) {
  asm volatile("fence.proxy.async.global;" ::: "memory");
  mbar_arrive_expect_tx(&g_sh.vbar[b], bytes);
  bulk_g2s(vb(b), src, bytes, &g_sh.vbar[b]);
}
__device__ __forceinline__ void vload_more(int b, int off_floats, const void *src, uint32_t bytes) {
  bulk_g2s(vb(b) + off_floats, src, bytes, &g_sh.vbar[b]);
}

__device__ __forceinline__ void rows_of(int R, int c, int n, int &r0, int &r1) {
  const int ng = (R + 3) >> 2;
  r0 = min(ng * c / n * 4, R);
  r1 = min(ng * (c + 1) / n * 4, R);
}

// GEMV tiling of a K-column matrix: column segments (a power of two dividing the warp
// count, <= 128 blocks each) and rows per ring slot
struct Tiling {
  int nblk, segs, sb, rt;
};
__device__ __forceinline__ Tiling tiling(int K) {
  Tiling t;
  t.nblk = K >> 5;
  t.segs = 1;
  while (t.segs * 128 < t.nblk) t.segs <<= 1;
  t.sb = (t.nblk + t.segs - 1) / t.segs;
  t.rt = min(16, SLOT / ((K >> 1) + (K >> 4)));
  return t;
}

// The attention split of one layer for the CTA: part j of KV head g over positions [c0, c1)
struct AttnPart {
  int g, j, npart, s0, n, cs, c0, c1;
  bool active;
};
__device__ __forceinline__ AttnPart attn_part(int c, int nctas, int NKV, int p, int win) {
  AttnPart r;
  r.g = c % NKV;
  r.j = c / NKV;
  const int avail = (nctas - 1 - r.g) / NKV + 1;
  r.s0 = (win >= 0 && p - win + 1 > 0) ? p - win + 1 : 0;
  r.n = p - r.s0 + 1;
  int np = min(avail, max(1, (r.n + MINP - 1) / MINP));
  r.cs = (r.n + np - 1) / np;
  r.npart = (r.n + r.cs - 1) / r.cs;
  r.active = r.j < r.npart;
  r.c0 = r.s0 + r.j * r.cs;
  r.c1 = min(r.c0 + r.cs, p + 1);
  return r;
}

// ------------------------------------------------------------------------------ producer
// Tile order of one step (the consumers take them in the same order):
//   embedding row of the token;
//   per layer: [norm weights] QKV | K slices | V slices | O | [norm weights] gate/up | down;
//   [final norm weights] LM head.
// The order is generated by a small state machine whose per-tile step is plain arithmetic.
struct Tile {
  const void *s0, *s1;
  uint32_t b0, b1;
};

struct TileGen {
  enum { EMB, VEC_A, QKV, KT, VT, OP, VEC_B, GU, DN, VEC_F, LM, DONE };
  int st = EMB, L = 0;
  // the current stage, read once from the layer table when the stage is entered, so that a
  // tile costs the producer thread only arithmetic
  const uint8_t *c0 = nullptr, *c1 = nullptr;   // codes of the matrix (and of up, for GU)
  const uint8_t *s0 = nullptr, *s1 = nullptr;   // block scales as bytes
  const void *v1 = nullptr, *v2 = nullptr;      // norm weight vectors
  const int32_t *kv = nullptr;                  // this head's K or V cache rows
  int K = 0, rt = 0, r = 0, r1 = 0, m = 0, pos = 0, ce = 0;

  __device__ void set_w(const DevQ4B &w, const DevQ4B *w2) {
    K = w.cols;
    rt = tiling(K).rt;
    rows_of(w.rows, blockIdx.x, gridDim.x, r, r1);
    c0 = w.codes;
    s0 = reinterpret_cast<const uint8_t *>(w.scales);
    c1 = w2 ? w2->codes : nullptr;
    s1 = w2 ? reinterpret_cast<const uint8_t *>(w2->scales) : nullptr;
    m = 0;
  }

  // read the stage just entered; false when it has no tile for this CTA
  __device__ bool enter(const DecodeArgs &a, int p) {
    const DecLayer *ly = a.layers + (L < a.NL ? L : a.NL - 1);
    switch (st) {
      case VEC_A:
        v1 = (L > 0 && a.gemma) ? (const void *)a.layers[L - 1].post_ffw : nullptr;
        v2 = ly->attn_norm;
        return true;
      case VEC_B:
        v1 = a.gemma ? (const void *)ly->post_attn : nullptr;
        v2 = ly->ffn_norm;
        return true;
      case VEC_F:
        v1 = a.gemma ? (const void *)a.layers[a.NL - 1].post_ffw : nullptr;
        v2 = a.out_norm;
        return true;
      case QKV: set_w(ly->qkv, nullptr); return r < r1;
      case OP: set_w(ly->o, nullptr); return r < r1;
      case GU: set_w(ly->g, &ly->u); return r < r1;
      case DN: set_w(ly->d, nullptr); return r < r1;
      case LM: set_w(a.out, nullptr); return r < r1;
      case KT:
      case VT: {
        const AttnPart ap = attn_part(blockIdx.x, gridDim.x, a.NKV, p, ly->win);
        if (!ap.active) return false;
        kv = (st == KT ? a.kc : a.vc) + (size_t)L * a.kvl + (size_t)ap.g * a.P * a.HD;
        pos = ap.c0;
        ce = min(ap.c1, p);
        return pos < ce;
      }
      default: return true;
    }
  }

  __device__ void advance_stage(const DecodeArgs &a, int p) {
    for (;;) {
      if (st == DN) {
        L++;
        st = L < a.NL ? VEC_A : VEC_F;
      } else if (st == LM || st == DONE) {
        st = DONE;
        return;
      } else {
        st++;
      }
      if (enter(a, p)) return;
    }
  }

  // the next tile; false when the step has no more
  __device__ bool next(const DecodeArgs &a, int p, int tok, Tile &t) {
    t.s1 = nullptr;
    t.b1 = 0;
    switch (st) {
      case DONE: return false;
      case EMB: {
        const int E = a.E;
        t.s0 = a.embd.codes + (size_t)tok * (E >> 1);
        t.b0 = (uint32_t)(E >> 1);
        t.s1 = reinterpret_cast<const uint8_t *>(a.embd.scales) + (size_t)tok * (E >> 4);
        t.b1 = (uint32_t)(E >> 4);
        advance_stage(a, p);
        return true;
      }
      case VEC_A:
      case VEC_B:
      case VEC_F: {
        const uint32_t b = (uint32_t)a.E * 4;
        t.s0 = v1 ? v1 : v2;
        t.b0 = b;
        if (v1) { t.s1 = v2; t.b1 = b; }
        advance_stage(a, p);
        return true;
      }
      case KT:
      case VT: {
        const int HD = a.HD, sub = SLOT / (HD * 4);
        const int len = min(sub, ce - pos);
        t.s0 = kv + (size_t)pos * HD;
        t.b0 = (uint32_t)len * HD * 4;
        pos += len;
        if (pos >= ce) advance_stage(a, p);
        return true;
      }
      default: {   // GEMV row tiles (gate and up alternate per row range)
        const int rows = min(rt, r1 - r);
        const uint8_t *cc = m ? c1 : c0, *ss = m ? s1 : s0;
        t.s0 = cc + (size_t)r * (K >> 1);
        t.b0 = (uint32_t)rows * (K >> 1);
        t.s1 = ss + (size_t)r * (K >> 4);
        t.b1 = (uint32_t)rows * (K >> 4);
        if (c1 && m == 0) {
          m = 1;
        } else {
          m = 0;
          r += rt;
          if (r >= r1) advance_stage(a, p);
        }
        return true;
      }
    }
  }
};

// put tile T into its ring slot once the consumers have released the slot's previous tile;
// false (and the step aborted) if that wait gives up
__device__ bool ring_issue(const DecodeArgs &a, uint32_t T, const Tile &t) {
  const int slot = (int)(T % NSLOT);
  const uint32_t n = T / NSLOT;
  if (n > 0) {
    bool got = false;
    const uint64_t t0 = now_ns();
    for (;;) {
      if (mbar_try_wait_sleep(&g_sh.empty[slot], (n - 1) & 1u, SLEEP_NS)) { got = true; break; }
      if (aborted()) break;
      if (now_ns() - t0 > WAIT_LIMIT_NS) break;
    }
    if (!got) {
      if (!aborted()) set_abort(a);
      return false;
    }
  }
  if (a.trace && blockIdx.x == 0 && T < DEC_TRACE_TILES) a.trace[3 * decode_trace_points(a.NL) + 2 * T] = now_ns();
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(&g_sh.full[slot], t.b0 + t.b1);
  bulk_g2s(ring_slot(slot), t.s0, t.b0, &g_sh.full[slot]);
  if (t.b1) bulk_g2s(ring_slot(slot) + t.b0, t.s1, t.b1, &g_sh.full[slot]);
  return true;
}

__device__ uint32_t produce(const DecodeArgs &a, int p, int tok) {
  TileGen gen;
  Tile t;
  uint32_t T = 0;
  while (gen.next(a, p, tok, t)) {
    if (!ring_issue(a, T, t)) return T;
    T++;
  }
  return T;
}

// ------------------------------------------------------------------------------ consumers
__device__ acc128 csum128(acc128 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc128 r;
    r.lo = __shfl_xor_sync(0xffffffffu, v.lo, o);
    r.hi = __shfl_xor_sync(0xffffffffu, v.hi, o);
    acc128_add(v, r);
  }
  if (lane_() == 0) g_sh.red128[warp_()] = v;
  cbar();
  acc128 s{0ull, 0ll};
  for (int i = 0; i < CW; i++) acc128_add(s, g_sh.red128[i]);
  cbar();
  return s;
}

__device__ float cmax_f(float v) {
  v = warp_max_f(v);
  if (lane_() == 0) g_sh.redf[warp_()] = v;
  cbar();
  float m = 0.0f;
  for (int i = 0; i < CW; i++) m = fmaxf(m, g_sh.redf[i]);
  cbar();
  return m;
}

__device__ __noinline__ uint64_t rms_inv_dec(acc128 tot, int n, uint32_t *err) { return rms_inv(tot, n, err); }

// trace point k (only when a trace buffer is given): all compute threads of the CTA are past
// the point when its time is taken
__device__ __noinline__ void trace_point(const DecodeArgs &a, int k) {
  if (!a.trace) return;
  cbar();
  if (tid_() == 0) {
    const unsigned long long t = now_ns();
    unsigned long long *e = a.trace + 3 * k;
    if (blockIdx.x == 0) e[0] = (unsigned long long)clock64();   // CTA 0: SM cycles (exact)
    atomicMax(e + 1, t);
    atomicMin(e + 2, t);
  }
}

// copy layer L's descriptor into its shared-memory slot (threads of the last two warps; the
// slot is read after the next compute barrier)
__device__ __forceinline__ void load_layer(const DecodeArgs &a, int L) {
  constexpr int W = (int)(sizeof(DecLayer) / 4);
  static_assert(W <= 64, "layer descriptor");
  const int t = tid_() - (CT - 64);
  if (L < a.NL && t >= 0 && t < W)
    reinterpret_cast<uint32_t *>(&g_sh.ly[L % 3])[t] = __ldg(reinterpret_cast<const uint32_t *>(a.layers + L) + t);
}

__device__ __forceinline__ void put_code(int b, int lane, int32_t q) {
  const int pos = perm_pos(lane);
  xa()[(pos >> 4) * PLANE + b * 16 + (pos & 15)] = (int8_t)q;
  const int32_t sum = warp_sum_i32(q);
  if (lane == 0) xs()[b] = sum;
}

// quantize n values of shared memory into activation blocks [b0, b0 + n/32)
__device__ __forceinline__ void quant_smem(const float *src, int n, int b0, float s) {
  for (int b = warp_(); b < (n >> 5); b += CW) put_code(b0 + b, lane_(), quant1(src[b * 32 + lane_()], s));
}

__device__ __forceinline__ double act_dscale(float s) { return __dmul_rn(__ddiv_rn((double)s, 127.0), 0x1p-24); }

__device__ __forceinline__ float acc_to_f32(long long acc, double d) {
  return __double2float_rn(__dmul_rn(__ll2double_rn(acc), d));
}

__device__ __forceinline__ void take_tile(const DecodeArgs &a, Cnt &c, int &slot, bool &ready) {
  const uint32_t T = c.T++;
  slot = (int)(T % NSLOT);
  ready = wait_bar(a, &g_sh.full[slot], (T / NSLOT) & 1u);
  if (a.trace && blockIdx.x == 0 && tid_() == 0 && T < DEC_TRACE_TILES)
    a.trace[3 * decode_trace_points(a.NL) + 2 * T + 1] = now_ns();
}
__device__ __forceinline__ void release_tile(int slot) {
  __syncwarp();
  if (lane_() == 0) mbar_arrive(&g_sh.empty[slot]);
}

// Residual add + RMSNorm island + quantizer. The residual row comes from xin (or the
// embedding tile when embed), add (nullable) from the previous block's output; with
// sandwich, add goes through the post-norm island first. CTA c writes slice c of the new
// residual to xout. The quantized row lands in the activation blocks; returns its scale.
__device__ __noinline__ float norm_phase(const DecodeArgs &a, Cnt &c, bool embed, const float *xin,
                                         const float *add, bool sandwich, float *xout, int tr = -1) {
  const int E = a.E, tid = tid_();
  float *X = vb(0), *A = vb(1);
  if (tid == 0) {
    fence_proxy_async_smem();
    if (!embed) vload(0, xin, (uint32_t)E * 4);
    if (add) vload(1, add, (uint32_t)E * 4);
  }
  int slot;
  bool ready;
  if (embed) {   // x = code * f16 scale (* sqrt(E) for Gemma), from the embedding row tile
    take_tile(a, c, slot, ready);
    const uint8_t *cr = ring_slot(slot);
    const uint16_t *sr = reinterpret_cast<const uint16_t *>(cr + (E >> 1));
    for (int i = tid; i < E && ready; i += CT) {
      const uint32_t nib = (i & 1) ? (cr[i >> 1] >> 4) : (cr[i >> 1] & 0xFu);
      const int code = nib >= 8 ? (int)nib - 16 : (int)nib;
      float v = __fmul_rn((float)code, f16_value(sr[i >> 5]));
      if (a.gemma) v = __fmul_rn(v, a.es);
      X[i] = v;
    }
    release_tile(slot);
  }
  take_tile(a, c, slot, ready);   // norm weights
  const float *aw = reinterpret_cast<const float *>(ring_slot(slot));
  const float *ow = aw + (sandwich ? E : 0);
  bool vok = true;
  if (!embed) vok = wait_bar(a, &g_sh.vbar[0], (c.vp0++) & 1u) && vok;
  if (add) vok = wait_bar(a, &g_sh.vbar[1], (c.vp1++) & 1u) && vok;
  cbar();   // X complete (embedding written by all threads)
  if (tr >= 0) trace_point(a, tr);
  bool bad = false;
  uint64_t inv = 0;
  if (add && sandwich) {
    acc128 ss{0ull, 0ll};
    for (int i = tid; i < E; i += CT) {
      const float v = A[i];
      if (!(fabsf(v) < 32768.0f)) { bad = true; continue; }
      const int64_t q = q16_round(v);
      acc128_add(ss, q * q);
    }
    inv = rms_inv_dec(csum128(ss), E, tid == 0 ? a.err : nullptr);
  }
  if (tr >= 0) trace_point(a, tr + 1);
  const int per = (E + (int)gridDim.x - 1) / (int)gridDim.x;
  const int lo = (int)blockIdx.x * per, hi = min(lo + per, E);
  acc128 ss{0ull, 0ll};
  for (int i = tid; i < E; i += CT) {
    float x = X[i];
    if (add) x = __fadd_rn(x, sandwich ? rms_apply(A[i], aw[i], inv, a.err) : A[i]);
    X[i] = x;
    if (i >= lo && i < hi) __stcg(xout + i, x);
    if (!(fabsf(x) < 32768.0f)) { bad = true; continue; }
    const int64_t q = q16_round(x);
    acc128_add(ss, q * q);
  }
  if (bad) raise_err(a.err, ERR_NORM_RANGE);
  inv = rms_inv_dec(csum128(ss), E, tid == 0 ? a.err : nullptr);
  if (tr >= 0) trace_point(a, tr + 2);
  float m = 0.0f;
  for (int i = tid; i < E; i += CT) {
    const float y = rms_apply(X[i], ow[i], inv, a.err);
    X[i] = y;
    m = fmaxf(m, fabsf(y));
  }
  release_tile(slot);
  const float s = cmax_f(m);
  if (tr >= 0) trace_point(a, tr + 3);
  if (vok) quant_smem(X, E, 0, s);
  return s;
}

// quantize a row of K floats written by other CTAs in this step (bulk copies through the two
// vector buffers, 4096 floats at a time)
__device__ __noinline__ void quant_vec(const DecodeArgs &a, Cnt &c, const float *src, int K, float s) {
  const int nch = (K + VBUF - 1) / VBUF;
  if (tid_() == 0) {
    fence_proxy_async_smem();
    for (int ch = 0; ch < 2 && ch < nch; ch++)
      vload(ch, src + (size_t)ch * VBUF, (uint32_t)min(VBUF, K - ch * VBUF) * 4);
  }
  for (int ch = 0; ch < nch; ch++) {
    const int b = ch & 1;
    const bool ok = wait_bar(a, &g_sh.vbar[b], (b ? c.vp1++ : c.vp0++) & 1u);
    const int len = min(VBUF, K - ch * VBUF);
    if (ok) quant_smem(vb(b), len, ch * (VBUF / 32), s);
    cbar();
    if (tid_() == 0 && ch + 2 < nch) {
      fence_proxy_async_smem();
      vload(b, src + (size_t)(ch + 2) * VBUF, (uint32_t)min(VBUF, K - (ch + 2) * VBUF) * 4);
    }
  }
}

// per-lane partial dot of one (row, segment) unit: the warp's lanes own 32-column blocks b0 + 32 j
__device__ __forceinline__ int64_t unit_part(const uint8_t *crow, const uint16_t *srow, const int4 (&x0)[4],
                                             const int4 (&x1)[4], const int32_t (&xc)[4], const bool (&val)[4],
                                             int b0) {
  int64_t acc = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    if (val[j]) {
      const int b = b0 + 32 * j;
      const uint4 cw = *reinterpret_cast<const uint4 *>(crow + (size_t)b * 16);
      scale_acc(acc, srow[b], block_dot(cw, x0[j], x1[j]) + xc[j]);
    }
  }
  return acc;
}

// two units of two different tiles at once (independent chains the scheduler interleaves)
__device__ __forceinline__ void unit_part2(const uint8_t *ca, const uint16_t *sa_, const uint8_t *cb, const uint16_t *sb,
                                           const int4 (&x0)[4], const int4 (&x1)[4], const int32_t (&xc)[4],
                                           const bool (&val)[4], int b0, int64_t &pa, int64_t &pb) {
  int64_t acc_a = 0, acc_b = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    if (val[j]) {
      const int b = b0 + 32 * j;
      const uint4 wa = *reinterpret_cast<const uint4 *>(ca + (size_t)b * 16);
      const uint4 wb = *reinterpret_cast<const uint4 *>(cb + (size_t)b * 16);
      const uint32_t ha = sa_[b], hb = sb[b];
      scale_acc(acc_a, ha, block_dot(wa, x0[j], x1[j]) + xc[j]);
      scale_acc(acc_b, hb, block_dot(wb, x0[j], x1[j]) + xc[j]);
    }
  }
  pa = acc_a;
  pb = acc_b;
}

enum { PH_STORE = 0, PH_GELU = 1, PH_SILU = 2, PH_LM = 3 };

// One GEMV over this CTA's rows of w (and w2 for the gated phases), input = the activation
// codes in shared memory with scale factor dsc. STORE/GELU/SILU: y[row] after the phase
// (ymax: atomicMax of the CTA's max |y|); LM: logits and the greedy-argmax key per row.
// Tiles are taken two at a time (a gate tile and the up tile of the same rows in the gated
// phases) and every warp works on both at once; a warp releases the two slots as soon as it
// has read them, before its warp reductions, so the next copies start earlier.
template <int PH>
__device__ __noinline__ void gemv_phase(const DecodeArgs &a, Cnt &c, const DevQ4B &w, const DevQ4B &w2,
                                        double dsc, float *y, uint32_t *ymax) {
  const int warp = warp_(), lane = lane_(), tid = tid_();
  const int K = w.cols;
  const Tiling tl = tiling(K);
  int r0, r1;
  rows_of(w.rows, blockIdx.x, gridDim.x, r0, r1);
  const int seg = warp & (tl.segs - 1);
  const int b0 = seg * tl.sb + lane;
  int lsegs = 0;
  while ((1 << lsegs) < tl.segs) lsegs++;
  int4 x0[4], x1[4];
  int32_t xc[4];
  bool val[4];
  const int4 *p0 = reinterpret_cast<const int4 *>(xa()), *p1 = reinterpret_cast<const int4 *>(xa() + PLANE);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int bl = lane + 32 * j, b = b0 + 32 * j;
    val[j] = bl < tl.sb && b < tl.nblk;
    x0[j] = val[j] ? p0[b] : make_int4(0, 0, 0, 0);
    x1[j] = val[j] ? p1[b] : make_int4(0, 0, 0, 0);
    xc[j] = val[j] ? -8 * xs()[b] : 0;
  }
  constexpr int NM = (PH == PH_GELU || PH == PH_SILU) ? 2 : 1;
  unsigned long long *ra_ = racc();
  unsigned long long best = 0ull;
  const int nchunk = (r1 - r0 + tl.rt - 1) / tl.rt;
  const int ntiles = nchunk * NM;
  for (int t = 0; t < ntiles; t += 2) {
    const bool hasB = t + 1 < ntiles;
    // tile q (0: t, 1: t+1): matrix m and first row
    int slot[2] = {0, 0}, rows[2] = {0, 0}, m[2] = {0, 0}, ra[2] = {0, 0};
    bool rdy[2] = {false, false};
    for (int q = 0; q < 2; q++) {
      if (q == 1 && !hasB) break;
      const int tt = t + q;
      m[q] = NM == 2 ? (tt & 1) : 0;
      ra[q] = r0 + (NM == 2 ? (tt >> 1) : tt) * tl.rt;
      rows[q] = min(tl.rt, r1 - ra[q]);
      take_tile(a, c, slot[q], rdy[q]);
    }
    // per-lane partials of up to two units per tile: [tile][k] with unit = warp + CW k
    int64_t part[2][2] = {{0, 0}, {0, 0}};
    bool has[2][2];
#pragma unroll
    for (int q = 0; q < 2; q++)
#pragma unroll
      for (int k = 0; k < 2; k++) has[q][k] = rdy[q] && (warp + CW * k) < rows[q] * tl.segs;
    if (has[0][0] && has[1][0] && !has[0][1] && !has[1][1]) {   // the common case: one unit per tile
      const int rl = warp >> lsegs;
      const uint8_t *ca = ring_slot(slot[0]), *cb = ring_slot(slot[1]);
      const uint16_t *sa_ = reinterpret_cast<const uint16_t *>(ca + (size_t)rows[0] * (K >> 1));
      const uint16_t *sb = reinterpret_cast<const uint16_t *>(cb + (size_t)rows[1] * (K >> 1));
      unit_part2(ca + (size_t)rl * (K >> 1), sa_ + (size_t)rl * tl.nblk, cb + (size_t)rl * (K >> 1),
                 sb + (size_t)rl * tl.nblk, x0, x1, xc, val, b0, part[0][0], part[1][0]);
    } else {
#pragma unroll
      for (int k = 0; k < 2; k++) {
#pragma unroll
        for (int q = 0; q < 2; q++) {
          if (has[q][k]) {
            const int rl = (warp + CW * k) >> lsegs;
            const uint8_t *codes = ring_slot(slot[q]);
            const uint16_t *scl = reinterpret_cast<const uint16_t *>(codes + (size_t)rows[q] * (K >> 1));
            part[q][k] = unit_part(codes + (size_t)rl * (K >> 1), scl + (size_t)rl * tl.nblk, x0, x1, xc, val, b0);
          }
        }
      }
    }
    release_tile(slot[0]);
    if (hasB) release_tile(slot[1]);
#pragma unroll
    for (int k = 0; k < 2; k++) {
#pragma unroll
      for (int q = 0; q < 2; q++) {
        if (!has[q][k]) continue;
        const int64_t acc = warp_sum_i64(part[q][k]);
        if (lane == 0) {
          const int rl = (warp + CW * k) >> lsegs;
          const int row = ra[q] - r0 + rl;
          if (PH == PH_LM) {
            const float v = acc_to_f32(acc, dsc);
            y[ra[q] + rl] = v;
            const unsigned long long key = argmax_key(v, ra[q] + rl);
            best = key > best ? key : best;
          } else if (tl.segs == 1) {
            ra_[m[q] * RACC + row] = (unsigned long long)acc;
          } else {
            atomicAdd(ra_ + m[q] * RACC + row, (unsigned long long)acc);
          }
        }
      }
    }
  }
  if (PH == PH_LM) {
    if (tid == 0) g_sh.key = 0ull;
    cbar();
    if (lane == 0 && best) atomicMax(&g_sh.key, best);
    cbar();
    if (tid == 0 && g_sh.key) atomicMax(a.amax, g_sh.key);
    return;
  }
  cbar();
  float mx = 0.0f;
  for (int row = tid; row < r1 - r0; row += CT) {
    float v = acc_to_f32((long long)ra_[row], dsc);
    if (NM == 2) {
      const float u = acc_to_f32((long long)ra_[RACC + row], dsc);
      if (!(fabsf(v) < 2048.0f)) { raise_err(a.err, ERR_ACT_RANGE); v = 0.0f; }
      v = __fmul_rn(PH == PH_GELU ? gelu_exact(v) : silu_exact(v), u);
      ra_[RACC + row] = 0ull;
    }
    ra_[row] = 0ull;
    __stcg(y + r0 + row, v);
    mx = fmaxf(mx, fabsf(v));
  }
  if (ymax) {
    mx = cmax_f(mx);
    if (tid == 0) {
      if (!(mx <= 3.402823466e38f)) raise_err(a.err, ERR_ACT_RANGE);
      else atomicMax(ymax, __float_as_uint(mx));
    }
  }
}

// score of one cached or new key row against the G rotated queries
template <int HD>
__device__ __forceinline__ void score_row(const DecodeArgs &a, const int32_t *krow, int G, int idx, int SCS) {
  constexpr int EPL = HD / 32;
  const int lane = lane_();
  int32_t kv[EPL];
#pragma unroll
  for (int e = 0; e < EPL; e++) kv[e] = krow[lane * EPL + e];
  for (int h = 0; h < G; h++) {
    const int32_t *q = qs() + h * HD + lane * EPL;
    int64_t s = 0;
#pragma unroll
    for (int e = 0; e < EPL; e++) s += (int64_t)q[e] * (int64_t)kv[e];
    s = warp_sum_i64(s);
    if (lane == 0) {
      float z = __fmul_rn(__double2float_rn(__dmul_rn(__ll2double_rn(s), 0x1p-32)), a.ascale);
      if (!(fabsf(z) < 131072.0f)) { raise_err(a.err, ERR_SCORE_RANGE); z = 0.0f; }
      const int32_t zi = (int32_t)llround_d((double)z * 16384.0);
      sc()[h * SCS + idx] = zi;
      atomicMax(&g_sh.mx[h], zi);
    }
  }
}

__device__ __noinline__ int64_t floordiv_dec(int64_t hi, uint64_t lo, uint64_t d) { return floordiv_s128(hi, lo, d); }

// attention of layer L for this CTA's part; the outputs of the head land in a.ao and the
// layer's max |ao| slot. Returns false on abort.
template <int HD>
__device__ __noinline__ bool attn_phase(const DecodeArgs &a, Cnt &c, int L, const DecLayer &ly, int p) {
  const int tr = 1 + L * DEC_TRACE_PER_LAYER + 14;   // sub-phase trace points
  const int tid = tid_(), warp = warp_(), lane = lane_();
  const int G = a.NH / a.NKV, half = HD / 2;
  const int SCS = SCMAX / G;
  const AttnPart ap = attn_part(blockIdx.x, gridDim.x, a.NKV, p, ly.win);
  // the head counter collects 2 * npart arrivals per layer whether or not this CTA is a part
  uint32_t *hctr = a.sync + SYNC_HEAD + DEC_SYNC_WORDS_PER * ap.g;
  const uint32_t t1 = c.hep + ap.npart, t2 = c.hep + 2 * ap.npart;
  c.hep = t2;
  if (!ap.active) return true;
  const int cn = ap.c1 - ap.c0, ce = min(ap.c1, p), ncached = ce - ap.c0;
  const bool has_new = ap.c1 == p + 1;
  const size_t hoff = (size_t)L * a.kvl + (size_t)ap.g * a.P * HD;
  // the host checks this bound before choosing this kernel; past it the tiles are still
  // consumed and the barriers kept, only the arithmetic is skipped
  const bool fits = cn <= SCS;
  if (!fits && tid == 0) raise_err(a.err, ERR_SCORE_RANGE);
  // ---- raw q (G heads) [+ k, v of the new position] by one bulk copy
  const int nh = G + (has_new ? 1 : 0);   // rows: G query heads, then the key
  float *raw = vb(0);
  if (tid == 0) {
    fence_proxy_async_smem();
    asm volatile("fence.proxy.async.global;" ::: "memory");
    const uint32_t qb = (uint32_t)(G * HD) * 4, kb = (uint32_t)HD * 4;
    mbar_arrive_expect_tx(&g_sh.vbar[0], qb + (has_new ? 2 * kb : 0));
    bulk_g2s(raw, a.qkv + (size_t)ap.g * G * HD, qb, &g_sh.vbar[0]);
    if (has_new) {
      vload_more(0, G * HD, a.qkv + a.QD + (size_t)ap.g * HD, kb);
      vload_more(0, (G + 1) * HD, a.qkv + a.QD + a.KVD + (size_t)ap.g * HD, kb);
    }
  }
  if (tid < G) { g_sh.mx[tid] = INT32_MIN; g_sh.ssum[tid] = 0ull; }
  wait_bar(a, &g_sh.vbar[0], (c.vp0++) & 1u);
  cbar();
  if (warp < nh) {   // one warp per head row: the QK-norm island's inverse rms
    const float *nw = warp < G ? ly.q_norm : ly.k_norm;
    uint64_t inv = 0;
    if (nw) {
      acc128 ss{0ull, 0ll};
      bool bad = false;
      for (int d = lane; d < HD; d += 32) {
        const float x = raw[warp * HD + d];
        if (!(fabsf(x) < 32768.0f)) { bad = true; continue; }
        const int64_t q = q16_round(x);
        acc128_add(ss, q * q);
      }
      if (bad) raise_err(a.err, ERR_NORM_RANGE);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        acc128 r;
        r.lo = __shfl_xor_sync(0xffffffffu, ss.lo, o);
        r.hi = __shfl_xor_sync(0xffffffffu, ss.hi, o);
        acc128_add(ss, r);
      }
      if (lane == 0) inv = rms_inv_dec(ss, HD, a.err);
    }
    if (lane == 0) g_sh.inv[warp] = inv;
  }
  cbar();
  for (int i = tid; i < nh * half; i += CT) {
    const int r = i / half, d = i % half;
    const float *nw = r < G ? ly.q_norm : ly.k_norm;
    float va = raw[r * HD + d], vb_ = raw[r * HD + d + half];
    if (nw) {
      const uint64_t inv = g_sh.inv[r];
      va = rms_apply(va, __ldg(nw + d), inv, a.err);
      vb_ = rms_apply(vb_, __ldg(nw + d + half), inv, a.err);
    }
    int32_t oa, ob;
    cordic_rotate<1>(va, vb_, (uint64_t)(int64_t)p * __ldg(ly.W + d), g_sh.T, a.gain, oa, ob, a.err);
    if (r < G) {
      qs()[r * HD + d] = oa;
      qs()[r * HD + d + half] = ob;
    } else {
      kn()[d] = oa;
      kn()[d + half] = ob;
      int32_t *dst = a.kc + hoff + (size_t)p * HD;
      dst[d] = oa;
      dst[d + half] = ob;
    }
  }
  if (has_new) {
    for (int d = tid; d < HD; d += CT) {
      const float v = raw[(G + 1) * HD + d];
      int32_t q = 0;
      if (!(fabsf(v) < 16384.0f)) raise_err(a.err, ERR_V_RANGE);
      else q = __float2int_rn(__fmul_rn(v, 65536.0f));
      vn()[d] = q;
      a.vc[hoff + (size_t)p * HD + d] = q;
    }
  }
  cbar();
  trace_point(a, tr);
  // ---- exact scores -> the 2^14 grid; K slices through the ring
  const int sub = SLOT / (HD * 4);
  const int nsub = (ncached + sub - 1) / sub;
  for (int t = 0; t < nsub; t++) {
    int slot;
    bool ready;
    take_tile(a, c, slot, ready);
    const int len = min(sub, ncached - t * sub);
    const int32_t *buf = reinterpret_cast<const int32_t *>(ring_slot(slot));
    if (ready && fits)
      for (int pp = warp; pp < len; pp += CW) score_row<HD>(a, buf + pp * HD, G, t * sub + pp, SCS);
    release_tile(slot);
  }
  if (fits && has_new && warp == 0) score_row<HD>(a, kn(), G, ncached, SCS);
  cbar();
  trace_point(a, tr + 1);
  if (tid < G) a.pmx[blockIdx.x * G + tid] = g_sh.mx[tid];
  if (!counter_sync(a, hctr, t1)) return false;
  trace_point(a, tr + 2);
  // ---- head maximum (one warp per query head gathers the parts), integer exponentials,
  // their exact sum
  if (warp < G) {
    int32_t m = INT32_MIN;
    for (int jj = lane; jj < ap.npart; jj += 32) m = max(m, __ldcg(a.pmx + (ap.g + a.NKV * jj) * G + warp));
    m = warp_max_i32(m);
    if (lane == 0) g_sh.mg[warp] = m;
  }
  cbar();
  for (int h = 0; h < G && fits; h++) {
    int64_t part = 0;
    const int64_t mg = g_sh.mg[h];
    for (int i = tid; i < cn; i += CT) {
      const int64_t d = (((int64_t)sc()[h * SCS + i] - mg) * ONE) >> 14;
      const int32_t e = (int32_t)exp_fixed(d);
      sc()[h * SCS + i] = e;
      part += e;
    }
    part = warp_sum_i64(part);
    if (lane == 0 && part) atomicAdd(&g_sh.ssum[h], (unsigned long long)part);
  }
  cbar();
  trace_point(a, tr + 3);
  // ---- exact V-sum: e * v split at bit 16 so both halves accumulate in int64
  const int GH = G * HD;
  int64_t vh0 = 0, vl0 = 0, vh1 = 0, vl1 = 0;   // outputs tid and tid + CT
  for (int t = 0; t < nsub; t++) {
    int slot;
    bool ready;
    take_tile(a, c, slot, ready);
    const int len = min(sub, ncached - t * sub);
    const int32_t *buf = reinterpret_cast<const int32_t *>(ring_slot(slot));
    if (ready && fits) {
      for (int r = 0; r < 2; r++) {
        const int o = tid + r * CT;
        if (o >= GH) break;
        const int h = o / HD, d = o % HD;
        const int32_t *e = sc() + h * SCS + t * sub;
        int64_t vh = 0, vl = 0;
        for (int pp = 0; pp < len; pp++) {
          const int32_t v = buf[pp * HD + d];
          const int64_t ev = e[pp];
          vh += ev * (int64_t)(v >> 16);
          vl += ev * (int64_t)(v & 0xFFFF);
        }
        if (r) { vh1 += vh; vl1 += vl; }
        else { vh0 += vh; vl0 += vl; }
      }
    }
    release_tile(slot);
  }
  for (int r = 0; r < 2; r++) {
    const int o = tid + r * CT;
    if (o >= GH) break;
    const int h = o / HD, d = o % HD;
    int64_t vh = r ? vh1 : vh0, vl = r ? vl1 : vl0;
    if (has_new && fits) {
      const int32_t v = vn()[d];
      const int64_t ev = sc()[h * SCS + ncached];
      vh += ev * (int64_t)(v >> 16);
      vl += ev * (int64_t)(v & 0xFFFF);
    }
    // N = vh * 2^16 + vl as a 128-bit value
    acc128 N{(uint64_t)vh << 16, vh >> 48};
    acc128_add(N, vl);
    uint64_t *dst = a.pnum + ((size_t)blockIdx.x * GH + o) * 2;
    __stcg(dst, N.lo);
    __stcg(dst + 1, (uint64_t)N.hi);
  }
  if (tid < G) __stcg(reinterpret_cast<unsigned long long *>(a.psum) + blockIdx.x * G + tid, g_sh.ssum[tid]);
  trace_point(a, tr + 4);
  if (!counter_sync(a, hctr, t2)) return false;
  trace_point(a, tr + 5);
  // ---- this part finalizes outputs [j*fo, (j+1)*fo) of the head group: one warp per
  // output, its lanes gather the parts' partial sums in parallel
  const int fo = (GH + ap.npart - 1) / ap.npart;
  const int o0 = ap.j * fo, o1 = min(o0 + fo, GH);
  float omax = 0.0f;
  for (int o = o0 + warp; o < o1; o += CW) {
    const int h = o / HD, d = o % HD;
    acc128 N{0ull, 0ll};
    int64_t S = 0;
    for (int jj = lane; jj < ap.npart; jj += 32) {
      const int cc = ap.g + a.NKV * jj;
      const uint64_t *src = a.pnum + ((size_t)cc * GH + o) * 2;
      acc128_add(N, acc128{__ldcg(src), (int64_t)__ldcg(src + 1)});
      S += (int64_t)__ldcg(reinterpret_cast<const unsigned long long *>(a.psum) + cc * G + h);
    }
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) {
      acc128 r;
      r.lo = __shfl_xor_sync(0xffffffffu, N.lo, sh);
      r.hi = __shfl_xor_sync(0xffffffffu, N.hi, sh);
      acc128_add(N, r);
    }
    S = warp_sum_i64(S);
    if (lane == 0) {
      const int64_t hi = (int64_t)(((uint64_t)N.hi << 16) | (N.lo >> 48));   // N * 2^16, |N| < 2^78
      const uint64_t lo = N.lo << 16;
      const int64_t qd = S > 0 ? floordiv_dec(hi, lo, (uint64_t)S) : 0;
      const float out = __double2float_rn(__dmul_rn(__ll2double_rn(qd), 0x1p-32));
      __stcg(a.ao + (size_t)(ap.g * G + h) * HD + d, out);
      omax = fmaxf(omax, fabsf(out));
    }
  }
  omax = cmax_f(omax);
  if (tid == 0) atomicMax(a.slots + 2 * L, __float_as_uint(omax));
  return true;
}

__device__ bool attn_dispatch(const DecodeArgs &a, Cnt &c, int L, const DecLayer &ly, int p) {
  switch (a.HD) {
    case 64: return attn_phase<64>(a, c, L, ly, p);
    case 128: return attn_phase<128>(a, c, L, ly, p);
    default: return attn_phase<256>(a, c, L, ly, p);
  }
}

__device__ void consumer(const DecodeArgs &a, int p) {
  float *xb[2] = {a.x2, a.x2 + a.E};
  int cur = 0;
  const DevQ4B none{nullptr, nullptr, 0, 0};
  Cnt c{0u, 0u, 0u, 0u, 0u};
  load_layer(a, 0);
  if (tid_() < CORDIC_ITERS) g_sh.T[tid_()] = __ldg(a.T + tid_());
  cbar();
  trace_point(a, 0);
  for (int L = 0; L < a.NL; L++) {
    const DecLayer &ly = g_sh.ly[L % 3];
    const int tk = 1 + L * DEC_TRACE_PER_LAYER;
    // attention block
    float s = norm_phase(a, c, L == 0, xb[cur], L ? a.dn : nullptr, L && a.gemma, xb[cur ^ 1],
                         a.trace ? tk + 20 : -1);
    cur ^= 1;
    cbar();
    trace_point(a, tk + 0);
    gemv_phase<PH_STORE>(a, c, ly.qkv, none, act_dscale(s), a.qkv, nullptr);
    trace_point(a, tk + 1);
    load_layer(a, L + 1);   // overlaps the barrier wait
    if (!grid_sync(a, c)) return;
    trace_point(a, tk + 2);
    if (!attn_dispatch(a, c, L, ly, p)) return;
    trace_point(a, tk + 3);
    if (!grid_sync(a, c)) return;
    trace_point(a, tk + 4);
    s = __uint_as_float(__ldcg(a.slots + 2 * L));
    quant_vec(a, c, a.ao, a.QD, s);
    cbar();
    trace_point(a, tk + 5);
    gemv_phase<PH_STORE>(a, c, ly.o, none, act_dscale(s), a.ap, nullptr);
    trace_point(a, tk + 6);
    if (!grid_sync(a, c)) return;
    trace_point(a, tk + 7);
    // feed-forward block
    s = norm_phase(a, c, false, xb[cur], a.ap, a.gemma != 0, xb[cur ^ 1]);
    cur ^= 1;
    cbar();
    trace_point(a, tk + 8);
    if (a.gemma) gemv_phase<PH_GELU>(a, c, ly.g, ly.u, act_dscale(s), a.gg, a.slots + 2 * L + 1);
    else gemv_phase<PH_SILU>(a, c, ly.g, ly.u, act_dscale(s), a.gg, a.slots + 2 * L + 1);
    trace_point(a, tk + 9);
    if (!grid_sync(a, c)) return;
    trace_point(a, tk + 10);
    s = __uint_as_float(__ldcg(a.slots + 2 * L + 1));
    quant_vec(a, c, a.gg, a.FF, s);
    cbar();
    trace_point(a, tk + 11);
    gemv_phase<PH_STORE>(a, c, ly.d, none, act_dscale(s), a.dn, nullptr);
    trace_point(a, tk + 12);
    if (!grid_sync(a, c)) return;
    trace_point(a, tk + 13);
  }
  const int tf = 1 + a.NL * DEC_TRACE_PER_LAYER;
  const float s = norm_phase(a, c, false, xb[cur], a.dn, a.gemma != 0, xb[cur ^ 1]);
  cbar();
  trace_point(a, tf);
  gemv_phase<PH_LM>(a, c, a.out, none, act_dscale(s), a.logits, nullptr);
  trace_point(a, tf + 1);
  if (!grid_sync(a, c)) return;
  trace_point(a, tf + 2);
  if (blockIdx.x == 0 && tid_() == 0) {
    const unsigned long long key = *(volatile unsigned long long *)a.amax;
    const int32_t next = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
    *a.argmax_dev = next;
    *a.tok_dev = next;
    *a.pos_dev = p + 1;
  }
}

__global__ void __launch_bounds__(NTHREADS, 1) k_decode(const __grid_constant__ DecodeArgs a) {
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    for (int s = 0; s < NSLOT; s++) {
      mbar_init(&g_sh.full[s], 1);
      mbar_init(&g_sh.empty[s], CW);
    }
    mbar_init(&g_sh.vbar[0], 1);
    mbar_init(&g_sh.vbar[1], 1);
    g_sh.abort = 0;
    g_sh.issued = 0;
    mbar_init_fence();
  }
  for (int i = tid; i < 2 * RACC; i += NTHREADS) racc()[i] = 0ull;
  __syncthreads();
  const int p = a.pos_dev[0];
  int tok = a.tok_dev[0];
  if (tok < 0 || tok >= a.V) {
    if (tid == 0) raise_err(a.err, ERR_TOKEN);
    tok = 0;
  }
  if (warp == CW) {
    if ((tid & 31) == 0) g_sh.issued = produce(a, p, tok);
    __syncwarp();
  } else {
    consumer(a, p);
  }
  __syncthreads();
  if (tid == 0) {
    // copies still in flight (only after an abort): wait for the last one of each slot
    const uint32_t issued = g_sh.issued;
    for (int s = 0; s < NSLOT; s++) {
      if ((uint32_t)s >= issued) break;
      const uint32_t last = issued - 1 - ((issued - 1 - (uint32_t)s) % NSLOT);
      const uint64_t t0 = now_ns();
      while (!mbar_try_wait(&g_sh.full[s], (last / NSLOT) & 1u))
        if (now_ns() - t0 > WAIT_LIMIT_NS) break;
    }
    // the last CTA out resets the counters and the per-layer slots for the next step
    __threadfence();
    const uint32_t t = atomicAdd(a.sync + SYNC_EXIT, 1u);
    if (t == gridDim.x - 1) {
      __threadfence();
      a.sync[SYNC_GRID] = 0u;
      for (int g = 0; g < a.NKV; g++) a.sync[SYNC_HEAD + DEC_SYNC_WORDS_PER * g] = 0u;
      for (int i = 0; i < 2 * a.NL; i++) a.slots[i] = 0u;
      *a.amax = 0ull;
      a.sync[SYNC_ABORT] = 0u;
      __threadfence();
      a.sync[SYNC_EXIT] = 0u;
    }
  }
}

// ------------------------------------------------------------------------------ ring GEMV
// The GEMV phase as a kernel of its own (batch-1 GEMVs of the multi-kernel schedule): the
// producer warp streams this CTA's row tiles into the ring before the programmatic-dependent-
// launch wait (the weights do not depend on the previous kernel), the consumers wait, stage
// the quantized activation row and run gemv_phase.
__global__ void __launch_bounds__(NTHREADS, 1) k_gemv_ring(const __grid_constant__ GemvRingArgs g) {
  __shared__ DecodeArgs sa;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    for (int s = 0; s < NSLOT; s++) {
      mbar_init(&g_sh.full[s], 1);
      mbar_init(&g_sh.empty[s], CW);
    }
    g_sh.abort = 0;
    g_sh.issued = 0;
    mbar_init_fence();
    memset(&sa, 0, sizeof sa);
    sa.err = g.err;
    sa.amax = g.amax;
  }
  for (int i = tid; i < 2 * RACC; i += NTHREADS) racc()[i] = 0ull;
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == CW) {
    if ((tid & 31) == 0) {
      const DevQ4B *w2 = g.mode == 1 || g.mode == 2 ? &g.w2 : nullptr;
      int r, r1;
      rows_of(g.w.rows, blockIdx.x, gridDim.x, r, r1);
      const int K = g.w.cols, rt = tiling(K).rt;
      uint32_t T = 0;
      for (; r < r1; r += rt) {
        const int rows = min(rt, r1 - r);
        for (int m = 0; m < (w2 ? 2 : 1); m++) {
          const DevQ4B &q = m ? *w2 : g.w;
          Tile t{q.codes + (size_t)r * (K >> 1), reinterpret_cast<const uint8_t *>(q.scales) + (size_t)r * (K >> 4),
                 (uint32_t)rows * (K >> 1), (uint32_t)rows * (K >> 4)};
          if (!ring_issue(sa, T, t)) break;
          T++;
        }
        if (aborted()) break;
      }
      g_sh.issued = T;
    }
    __syncwarp();
  } else {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the activation row: per 32-column block, bytes 0-15 to plane 0 and 16-31 to plane 1
    const int nblk = g.w.cols >> 5;
    const int4 *q4 = reinterpret_cast<const int4 *>(g.act.q);
    int4 *p0 = reinterpret_cast<int4 *>(xa()), *p1 = reinterpret_cast<int4 *>(xa() + PLANE);
    for (int b = tid; b < nblk; b += CT) {
      p0[b] = q4[2 * b];
      p1[b] = q4[2 * b + 1];
      xs()[b] = g.act.bsum[b];
    }
    const double dsc = act_dscale(g.act.scale[0]);
    cbar();
    Cnt c{0u, 0u, 0u, 0u, 0u};
    switch (g.mode) {
      case 0: gemv_phase<PH_STORE>(sa, c, g.w, g.w, dsc, g.y, g.ymax); break;
      case 1: gemv_phase<PH_GELU>(sa, c, g.w, g.w2, dsc, g.y, g.ymax); break;
      case 2: gemv_phase<PH_SILU>(sa, c, g.w, g.w2, dsc, g.y, g.ymax); break;
      default: gemv_phase<PH_LM>(sa, c, g.w, g.w, dsc, g.y, nullptr); break;
    }
  }
  __syncthreads();
  if (tid == 0) {   // copies still in flight (only after an abort)
    const uint32_t issued = g_sh.issued;
    for (int s = 0; s < NSLOT; s++) {
      if ((uint32_t)s >= issued) break;
      const uint32_t last = issued - 1 - ((issued - 1 - (uint32_t)s) % NSLOT);
      const uint64_t t0 = now_ns();
      while (!mbar_try_wait(&g_sh.full[s], (last / NSLOT) & 1u))
        if (now_ns() - t0 > WAIT_LIMIT_NS) break;
    }
  }
}

}  // namespace

bool gemv_ring_covers(const DevQ4B &w, int mode) {
  const int K = w.cols;
  if (K > KMAX || (K & 255) || w.rows <= 0) return false;
  int segs = 1;
  while (segs * 128 < K / 32) segs <<= 1;
  const int rt = std::min(16, SLOT / (K / 2 + K / 16));
  if (rt * segs > 2 * CW) return false;
  const int grid = decode_grid();
  if (grid <= 0) return false;
  if (mode != 3 && (((w.rows + 3) / 4 + grid - 1) / grid) * 4 > RACC) return false;
  return (long long)((w.rows + 3) / 4) * grid <= 0x7fffffffLL;
}

cudaError_t launch_gemv_ring(const GemvRingArgs &g, cudaStream_t st, bool pdl) {
  static int grid = 0;
  if (grid == 0) grid = decode_grid();
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv_ring, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_gemv_ring, g);
}

const char *decode_unsupported(const DecodeArgs &a, int grid, int ctx) {
  if (grid <= 0) return "the persistent decode kernel cannot be resident on this device";
  if (a.E > EMAX || (a.E & 31)) return "d_model above 4096 or not a multiple of 32";
  const int Ks[3] = {a.E, a.QD, a.FF};
  for (int K : Ks)
    if (K > KMAX || (K & 255)) return "a GEMV width above 16384 or not a multiple of 256";
  if (a.NH % a.NKV || a.NKV > grid) return "head layout";
  const int G = a.NH / a.NKV;
  if (G > 8 || G * a.HD > GHMAX || a.HD > HDMAX || (a.HD != 64 && a.HD != 128 && a.HD != 256))
    return "query heads per KV head x head_dim above 512";
  if ((G + 2) * a.HD > VBUF) return "query/key/value rows above the vector buffer";
  const int Kw[3] = {a.E, a.QD, a.FF};
  for (int K : Kw) {   // units per tile (rows x column segments) at most 2 per compute warp
    int segs = 1;
    while (segs * 128 < K / 32) segs <<= 1;
    if (std::min(16, SLOT / (K / 2 + K / 16)) * segs > 2 * CW) return "GEMV tile above two units per warp";
  }
  const int rmax[3] = {a.E, a.FF, a.QD + 2 * a.KVD};
  for (int R : rmax)
    if ((((R + 3) / 4 + grid - 1) / grid) * 4 > RACC) return "rows per CTA above the accumulator capacity";
  if ((long long)((a.V + 3) / 4) * grid > 0x7fffffffLL) return "vocabulary too large for the row split";
  // scores per part: ceil(n / parts) with at least MINP positions per part
  const int avail = grid / a.NKV;
  const int cs = std::max(MINP, (ctx + avail - 1) / avail);
  if (cs * G > SCMAX) return "context too long for the per-CTA score buffer";
  return nullptr;
}

int decode_grid() {
  int dev = 0, nsm = 0, coop = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !coop) return 0;
  if (cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  int per = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_decode, NTHREADS, SMEM) != cudaSuccess || per < 1) {
    (void)cudaGetLastError();
    return 0;
  }
  return nsm;
}

cudaError_t launch_decode(const DecodeArgs &a, int grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_decode, a);
}

}  // namespace spb
