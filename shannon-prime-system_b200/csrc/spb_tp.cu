// spb_tp.cu -- tensor-parallel group: one process per GPU, NCCL over NVLink for the exchanges.
//
// The row-split matrices (attention output projection, FFN down projection) end in an
// all-reduce of their exact int64 partial sums, which is byte-exact in any order or topology;
// the activation quantizer's per-row max |u| of a column-split producer is a max all-reduce of
// the f32 bit patterns (non-negative floats order as their bits); the vocabulary-split LM head
// ends in a max all-reduce of its greedy-argmax keys and an all-gather of its logits.
//
// Small messages (the decode step's) go through a one-shot exchange over peer memory once the
// group has connected its mailboxes (spb_tp_p2p_init / _connect); larger ones and groups without
// mailboxes use NCCL, resolved at run time (dlopen of libnccl.so.2): a process that already
// loaded one (torch does) shares it, and single-GPU use never needs the library.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/spb200.h"
#include "spb_kernels.cuh"
#include "spb_tp.cuh"

namespace {

struct NcclApi {
  bool ok = false;
  char why[256] = {0};
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRank) commInitRank = nullptr;
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclAllReduce) allReduce = nullptr;
  decltype(&ncclAllGather) allGather = nullptr;
  decltype(&ncclGetErrorString) errorString = nullptr;
};

const NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      snprintf(api.why, sizeof(api.why), "dlopen libnccl.so.2: %s", dlerror());
      return;
    }
#define SPB_SYM(field, name)                                                  \
  api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name));          \
  if (!api.field) {                                                           \
    snprintf(api.why, sizeof(api.why), "libnccl: missing symbol %s", name);   \
    return;                                                                   \
  }
    SPB_SYM(getUniqueId, "ncclGetUniqueId");
    SPB_SYM(commInitRank, "ncclCommInitRank");
    SPB_SYM(commDestroy, "ncclCommDestroy");
    SPB_SYM(allReduce, "ncclAllReduce");
    SPB_SYM(allGather, "ncclAllGather");
    SPB_SYM(errorString, "ncclGetErrorString");
#undef SPB_SYM
    api.ok = true;
  });
  return api;
}

int nccl_fail(const char *what, ncclResult_t r) {
  char msg[320];
  snprintf(msg, sizeof(msg), "spb_tp: %s: %s", what, nccl().errorString ? nccl().errorString(r) : "nccl error");
  return spb::record_error(SPB_ECUDA, msg);
}

}  // namespace

// ---- one-shot exchange over peer memory (small messages: the decode-step exchanges) ----
// Each rank owns a mailbox in its HBM, mapped into every other rank through CUDA IPC:
// words [16 p] hold source p's flag (128 bytes apart), then data[2][world][cap] uint64. One CTA
// pushes this rank's n values into slot [parity][rank] of every mailbox, fences at system
// scope and raises its flag in each; then it waits for every source's flag in its own mailbox
// (bounded by %globaltimer: ERR_TIMEOUT after 2 s, the wait then ends and the kernel returns
// with the missing sources' slots unread) and reduces the world slots locally. The
// exchange number e comes from a device counter (so graph replays stay in step); slots
// alternate with e's parity, so a rank that is one exchange ahead never overwrites a slot that
// is still being read.
constexpr int P2P_MAX = 8;
constexpr int P2P_FLAG_WORDS = 16 * P2P_MAX;
constexpr int P2P_THREADS = 1024;

enum P2POp : int { P2P_SUM_I64 = 0, P2P_MAX_U32 = 1, P2P_MAX_U64 = 2 };

struct P2PArgs {
  uint64_t *mbox[P2P_MAX];   // every rank's mailbox (this rank's own included) in this address space
  uint64_t *epoch;
  uint32_t *err;
  const void *src;
  void *dst;
  int n, cap, rank, world, op;
  uint64_t timeout_ns;       // the bounded wait's limit
};

constexpr uint64_t P2P_TIMEOUT_NS = 2000000000ull;

__device__ __forceinline__ uint64_t p2p_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(P2P_THREADS) k_p2p_exchange(P2PArgs a) {
  const uint64_t e = *(volatile uint64_t *)a.epoch + 1;
  const size_t par = e & 1;
  for (int p = 0; p < a.world; p++) {
    uint64_t *slot = a.mbox[p] + P2P_FLAG_WORDS + (par * a.world + a.rank) * (size_t)a.cap;
    for (int i = threadIdx.x; i < a.n; i += P2P_THREADS)
      slot[i] = a.op == P2P_MAX_U32 ? (uint64_t)static_cast<const uint32_t *>(a.src)[i]
                                    : static_cast<const uint64_t *>(a.src)[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < a.world) {
    uint64_t *flag = a.mbox[threadIdx.x] + 16 * a.rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(e) : "memory");
    const uint64_t *mine = a.mbox[a.rank] + 16 * threadIdx.x;
    const uint64_t t0 = p2p_now();
    for (;;) {
      uint64_t v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
      if (v >= e) break;
      if (p2p_now() - t0 > a.timeout_ns) {
        atomicOr(a.err, spb::ERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
  const uint64_t *data = a.mbox[a.rank] + P2P_FLAG_WORDS + par * a.world * (size_t)a.cap;
  for (int i = threadIdx.x; i < a.n; i += P2P_THREADS) {
    uint64_t acc = data[i];
    for (int s = 1; s < a.world; s++) {
      const uint64_t v = data[(size_t)s * a.cap + i];
      if (a.op == P2P_SUM_I64) acc += v;   // two's complement: the int64 sum
      else acc = v > acc ? v : acc;
    }
    if (a.op == P2P_MAX_U32) static_cast<uint32_t *>(a.dst)[i] = (uint32_t)acc;
    else static_cast<uint64_t *>(a.dst)[i] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) *a.epoch = e;
}

struct spb_tp {
  int rank = 0, world = 1, device = 0;
  ncclComm_t comm = nullptr;
  // peer-memory exchange (after spb_tp_p2p_connect)
  int cap = 0;
  uint64_t *mbox = nullptr;            // own mailbox
  uint64_t *peer[P2P_MAX] = {};        // mapped mailboxes (peer[rank] == mbox)
  uint64_t *epoch = nullptr;
  uint32_t *err = nullptr;
  bool p2p = false;
};

static_assert(sizeof(ncclUniqueId) == SPB_TP_ID_BYTES, "NCCL unique id size");

extern "C" int spb_tp_shard(const spb_config *cfg, int rank, int world, int32_t out[8]) {
  if (!cfg || !out) return spb::record_error(SPB_EBADARG, "spb_tp_shard: null arg");
  if (world <= 0 || rank < 0 || rank >= world) return spb::record_error(SPB_EBADARG, "spb_tp_shard: bad rank/world");
  if (cfg->n_head_kv % world)
    return spb::record_error(SPB_EUNSUPPORTED, "spb_tp_shard: n_head_kv is not a multiple of the group size");
  if (cfg->n_ff % (32 * world))
    return spb::record_error(SPB_EUNSUPPORTED, "spb_tp_shard: n_ff is not a multiple of 32 x the group size");
  if (cfg->n_vocab % world) return spb::record_error(SPB_EUNSUPPORTED, "spb_tp_shard: n_vocab % group size != 0");
  const int nkv = cfg->n_head_kv / world, nh = nkv * (cfg->n_head / cfg->n_head_kv);
  if ((nh * cfg->head_dim) & 31)
    return spb::record_error(SPB_EUNSUPPORTED, "spb_tp_shard: a rank's heads are not whole 32-column blocks");
  const int nff = cfg->n_ff / world, nv = cfg->n_vocab / world;
  out[0] = rank * nh;   out[1] = nh;    // query heads
  out[2] = rank * nkv;  out[3] = nkv;   // KV heads (the query heads' GQA groups)
  out[4] = rank * nff;  out[5] = nff;   // FFN columns (gate/up rows, down columns)
  out[6] = rank * nv;   out[7] = nv;    // LM-head rows
  return SPB_OK;
}

extern "C" int spb_tp_unique_id(uint8_t *id) {
  if (!id) return spb::record_error(SPB_EBADARG, "spb_tp_unique_id: null arg");
  if (!nccl().ok) return spb::record_error(SPB_EUNSUPPORTED, nccl().why);
  ncclUniqueId u;
  const ncclResult_t r = nccl().getUniqueId(&u);
  if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
  memcpy(id, &u, sizeof(u));
  return SPB_OK;
}

extern "C" int spb_tp_open(const uint8_t *id, int rank, int world, int device, spb_tp **out) {
  if (!id || !out || world <= 0 || rank < 0 || rank >= world)
    return spb::record_error(SPB_EBADARG, "spb_tp_open: bad arg");
  *out = nullptr;
  if (!nccl().ok) return spb::record_error(SPB_EUNSUPPORTED, nccl().why);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return spb::record_error(SPB_ECUDA, cudaGetErrorString(e));
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  spb_tp *tp = new spb_tp();
  tp->rank = rank;
  tp->world = world;
  tp->device = device;
  const ncclResult_t r = nccl().commInitRank(&tp->comm, world, u, rank);
  if (r != ncclSuccess) {
    delete tp;
    return nccl_fail("ncclCommInitRank", r);
  }
  *out = tp;
  return SPB_OK;
}

extern "C" void spb_tp_close(spb_tp *tp) {
  if (!tp) return;
  cudaSetDevice(tp->device);
  cudaDeviceSynchronize();
  for (int p = 0; p < tp->world && p < P2P_MAX; p++)
    if (tp->peer[p] && tp->peer[p] != tp->mbox) cudaIpcCloseMemHandle(tp->peer[p]);
  cudaFree(tp->mbox);
  cudaFree(tp->epoch);
  if (tp->comm) nccl().commDestroy(tp->comm);
  delete tp;
}

// blob = cudaIpcMemHandle_t of the mailbox, then the device UUID
extern "C" int spb_tp_p2p_init(spb_tp *tp, int cap, uint8_t *blob) {
  if (!tp || !blob || cap <= 0) return spb::record_error(SPB_EBADARG, "spb_tp_p2p_init: bad arg");
  if (tp->world > P2P_MAX) return spb::record_error(SPB_EUNSUPPORTED, "spb_tp_p2p_init: more than 8 ranks");
  if (tp->mbox) return spb::record_error(SPB_EBADSTATE, "spb_tp_p2p_init: already initialised");
  cudaError_t e = cudaSetDevice(tp->device);
  const size_t words = P2P_FLAG_WORDS + (size_t)2 * tp->world * cap;
  if (e == cudaSuccess) e = cudaMalloc(&tp->mbox, words * 8);
  if (e == cudaSuccess) e = cudaMemset(tp->mbox, 0, words * 8);
  if (e == cudaSuccess) e = cudaMalloc(&tp->epoch, 64);
  if (e == cudaSuccess) e = cudaMemset(tp->epoch, 0, 64);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, tp->mbox);
  cudaDeviceProp prop;
  if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, tp->device);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return spb::record_error(SPB_ECUDA, cudaGetErrorString(e));
  tp->err = reinterpret_cast<uint32_t *>(tp->epoch + 1);
  tp->cap = cap;
  memcpy(blob, &h, sizeof(h));
  memcpy(blob + sizeof(h), &prop.uuid, 16);
  return SPB_OK;
}

extern "C" int spb_tp_p2p_connect(spb_tp *tp, const uint8_t *blobs) {
  if (!tp || !blobs || !tp->mbox) return spb::record_error(SPB_EBADSTATE, "spb_tp_p2p_connect: call spb_tp_p2p_init first");
  const size_t B = SPB_TP_P2P_BLOB_BYTES;
  // ranks that wait on one another must sit on distinct GPUs
  for (int p = 0; p < tp->world; p++)
    for (int q = p + 1; q < tp->world; q++)
      if (!memcmp(blobs + p * B + sizeof(cudaIpcMemHandle_t), blobs + q * B + sizeof(cudaIpcMemHandle_t), 16))
        return spb::record_error(SPB_EUNSUPPORTED, "spb_tp_p2p_connect: two ranks share one GPU");
  cudaError_t e = cudaSetDevice(tp->device);
  for (int p = 0; p < tp->world && e == cudaSuccess; p++) {
    if (p == tp->rank) {
      tp->peer[p] = tp->mbox;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, blobs + p * B, sizeof(h));
    void *ptr = nullptr;
    e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    tp->peer[p] = static_cast<uint64_t *>(ptr);
  }
  if (e != cudaSuccess) return spb::record_error(SPB_ECUDA, cudaGetErrorString(e));
  tp->p2p = true;
  return SPB_OK;
}

// Diagnostics of the bounded wait: rank 0 of a group of `world` mailboxes that all live on the
// current device. The sources not in absent_mask have already arrived (their flag and n values
// are in place before the launch); the absent ones never do, so the kernel's wait runs out after
// timeout_ms and it raises ERR_TIMEOUT. No second process or GPU takes part, so nothing else
// can hang.
extern "C" int spb_tp_p2p_loopback(int world, uint32_t absent_mask, int timeout_ms, int n) {
  if (world < 2 || world > P2P_MAX || timeout_ms <= 0 || timeout_ms > 10000 || n <= 0 || n > 4096 ||
      (absent_mask & 1u) || (absent_mask >> world))
    return spb::record_error(SPB_EBADARG, "spb_tp_p2p_loopback: bad arg");
  const size_t words = P2P_FLAG_WORDS + (size_t)2 * world * n;
  uint64_t *mb = nullptr, *io = nullptr;
  cudaError_t e = cudaMalloc(&mb, words * 8 * world);
  if (e == cudaSuccess) e = cudaMalloc(&io, (size_t)(2 * n + 16) * 8);
  std::vector<uint64_t> h0(words, 0), src(n), got(n);
  for (int i = 0; i < n; i++) src[i] = (uint64_t)(i * 7 + 1);
  uint64_t want_sum = 0;
  for (int p = 1; p < world; p++) {
    if (absent_mask & (1u << p)) continue;
    h0[16 * p] = 1;   // exchange 1 (odd parity): this source has arrived
    for (int i = 0; i < n; i++) h0[P2P_FLAG_WORDS + ((size_t)world + p) * n + i] = (uint64_t)(1000 * p + i);
  }
  if (e == cudaSuccess) e = cudaMemset(mb, 0, words * 8 * world);
  if (e == cudaSuccess) e = cudaMemset(io, 0, (size_t)(2 * n + 16) * 8);
  if (e == cudaSuccess) e = cudaMemcpy(mb, h0.data(), words * 8, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(io, src.data(), (size_t)n * 8, cudaMemcpyHostToDevice);
  uint32_t herr = 0;
  if (e == cudaSuccess) {
    P2PArgs a{};
    for (int p = 0; p < world; p++) a.mbox[p] = mb + (size_t)p * words;
    a.epoch = io + 2 * n;
    a.err = reinterpret_cast<uint32_t *>(io + 2 * n + 8);
    a.src = io;
    a.dst = io + n;
    a.n = n;
    a.cap = n;
    a.rank = 0;
    a.world = world;
    a.op = P2P_SUM_I64;
    a.timeout_ns = (uint64_t)timeout_ms * 1000000ull;
    k_p2p_exchange<<<1, P2P_THREADS>>>(a);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpy(got.data(), io + n, (size_t)n * 8, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&herr, a.err, 4, cudaMemcpyDeviceToHost);
  }
  cudaFree(mb);
  cudaFree(io);
  if (e != cudaSuccess) return spb::record_error(SPB_ECUDA, cudaGetErrorString(e));
  if (herr & spb::ERR_TIMEOUT)
    return spb::record_error(SPB_ECUDA, "spb_tp_p2p_loopback: a bounded wait gave up (timeout)");
  for (int i = 0; i < n; i++) {
    want_sum = src[i];
    for (int p = 1; p < world; p++) want_sum += (uint64_t)(1000 * p + i);
    if (got[i] != want_sum) return spb::record_error(SPB_ERANGE, "spb_tp_p2p_loopback: wrong sum");
  }
  return SPB_OK;
}

extern "C" int spb_tp_rank(const spb_tp *tp) { return tp ? tp->rank : -1; }
extern "C" int spb_tp_world(const spb_tp *tp) { return tp ? tp->world : 0; }

namespace spb {

int tp_device(const spb_tp *tp) { return tp->device; }

// the peer-memory exchange when connected and the message fits a slot, else NCCL
static bool p2p_takes(const spb_tp *tp, size_t n) { return tp->p2p && n <= (size_t)tp->cap; }

static cudaError_t p2p_launch(const spb_tp *tp, const void *src, void *dst, size_t n, int op, cudaStream_t st,
                              uint32_t *err) {
  P2PArgs a{};
  for (int p = 0; p < tp->world; p++) a.mbox[p] = tp->peer[p];
  a.epoch = tp->epoch;
  a.err = err ? err : tp->err;
  a.src = src;
  a.dst = dst;
  a.n = (int)n;
  a.cap = tp->cap;
  a.rank = tp->rank;
  a.world = tp->world;
  a.op = op;
  a.timeout_ns = P2P_TIMEOUT_NS;
  k_p2p_exchange<<<1, P2P_THREADS, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t tp_sum_i64(const spb_tp *tp, int64_t *buf, size_t n, cudaStream_t st, uint32_t *err) {
  if (p2p_takes(tp, n)) return p2p_launch(tp, buf, buf, n, P2P_SUM_I64, st, err);
  const ncclResult_t r = nccl().allReduce(buf, buf, n, ncclInt64, ncclSum, tp->comm, st);
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

cudaError_t tp_max_u32(const spb_tp *tp, uint32_t *buf, size_t n, cudaStream_t st, uint32_t *err) {
  if (p2p_takes(tp, n)) return p2p_launch(tp, buf, buf, n, P2P_MAX_U32, st, err);
  const ncclResult_t r = nccl().allReduce(buf, buf, n, ncclUint32, ncclMax, tp->comm, st);
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

cudaError_t tp_max_u64(const spb_tp *tp, unsigned long long *buf, size_t n, cudaStream_t st, uint32_t *err) {
  if (p2p_takes(tp, n)) return p2p_launch(tp, buf, buf, n, P2P_MAX_U64, st, err);
  const ncclResult_t r = nccl().allReduce(buf, buf, n, ncclUint64, ncclMax, tp->comm, st);
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}


cudaError_t tp_gather_f32(const spb_tp *tp, const float *send, float *recv, size_t n, cudaStream_t st) {
  const ncclResult_t r = nccl().allGather(send, recv, n, ncclFloat32, tp->comm, st);
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

}  // namespace spb
