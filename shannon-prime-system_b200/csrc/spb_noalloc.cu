// spb_noalloc.cu -- spb_gemv_q4b_noalloc: the OK_Q4B dequant-GEMV for callers that must not
// allocate device memory.
//
// Who needs it: a process whose device memory is already handed out (for example to a
// framework's own pool reserved at start-up), code on a latency-critical path where a
// cudaMalloc/cudaFree would add an implicit device synchronisation, or an integration whose
// rules forbid allocations after initialisation. spb_gemv_q4b grows a per-device workspace
// with cudaMalloc on first use; this variant instead keeps its scratch -- the quantized
// activations, their per-block sums and the per-row scales -- in one fixed array compiled
// into the library. The caller still provides the inputs and the output.
//
// Costs and limits: the array below is part of the module image, so every GPU that loads
// libspb200.so holds it until the process exits; it bounds n_tok * cols. All calls on a
// device share it and each call overwrites what the previous one left, so calls that can
// overlap on the GPU (for example from two streams) race and must be serialised by the
// caller. spb_gemv_q4b raises range-error bits into a per-device word that
// spb_take_device_errors() reads; that word is allocated, so this variant records none and its
// inputs must be finite.
//
// The scratch's device address is looked up once per device and CUDA context (the context in
// which the module holding the array was loaded): a cudaDeviceReset, or another context made
// current on the same device, gets a fresh lookup instead of a stale address.
#include "../../include/spb200.h"
#include "spb_kernels.cuh"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

using namespace spb;

namespace {

constexpr size_t NOALLOC_MAX_ELEMS = 262144;                 // n_tok * cols
constexpr int NOALLOC_MAX_COLS = 16384;                        // the GEMV's widest row
constexpr size_t NOALLOC_Q_BYTES = NOALLOC_MAX_ELEMS;         // int8 activations
constexpr size_t NOALLOC_BSUM_BYTES = NOALLOC_MAX_ELEMS / 32 * 4;
constexpr size_t NOALLOC_SCALE_BYTES = 256;                   // up to 16 f32 row scales
constexpr size_t NOALLOC_BYTES = NOALLOC_Q_BYTES + NOALLOC_BSUM_BYTES + NOALLOC_SCALE_BYTES;

// The scratch. In host code this name is only a stand-in for the symbol (not a device
// address); the host side obtains the device address with cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
unsigned char *g_addr[MAX_DEVICES];   // device address of the scratch, per device ...
CUcontext g_ctx[MAX_DEVICES];         // ... valid in this context

int fail(int code, const char *msg) { return spb::record_error(code, msg); }   // -> spb_last_error()

// the current CUDA context (driver entry point through the runtime: no libcuda link needed)
CUcontext current_context() {
  using Fn = CUresult (*)(CUcontext *);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(p);
  });
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

}  // namespace

// Declared in include/spb200.h. The first call on a device (and in each new context on it, e.g.
// after a cudaDeviceReset) looks up the scratch's device address with that device current
// (cudaGetSymbolAddress); make that first call before any stream capture on the device.
extern "C" int spb_gemv_q4b_noalloc(const uint8_t *codes, const uint16_t *bscale, int rows, int cols,
                                    const float *x, int n_tok, float *y, void *stream) {
  if (!codes || !bscale || !x || !y || rows <= 0 || cols <= 0 || (cols & 31))
    return fail(SPB_EBADARG, "spb_gemv_q4b_noalloc: bad arg (cols must be a positive multiple of 32)");
  if (n_tok != 1 && n_tok != 2 && n_tok != 4 && n_tok != 8 && n_tok != 16)
    return fail(SPB_EBADARG, "spb_gemv_q4b_noalloc: n_tok must be 1, 2, 4, 8 or 16");
  if (cols > NOALLOC_MAX_COLS)
    return fail(SPB_EBADARG, "spb_gemv_q4b_noalloc: cols exceeds the GEMV's 16384-column limit");
  if ((size_t)n_tok * (size_t)cols > NOALLOC_MAX_ELEMS)
    return fail(SPB_EBADARG, "spb_gemv_q4b_noalloc: n_tok * cols exceeds the fixed scratch (262144 elements)");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES)
    return fail(SPB_ECUDA, "spb_gemv_q4b_noalloc: no current CUDA device");
  unsigned char *base = nullptr;
  {
    const CUcontext ctx = current_context();   // null before the runtime made one current
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev] || !ctx || g_ctx[dev] != ctx) {
      void *p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // makes the context current
      if (e != cudaSuccess) return fail(SPB_ECUDA, "spb_gemv_q4b_noalloc: cudaGetSymbolAddress failed");
      g_addr[dev] = static_cast<unsigned char *>(p);
      g_ctx[dev] = current_context();
    }
    base = g_addr[dev];
  }
  cudaStream_t st = (cudaStream_t)stream;
  // Every scratch word the kernels read is written first in this call: the row max (as the
  // row scale) by the quantizer's max pass, the codes and block sums by the quantizer; the
  // previous call's contents are therefore never read and need no clearing.
  const DevAct act{reinterpret_cast<int8_t *>(base), reinterpret_cast<int32_t *>(base + NOALLOC_Q_BYTES),
                   reinterpret_cast<float *>(base + NOALLOC_Q_BYTES + NOALLOC_BSUM_BYTES)};
  cudaError_t e = launch_quant(x, cols, cols, n_tok, act, nullptr, nullptr, st);
  if (e == cudaSuccess) e = launch_gemv(DevQ4B{codes, bscale, rows, cols}, nullptr, act, n_tok, y, rows, EPI_STORE,
                                        nullptr, st);
  if (e != cudaSuccess) return fail(SPB_ECUDA, cudaGetErrorString(e));
  return SPB_OK;
}
