// spb_tp.cuh -- the tensor-parallel group's exchanges as the runtime enqueues them (spb_tp.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

struct spb_tp;

namespace spb {

int tp_device(const spb_tp *tp);
// in place on `st`; cudaErrorUnknown when NCCL refuses the call (detail from NCCL's own log);
// err: the caller's error word, which the peer-memory exchange's bounded wait raises
// ERR_TIMEOUT into when a rank does not arrive
cudaError_t tp_sum_i64(const spb_tp *tp, int64_t *buf, size_t n, cudaStream_t st, uint32_t *err);
cudaError_t tp_max_u32(const spb_tp *tp, uint32_t *buf, size_t n, cudaStream_t st, uint32_t *err);
cudaError_t tp_max_u64(const spb_tp *tp, unsigned long long *buf, size_t n, cudaStream_t st, uint32_t *err);
// recv = [rank 0's n][rank 1's n]...
cudaError_t tp_gather_f32(const spb_tp *tp, const float *send, float *recv, size_t n, cudaStream_t st);

}  // namespace spb
