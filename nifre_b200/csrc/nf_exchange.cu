// Cross-GPU exchange of the sharded attention output (one process per GPU).
//
// The reference runs attention on one device (src/inference/attention.py:77-104);
// sharded over N GPUs by KV head, each rank computes its query heads' columns
// of every output row and the ranks exchange them once per layer.  The
// attention kernels store their rows into every rank's gathered buffer
// directly (peer stores over NVLink, through CUDA IPC mappings made here) and
// signal completion through flag arrays in each rank's memory; this file
// holds the mappings and the stand-alone signal-and-wait.  No multicast, no
// bulk or tensor copies of peer memory: plain loads and stores only.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "nf_common.cuh"
#include "nf_internal.h"

namespace nf {

__global__ void exchange_barrier_kernel(NfGather g, int* status) {
  int* flags[kMaxRanks];
  for (int r = 0; r < g.n_ranks; ++r) flags[r] = g.flags[r];
  exchange_signal_wait(flags, g.n_ranks, g.rank, g.epoch, status, kWaitLimitCycles, g.epoch_counter);
}

static PFN_cuMemGetAddressRange_v3020 range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 3020, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  }
  return fn;
}

}  // namespace nf

extern "C" int nf_exchange_barrier(const NfGather* gather, int32_t* status, void* stream) {
  using namespace nf;
  if (!gather || !status) return fail(NF_EINVAL, "nf_exchange_barrier: null argument");
  if (gather->n_ranks < 1 || gather->n_ranks > kMaxRanks || gather->rank < 0 || gather->rank >= gather->n_ranks)
    return fail(NF_EINVAL, "nf_exchange_barrier: %d ranks (1..%d), rank %d", gather->n_ranks, kMaxRanks,
                gather->rank);
  if (gather->n_ranks == 1) return ok();
  for (int r = 0; r < gather->n_ranks; ++r)
    if (!gather->flags[r] || (reinterpret_cast<uintptr_t>(gather->flags[r]) & 3))
      return fail(NF_EINVAL, "nf_exchange_barrier: flags[%d] is null or unaligned", r);
  exchange_barrier_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(*gather, status);
  return check_launch("nf_exchange_barrier");
}

extern "C" int nf_ipc_handle(const void* ptr, void* handle64, int64_t* offset) {
  using namespace nf;
  if (!ptr || !handle64 || !offset) return fail(NF_EINVAL, "nf_ipc_handle: null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  auto range = range_fn();
  CUdeviceptr base = 0;
  size_t size = 0;
  if (!range || range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(NF_ECUDA, "nf_ipc_handle: the pointer is not in a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_ipc_handle: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle64, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return ok();
}

extern "C" int nf_ipc_open(const void* handle64, int64_t offset, void** ptr) {
  using namespace nf;
  if (!handle64 || !ptr || offset < 0) return fail(NF_EINVAL, "nf_ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_ipc_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *ptr = static_cast<char*>(base) + offset;
  return ok();
}

extern "C" int nf_ipc_close(void* ptr, int64_t offset) {
  using namespace nf;
  if (!ptr) return fail(NF_EINVAL, "nf_ipc_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_ipc_close: %s", cudaGetErrorString(e));
  return ok();
}
