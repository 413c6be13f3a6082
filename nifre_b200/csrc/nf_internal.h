// Host-side helpers shared by the entry points (not part of the ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nf {
// Records a message for nf_last_error() on this thread and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears the thread's message; returns NF_OK.
int ok();
// Checks cudaGetLastError() after a launch.
int check_launch(const char* what);
// Number of SMs of the current device (queried once per device).
int sm_count();
size_t dtype_size(int dtype);
// Which attention kernel the calling thread launched last (see nf_last_attention_path).
void set_attention_path(int path);
// Raises the dynamic shared memory limit of kernel `func` to `smem` bytes and
// returns in *per_sm its resident blocks per SM for `threads` threads (NULL:
// not needed), doing the CUDA calls once per (device, kernel, smem, threads):
// a launch path then costs no attribute or occupancy query per call.
cudaError_t prepare_launch(const void* func, int smem, int threads, int* per_sm);

// The cascade on the tensor cores (the prefill kernel's pipeline in its
// cascade mode, nf_prefill.cu); NF_EUNSUPPORTED when the shape needs the
// mma.sync kernel of nf_cascade.cu.
struct CascTcArgs {
  float* ws;
  const void* q;
  long long q_stride;
  int q_rows;
  const void* kp;
  const void* vp;
  int dtype, Hq, Hkv, D, bs, num_blocks;
  const int* bt;
  int max_blocks;
  const int* items;
  const int* counts;
  int max_items, max_units;
  const int* tasks;
  int n_tasks;
  const int* toks;
  int n_toks;
  float scale_log2;
  int* status;
  void* stream;
};
int cascade_tensor_core(const CascTcArgs& a);
}  // namespace nf
