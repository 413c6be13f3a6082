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
}  // namespace nf
