// Error reporting, versioning and small host helpers of the C ABI.
#include <stdarg.h>
#include <stdio.h>

#include "nf_internal.h"
#include "../../include/nifre_b200.h"

namespace nf {

static thread_local char g_err[512] = "";
static thread_local int g_attention_path = -1;

void set_attention_path(int path) { g_attention_path = path; }

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = '\0';
  return NF_OK;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NF_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return ok();
}

int sm_count() {
  // Cached per device; a benign race only repeats the same query.
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

size_t dtype_size(int dtype) {
  switch (dtype) {
    case NF_F32: return 4;
    case NF_F16: return 2;
    case NF_BF16: return 2;
    default: return 0;
  }
}

}  // namespace nf

extern "C" const char* nf_last_error(void) { return nf::g_err; }

extern "C" int nf_abi_version(void) { return 12; }

extern "C" int nf_last_attention_path(void) { return nf::g_attention_path; }
