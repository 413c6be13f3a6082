// Error reporting, versioning and small host helpers of the C ABI.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

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

cudaError_t prepare_launch(const void* func, int smem, int threads, int* per_sm) {
  // The dynamic shared memory limit is a setting of the function (per device): it is only ever raised, to the
  // largest size any launch asked for, so that a launch with a smaller size never lowers it under another's.
  struct Limit {
    int dev;
    const void* func;
    int smem;
  };
  struct Occ {
    int dev;
    const void* func;
    int smem, threads, per_sm;
  };
  static Limit limits[64];
  static Occ occs[128];
  static int n_lim = 0, n_occ = 0;
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  int li = -1;
  for (int i = 0; i < n_lim; ++i)
    if (limits[i].dev == dev && limits[i].func == func) li = i;
  const int have = li >= 0 ? limits[li].smem : 48 * 1024;
  if (smem > have) {
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (li >= 0)
      limits[li].smem = smem;
    else if (n_lim < 64)
      limits[n_lim++] = Limit{dev, func, smem};
  }
  if (!per_sm) return cudaSuccess;
  for (int i = 0; i < n_occ; ++i)
    if (occs[i].dev == dev && occs[i].func == func && occs[i].smem == smem && occs[i].threads == threads) {
      *per_sm = occs[i].per_sm;
      return cudaSuccess;
    }
  int occ = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, func, threads, smem) != cudaSuccess || occ < 1) occ = 1;
  (void)cudaGetLastError();
  *per_sm = occ;
  if (n_occ < 128) occs[n_occ++] = Occ{dev, func, smem, threads, occ};
  return cudaSuccess;
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

extern "C" int nf_abi_version(void) { return 14; }

extern "C" int nf_last_attention_path(void) { return nf::g_attention_path; }
