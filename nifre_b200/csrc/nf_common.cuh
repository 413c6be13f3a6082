// Shared device helpers for the nifre_b200 kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/nifre_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "nifre_b200 kernels are written for sm_100a (B200) only"
#endif

namespace nf {

// ---------------------------------------------------------------- element types
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// Pack two floats into one 32-bit register of two 16-bit values (lo = a).
template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ---------------------------------------------------------------- shared memory / PTX
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes initialised mbarriers visible to the TMA (async proxy) before use.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the kernel before it on the stream runs; it
// calls pdl_wait() before its first read of anything that kernel writes,
// which returns once that kernel has completed and its writes are visible
// (immediately when there is no such launch).  pdl_launch_dependents() lets
// the next such kernel start launching now.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Time limit of every pipeline wait: about two seconds at the B200's top SM
// clock.  A wait that runs out flags NF_STATUS_WAIT_TIMEOUT and returns false;
// the caller then leaves its loops, so no kernel can spin forever.
constexpr long long kWaitLimitCycles = 4000000000LL;

// Split-K unit records (nf_pack_step) carry an item's part count in the low
// 16 bits of their last field and its unit count in the high bits; more
// parts than this per item are flagged (NF_STATUS_UNIT_OVERFLOW).
constexpr int kMaxParts = (1 << 15) - 1;
__device__ __forceinline__ int rec_parts(int w) { return w & 0xffff; }
__device__ __forceinline__ int rec_units(int w) { return w >> 16; }

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* status,
                                          long long limit = kWaitLimitCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > limit) {
      atomicOr(status, NF_STATUS_WAIT_TIMEOUT);
      return false;
    }
  }
}

// Waits, with the same kind of time limit, until the global counter reaches
// `total` (the grid-wide wait of the attention kernels' end-of-launch merge).
// Returns false, with NF_STATUS_WAIT_TIMEOUT set, when the limit runs out.
__device__ __forceinline__ bool wait_count(const int* counter, int total, int* status,
                                           long long limit = kWaitLimitCycles) {
  const long long t0 = clock64();
  while (*reinterpret_cast<const volatile int*>(counter) < total) {
    if (clock64() - t0 > limit) {
      atomicOr(status, NF_STATUS_WAIT_TIMEOUT);
      return false;
    }
    __nanosleep(256);
  }
  return true;
}

// ---------------------------------------------------------------- cross-GPU exchange
// Ranks of one exchange (one process per GPU) publish the completion of a
// launch through flag arrays in each other's memory (CUDA IPC mappings over
// NVLink): flags[r] of every rank's array holds the last call number (epoch)
// that rank r finished.  Plain loads and stores over peer memory only.
constexpr int kMaxRanks = 8;

__device__ __forceinline__ void st_release_sys(int* addr, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* addr) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// One thread: makes this GPU's earlier writes (its own and, through the
// barrier before the call, its CTA's) visible system-wide, sets
// flags[rank] = epoch in every rank's array, then waits, with a time limit,
// until every rank has set its entry of this rank's array to epoch or later
// (epochs compared modulo 2^32).  Returns false (NF_STATUS_WAIT_TIMEOUT set)
// if the limit runs out.
__device__ __forceinline__ bool exchange_signal_wait(int* const* rank_flags, int n_ranks, int rank, int epoch,
                                                     int* status, long long limit = kWaitLimitCycles,
                                                     int* epoch_counter = nullptr) {
  if (epoch_counter) {  // the epoch kept on the device: this call's is the next one
    epoch = *reinterpret_cast<volatile int*>(epoch_counter) + 1;
    *reinterpret_cast<volatile int*>(epoch_counter) = epoch;
  }
  __threadfence_system();
  for (int r = 0; r < n_ranks; ++r) st_release_sys(rank_flags[r] + rank, epoch);
  const int* mine = rank_flags[rank];
  const long long t0 = clock64();
  for (int r = 0; r < n_ranks; ++r) {
    while (ld_acquire_sys(mine + r) - epoch < 0) {
      if (clock64() - t0 > limit) {
        atomicOr(status, NF_STATUS_WAIT_TIMEOUT);
        return false;
      }
      __nanosleep(32);
    }
  }
  return true;
}

// One-dimensional TMA bulk copy global -> shared, completing on an mbarrier.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// 16-byte asynchronous global -> shared copy (LDGSTS), L1 bypassed: K/V rows
// are read once.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most n of this thread's most recent copy groups are pending
// (n above 6 waits for 6, which only waits longer).
__device__ __forceinline__ void cp_async_wait(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
  }
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// D = A(16x16, row) * B(16x8, col) + D, fp32 accumulate.
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^x on the special-function unit (PTX ex2.approx; inputs here are <= 0,
// -inf maps to +0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ int elect_lane0() { return (threadIdx.x & 31) == 0; }

}  // namespace nf
