// Self-check of the tcgen05 path used by the prefill kernel: one 128 x N x K
// bf16 MMA chain from 128-byte-swizzled shared memory into tensor memory,
// read back with tcgen05.ld.  Exported as a diagnostic (no counterpart in the
// reference) so that a test can compare it with a host matmul.
#include "nf_common.cuh"
#include "nf_internal.h"
#include "nf_umma.cuh"

namespace nf {

// Byte offset of element (row, col) of a row-major operand with 64-element
// (128-byte) atoms along `col`: atom `col / 64` is a region of `rows` x 128 B,
// 16-byte chunks XOR-swizzled by the row.
__device__ __forceinline__ uint32_t sw128_off(int row, int col, int rows) {
  const int region = col >> 6, chunk = (col >> 3) & 7;
  return region * rows * 128 + row * 128 + ((chunk ^ (row & 7)) << 4) + (col & 7) * 2;
}

// mode 0: C[m][n] = sum_k A[m][k] B[n][k]  (B K-major, as K in S = Q K^T)
// mode 1: C[m][n] = sum_k A[m][k] B[k][n]  (B MN-major, as V in O = P V)
// mode 2: as mode 1 with A in tensor memory (row m in lane m, columns 128..),
//         written there by tcgen05.st (P in O = P V)
__global__ void __launch_bounds__(128) umma_selftest_kernel(const __nv_bfloat16* A, const __nv_bfloat16* B,
                                                             float* C, int N, int K, int mode, int* status) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint32_t tmem_base;
  __shared__ __align__(8) unsigned long long bar;
  unsigned char* As = base;                  // 128 x K
  unsigned char* Bs = base + 128 * K * 2;    // N x K (mode 0) or K x N (mode 1)
  const int tid = threadIdx.x, warp = tid >> 5;
  for (int i = tid; i < 128 * K; i += 128) {
    const int r = i / K, c = i % K;
    *reinterpret_cast<__nv_bfloat16*>(As + sw128_off(r, c, 128)) = A[i];
  }
  if (mode == 0) {
    for (int i = tid; i < N * K; i += 128) {
      const int r = i / K, c = i % K;
      *reinterpret_cast<__nv_bfloat16*>(Bs + sw128_off(r, c, N)) = B[i];
    }
  } else {
    for (int i = tid; i < K * N; i += 128) {
      const int r = i / N, c = i % N;  // row = k, col = n
      *reinterpret_cast<__nv_bfloat16*>(Bs + sw128_off(r, c, K)) = B[i];
    }
  }
  if (warp == 0) tmem_alloc(smem_u32(&tmem_base), 256);
  if (tid == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;
  if (mode == 2) {
    // row `tid` of A, packed in pairs, into columns 128 .. 128 + K/2 of lane `tid`
    const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
    for (int c0 = 0; c0 < K / 2; c0 += 32) {
      uint32_t r[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const __nv_bfloat162 v = __halves2bfloat162(A[tid * K + 2 * (c0 + j)], A[tid * K + 2 * (c0 + j) + 1]);
        r[j] = *reinterpret_cast<const uint32_t*>(&v);
      }
      tmem_st32(tbase + lane_addr + 128 + c0, r);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (tid == 0) {
    const uint32_t idesc = umma_idesc_f16(true, 128, N, false, mode != 0);
    for (int ks = 0; ks < K / 16; ++ks) {
      if (mode == 2) {
        umma_f16_ts(tbase, tbase + 128 + ks * 8, umma_sdesc_sw128(smem_u32(Bs) + ks * 16 * 128, K * 128, 1024),
                    idesc, ks > 0);
        continue;
      }
      const uint32_t a = smem_u32(As) + (ks >> 2) * 128 * 128 + (ks & 3) * 32;
      uint64_t bd;
      if (mode == 0) {
        bd = umma_sdesc_sw128(smem_u32(Bs) + (ks >> 2) * N * 128 + (ks & 3) * 32, 16, 1024);
      } else {
        // 16 k-rows from row 16*ks; MN atoms (64 columns) are regions of K rows x 128 B
        bd = umma_sdesc_sw128(smem_u32(Bs) + ks * 16 * 128, K * 128, 1024);
      }
      umma_f16_ss(tbase, umma_sdesc_sw128(a, 16, 1024), bd, idesc, ks > 0);
    }
    umma_commit(smem_u32(&bar));
  }
  __syncwarp();
  if (!mbar_wait(smem_u32(&bar), 0, status)) {
    // leave the accumulator unread; the status word reports the timeout
  } else {
    tc_fence_after();
    const int row = warp * 32 + (tid & 31);
    for (int c0 = 0; c0 < N; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tbase + ((uint32_t)(warp * 32) << 16) + c0, r);
      tmem_wait_ld();
      tmem_reg_fence(r);
#pragma unroll
      for (int j = 0; j < 32; ++j) C[row * N + c0 + j] = __uint_as_float(r[j]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

}  // namespace nf

extern "C" int nf_selftest_umma(const void* A, const void* B, float* C, int32_t N, int32_t K, int32_t mode,
                                int32_t* status, void* stream) {
  using namespace nf;
  if (!A || !B || !C || !status) return fail(NF_EINVAL, "nf_selftest_umma: null pointer");
  if ((N != 64 && N != 128) || (K != 64 && K != 128) || mode < 0 || mode > 2)
    return fail(NF_EINVAL, "nf_selftest_umma: N, K in {64, 128}, mode 0, 1 or 2");
  const int smem = 1024 + 128 * K * 2 + N * K * 2;
  cudaError_t e = cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_selftest_umma: %s", cudaGetErrorString(e));
  umma_selftest_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B), C, N, K, mode, status);
  return check_launch("nf_selftest_umma");
}
