// Tensor-map (TMA) copies of key/value blocks from the paged pools into
// shared memory, shared by the decode and prefill kernels.  Every copy lands in
// the issuing CTA only.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace nf {

// Keys and values are read once per launch: their lines go first when L2
// needs room, so the split-K parts and the queries stay cached.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Keys and values that several CTAs read in turn (a prefill chunk's prefix,
// read by every query tile of the chunk): keep them in L2 first.
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Starts the fetch of a tensor map (a __grid_constant__ kernel parameter)
// into the tensor-copy unit's descriptor cache, so that the first copy
// through it does not wait for the descriptor.
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar,
                                            uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar,
                                            uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            int c4, uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3, %4, %5, %6}], [%7], %8;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar), "l"(pol)
      : "memory");
}

// Tensor map over one pool (num_blocks, bs, Hkv, D), 16-bit elements,
// 128-byte swizzle.  permuted: dims (d_lo, token, [d_hi,] head, block) with a
// box of 16 tokens x hg heads; else (d_lo, [d_hi,] head, token, block) with a
// box of one head (and one 64-element half of a 128-wide head) x 16 tokens.
bool encode_pool_map(CUtensorMap* map, const void* pool, int dtype, int D, int Hkv, int bs, int num_blocks, int hg,
                     bool permuted);

// Tensor map over query rows (rows, H, D) with row stride `row_stride`
// elements, 16-bit, 128-byte swizzle: dims (d_lo, [d_hi,] head, row), box of
// 64 elements x g heads x tt rows, landing as tt*g rows of 128 bytes (row
// major in (row, head)).
bool encode_rows_map(CUtensorMap* map, const void* base, int dtype, int D, int H, long long rows, long long row_stride,
                     int g, int tt);

// Tensor map over a row-major matrix of 16-bit elements (rows x cols, row
// stride `row_stride` elements), 128-byte swizzle, box of 64 columns x
// box_rows rows (one 128-byte row of the box per matrix row).
bool encode_matrix_map(CUtensorMap* map, const void* base, int dtype, long long cols, long long rows,
                       long long row_stride, int box_rows);

}  // namespace nf
