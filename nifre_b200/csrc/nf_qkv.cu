// The QKV projection fused with the KV append (tcgen05 / TMEM).
//
// Reference: GptAttention.forward (src/inference/models/gpt.py:38-51) runs
// three nn.Linear projections, then Attention appends the new K/V to the
// cache (paged_kv_cache.py:107-121) and attends.  Here one kernel computes
// [q | k | v] = x W^T (+ b) for the step's rows, with W the three weights
// stacked (nn.Linear layout: out_features x in_features), and its epilogue
// writes the q columns to q_out and the k / v columns straight into their
// pool rows through the step's slot mapping -- so new keys and values never
// make a round trip through HBM between the projection and the append.
//
// One CTA per 128-row x BN-column output tile (BN = 64, or 32 for steps with
// few rows so that more SMs stream the weights): a producer warp streams
// 64-wide K slices of the x tile and the weight tile into a 6-stage ring by
// TMA (128-byte swizzle), one elected lane of the MMA warp issues
// tcgen05.mma kind::f16 (M = 128, N = BN, K = 16, fp32 accumulator in
// tensor memory) and releases each stage with a commit, and four epilogue
// warps (thread = row) read the accumulator, add the bias, round to the
// output type and store 2*BN bytes per row.  Every wait is time-limited.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>

#include "nf_common.cuh"
#include "nf_internal.h"
#include "nf_tma.cuh"
#include "nf_umma.cuh"

namespace nf {

struct QkvParams {
  int rows, K, Nq, Nkv;     // output columns: [0, Nq) q, [Nq, Nq+Nkv) k, [Nq+Nkv, Nq+2Nkv) v
  const char* bias;         // Nq + 2 Nkv elements of the output type, or null
  char* q_out;
  long long q_stride;       // elements
  char* k_pool;
  char* v_pool;             // pool rows of Nkv elements
  long long pool_rows;
  const int* slot_mapping;  // pool row of row r (token r of the step)
  const int* seqs;          // step records (slot, q_start, q_len, ctx_before), for pos_out
  int n_seqs;
  long long* pos_out;       // optional: pos_out[slot] = ctx_before + q_len
  int* status;
};

// Output tiles are 128 rows x BN columns (BN = 64, or 32 when 64-wide tiles
// would leave SMs idle: a decode step has few rows, and the weights are the
// bytes to stream).
constexpr int kQkvBM = 128, kQkvStages = 6;
constexpr uint32_t kQkvA = kQkvBM * 128;  // bytes of one 64-wide K slice of the x tile
template <int BN>
struct QkvCfg {
  static constexpr uint32_t B = BN * 128;  // one 64-wide K slice of the weight tile
  static constexpr uint32_t STAGE = kQkvA + B;
  static constexpr uint32_t SMEM = 1024 + kQkvStages * STAGE + 1024;  // header + ring + alignment slack
};

template <typename T, int BN>
__global__ void __launch_bounds__(192, 1)
    qkv_append_kernel(const QkvParams p, const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw) {
  constexpr uint32_t kQkvStage = QkvCfg<BN>::STAGE;
  constexpr int kQkvBN = BN;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t hdr = smem_u32(base);
  auto full = [&](int s) { return hdr + 8 * s; };
  auto empty = [&](int s) { return hdr + 64 + 8 * s; };
  const uint32_t acc_done = hdr + 128, tmem_slot = hdr + 256;
  const uint32_t ring = hdr + 1024;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kQkvBM, n0 = blockIdx.y * kQkvBN;
  const int nk = (p.K + 63) >> 6;
  if (threadIdx.x == 32) {
    tma_prefetch_map(&tx);
    tma_prefetch_map(&tw);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kQkvStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(acc_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 64);  // >= BN fp32 columns (allocations are powers of two >= 32)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(base + 256);
  if (warp == 0) {
    // producer: K slices of the x tile (evict first: read by the N tiles of
    // this row block only) and of the weight tile (kept: every row block reads it)
    const uint64_t pol_x = l2_evict_first(), pol_w = l2_evict_last();
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kQkvStages;
      const uint32_t ph = (uint32_t)(kb / kQkvStages) & 1u;
      if (!mbar_wait(empty(s), ph ^ 1u, p.status)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(full(s), kQkvStage);
        tma_load_2d(ring + s * kQkvStage, &tx, kb * 64, m0, full(s), pol_x);
        tma_load_2d(ring + s * kQkvStage + kQkvA, &tw, kb * 64, n0, full(s), pol_w);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    const bool leader = elect_one();
    const uint32_t idesc = umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, kQkvBM, kQkvBN, false, false);
    const uint32_t ring0 = __shfl_sync(0xffffffffu, ring, 0);
    const uint64_t da = umma_sdesc_sw128(ring0, 16, 1024), db = umma_sdesc_sw128(ring0 + kQkvA, 16, 1024);
    bool ok = true;
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % kQkvStages;
      const uint32_t ph = (uint32_t)(kb / kQkvStages) & 1u;
      ok = mbar_wait(full(s), ph, p.status);
      if (!ok) break;
      tc_fence_after();
      if (leader) {
        const uint64_t so = (uint64_t)((s * kQkvStage) >> 4);
#pragma unroll
        for (int k = 0; k < 4; ++k)  // K = 16 per instruction: 32 bytes along the swizzled row
          umma_f16_ss(tmem, da + so + 2 * k, db + so + 2 * k, idesc, (kb | k) ? 1u : 0u);
        umma_commit(empty(s));
      }
      __syncwarp();
    }
    if (leader) umma_commit(acc_done);
    __syncwarp();
  } else {
    // epilogue warps 2..5: tensor-memory lanes 32 * (warp % 4) .. +31 = rows of the tile
    const int quad = warp & 3;
    const int r = m0 + quad * 32 + lane;
    const bool ok = mbar_wait(acc_done, 0, p.status);
    tc_fence_after();
    constexpr int NC = BN / 32;  // 32-column tensor-memory loads
    uint32_t a[NC][32];
    if (ok) {
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16);
#pragma unroll
      for (int c = 0; c < NC; ++c) tmem_ld32(taddr + 32 * c, a[c]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < NC; ++c) tmem_reg_fence(a[c]);
    }
    if (ok && r < p.rows) {
      T* dst = nullptr;
      if (n0 < p.Nq) {
        dst = reinterpret_cast<T*>(p.q_out) + (long long)r * p.q_stride + n0;
      } else {
        const int slot = __ldg(p.slot_mapping + r);
        if (slot < 0 || slot >= p.pool_rows) {
          atomicOr(p.status, NF_STATUS_BAD_SLOT);
        } else {
          const bool is_k = n0 < p.Nq + p.Nkv;
          const int c0 = n0 - p.Nq - (is_k ? 0 : p.Nkv);
          dst = reinterpret_cast<T*>(is_k ? p.k_pool : p.v_pool) + (long long)slot * p.Nkv + c0;
        }
      }
      if (dst) {
        const T* b = reinterpret_cast<const T*>(p.bias);
        uint32_t wv[BN / 2];
#pragma unroll
        for (int i = 0; i < BN / 2; ++i) {
          const int c = 2 * i;
          float v0 = __uint_as_float(a[c >> 5][c & 31]), v1 = __uint_as_float(a[(c + 1) >> 5][(c + 1) & 31]);
          if (b) {
            v0 += Elem<T>::to_f(b[n0 + c]);
            v1 += Elem<T>::to_f(b[n0 + c + 1]);
          }
          wv[i] = pack2<T>(v0, v1);
        }
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int i = 0; i < BN / 8; ++i) d4[i] = make_uint4(wv[4 * i], wv[4 * i + 1], wv[4 * i + 2], wv[4 * i + 3]);
      }
    }
    // the reference advances pos when the last layer appends (paged_kv_cache.py:120-121)
    if (p.pos_out && blockIdx.x == 0 && blockIdx.y == 0)
      for (int i = threadIdx.x - 64; i < p.n_seqs; i += 128) {
        const int4 sq = __ldg(reinterpret_cast<const int4*>(p.seqs) + i);
        p.pos_out[sq.x] = (long long)sq.w + sq.z;
      }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 64);
}

}  // namespace nf

extern "C" int nf_qkv_append(const void* x, int64_t x_row_stride, int32_t rows, const void* weight, const void* bias,
                             int32_t k_dim, int32_t n_q, int32_t n_kv, void* q_out, int64_t q_out_row_stride,
                             void* k_pool, void* v_pool, int64_t pool_rows, int32_t dtype,
                             const int32_t* slot_mapping, const int32_t* seqs, int32_t n_seqs, int64_t* pos_out,
                             int32_t* status, void* stream) {
  using namespace nf;
  if (dtype != NF_BF16 && dtype != NF_F16)
    return fail(NF_EUNSUPPORTED, "nf_qkv_append: 16-bit operands only (dtype %d)", dtype);
  if (rows < 0 || k_dim <= 0 || n_q <= 0 || n_kv <= 0 || pool_rows <= 0 || n_seqs < 0)
    return fail(NF_EINVAL, "nf_qkv_append: sizes must be positive");
  if (n_q % 64 || n_kv % 64)
    return fail(NF_EUNSUPPORTED, "nf_qkv_append: q and k/v widths (%d, %d) must be multiples of 64", n_q, n_kv);
  if (k_dim % 8) return fail(NF_EUNSUPPORTED, "nf_qkv_append: in_features %d is not a multiple of 8", k_dim);
  if (!x || !weight || !q_out || !k_pool || !v_pool || !slot_mapping || !status || (pos_out && !seqs))
    return fail(NF_EINVAL, "nf_qkv_append: null pointer argument");
  auto al = [](const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
  if (!al(x, 16) || (x_row_stride * 2) % 16 || !al(weight, 16) || !al(q_out, 16) || (q_out_row_stride * 2) % 16 ||
      !al(k_pool, 16) || !al(v_pool, 16) || (seqs && !al(seqs, 16)) || (bias && !al(bias, 4)))
    return fail(NF_EINVAL, "nf_qkv_append: x, weight, q_out rows and pools must be 16-byte aligned");
  if (x_row_stride < k_dim) return fail(NF_EINVAL, "nf_qkv_append: x row stride below in_features");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  QkvParams p;
  p.rows = rows;
  p.K = k_dim;
  p.Nq = n_q;
  p.Nkv = n_kv;
  p.bias = static_cast<const char*>(bias);
  p.q_out = static_cast<char*>(q_out);
  p.q_stride = q_out_row_stride;
  p.k_pool = static_cast<char*>(k_pool);
  p.v_pool = static_cast<char*>(v_pool);
  p.pool_rows = pool_rows;
  p.slot_mapping = slot_mapping;
  p.seqs = seqs;
  p.n_seqs = pos_out ? n_seqs : 0;
  p.pos_out = reinterpret_cast<long long*>(pos_out);
  p.status = status;
  if (rows == 0) return ok();
  const long long n_all = (long long)n_q + 2LL * n_kv;
  const long long row_tiles = (rows + kQkvBM - 1) / kQkvBM;
  const int bn = row_tiles * (n_all / 64) < sm_count() ? 32 : 64;
  CUtensorMap tx, tw;
  if (!encode_matrix_map(&tx, x, dtype, k_dim, rows, x_row_stride, kQkvBM) ||
      !encode_matrix_map(&tw, weight, dtype, k_dim, n_all, k_dim, bn))
    return fail(NF_ECUDA, "nf_qkv_append: tensor map encoding failed");
  auto kern = dtype == NF_BF16 ? (bn == 32 ? qkv_append_kernel<__nv_bfloat16, 32> : qkv_append_kernel<__nv_bfloat16, 64>)
                               : (bn == 32 ? qkv_append_kernel<__half, 32> : qkv_append_kernel<__half, 64>);
  const int smem = bn == 32 ? (int)QkvCfg<32>::SMEM : (int)QkvCfg<64>::SMEM;
  cudaError_t e = prepare_launch(reinterpret_cast<const void*>(kern), smem, 192, nullptr);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_qkv_append: smem attribute: %s", cudaGetErrorString(e));
  const dim3 grid((unsigned)row_tiles, (unsigned)(n_all / bn));
  kern<<<grid, 192, smem, st>>>(p, tx, tw);
  return check_launch("nf_qkv_append");
}
