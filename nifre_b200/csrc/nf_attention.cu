// Paged attention over a ragged batch: split-K, grouped-query, online softmax.
//
// Computes what Attention._forward_with_cache_row does per row
// (jyotilakra92/nifre src/inference/attention.py:106-142): scores q.k over the
// past and new keys, the causal mask of attention.py:144-152 (a query at
// absolute position p sees keys 0..p), softmax(scores / sqrt(D)) and the
// weighted sum of values -- but reading K/V in place from the block pool
// (paged_kv_cache.py:72-85 layout) instead of PagedKVCache.get's gather and
// torch.cat (paged_kv_cache.py:123-142, attention.py:121-127).
//
// Work decomposition.  nf_pack_step emits one work item per query token
// (slot, query row, kv_len) and cuts each item's keys into units of
// `split` keys.  A persistent grid (one CTA per SM) walks the units; each
// CTA covers a group of HG KV heads, so every staged key row is one
// contiguous run of HG*D elements of the pool.
//
// Inside a CTA (warp specialised):
//   * warp W (producer): for each stage of R = 16*SUB keys, looks up the
//     block table and issues one TMA bulk copy (cp.async.bulk) per K row and
//     per V row into a padded shared-memory row (pitch = HG*D*size + 16 so the
//     fragment loads below hit 8 distinct bank groups); completion is counted
//     in bytes on the stage's "full" mbarrier.
//   * warps 0..W-1 (consumers): warp w owns KV head (w % HG) of the group and
//     the 16-key sub-tile (w / HG) of each stage.  For 16-bit pools, the
//     scores S^T = K Q^T (16 keys x 8 query heads of the group) and the output
//     O^T += V^T P^T (D x 8) are mma.sync m16n8k16 tiles: GQA groups of up to
//     8 query heads share one K/V read.  The probabilities go from the S^T
//     accumulator layout to the B-operand layout with two movmatrix
//     transposes.  For float32 pools the same stages are consumed with
//     CUDA-core FMAs (the reference's float32 model must keep full precision).
//   * split-K merge: a unit whose item has more than one partial writes
//     (m, l, acc) to the caller's workspace; the last warp to finish an
//     (item, KV head) -- counted with one atomic per warp -- merges all
//     partials and writes the output.  There is no second launch and no
//     cross-warp barrier; every wait in the kernel is an mbarrier wait with a
//     time limit.
#include <math.h>

#include "nf_common.cuh"
#include "nf_internal.h"

namespace nf {

struct AttnParams {
  char* out;
  long long out_stride;
  const char* q;
  long long q_stride;
  const char* kp;
  const char* vp;
  int Hq, Hkv, D, G, bs, num_blocks;
  const int* bt;
  int max_blocks;
  const int* items;
  const int* units;
  const int* counts;
  int max_units, split;
  float scale_log2;
  float* ws;
  int* cnt;
  int* status;
  // launch plan
  int HG, SUB, W, n_hg, stages, R, pitch, row_bytes, stage_bytes;
};

constexpr int kBarrierBytes = 256;  // full[8] + empty[8] mbarriers
constexpr int kMaxStages = 8;
constexpr float kNegInf = -INFINITY;

__device__ __forceinline__ uint32_t full_bar(unsigned char* smem, int s) { return smem_u32(smem) + 8 * s; }
__device__ __forceinline__ uint32_t empty_bar(unsigned char* smem, int s) { return smem_u32(smem) + 64 + 8 * s; }

// ---------------------------------------------------------------- producer
template <typename T>
__device__ void producer_loop(const AttnParams& p, unsigned char* smem, int total) {
  const int lane = threadIdx.x & 31;
  const uint32_t tx_bytes = 2u * p.R * p.row_bytes;
  const uint32_t stage0 = smem_u32(smem) + kBarrierBytes;
  int k = 0;
  bool ok = true;
  for (int v = blockIdx.x; v < total && ok; v += gridDim.x) {
    const int u = v / p.n_hg, hg = v % p.n_hg;
    const int item = p.units[2 * u], split = p.units[2 * u + 1];
    const int slot = p.items[4 * item], kv_len = p.items[4 * item + 2];
    const int t0 = split * p.split, t1 = min(t0 + p.split, kv_len);
    const int* btrow = p.bt + (long long)slot * p.max_blocks;
    const long long head_off = (long long)hg * p.HG * p.D;
    for (int t = t0; t < t1; t += p.R, ++k) {
      const int s = k % p.stages, round = k / p.stages;
      if (!mbar_wait(empty_bar(smem, s), (round & 1) ^ 1, p.status)) {
        ok = false;
        break;
      }
      if (lane == 0) mbar_arrive_expect_tx(full_bar(smem, s), tx_bytes);
      __syncwarp();
      const uint32_t sbase = stage0 + s * p.stage_bytes;
      for (int i = lane; i < 2 * p.R; i += 32) {
        const int kv = i >= p.R;
        const int r = kv ? i - p.R : i;
        const int tok = min(t + r, t1 - 1);  // rows past the end repeat the last key (masked)
        const int lb = tok / p.bs;
        int phys = lb < p.max_blocks ? btrow[lb] : -1;
        if (phys < 0 || phys >= p.num_blocks) {
          atomicOr(p.status, NF_STATUS_BAD_BLOCK);
          phys = 0;
        }
        const long long row = (long long)phys * p.bs + tok % p.bs;
        const T* src = reinterpret_cast<const T*>(kv ? p.vp : p.kp) + row * p.Hkv * p.D + head_off;
        bulk_g2s(sbase + (kv * p.R + r) * p.pitch, src, p.row_bytes, full_bar(smem, s));
      }
    }
  }
  if (!ok) {
    // leave no bulk copy in flight into this CTA's shared memory
    for (int j = max(0, k - p.stages); j < k; ++j) mbar_wait(full_bar(smem, j % p.stages), (j / p.stages) & 1, p.status);
  }
}

// ---------------------------------------------------------------- shared epilogue
// Writes one query head's result for this warp's part of a unit.  `acc(d)`
// returns the unnormalised accumulator of element d held by this lane (the
// caller only calls for elements it owns).
struct UnitCtx {
  int u, item, q_row, kv_len, unit_base, nparts, kvh, sub;
};

// Merge of all partials of (item, kvh) by the last warp to finish.
template <typename T>
__device__ void merge_partials(const AttnParams& p, const UnitCtx& c) {
  const int lane = threadIdx.x & 31;
  const int DP = p.D + 2;
  for (int n = 0; n < p.G; ++n) {
    const int qh = c.kvh * p.G + n;
    float M = kNegInf;
    for (int j = 0; j < c.nparts; ++j) {
      const float* pb = p.ws + ((long long)(c.unit_base * p.SUB + j) * p.Hq + qh) * DP;
      M = fmaxf(M, __ldcg(pb + p.D));
    }
    float L = 0.f;
    for (int j = 0; j < c.nparts; ++j) {
      const float* pb = p.ws + ((long long)(c.unit_base * p.SUB + j) * p.Hq + qh) * DP;
      const float mj = __ldcg(pb + p.D);
      if (mj != kNegInf) L += __ldcg(pb + p.D + 1) * ex2(mj - M);
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    T* o = reinterpret_cast<T*>(p.out) + (long long)c.q_row * p.out_stride + (long long)qh * p.D;
    for (int d = lane; d < p.D; d += 32) {
      float a = 0.f;
      for (int j = 0; j < c.nparts; ++j) {
        const float* pb = p.ws + ((long long)(c.unit_base * p.SUB + j) * p.Hq + qh) * DP;
        const float mj = __ldcg(pb + p.D);
        if (mj != kNegInf) a += __ldcg(pb + d) * ex2(mj - M);
      }
      o[d] = Elem<T>::from_f(a * inv);
    }
  }
}

// After this warp wrote its partial: count it; the last one merges.
template <typename T>
__device__ void finish_partial(const AttnParams& p, const UnitCtx& c) {
  __threadfence();
  __syncwarp();
  int last = 0;
  int* ctr = p.cnt + (long long)c.item * p.Hkv + c.kvh;
  if ((threadIdx.x & 31) == 0) last = (atomicAdd(ctr, 1) == c.nparts - 1);
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence();
    merge_partials<T>(p, c);
    if ((threadIdx.x & 31) == 0) *ctr = 0;  // workspace left clean for the next launch
  }
}

// ---------------------------------------------------------------- consumers
__device__ __forceinline__ UnitCtx unit_ctx(const AttnParams& p, int v, int warp) {
  UnitCtx c;
  c.u = v / p.n_hg;
  const int hg = v % p.n_hg;
  c.item = p.units[2 * c.u];
  c.q_row = p.items[4 * c.item + 1];
  c.kv_len = p.items[4 * c.item + 2];
  c.unit_base = p.items[4 * c.item + 3];
  c.nparts = ((c.kv_len + p.split - 1) / p.split) * p.SUB;
  c.kvh = hg * p.HG + warp % p.HG;
  c.sub = warp / p.HG;
  return c;
}

// 16-bit pools: tensor-core tiles.  D_ is the head dimension (64 or 128).
template <typename T, int D_>
__device__ void consumer_mma(const AttnParams& p, unsigned char* smem, int total) {
  constexpr int KS = D_ / 16;  // k-steps of S^T and m-tiles of O^T
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t stage0 = smem_u32(smem) + kBarrierBytes;
  const int n0 = 2 * (lane & 3);       // query heads of this lane's accumulator columns
  const int tq = lane >> 2;            // key row / d row of this lane in a fragment
  int k = 0;
  for (int v = blockIdx.x; v < total; v += gridDim.x) {
    const UnitCtx c = unit_ctx(p, v, warp);
    const int split = p.units[2 * c.u + 1];
    const int t0 = split * p.split, t1 = min(t0 + p.split, c.kv_len);
    // Q^T as the B operand: column n = query head tq of the group.
    uint32_t qf[KS][2];
    {
      const T* qp = reinterpret_cast<const T*>(p.q) + (long long)c.q_row * p.q_stride +
                    (long long)(c.kvh * p.G + tq) * D_ + n0;
      const bool has = tq < p.G;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qf[ks][0] = has ? *reinterpret_cast<const uint32_t*>(qp + ks * 16) : 0u;
        qf[ks][1] = has ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 8) : 0u;
      }
    }
    float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;
    float o[KS][4];
#pragma unroll
    for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    for (int t = t0; t < t1; t += p.R, ++k) {
      const int s = k % p.stages, round = k / p.stages;
      if (!mbar_wait(full_bar(smem, s), round & 1, p.status)) return;
      const int tb = t + c.sub * 16;
      if (tb < t1) {
        const uint32_t kbase = stage0 + s * p.stage_bytes + (c.sub * 16) * p.pitch + (warp % p.HG) * D_ * 2;
        const uint32_t vbase = kbase + p.R * p.pitch;
        // S^T = K Q^T : 16 keys x 8 query heads
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
        {
          const int r = (lane & 7) + ((lane >> 3) & 1) * 8;  // key row supplied by this lane
          const int cb = (lane >> 4) * 8;                       // column half
          const uint32_t a_addr = kbase + r * p.pitch + cb * 2;
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(a_addr + ks * 32, a0, a1, a2, a3);
            mma16816<T>(sc, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
          }
        }
        const bool v0 = tb + tq < t1, v1 = tb + tq + 8 < t1;
        const float x0 = v0 ? sc[0] * p.scale_log2 : kNegInf;
        const float x1 = v0 ? sc[1] * p.scale_log2 : kNegInf;
        const float x2 = v1 ? sc[2] * p.scale_log2 : kNegInf;
        const float x3 = v1 ? sc[3] * p.scale_log2 : kNegInf;
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
        for (int o_ = 4; o_ < 32; o_ <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o_));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o_));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float b0 = mn0 == kNegInf ? 0.f : mn0, b1 = mn1 == kNegInf ? 0.f : mn1;
        const float al0 = ex2(m0 - b0), al1 = ex2(m1 - b1);
        const float p0 = ex2(x0 - b0), p1 = ex2(x1 - b1), p2 = ex2(x2 - b0), p3 = ex2(x3 - b1);
        l0 = l0 * al0 + p0 + p2;
        l1 = l1 * al1 + p1 + p3;
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int i = 0; i < KS; ++i) {
          o[i][0] *= al0;
          o[i][1] *= al1;
          o[i][2] *= al0;
          o[i][3] *= al1;
        }
        // P^T (keys x heads) as the B operand: transpose the two 8x8 halves.
        const uint32_t pb0 = movmatrix_t(pack2<T>(p0, p1));
        const uint32_t pb1 = movmatrix_t(pack2<T>(p2, p3));
        // O^T += V^T P^T
        {
          const int r = (lane & 7) + ((lane >> 4) & 1) * 8;  // key row supplied by this lane
          const int cb = ((lane >> 3) & 1) * 8;               // d offset within the m-tile
          const uint32_t a_addr = vbase + r * p.pitch + cb * 2;
#pragma unroll
          for (int i = 0; i < KS; ++i) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4_t(a_addr + i * 32, a0, a1, a2, a3);
            mma16816<T>(o[i], a0, a1, a2, a3, pb0, pb1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(smem, s));
    }
    // row sums: lanes sharing lane&3 hold the same query heads
#pragma unroll
    for (int o_ = 4; o_ < 32; o_ <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o_);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o_);
    }
    const bool h0 = n0 < p.G, h1 = n0 + 1 < p.G;
    if (c.nparts == 1) {
      T* ob = reinterpret_cast<T*>(p.out) + (long long)c.q_row * p.out_stride + (long long)(c.kvh * p.G) * D_;
      const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        const int d = 16 * i + tq;
        if (h0) {
          ob[n0 * D_ + d] = Elem<T>::from_f(o[i][0] * i0);
          ob[n0 * D_ + d + 8] = Elem<T>::from_f(o[i][2] * i0);
        }
        if (h1) {
          ob[(n0 + 1) * D_ + d] = Elem<T>::from_f(o[i][1] * i1);
          ob[(n0 + 1) * D_ + d + 8] = Elem<T>::from_f(o[i][3] * i1);
        }
      }
    } else {
      const int DP = D_ + 2;
      float* wb = p.ws + ((long long)(c.u * p.SUB + c.sub) * p.Hq + c.kvh * p.G) * DP;
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        const int d = 16 * i + tq;
        if (h0) {
          __stcg(wb + n0 * DP + d, o[i][0]);
          __stcg(wb + n0 * DP + d + 8, o[i][2]);
        }
        if (h1) {
          __stcg(wb + (n0 + 1) * DP + d, o[i][1]);
          __stcg(wb + (n0 + 1) * DP + d + 8, o[i][3]);
        }
      }
      if (tq == 0) {
        if (h0) {
          __stcg(wb + n0 * DP + D_, m0);
          __stcg(wb + n0 * DP + D_ + 1, l0);
        }
        if (h1) {
          __stcg(wb + (n0 + 1) * DP + D_, m1);
          __stcg(wb + (n0 + 1) * DP + D_ + 1, l1);
        }
      }
      finish_partial<T>(p, c);
    }
  }
}

// Any dtype, any head_dim <= 32*DPL, up to 8 query heads per KV head:
// CUDA-core FMAs, lanes split the head dimension.
template <typename T, int DPL>
__device__ void consumer_simt(const AttnParams& p, unsigned char* smem, int total) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* stage0 = smem + kBarrierBytes;
  int k = 0;
  for (int v = blockIdx.x; v < total; v += gridDim.x) {
    const UnitCtx c = unit_ctx(p, v, warp);
    const int split = p.units[2 * c.u + 1];
    const int t0 = split * p.split, t1 = min(t0 + p.split, c.kv_len);
    float qv[8][DPL], acc[8][DPL], m[8], l[8];
    const T* qp = reinterpret_cast<const T*>(p.q) + (long long)c.q_row * p.q_stride + (long long)(c.kvh * p.G) * p.D;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      m[n] = kNegInf;
      l[n] = 0.f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int d = lane + 32 * i;
        qv[n][i] = (n < p.G && d < p.D) ? Elem<T>::to_f(qp[n * p.D + d]) * p.scale_log2 : 0.f;
        acc[n][i] = 0.f;
      }
    }
    for (int t = t0; t < t1; t += p.R, ++k) {
      const int s = k % p.stages, round = k / p.stages;
      if (!mbar_wait(full_bar(smem, s), round & 1, p.status)) return;
      const int tb = t + c.sub * 16;
      const int nv = min(16, t1 - tb);
      const unsigned char* kb = stage0 + s * p.stage_bytes + (c.sub * 16) * p.pitch + (warp % p.HG) * p.D * sizeof(T);
      const unsigned char* vb = kb + p.R * p.pitch;
      for (int j = 0; j < nv; ++j) {
        const T* kr = reinterpret_cast<const T*>(kb + j * p.pitch);
        const T* vr = reinterpret_cast<const T*>(vb + j * p.pitch);
        float kk[DPL], vv[DPL];
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int d = lane + 32 * i;
          kk[i] = d < p.D ? Elem<T>::to_f(kr[d]) : 0.f;
          vv[i] = d < p.D ? Elem<T>::to_f(vr[d]) : 0.f;
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          if (n < p.G) {
            float sdot = 0.f;
#pragma unroll
            for (int i = 0; i < DPL; ++i) sdot = fmaf(qv[n][i], kk[i], sdot);
#pragma unroll
            for (int o_ = 16; o_ > 0; o_ >>= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, o_);
            const float mn = fmaxf(m[n], sdot);
            const float al = ex2(m[n] - mn), pj = ex2(sdot - mn);
            l[n] = l[n] * al + pj;
            m[n] = mn;
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[n][i] = fmaf(pj, vv[i], acc[n][i] * al);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(smem, s));
    }
    if (c.nparts == 1) {
      T* ob = reinterpret_cast<T*>(p.out) + (long long)c.q_row * p.out_stride + (long long)(c.kvh * p.G) * p.D;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        if (n < p.G) {
          const float inv = l[n] > 0.f ? 1.f / l[n] : 0.f;
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            if (d < p.D) ob[n * p.D + d] = Elem<T>::from_f(acc[n][i] * inv);
          }
        }
      }
    } else {
      const int DP = p.D + 2;
      float* wb = p.ws + ((long long)(c.u * p.SUB + c.sub) * p.Hq + c.kvh * p.G) * DP;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        if (n < p.G) {
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            if (d < p.D) __stcg(wb + n * DP + d, acc[n][i]);
          }
          if (lane == 0) {
            __stcg(wb + n * DP + p.D, m[n]);
            __stcg(wb + n * DP + p.D + 1, l[n]);
          }
        }
      }
      finish_partial<T>(p, c);
    }
  }
}

// ---------------------------------------------------------------- kernel
template <typename T, int D_, bool MMA, int DPL>
__global__ void __launch_bounds__(288, 1) paged_attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full_bar(smem, s), 1);
      mbar_init(empty_bar(smem, s), p.W);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int n_units = min(p.counts[1], p.max_units);
  const int total = n_units * p.n_hg;
  if (warp == p.W) {
    producer_loop<T>(p, smem, total);
  } else if (warp < p.W) {
    if constexpr (MMA) consumer_mma<T, D_>(p, smem, total);
    else consumer_simt<T, DPL>(p, smem, total);
  }
}

// ---------------------------------------------------------------- host plan
struct Plan {
  int HG, SUB, W, n_hg, stages, R, pitch, row_bytes, stage_bytes, smem;
  bool mma;
  int dpl;
};

constexpr int kSmemBudget = 227 * 1024;

static int make_plan(int dtype, int Hq, int Hkv, int D, Plan& pl) {
  const size_t es = dtype_size(dtype);
  if (!es) return fail(NF_EINVAL, "nf_paged_attention: bad dtype %d", dtype);
  if (Hq <= 0 || Hkv <= 0 || D <= 0 || Hq % Hkv != 0)
    return fail(NF_EINVAL, "nf_paged_attention: num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)", Hq, Hkv);
  const int G = Hq / Hkv;
  if (G > 8) return fail(NF_EUNSUPPORTED, "nf_paged_attention: more than 8 query heads per KV head (%d)", G);
  if (D > 256) return fail(NF_EUNSUPPORTED, "nf_paged_attention: head_dim %d > 256", D);
  pl.mma = (dtype != NF_F32) && (D == 64 || D == 128);
  pl.dpl = D <= 32 ? 1 : D <= 64 ? 2 : D <= 128 ? 4 : 8;
  // Pick the head group (HG KV heads per CTA, rows contiguous in the pool) and
  // the number of 16-key sub-tiles per stage (SUB) with the most consumer
  // warps (W = HG * SUB <= 8) whose stage still fits three times in shared
  // memory (twice as a last resort).
  pl.HG = 0;
  for (int need = 3; need >= 2 && !pl.HG; --need) {
    for (int w = 8; w >= 1 && !pl.HG; w >>= 1) {
      for (int hg = (Hkv < 8 ? Hkv : 8); hg >= 1; --hg) {
        if (Hkv % hg || (hg * D * (int)es) % 16) continue;
        const int sub = w / hg > 0 ? w / hg : 1;
        if (hg * sub > 8) continue;
        const int pitch = hg * D * (int)es + 16;
        const int stage = 2 * 16 * sub * pitch;
        if ((kSmemBudget - kBarrierBytes) / stage < need) continue;
        pl.HG = hg;
        pl.SUB = sub;
        break;
      }
    }
  }
  if (!pl.HG) return fail(NF_EUNSUPPORTED, "nf_paged_attention: no stage layout fits for %d KV heads x %d elements", Hkv, D);
  pl.W = pl.HG * pl.SUB;
  pl.n_hg = Hkv / pl.HG;
  pl.R = 16 * pl.SUB;
  pl.row_bytes = pl.HG * D * (int)es;
  pl.pitch = pl.row_bytes + 16;
  pl.stage_bytes = 2 * pl.R * pl.pitch;
  pl.stages = (kSmemBudget - kBarrierBytes) / pl.stage_bytes;
  if (pl.stages > kMaxStages) pl.stages = kMaxStages;
  pl.smem = kBarrierBytes + pl.stages * pl.stage_bytes;
  return ok();
}

template <typename T, int D_, bool MMA, int DPL>
static int launch_attn(const AttnParams& p, const Plan& pl, int grid, cudaStream_t st) {
  auto kern = paged_attention_kernel<T, D_, MMA, DPL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_paged_attention: smem attribute: %s", cudaGetErrorString(e));
  kern<<<grid, (pl.W + 1) * 32, pl.smem, st>>>(p);
  return check_launch("nf_paged_attention");
}

template <typename T>
static int dispatch_attn(const AttnParams& p, const Plan& pl, int grid, cudaStream_t st) {
  if constexpr (!std::is_same<T, float>::value) {
    if (pl.mma && p.D == 64) return launch_attn<T, 64, true, 2>(p, pl, grid, st);
    if (pl.mma && p.D == 128) return launch_attn<T, 128, true, 4>(p, pl, grid, st);
  }
  switch (pl.dpl) {
    case 1: return launch_attn<T, 0, false, 1>(p, pl, grid, st);
    case 2: return launch_attn<T, 0, false, 2>(p, pl, grid, st);
    case 4: return launch_attn<T, 0, false, 4>(p, pl, grid, st);
    default: return launch_attn<T, 0, false, 8>(p, pl, grid, st);
  }
}

}  // namespace nf

extern "C" int nf_attention_workspace(int32_t max_units, int32_t max_items, int32_t num_q_heads,
                                      int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                                      int64_t* partial_floats, int64_t* counter_ints) {
  using namespace nf;
  Plan pl;
  int rc = make_plan(dtype, num_q_heads, num_kv_heads, head_dim, pl);
  if (rc) return rc;
  if (max_units <= 0 || max_items <= 0 || !partial_floats || !counter_ints)
    return fail(NF_EINVAL, "nf_attention_workspace: bad arguments");
  *partial_floats = (int64_t)max_units * pl.SUB * num_q_heads * (head_dim + 2);
  *counter_ints = (int64_t)max_items * num_kv_heads;
  return ok();
}

extern "C" int nf_paged_attention(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                  const void* k_pool, const void* v_pool, int32_t dtype, int32_t num_q_heads,
                                  int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                  const int32_t* block_tables, int32_t max_blocks_per_seq, const int32_t* items,
                                  const int32_t* units, const int32_t* counts, int32_t max_items, int32_t max_units,
                                  int32_t split_tokens, float scale, float* ws_partials, int64_t ws_partial_floats,
                                  int32_t* ws_counters, int64_t ws_counter_ints, int32_t* status, void* stream) {
  using namespace nf;
  Plan pl;
  int rc = make_plan(dtype, num_q_heads, num_kv_heads, head_dim, pl);
  if (rc) return rc;
  if (!out || !q || !k_pool || !v_pool || !block_tables || !items || !units || !counts || !status)
    return fail(NF_EINVAL, "nf_paged_attention: null pointer argument");
  if (block_size <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0 || max_units <= 0 || max_items <= 0)
    return fail(NF_EINVAL, "nf_paged_attention: sizes must be positive");
  if (split_tokens <= 0 || split_tokens % pl.R != 0)
    return fail(NF_EINVAL, "nf_paged_attention: split_tokens (%d) must be a positive multiple of %d", split_tokens, pl.R);
  const int64_t need_p = (int64_t)max_units * pl.SUB * num_q_heads * (head_dim + 2);
  const int64_t need_c = (int64_t)max_items * num_kv_heads;
  if (!ws_partials || ws_partial_floats < need_p || !ws_counters || ws_counter_ints < need_c)
    return fail(NF_EINVAL, "nf_paged_attention: workspace too small (need %lld floats, %lld counters)",
                (long long)need_p, (long long)need_c);
  const size_t es = dtype_size(dtype);
  auto al = [](const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
  if (!al(k_pool, 16) || !al(v_pool, 16)) return fail(NF_EINVAL, "nf_paged_attention: pools must be 16-byte aligned");
  if (pl.mma && (!al(q, 4) || (q_row_stride * (int64_t)es) % 4 != 0))
    return fail(NF_EINVAL, "nf_paged_attention: q rows must be 4-byte aligned");
  AttnParams p;
  p.out = static_cast<char*>(out);
  p.out_stride = out_row_stride;
  p.q = static_cast<const char*>(q);
  p.q_stride = q_row_stride;
  p.kp = static_cast<const char*>(k_pool);
  p.vp = static_cast<const char*>(v_pool);
  p.Hq = num_q_heads;
  p.Hkv = num_kv_heads;
  p.D = head_dim;
  p.G = num_q_heads / num_kv_heads;
  p.bs = block_size;
  p.num_blocks = num_blocks;
  p.bt = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.items = items;
  p.units = units;
  p.counts = counts;
  p.max_units = max_units;
  p.split = split_tokens;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.ws = ws_partials;
  p.cnt = ws_counters;
  p.status = status;
  p.HG = pl.HG;
  p.SUB = pl.SUB;
  p.W = pl.W;
  p.n_hg = pl.n_hg;
  p.stages = pl.stages;
  p.R = pl.R;
  p.pitch = pl.pitch;
  p.row_bytes = pl.row_bytes;
  p.stage_bytes = pl.stage_bytes;
  long long want = (long long)max_units * pl.n_hg;
  int grid = sm_count();
  if (want < grid) grid = (int)want;
  if (grid < 1) grid = 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NF_F32: return dispatch_attn<float>(p, pl, grid, st);
    case NF_F16: return dispatch_attn<__half>(p, pl, grid, st);
    case NF_BF16: return dispatch_attn<__nv_bfloat16>(p, pl, grid, st);
  }
  return fail(NF_EINVAL, "nf_paged_attention: bad dtype %d", dtype);
}
