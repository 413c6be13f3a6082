// Device code shared by the paged-attention kernels (cp.async and tensor-map
// staging): launch parameters, work records and the split-K epilogue/merge.
#pragma once

#include <math.h>

#include "nf_common.cuh"

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
  const int* units;
  const int* counts;
  int max_units, split;
  float scale_log2;
  float* ws;    // partials [max_units][Hq][D + 4]: acc[D], m, l, pad
  int* cnt;     // parts finished per (item, KV head)
  int* queue;   // {next work item, warps finished}; zero between launches
  int* status;
  // launch plan
  int W, stages, head_bytes, stage_bytes, swz, tile, bs16, q_smem;
  int HG, n_hg;  // tensor-map path: KV heads per CTA and head groups
};

constexpr float kNegInf = -INFINITY;

// Byte offset of 16-byte chunk c of row r inside a tile (rows of head_bytes).
__device__ __forceinline__ int tile_off(int r, int c, int head_bytes, int swz) {
  const int pc = swz ? ((c & ~7) | ((c & 7) ^ (r & 7))) : c;
  return r * head_bytes + pc * 16;
}

// One work item as both cursors see it.
struct Work {
  int w;  // work item index; < 0 marks the end of this warp's work
  int u, item, slot, q_row, t0, t1, unit_base, nparts, kvh;
};

__device__ __forceinline__ int checked_block(const AttnParams& p, const int* btrow, int lb) {
  int phys = lb < p.max_blocks ? __ldg(btrow + lb) : -1;
  if (phys < 0 || phys >= p.num_blocks) {
    atomicOr(p.status, NF_STATUS_BAD_BLOCK);
    phys = 0;
  }
  return phys;
}

// ---------------------------------------------------------------- split-K merge
// Merges the nparts (acc, m, l) records of one (item, KV head) into the
// output.  Warp-parallel: lanes read the parts' maxima and sums for all heads
// of the group at once, then every lane accumulates its float4 chunks of the
// output with four parts' loads in flight.
template <typename T>
__device__ void merge_partials(const AttnParams& p, const Work& c) {
  const int lane = threadIdx.x & 31;
  const int D = p.D, DP = D + 4, G = p.G;
  const float* part0 = p.ws + ((long long)c.unit_base * p.Hq + (long long)c.kvh * G) * DP;
  const long long ps = (long long)p.Hq * DP;  // between consecutive parts
  const int GP = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;  // heads rounded up to a power of two
  const int n = lane % GP, jj = lane / GP, PP = 32 / GP;
  float mx = kNegInf;
  if (n < G)
    for (int j = jj; j < c.nparts; j += PP) mx = fmaxf(mx, __ldcg(part0 + j * ps + n * DP + D));
  for (int o_ = GP; o_ < 32; o_ <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o_));
  float sm = 0.f;
  if (n < G)
    for (int j = jj; j < c.nparts; j += PP) {
      const float* pb = part0 + j * ps + n * DP;
      const float mj = __ldcg(pb + D);
      if (mj != kNegInf) sm += __ldcg(pb + D + 1) * ex2(mj - mx);
    }
  for (int o_ = GP; o_ < 32; o_ <<= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o_);
  // lane n (< GP) now holds head n's max and normaliser
  T* o = reinterpret_cast<T*>(p.out) + (long long)c.q_row * p.out_stride + (long long)c.kvh * G * D;
  const int D4 = D >> 2, GD4 = G * D4;
  for (int e0 = 0; e0 < GD4; e0 += 32) {
    const int e = min(e0 + lane, GD4 - 1);
    const int hn = e / D4, d = (e - hn * D4) * 4;
    const float Mn = __shfl_sync(0xffffffffu, mx, hn);
    const float Ln = __shfl_sync(0xffffffffu, sm, hn);
    if (e0 + lane < GD4) {
      const float* pe = part0 + hn * DP;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      int j = 0;
      for (; j + 4 <= c.nparts; j += 4) {
        float4 x[4];
        float mm[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          x[u] = __ldcg(reinterpret_cast<const float4*>(pe + (j + u) * ps + d));
          mm[u] = __ldcg(pe + (j + u) * ps + D);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float wgt = mm[u] == kNegInf ? 0.f : ex2(mm[u] - Mn);
          a.x += x[u].x * wgt; a.y += x[u].y * wgt; a.z += x[u].z * wgt; a.w += x[u].w * wgt;
        }
      }
      for (; j < c.nparts; ++j) {
        const float mj = __ldcg(pe + j * ps + D);
        if (mj != kNegInf) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(pe + j * ps + d));
          const float wgt = ex2(mj - Mn);
          a.x += x.x * wgt; a.y += x.y * wgt; a.z += x.z * wgt; a.w += x.w * wgt;
        }
      }
      const float inv = Ln > 0.f ? 1.f / Ln : 0.f;
      T* od = o + hn * D + d;
      od[0] = Elem<T>::from_f(a.x * inv);
      od[1] = Elem<T>::from_f(a.y * inv);
      od[2] = Elem<T>::from_f(a.z * inv);
      od[3] = Elem<T>::from_f(a.w * inv);
    }
  }
}

// After this warp wrote its part: count it; the last part merges.
template <typename T>
__device__ void finish_partial(const AttnParams& p, const Work& c) {
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

// The last of `participants` queue users (warps or CTAs) to run out of work
// resets the queue for the next launch.
__device__ __forceinline__ void retire_worker(const AttnParams& p, int participants) {
  if ((threadIdx.x & 31) == 0) {
    __threadfence();
    if (atomicAdd(p.queue + 1, 1) == participants - 1) {
      p.queue[0] = 0;
      p.queue[1] = 0;
      __threadfence();
    }
  }
}

// Output of one warp's (unit, KV head) from the O^T accumulators of the
// tensor-core path: normalised rows when the item has one part, else the
// part's (acc, m, l) record and the split-K bookkeeping.  Lane layout of
// o[i][*]: d = 16 i + lane/4 (+8), query heads 2 (lane % 4) (+1).
template <typename T, int D_>
__device__ __forceinline__ void mma_epilogue(const AttnParams& p, const Work& c, float (&o)[D_ / 16][4], float m0,
                                             float m1, float l0, float l1) {
  constexpr int KS = D_ / 16;
  const int lane = threadIdx.x & 31;
  const int n0 = 2 * (lane & 3), tq = lane >> 2;
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
    const int DP = D_ + 4;
    float* wb = p.ws + ((long long)c.u * p.Hq + c.kvh * p.G) * DP;
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

}  // namespace nf
