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

// Split-K part slot of a unit in the workspace: the parts of one item are
// contiguous from its unit_base, in key order, wherever the unit sits in the
// unit list.
__device__ __forceinline__ int part_index(const AttnParams& p, const Work& c) { return c.unit_base + c.t0 / p.split; }

// ---------------------------------------------------------------- split-K merge
// Merges the nparts (acc, m, l) records of one (item, KV head) into the
// output: out = sum_j 2^(m_j - M) acc_j / sum_j 2^(m_j - M) l_j.  Lane e owns
// float4 chunks e and e + 32 of the group's G x D outputs; one pass over the
// parts with PB parts' loads in flight per lane and a running maximum (the
// sums are rescaled when it grows), so the merge costs about nparts / PB
// round trips to L2.
template <typename T, int PB>
__device__ void merge_partials(const AttnParams& p, const Work& c) {
  const int lane = threadIdx.x & 31;
  const int D = p.D, DP = D + 4, G = p.G;
  const float* part0 = p.ws + ((long long)c.unit_base * p.Hq + (long long)c.kvh * G) * DP;
  const long long ps = (long long)p.Hq * DP;  // between consecutive parts
  T* o = reinterpret_cast<T*>(p.out) + (long long)c.q_row * p.out_stride + (long long)c.kvh * G * D;
  const int D4 = D >> 2, GD4 = G * D4;
  for (int e0 = 0; e0 < GD4; e0 += 64) {
    const int ea = min(e0 + lane, GD4 - 1), eb = min(e0 + 32 + lane, GD4 - 1);
    const int ha = ea / D4, hb = eb / D4;
    const float* pa = part0 + ha * DP + (ea - ha * D4) * 4;
    const float* pb = part0 + hb * DP + (eb - hb * D4) * 4;
    const float* ma = part0 + ha * DP + D;
    const float* mb = part0 + hb * DP + D;
    float Ma = kNegInf, Mb = kNegInf, La = 0.f, Lb = 0.f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f), B = A;
    for (int j = 0; j < c.nparts; j += PB) {
      float4 xa[PB], xb[PB];
      float2 la[PB], lb[PB];
#pragma unroll
      for (int u = 0; u < PB; ++u) {
        if (j + u < c.nparts) {
          const long long off = (long long)(j + u) * ps;
          la[u] = __ldcg(reinterpret_cast<const float2*>(ma + off));
          lb[u] = __ldcg(reinterpret_cast<const float2*>(mb + off));
          xa[u] = __ldcg(reinterpret_cast<const float4*>(pa + off));
          xb[u] = __ldcg(reinterpret_cast<const float4*>(pb + off));
        } else {
          la[u] = lb[u] = make_float2(kNegInf, 0.f);
          xa[u] = xb[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      float na = Ma, nb = Mb;
#pragma unroll
      for (int u = 0; u < PB; ++u) {
        na = fmaxf(na, la[u].x);
        nb = fmaxf(nb, lb[u].x);
      }
      // parts with m = -inf saw no key; 2^(-inf) = 0 drops them
      const float ba = na == kNegInf ? 0.f : na, bb = nb == kNegInf ? 0.f : nb;
      const float sa = ex2(Ma - ba), sb = ex2(Mb - bb);
      A.x *= sa; A.y *= sa; A.z *= sa; A.w *= sa; La *= sa;
      B.x *= sb; B.y *= sb; B.z *= sb; B.w *= sb; Lb *= sb;
#pragma unroll
      for (int u = 0; u < PB; ++u) {
        const float wa = la[u].x == kNegInf ? 0.f : ex2(la[u].x - ba);
        const float wb = lb[u].x == kNegInf ? 0.f : ex2(lb[u].x - bb);
        A.x += xa[u].x * wa; A.y += xa[u].y * wa; A.z += xa[u].z * wa; A.w += xa[u].w * wa; La += la[u].y * wa;
        B.x += xb[u].x * wb; B.y += xb[u].y * wb; B.z += xb[u].z * wb; B.w += xb[u].w * wb; Lb += lb[u].y * wb;
      }
      Ma = na;
      Mb = nb;
    }
    if (e0 + lane < GD4) {
      const float inv = La > 0.f ? 1.f / La : 0.f;
      T* od = o + ha * D + (ea - ha * D4) * 4;
      od[0] = Elem<T>::from_f(A.x * inv);
      od[1] = Elem<T>::from_f(A.y * inv);
      od[2] = Elem<T>::from_f(A.z * inv);
      od[3] = Elem<T>::from_f(A.w * inv);
    }
    if (e0 + 32 + lane < GD4) {
      const float inv = Lb > 0.f ? 1.f / Lb : 0.f;
      T* od = o + hb * D + (eb - hb * D4) * 4;
      od[0] = Elem<T>::from_f(B.x * inv);
      od[1] = Elem<T>::from_f(B.y * inv);
      od[2] = Elem<T>::from_f(B.z * inv);
      od[3] = Elem<T>::from_f(B.w * inv);
    }
  }
}

// After this warp wrote its part: count it; the last part merges (PB: parts'
// loads in flight per lane, see merge_partials).
template <typename T, int PB>
__device__ void finish_partial(const AttnParams& p, const Work& c) {
  __threadfence();
  __syncwarp();
  int last = 0;
  int* ctr = p.cnt + (long long)c.item * p.Hkv + c.kvh;
  if ((threadIdx.x & 31) == 0) last = (atomicAdd(ctr, 1) == c.nparts - 1);
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence();
    merge_partials<T, PB>(p, c);
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

// Stores of one warp's (unit, KV head) from the O^T accumulators of the
// tensor-core path.  Lane layout of o[i][*]: d = 16 i + lane/4 (+8), query
// heads 2 (lane % 4) (+1).

// Normalised output rows (the item has one part).
template <typename T, int D_>
__device__ __forceinline__ void mma_store_output(const AttnParams& p, const Work& c, float (&o)[D_ / 16][4], float l0,
                                                 float l1) {
  constexpr int KS = D_ / 16;
  const int lane = threadIdx.x & 31;
  const int n0 = 2 * (lane & 3), tq = lane >> 2;
  const bool h0 = n0 < p.G, h1 = n0 + 1 < p.G;
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
}

// The unit's split-K part record (acc, m, l) in the workspace.
template <typename T, int D_>
__device__ __forceinline__ void mma_store_part(const AttnParams& p, const Work& c, float (&o)[D_ / 16][4], float m0,
                                               float m1, float l0, float l1) {
  constexpr int KS = D_ / 16;
  const int lane = threadIdx.x & 31;
  const int n0 = 2 * (lane & 3), tq = lane >> 2;
  const bool h0 = n0 < p.G, h1 = n0 + 1 < p.G;
  const int DP = D_ + 4;
  float* wb = p.ws + ((long long)part_index(p, c) * p.Hq + c.kvh * p.G) * DP;
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
}

// Output rows when the item has one part, else the part record and the
// split-K bookkeeping (the last part merges).
template <typename T, int D_>
__device__ __forceinline__ void mma_epilogue(const AttnParams& p, const Work& c, float (&o)[D_ / 16][4], float m0,
                                             float m1, float l0, float l1) {
  if (c.nparts == 1) {
    mma_store_output<T, D_>(p, c, o, l0, l1);
  } else {
    mma_store_part<T, D_>(p, c, o, m0, m1, l0, l1);
    finish_partial<T, 2>(p, c);
  }
}

}  // namespace nf
