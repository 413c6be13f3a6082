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
  int* cnt;     // reserved (per (item, KV head) counters of the workspace layout)
  int* queue;   // {next work item, spare, work items finished, CTAs done}; zero between launches
  int* status;
  const int* items;  // per query: slot, q_row, kv_len, unit_base
  int max_items;
  // launch plan
  int W, stages, head_bytes, stage_bytes, swz, tile, bs16, q_smem;
  int HG, n_hg;  // tensor-map path: KV heads per CTA and head groups
  int vec_out;         // 1: out rows and strides allow 8-byte (16-bit types) / 16-byte (float) stores
  int stage_out;       // tensor-map path: byte offset of the consumer warps' output staging (0: none)
  int pdl;             // 1: may be launched with programmatic stream serialization
  int own_parts_only;  // 1: the workspace holds only this launch's parts (no cascade parts to merge)
  // Gathered output over several GPUs: every output row is also stored at
  // peer_out[r] (another rank's buffer, same row stride and column offset as
  // out) for r < n_peers; when the launch is done its last CTA sets this
  // rank's entry of every rank's flag array to epoch and waits until all
  // ranks have set theirs (n_ranks > 1).
  int n_peers, n_ranks, rank, epoch;
  int* epoch_counter;  // device epoch (NfGather.epoch_counter), or null: epoch
  char* peer_out[kMaxRanks - 1];
  int* rank_flags[kMaxRanks];
};

// Stores of output elements at offset `off` (elements from out) on this GPU
// and on every peer of a gathered output.
template <typename T>
__device__ __forceinline__ void store_out(const AttnParams& p, long long off, T v) {
  reinterpret_cast<T*>(p.out)[off] = v;
  for (int r = 0; r < p.n_peers; ++r) reinterpret_cast<T*>(p.peer_out[r])[off] = v;
}
template <typename T>
__device__ __forceinline__ void store_out4(const AttnParams& p, long long off, float a, float b, float c, float d) {
  // four consecutive elements (off a multiple of 4): one 8- or 16-byte store per destination
  if constexpr (sizeof(T) == 2) {
    const uint2 v = make_uint2(pack2<T>(a, b), pack2<T>(c, d));
    *reinterpret_cast<uint2*>(reinterpret_cast<T*>(p.out) + off) = v;
    for (int r = 0; r < p.n_peers; ++r) *reinterpret_cast<uint2*>(reinterpret_cast<T*>(p.peer_out[r]) + off) = v;
  } else {
    const float4 v = make_float4(a, b, c, d);
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + off) = v;
    for (int r = 0; r < p.n_peers; ++r) *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.peer_out[r]) + off) = v;
  }
}

// A launch whose workspace cannot hold partial slots written by another
// kernel (own_parts_only) refuses a plan with cascade parts (partial slots
// beyond its own units, counts[3] > counts[1]): it flags
// NF_STATUS_FOREIGN_PARTS and does no work, instead of merging slots that
// were never written.
__device__ __forceinline__ bool parts_refused(const AttnParams& p) {
  return p.own_parts_only && __ldg(p.counts + 3) > __ldg(p.counts + 1);
}

// Units of the launch (0 for a refused plan, which is flagged once).
__device__ __forceinline__ int launch_units(const AttnParams& p) {
  if (parts_refused(p)) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(p.status, NF_STATUS_FOREIGN_PARTS);
    return 0;
  }
  return min(__ldg(p.counts + 1), p.max_units);
}

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
  int part;  // index of this unit among its item's parts
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
__device__ __forceinline__ int part_index(const AttnParams&, const Work& c) { return c.unit_base + c.part; }

// ---------------------------------------------------------------- split-K merge
// Merges float4 chunks c0 .. c0+31 (one per lane) of the G x D outputs of
// one (item, KV head): out = sum_j 2^(m_j - M) acc_j / sum_j 2^(m_j - M) l_j,
// one pass over the parts with PB parts' loads in flight and a running
// maximum (the sums are rescaled when it grows).
template <typename T, int PB>
__device__ void merge_chunk(const AttnParams& p, const Work& c, int c0) {
  const int lane = threadIdx.x & 31;
  const int D = p.D, DP = D + 4, D4 = D >> 2, GD4 = p.G * D4;
  const int e = min(c0 + lane, GD4 - 1), hn = e / D4, d = (e - hn * D4) * 4;
  const float* pe = p.ws + ((long long)c.unit_base * p.Hq + (long long)c.kvh * p.G + hn) * DP;
  const long long ps = (long long)p.Hq * DP;  // between consecutive parts
  float M = kNegInf, L = 0.f;
  float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < c.nparts; j += PB) {
    float4 x[PB];
    float2 ml[PB];
#pragma unroll
    for (int u = 0; u < PB; ++u) {
      if (j + u < c.nparts) {
        const float* pj = pe + (j + u) * ps;
        ml[u] = __ldcg(reinterpret_cast<const float2*>(pj + D));
        x[u] = __ldcg(reinterpret_cast<const float4*>(pj + d));
      } else {
        ml[u] = make_float2(kNegInf, 0.f);
        x[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float nm = M;
#pragma unroll
    for (int u = 0; u < PB; ++u) nm = fmaxf(nm, ml[u].x);
    const float b = nm == kNegInf ? 0.f : nm;  // parts with m = -inf saw no key: 2^(-inf) = 0
    const float sc = ex2(M - b);
    A.x *= sc; A.y *= sc; A.z *= sc; A.w *= sc; L *= sc;
#pragma unroll
    for (int u = 0; u < PB; ++u) {
      const float w = ml[u].x == kNegInf ? 0.f : ex2(ml[u].x - b);
      A.x += x[u].x * w; A.y += x[u].y * w; A.z += x[u].z * w; A.w += x[u].w * w; L += ml[u].y * w;
    }
    M = nm;
  }
  if (c0 + lane < GD4) {
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const long long off = (long long)c.q_row * p.out_stride + ((long long)c.kvh * p.G + hn) * D + d;
    if (p.vec_out)
      store_out4<T>(p, off, A.x * inv, A.y * inv, A.z * inv, A.w * inv);
    else {
      store_out<T>(p, off, Elem<T>::from_f(A.x * inv));
      store_out<T>(p, off + 1, Elem<T>::from_f(A.y * inv));
      store_out<T>(p, off + 2, Elem<T>::from_f(A.z * inv));
      store_out<T>(p, off + 3, Elem<T>::from_f(A.w * inv));
    }
  }
}

// End of a launch, called by every thread of every CTA once the CTA's work
// items are done (my_done of them, summed over the CTA by the caller in
// *cta_done).  Thread 0 adds them to the grid count and waits, with a time
// limit, until all `total` work items have stored their outputs or parts;
// then every warp of the grid takes a share of the split-K merges (one warp
// per (item, KV head, group of 32 output chunks) with more than one part).
// The counts and each warp's first merge task's item records (the step's
// pack wrote them before the launch) are requested before the wait, and
// each task's successor's records before the task's parts, so that a merge
// costs about one round trip once the wait ends.  `merge_bits` selects the
// pack's flags (counts[2]) that call for this merge: bit 0, an item with
// several parts; bit 1, an item with several units (a kernel whose units
// merge an item's cascade parts themselves when they are its only unit).
// The last CTA out resets the queue and the counts for the next launch.  The
// wait needs every CTA resident at once: the kernels are launched
// cooperatively.
template <typename T, int PB>
__device__ void finish_launch(const AttnParams& p, int* cta_done, int total, int merge_bits) {
  __shared__ int go;
  const int c_items = __ldg(p.counts), c_multi = __ldg(p.counts + 2), c_units = __ldg(p.counts + 3);
  // items before the first one with units (a step's prefill rows) have no parts: the tasks start after them
  const int t_first = max(0, c_multi >> 2);
  const int groups = (p.G * (p.D >> 2) + 31) >> 5;
  const int stride = gridDim.x * (blockDim.x >> 5);
  const int task0 = (threadIdx.x >> 5) * gridDim.x + blockIdx.x;
  const int4* items4 = reinterpret_cast<const int4*>(p.items);
  // records of a task's item t and the unit base of item t + 1 (within the buffers; checked against the counts
  // when used)
  auto records = [&](int task, int4& it, int& nx) {
    const int t = t_first + task / groups / p.Hkv;
    it = make_int4(0, 0, 0, -1);
    nx = 0;
    if (t < p.max_items) {
      it = __ldg(items4 + t);
      if (t + 1 < p.max_items) nx = __ldg(p.items + 4 * (t + 1) + 3);
    }
  };
  int4 it;
  int nx;
  records(task0, it, nx);
  __syncthreads();  // the CTA's output and part stores are issued
  const bool merge = (c_multi & merge_bits) != 0 && !parts_refused(p);
  if (threadIdx.x == 0) {
    __threadfence();
    const int mine = *cta_done;
    const int now = atomicAdd(p.queue + 2, mine) + mine;  // the last CTA in needs no further poll
    const bool ok = !merge || now >= total || wait_count(p.queue + 2, total, p.status);
    __threadfence();
    go = ok;
  }
  __syncthreads();
  if (go && merge) {
    const int n_items = min(c_items, p.max_items);
    const int n_units = min(c_units, p.max_units);  // partial slots, cascade parts included
    const int tasks = max(0, n_items - t_first) * p.Hkv * groups;
    // tasks dealt round-robin over the CTAs so that every SM takes a share
    for (int task = task0; task < tasks; task += stride) {
      const int pair = task / groups, grp = task - pair * groups;
      const int tl = pair / p.Hkv, t = t_first + tl;
      const int next = t + 1 < n_items ? nx : n_units;
      const int4 cur = it;
      if (task + stride < tasks) records(task + stride, it, nx);
      const int nparts = next - cur.w;
      if (nparts <= 1 || cur.w < 0 || next > p.max_units) continue;  // written directly, or a flagged overflow
      Work c;
      c.w = task;
      c.u = 0;
      c.item = t;
      c.slot = cur.x;
      c.q_row = cur.y;
      c.t0 = c.t1 = 0;
      c.unit_base = cur.w;
      c.nparts = nparts;
      c.kvh = pair - tl * p.Hkv;
      c.part = 0;
      merge_chunk<T, PB>(p, c, grp * 32);
    }
  }
  // a gathered output: the CTA's stores, to this GPU and to its peers, are
  // ordered before the CTA counts itself done by the CTA barrier and a
  // device-scope fence of the counting thread; the last CTA out observes
  // every count and fences at system scope before it signals the peers
  // (exchange_signal_wait), and as fences are cumulative that release covers
  // the stores of every CTA of the grid.  One system-scope fence per launch:
  // a fence in every CTA cost 7 us per two-GPU launch.
  __syncthreads();
  if (threadIdx.x == 0 && p.n_ranks > 1) __threadfence();
  if (threadIdx.x == 0 && atomicAdd(p.queue + 3, 1) == (int)gridDim.x - 1) {
    __threadfence();
    p.queue[0] = 0;
    p.queue[1] = 0;
    p.queue[2] = 0;
    p.queue[3] = 0;
    __threadfence();
    // the last CTA out: this rank's rows are in every rank's buffer; signal
    // the peers and wait for theirs, so that the launch ends with the whole
    // gathered output in place on this GPU
    if (p.n_ranks > 1)
      exchange_signal_wait(p.rank_flags, p.n_ranks, p.rank, p.epoch, p.status, kWaitLimitCycles, p.epoch_counter);
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
  const long long ob = (long long)c.q_row * p.out_stride + (long long)(c.kvh * p.G) * D_;
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
  for (int i = 0; i < KS; ++i) {
    const int d = 16 * i + tq;
    if (h0) {
      store_out<T>(p, ob + n0 * D_ + d, Elem<T>::from_f(o[i][0] * i0));
      store_out<T>(p, ob + n0 * D_ + d + 8, Elem<T>::from_f(o[i][2] * i0));
    }
    if (h1) {
      store_out<T>(p, ob + (n0 + 1) * D_ + d, Elem<T>::from_f(o[i][1] * i1));
      store_out<T>(p, ob + (n0 + 1) * D_ + d + 8, Elem<T>::from_f(o[i][3] * i1));
    }
  }
}

// Normalised output rows (the item has one part) staged in shared memory:
// the warp's G x D block of the output row (contiguous: the KV head's query
// heads) is written to its staging area, then copied out in 16-byte stores,
// one per lane and destination -- over NVLink to a gathered output's peers
// a 16-byte store carries eight times what a 2-byte one does.
template <typename T, int D_>
__device__ __forceinline__ void mma_store_output_staged(const AttnParams& p, const Work& c, float (&o)[D_ / 16][4],
                                                        float l0, float l1, uint32_t stage) {
  constexpr int KS = D_ / 16;
  const int lane = threadIdx.x & 31;
  const int n0 = 2 * (lane & 3), tq = lane >> 2;
  const bool h0 = n0 < p.G, h1 = n0 + 1 < p.G;
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
  auto st16 = [](uint32_t a, T v) {
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(a), "h"(*reinterpret_cast<unsigned short*>(&v)) : "memory");
  };
#pragma unroll
  for (int i = 0; i < KS; ++i) {
    const int d = 16 * i + tq;
    if (h0) {
      st16(stage + (n0 * D_ + d) * 2, Elem<T>::from_f(o[i][0] * i0));
      st16(stage + (n0 * D_ + d + 8) * 2, Elem<T>::from_f(o[i][2] * i0));
    }
    if (h1) {
      st16(stage + ((n0 + 1) * D_ + d) * 2, Elem<T>::from_f(o[i][1] * i1));
      st16(stage + ((n0 + 1) * D_ + d + 8) * 2, Elem<T>::from_f(o[i][3] * i1));
    }
  }
  __syncwarp();
  const long long ob = (long long)c.q_row * p.out_stride + (long long)(c.kvh * p.G) * D_;
  for (int ch = lane; ch < p.G * D_ / 8; ch += 32) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(stage + ch * 16));
    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + ob + ch * 8) = v;
    for (int r = 0; r < p.n_peers; ++r) *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.peer_out[r]) + ob + ch * 8) = v;
  }
  __syncwarp();  // the staging area is free for the warp's next output
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

// The output rows of an item whose only unit this is, beside its cascade
// parts: every other part of the item (slots unit_base .. unit_base +
// nparts - 1 but this unit's own, c.part), written by the cascade launch
// before this one, is merged into this unit's running state (o, m, l; l
// summed over the lanes) in registers -- PB parts' loads in flight at a
// time, rescaled as the maximum grows -- and the rows are written, with no
// wait for any other worker.
template <typename T, int D_>
__device__ __forceinline__ void mma_merge_parts(const AttnParams& p, const Work& c, float (&o)[D_ / 16][4],
                                                float m0, float m1, float l0, float l1, uint32_t stage) {
  constexpr int KS = D_ / 16;
  constexpr int PB = D_ == 64 ? 4 : 2;
  const int lane = threadIdx.x & 31;
  const int n0 = 2 * (lane & 3), tq = lane >> 2;
  const bool h0 = n0 < p.G, h1 = n0 + 1 < p.G;
  const int DP = D_ + 4, nc = c.nparts - 1;  // the other parts
  const float* wb = p.ws + ((long long)c.unit_base * p.Hq + c.kvh * p.G) * DP;
  const long long ps = (long long)p.Hq * DP;  // between consecutive parts
  float M0 = m0, M1 = m1;
  for (int j = 0; j < nc; j += PB) {
    float2 ml0[PB], ml1[PB];
    float a[PB][KS][4];
#pragma unroll
    for (int u = 0; u < PB; ++u) {
      const bool in = j + u < nc;
      const int part = j + u < c.part ? j + u : j + u + 1;  // skipping this unit's own
      const float* w0 = wb + part * ps + n0 * DP;
      const float* w1 = w0 + DP;
      ml0[u] = in && h0 ? __ldcg(reinterpret_cast<const float2*>(w0 + D_)) : make_float2(kNegInf, 0.f);
      ml1[u] = in && h1 ? __ldcg(reinterpret_cast<const float2*>(w1 + D_)) : make_float2(kNegInf, 0.f);
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        const int d = 16 * i + tq;
        a[u][i][0] = in && h0 ? __ldcg(w0 + d) : 0.f;
        a[u][i][2] = in && h0 ? __ldcg(w0 + d + 8) : 0.f;
        a[u][i][1] = in && h1 ? __ldcg(w1 + d) : 0.f;
        a[u][i][3] = in && h1 ? __ldcg(w1 + d + 8) : 0.f;
      }
    }
    float nm0 = M0, nm1 = M1;
#pragma unroll
    for (int u = 0; u < PB; ++u) {
      nm0 = fmaxf(nm0, ml0[u].x);
      nm1 = fmaxf(nm1, ml1[u].x);
    }
    const float b0 = nm0 == kNegInf ? 0.f : nm0, b1 = nm1 == kNegInf ? 0.f : nm1;
    const float s0 = ex2(M0 - b0), s1 = ex2(M1 - b1);  // 2^(-inf) = 0: a state that saw no key
    l0 *= s0;
    l1 *= s1;
#pragma unroll
    for (int i = 0; i < KS; ++i) {
      o[i][0] *= s0; o[i][2] *= s0;
      o[i][1] *= s1; o[i][3] *= s1;
    }
#pragma unroll
    for (int u = 0; u < PB; ++u) {
      const float w0 = ml0[u].x == kNegInf ? 0.f : ex2(ml0[u].x - b0);
      const float w1 = ml1[u].x == kNegInf ? 0.f : ex2(ml1[u].x - b1);
      l0 += ml0[u].y * w0;
      l1 += ml1[u].y * w1;
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        o[i][0] += a[u][i][0] * w0; o[i][2] += a[u][i][2] * w0;
        o[i][1] += a[u][i][1] * w1; o[i][3] += a[u][i][3] * w1;
      }
    }
    M0 = nm0;
    M1 = nm1;
  }
  if (stage)
    mma_store_output_staged<T, D_>(p, c, o, l0, l1, stage);
  else
    mma_store_output<T, D_>(p, c, o, l0, l1);
}

// Output rows when the item has one part, else the part record (merged at
// the end of the launch, finish_launch).
template <typename T, int D_>
__device__ __forceinline__ void mma_epilogue(const AttnParams& p, const Work& c, float (&o)[D_ / 16][4], float m0,
                                             float m1, float l0, float l1) {
  if (c.nparts == 1)
    mma_store_output<T, D_>(p, c, o, l0, l1);
  else
    mma_store_part<T, D_>(p, c, o, m0, m1, l0, l1);
}

}  // namespace nf
