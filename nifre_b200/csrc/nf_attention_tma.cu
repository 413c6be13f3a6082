// Paged attention with tensor-map (TMA) staging of whole key blocks.
//
// Same computation and work records as nf_attention.cu (see there for the
// reference mapping: attention.py:106-152 over the paged_kv_cache.py pools);
// this file only changes how keys reach shared memory, for 16-bit pools with
// head_dim 64 or 128 and a block size that is a multiple of 16.
//
// A CTA owns HG KV heads.  Its producer warp takes (unit, head group) work
// items from the queue and, for each 16-key step of a unit, issues one TMA
// tensor copy for K and one for V: the box is 16 tokens of one block x HG
// heads x head_dim, read through a tensor map whose dimensions are
// (head_dim, token in block, head, block) -- strides 2 B, Hkv*D*2, D*2,
// bs*Hkv*D*2 -- so the copy lands head-major: for every head, 16 rows of
// 128 bytes (two such halves for head_dim 128) with the hardware 128-byte
// swizzle, which is the bank-conflict-free layout the ldmatrix fragment
// loads expect.  Two requests move 16 KB (head_dim 64, 8 heads) where
// per-row copies needed 256 instructions per lane-set.  If the driver refuses
// that permuted-stride map, a map with increasing strides and one box per
// head (and per 64-element half of the head) gives the same layout.
//
// Consumer warp h computes KV head h of the group exactly as the per-warp
// path does (mma.sync S^T = K Q^T, online softmax, O^T += V^T P^T), two
// staged 16-key tiles per update.  A unit that is one split-K part of a
// longer item ends with the part's (acc, m, l) store; once every unit of the
// launch is done, all warps of the grid merge the parts (finish_launch).  Every wait is an mbarrier wait with a
// time limit: a wait that runs out sets NF_STATUS_WAIT_TIMEOUT and the warp
// leaves its loop.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "nf_attn_common.cuh"
#include "nf_internal.h"
#include "nf_tma.cuh"

namespace nf {

// Shared-memory header: stage barriers (full[8] at 0, empty[8] at 64) and
// step records (8 x 64 B at 128).
constexpr int kTmaHeader = 1024;
constexpr int kTmaMaxStages = 8;
constexpr int kTmaMaxThreads = (8 + 1) * 32;

struct StepRec {  // one 16-key step as the producer describes it to the consumers
  int u, item, q_row, t0, t1, unit_base, nsplits, hg, t, first, last, part, pad[4];
};

// Byte offset of key row r, 16-byte chunk c, in one head's staged tile:
// [d_hi][16 rows][128 B], chunks XOR-swizzled by the row (the TMA 128B mode).
__device__ __forceinline__ int tma_off(int r, int c) {
  return (c >> 3) * 2048 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

// Returns the number of work items this CTA took.
template <typename T, int D_>
__device__ int tma_producer(const AttnParams& p, const CUtensorMap* tk, const CUtensorMap* tv, unsigned char* base,
                            int total, int box_bytes, int q_bytes) {
  constexpr int NDH = D_ / 64;  // 64-element halves of a head row
  const uint32_t hdr = smem_u32(base);
  auto full = [&](int s) { return hdr + 8 * s; };
  auto empty = [&](int s) { return hdr + 64 + 8 * s; };
  StepRec* recs = reinterpret_cast<StepRec*>(base + 128);
  const uint32_t stage0 = hdr + kTmaHeader;
  const int S = p.stages;
  // The switch to the next unit needs three dependent round trips (ticket,
  // unit record, first block-table entry) of 1-2 us each under full load,
  // and this thread stalls on each result while no copy is issued.  So the
  // next ticket is requested kAhead steps (about 6 us of streaming) before the
  // current unit's last step, its record is loaded kGap steps later and its
  // first block-table entry kGap steps after that, each once the previous
  // result has had time to arrive.  Short units take the stalls.
  constexpr int kAhead = 8, kGap = 2;
  const uint64_t pol = l2_evict_first();
  const int4* urec = reinterpret_cast<const int4*>(p.units);
  int k = 0;           // steps issued
  int s = 0;           // slot of step k (k mod S)
  uint32_t pe = 1;     // parity that frees slot s for step k: ((k / S) & 1) ^ 1
  bool ok = true;
  // the first work item is this CTA's own (no round trip to the queue); the
  // queue hands out the rest, from gridDim.x on
  int w = blockIdx.x;
  int4 ra = make_int4(0, 0, 0, 0), rb = ra;
  if (w < total) {
    ra = __ldg(urec + 2 * (w / p.n_hg));
    rb = __ldg(urec + 2 * (w / p.n_hg) + 1);
  }
  // This launch may overlap the kernel before it on the stream (the KV
  // append of this layer, or the cascade, with programmatic stream
  // serialization).  The unit records and block tables come from the step's
  // pack, which completed before that kernel began; the pools (where the
  // append writes the new keys and values), the cascade's partial records
  // and the queue are touched only after the wait.  A launch whose queue is
  // cleared by the operation just before it (the allocation-free entry
  // point's memset) goes without programmatic serialization (p.pdl = 0).
  if (w < total) {
    const int lb = rb.x / p.bs;
    if (lb < p.max_blocks) asm volatile("prefetch.global.L1 [%0];" ::"l"(p.bt + (long long)ra.y * p.max_blocks + lb));
  }
  pdl_wait();
  int taken = 0;
  while (w < total) {
    ++taken;
    const int u = w / p.n_hg, hg = w - u * p.n_hg;
    const int* btrow = p.bt + (long long)ra.y * p.max_blocks;
    const int h0 = hg * p.HG;
    const int nsteps = (rb.y - rb.x + 15) >> 4;
    const int ask = nsteps - 1 - min(kAhead, nsteps - 1);  // step that requests the next ticket
    int wn = total;
    int4 na = make_int4(0, 0, 0, 0), nb = na;
    for (int i = 0, t = rb.x; i < nsteps; ++i, t += 16, ++k) {
      if (i == ask) {
        wn = (int)gridDim.x + atomicAdd(p.queue, 1);
      } else if (i == ask + kGap && wn < total) {
        na = __ldg(urec + 2 * (wn / p.n_hg));
        nb = __ldg(urec + 2 * (wn / p.n_hg) + 1);
      } else if (i == ask + 2 * kGap && wn < total) {
        const int lb = nb.x / p.bs;
        if (lb < p.max_blocks)
          asm volatile("prefetch.global.L1 [%0];" ::"l"(p.bt + (long long)na.y * p.max_blocks + lb));
      }
      if (!mbar_wait(empty(s), pe, p.status)) {
        ok = false;
        break;
      }
      StepRec& r = recs[s];
      r.u = u; r.item = ra.x; r.q_row = ra.z; r.t0 = rb.x; r.t1 = rb.y; r.unit_base = rb.z;
      r.nsplits = rb.w; r.hg = hg; r.t = t; r.first = i == 0; r.last = i == nsteps - 1; r.part = ra.w;
      const int lb = t / p.bs, off = t - lb * p.bs;
      const int phys = checked_block(p, btrow, lb);
      const uint32_t sb = stage0 + s * p.stage_bytes;
      mbar_arrive_expect_tx(full(s), 2 * box_bytes + (r.first ? q_bytes : 0));
      if (p.swz) {  // permuted-stride map: one box = 16 tokens x HG heads
        if constexpr (D_ == 64) {
          tma_load_4d(sb, tk, 0, off, h0, phys, full(s), pol);
          tma_load_4d(sb + box_bytes, tv, 0, off, h0, phys, full(s), pol);
        } else {
          tma_load_5d(sb, tk, 0, off, 0, h0, phys, full(s), pol);
          tma_load_5d(sb + box_bytes, tv, 0, off, 0, h0, phys, full(s), pol);
        }
      } else {  // increasing-stride map: one box per head (and per half of a 128-wide head)
        for (int h = 0; h < p.HG; ++h)
#pragma unroll
          for (int dh = 0; dh < NDH; ++dh) {
            const uint32_t d = sb + (h * NDH + dh) * 2048;
            if constexpr (D_ == 64) {
              tma_load_4d(d, tk, 0, h0 + h, off, phys, full(s), pol);
              tma_load_4d(d + box_bytes, tv, 0, h0 + h, off, phys, full(s), pol);
            } else {
              tma_load_5d(d, tk, 0, dh, h0 + h, off, phys, full(s), pol);
              tma_load_5d(d + box_bytes, tv, 0, dh, h0 + h, off, phys, full(s), pol);
            }
          }
      }
      if (r.first) {
        const char* qrow = p.q + ((long long)ra.z * p.q_stride + (long long)h0 * p.G * p.D) * (long long)sizeof(T);
        bulk_g2s(sb + 2 * box_bytes, qrow, q_bytes, full(s));
      }
      if (++s == S) {
        s = 0;
        pe ^= 1;
      }
    }
    if (!ok) break;
    if (ask + kGap > nsteps - 1 && wn < total) {  // a short unit: the record was not loaded yet
      na = __ldg(urec + 2 * (wn / p.n_hg));
      nb = __ldg(urec + 2 * (wn / p.n_hg) + 1);
    }
    w = wn;
    ra = na;
    rb = nb;
  }
  if (ok) {
    // end of work: a record with u = -1, published by a plain arrive
    if (mbar_wait(empty(s), pe, p.status)) {
      recs[s].u = -1;
      mbar_arrive(full(s));
      return taken;
    }
  }
  // a wait ran out: leave no copy in flight into this CTA's shared memory
  for (int j = max(0, k - S); j < k; ++j) mbar_wait(full(j % S), (j / S) & 1, p.status);
  return taken;
}

// One consumer update over NT staged 16-key tiles of this warp's head (K
// tiles at kb[j], V tiles at vb[j]; keys at or past nv are masked): S^T = K
// Q^T per tile, one running-max update for all NT x 16 keys, O^T += V^T P^T.
// Two tiles give two independent MMA chains and halve the per-key cost of
// the max shuffles, the rescale of O and the barrier traffic.
template <typename T, int D_, int NT>
__device__ __forceinline__ void consume_tiles(const AttnParams& p, const uint32_t (&kb)[2], const uint32_t (&vb)[2],
                                              int nv, const uint32_t (&qf)[D_ / 16][2], float (&o)[D_ / 16][4],
                                              float& m0, float& m1, float& l0, float& l1) {
  constexpr int KS = D_ / 16;
  const int lane = threadIdx.x & 31;
  const int tq = lane >> 2;
  const int kr = (lane & 7) + ((lane >> 3) & 1) * 8, kc = lane >> 4;
  const int vr = (lane & 7) + ((lane >> 4) & 1) * 8, vc = (lane >> 3) & 1;
  float x[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(kb[j] + tma_off(kr, 2 * ks + kc), a0, a1, a2, a3);
      mma16816<T>(sc, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
    }
    const bool v0 = 16 * j + tq < nv, v1 = 16 * j + tq + 8 < nv;
    x[j][0] = v0 ? sc[0] * p.scale_log2 : kNegInf;
    x[j][1] = v0 ? sc[1] * p.scale_log2 : kNegInf;
    x[j][2] = v1 ? sc[2] * p.scale_log2 : kNegInf;
    x[j][3] = v1 ? sc[3] * p.scale_log2 : kNegInf;
  }
  float mx0 = fmaxf(x[0][0], x[0][2]), mx1 = fmaxf(x[0][1], x[0][3]);
#pragma unroll
  for (int j = 1; j < NT; ++j) {
    mx0 = fmaxf(mx0, fmaxf(x[j][0], x[j][2]));
    mx1 = fmaxf(mx1, fmaxf(x[j][1], x[j][3]));
  }
#pragma unroll
  for (int o_ = 4; o_ < 32; o_ <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o_));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o_));
  }
  const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
  const float b0 = mn0 == kNegInf ? 0.f : mn0, b1 = mn1 == kNegInf ? 0.f : mn1;
  const float al0 = ex2(m0 - b0), al1 = ex2(m1 - b1);
  l0 *= al0;
  l1 *= al1;
  uint32_t pb[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const float p0 = ex2(x[j][0] - b0), p1 = ex2(x[j][1] - b1), p2 = ex2(x[j][2] - b0), p3 = ex2(x[j][3] - b1);
    l0 += p0 + p2;
    l1 += p1 + p3;
    pb[j][0] = movmatrix_t(pack2<T>(p0, p1));
    pb[j][1] = movmatrix_t(pack2<T>(p2, p3));
  }
  m0 = mn0;
  m1 = mn1;
#pragma unroll
  for (int i = 0; i < KS; ++i) {
    o[i][0] *= al0;
    o[i][1] *= al1;
    o[i][2] *= al0;
    o[i][3] *= al1;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vb[j] + tma_off(vr, 2 * i + vc), a0, a1, a2, a3);
      mma16816<T>(o[i], a0, a1, a2, a3, pb[j][0], pb[j][1]);
    }
  }
}

template <typename T, int D_>
__device__ void tma_consumer(const AttnParams& p, unsigned char* base, int box_bytes) {
  constexpr int KS = D_ / 16;
  constexpr int NDH = D_ / 64;
  constexpr int HB = D_ * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t hdr = smem_u32(base);
  const StepRec* recs = reinterpret_cast<const StepRec*>(base + 128);
  const uint32_t stage0 = hdr + kTmaHeader;
  const int S = p.stages;
  const int n0 = 2 * (lane & 3), tq = lane >> 2;
  const bool has = tq < p.G;
  const int head_region = warp * NDH * 2048;
  uint32_t qf[KS][2];
  float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;
  float o[KS][4];
  int s = 0;        // slot of the next step
  uint32_t ph = 0;  // parity of its full barrier
  auto advance = [&]() {
    if (++s == S) {
      s = 0;
      ph ^= 1;
    }
  };
  for (;;) {
    if (!mbar_wait(hdr + 8 * s, ph, p.status)) return;
    const StepRec r = recs[s];
    if (r.u < 0) return;  // no more work
    // head_dim 64: take the unit's next step too when it has one (32 keys
    // per update); head_dim 128 has the instruction-level parallelism of
    // 8 k-steps per tile and too few stages per CTA to hold two
    const int s0 = s;
    advance();
    const bool pair = D_ == 64 && !r.last;
    int s1 = s0;
    bool last = r.last;
    if (pair) {
      if (!mbar_wait(hdr + 8 * s, ph, p.status)) return;
      s1 = s;
      last = recs[s1].last;
      advance();
    }
    const uint32_t sb0 = stage0 + s0 * p.stage_bytes, sb1 = stage0 + s1 * p.stage_bytes;
    const uint32_t kb[2] = {sb0 + head_region, sb1 + head_region};
    const uint32_t vb[2] = {sb0 + box_bytes + head_region, sb1 + box_bytes + head_region};
    if (r.first) {
      const uint32_t qs = sb0 + 2 * box_bytes + (warp * p.G + tq) * HB + n0 * 2;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qf[ks][0] = has ? lds32(qs + ks * 32) : 0u;
        qf[ks][1] = has ? lds32(qs + ks * 32 + 16) : 0u;
      }
      m0 = m1 = kNegInf;
      l0 = l1 = 0.f;
#pragma unroll
      for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    }
    const int nv = min(pair ? 32 : 16, r.t1 - r.t);
    const int nvl = nv - (pair ? 16 : 0);  // valid rows of the last tile
    if (nvl < 16) {
      // rows past the unit's end hold whatever the block holds: zero them in V
      // (their scores are masked, but 0 * NaN would still poison the sum)
      const uint32_t vl = pair ? vb[1] : vb[0];
      for (int idx = lane; idx < (16 - nvl) * NDH * 8; idx += 32) {
        const int row = nvl + idx / (NDH * 8), rest = idx % (NDH * 8);
        const uint32_t a = vl + (rest >> 3) * 2048 + row * 128 + (rest & 7) * 16;
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0) : "memory");
      }
      __syncwarp();
    }
    if (pair)
      consume_tiles<T, D_, 2>(p, kb, vb, nv, qf, o, m0, m1, l0, l1);
    else
      consume_tiles<T, D_, 1>(p, kb, vb, nv, qf, o, m0, m1, l0, l1);
    // release the slots (the tail zeroing wrote with the generic proxy: order
    // it before the next tensor copy into the slot)
    if (nvl < 16) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(hdr + 64 + 8 * s0);
      if (pair) mbar_arrive(hdr + 64 + 8 * s1);
    }
    if (last) {
#pragma unroll
      for (int o_ = 4; o_ < 32; o_ <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o_);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o_);
      }
      Work c;
      c.w = 0;
      c.u = r.u;
      c.item = r.item;
      c.slot = 0;
      c.q_row = r.q_row;
      c.t0 = r.t0;
      c.t1 = r.t1;
      c.unit_base = r.unit_base;
      c.nparts = rec_parts(r.nsplits);
      c.kvh = r.hg * p.HG + warp;
      c.part = r.part;
      const int units = rec_units(r.nsplits);
      // output staging of this warp (a gathered output: 16-byte stores to the peers)
      const uint32_t stage = p.stage_out ? hdr + p.stage_out + warp * p.G * D_ * 2 : 0u;
      if (c.nparts == 1) {
        if (stage)
          mma_store_output_staged<T, D_>(p, c, o, l0, l1, stage);
        else
          mma_store_output<T, D_>(p, c, o, l0, l1);
      } else {
        // the part record (merged at the end of the launch), also for the
        // item's only unit beside its cascade parts, which merges those now:
        // a launch that also has items of several units merges every item
        // with several parts at its end (stalling a consumer warp to merge
        // many parts here would hold up its CTA's stream)
        mma_store_part<T, D_>(p, c, o, m0, m1, l0, l1);
        if (units == 1) mma_merge_parts<T, D_>(p, c, o, m0, m1, l0, l1, stage);
      }
    }
  }
}

// ONE_HEAD: the build for CTAs of one KV head (a pool sharded down to one
// KV head per GPU): 64 threads and registers capped so that the eight CTAs
// per SM the launch sizes its shared memory for are resident at once.
template <typename T, int D_, bool ONE_HEAD = false>
__global__ void __launch_bounds__(ONE_HEAD ? 64 : kTmaMaxThreads, ONE_HEAD ? 8 : 1) paged_attention_tma_kernel(const AttnParams p,
                                                                  const __grid_constant__ CUtensorMap tk,
                                                                  const __grid_constant__ CUtensorMap tv) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ int cta_done;
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int box_bytes = p.HG * 16 * D_ * 2;
  const int q_bytes = p.HG * p.G * D_ * 2;
  // the launch after this one (the next layer's KV append) may start as this
  // grid's CTAs leave; it waits for this grid before it reads or writes anything
  pdl_launch_dependents();
  if (threadIdx.x == 32 * p.HG) {  // the producer
    tma_prefetch_map(&tk);
    tma_prefetch_map(&tv);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(smem_u32(base) + 8 * s, 1);
      mbar_init(smem_u32(base) + 64 + 8 * s, p.HG);
    }
    fence_mbar_init();
    cta_done = 0;
  }
  __syncthreads();
  const int n_units = launch_units(p);
  const int total = n_units * p.n_hg;
  if (warp < p.HG) {
    tma_consumer<T, D_>(p, base, box_bytes);
  } else if ((threadIdx.x & 31) == 0) {
    cta_done = tma_producer<T, D_>(p, &tk, &tv, base, total, box_bytes, q_bytes);
  }
  finish_launch<T, 8>(p, &cta_done, total, 2);  // items of one unit merge in its epilogue
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

static bool encode_pool_map_uncached(CUtensorMap* map, const void* pool, int dtype, int D, int Hkv, int bs,
                                     int num_blocks, int hg, bool permuted);

// Pool maps depend only on the pool's address and shape: the last ones
// encoded are kept (a step reuses every layer's maps), so a launch encodes
// none in the steady state.  Keyed by everything the map encodes.
bool encode_pool_map(CUtensorMap* map, const void* pool, int dtype, int D, int Hkv, int bs, int num_blocks, int hg,
                     bool permuted) {
  struct Entry {
    const void* pool;
    int dtype, D, Hkv, bs, num_blocks, hg, permuted;
    bool ok;
    CUtensorMap map;
  };
  static Entry table[96];
  static int n = 0, next = 0;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n; ++i) {
      const Entry& t = table[i];
      if (t.pool == pool && t.dtype == dtype && t.D == D && t.Hkv == Hkv && t.bs == bs && t.num_blocks == num_blocks &&
          t.hg == hg && t.permuted == (int)permuted) {
        *map = t.map;
        return t.ok;
      }
    }
  }
  const bool ok = encode_pool_map_uncached(map, pool, dtype, D, Hkv, bs, num_blocks, hg, permuted);
  std::lock_guard<std::mutex> lock(mu);
  Entry& t = table[next];
  t = Entry{pool, dtype, D, Hkv, bs, num_blocks, hg, (int)permuted, ok, *map};
  next = (next + 1) % 96;
  if (n < 96) ++n;
  return ok;
}

static bool encode_pool_map_uncached(CUtensorMap* map, const void* pool, int dtype, int D, int Hkv, int bs,
                                     int num_blocks, int hg, bool permuted) {
  auto fn = encode_fn();
  if (!fn) return false;
  const CUtensorMapDataType dt = dtype == NF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t row = (cuuint64_t)Hkv * D * 2, head = (cuuint64_t)D * 2, blk = (cuuint64_t)bs * row;
  cuuint64_t dims[5], strides[4];
  cuuint32_t box[5], es[5] = {1, 1, 1, 1, 1};
  cuuint32_t rank;
  if (D == 64) {
    rank = 4;
    if (permuted) {
      cuuint64_t d[4] = {64, (cuuint64_t)bs, (cuuint64_t)Hkv, (cuuint64_t)num_blocks};
      cuuint64_t st[3] = {row, head, blk};
      cuuint32_t b[4] = {64, 16, (cuuint32_t)hg, 1};
      for (int i = 0; i < 4; ++i) { dims[i] = d[i]; box[i] = b[i]; }
      for (int i = 0; i < 3; ++i) strides[i] = st[i];
    } else {
      cuuint64_t d[4] = {64, (cuuint64_t)Hkv, (cuuint64_t)bs, (cuuint64_t)num_blocks};
      cuuint64_t st[3] = {head, row, blk};
      cuuint32_t b[4] = {64, 1, 16, 1};
      for (int i = 0; i < 4; ++i) { dims[i] = d[i]; box[i] = b[i]; }
      for (int i = 0; i < 3; ++i) strides[i] = st[i];
    }
  } else {
    rank = 5;
    if (permuted) {
      cuuint64_t d[5] = {64, (cuuint64_t)bs, 2, (cuuint64_t)Hkv, (cuuint64_t)num_blocks};
      cuuint64_t st[4] = {row, 128, head, blk};
      cuuint32_t b[5] = {64, 16, 2, (cuuint32_t)hg, 1};
      for (int i = 0; i < 5; ++i) { dims[i] = d[i]; box[i] = b[i]; }
      for (int i = 0; i < 4; ++i) strides[i] = st[i];
    } else {
      cuuint64_t d[5] = {64, 2, (cuuint64_t)Hkv, (cuuint64_t)bs, (cuuint64_t)num_blocks};
      cuuint64_t st[4] = {128, head, row, blk};
      cuuint32_t b[5] = {64, 1, 1, 16, 1};
      for (int i = 0; i < 5; ++i) { dims[i] = d[i]; box[i] = b[i]; }
      for (int i = 0; i < 4; ++i) strides[i] = st[i];
    }
  }
  const CUresult r = fn(map, dt, rank, const_cast<void*>(pool), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_matrix_map(CUtensorMap* map, const void* base, int dtype, long long cols, long long rows,
                       long long row_stride, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const CUtensorMapDataType dt = dtype == NF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows}, es[2] = {1, 1};
  const CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_rows_map(CUtensorMap* map, const void* base, int dtype, int D, int H, long long rows, long long row_stride,
                     int g, int tt) {
  auto fn = encode_fn();
  if (!fn) return false;
  const CUtensorMapDataType dt = dtype == NF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4], es[4] = {1, 1, 1, 1};
  cuuint32_t rank;
  if (D == 64) {
    rank = 3;
    cuuint64_t d[3] = {64, (cuuint64_t)H, (cuuint64_t)rows};
    cuuint64_t st[2] = {(cuuint64_t)D * 2, (cuuint64_t)row_stride * 2};
    cuuint32_t b[3] = {64, (cuuint32_t)g, (cuuint32_t)tt};
    for (int i = 0; i < 3; ++i) { dims[i] = d[i]; box[i] = b[i]; }
    for (int i = 0; i < 2; ++i) strides[i] = st[i];
  } else {
    rank = 4;
    cuuint64_t d[4] = {64, 2, (cuuint64_t)H, (cuuint64_t)rows};
    cuuint64_t st[3] = {128, (cuuint64_t)D * 2, (cuuint64_t)row_stride * 2};
    cuuint32_t b[4] = {64, 1, (cuuint32_t)g, (cuuint32_t)tt};
    for (int i = 0; i < 4; ++i) { dims[i] = d[i]; box[i] = b[i]; }
    for (int i = 0; i < 3; ++i) strides[i] = st[i];
  }
  const CUresult r = fn(map, dt, rank, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Launches the tensor-map kernel.  Returns NF_EUNSUPPORTED (nothing launched)
// when the shape or the driver rules it out; the caller then uses the
// per-warp cp.async kernel.
int launch_attention_tma(AttnParams p, int dtype, long long want, cudaStream_t st, int* path) {
  if (dtype != NF_BF16 && dtype != NF_F16) return NF_EUNSUPPORTED;
  if ((p.D != 64 && p.D != 128) || p.bs % 16 != 0 || !p.q_smem || p.G > 8) return NF_EUNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(p.kp) | reinterpret_cast<uintptr_t>(p.vp)) & 15) return NF_EUNSUPPORTED;
  // head_dim 64: one CTA per SM with up to 8 KV heads and 6 stages of 36 KB;
  // head_dim 128: two CTAs per SM with up to 4 KV heads and 3 stages of 36 KB
  // each.  Either way about four stages (128 KB) per SM are in flight while
  // the consumers hold the ones they compute on, and 8 consumer warps share
  // the SM.  With fewer KV heads (a shard of the heads on each of several
  // GPUs) the CTAs get smaller and more of them share an SM, so that 8
  // consumer warps still stream per SM.
  const int max_hg = p.D == 64 ? 8 : 4;
  int hg = 0;
  for (int h = p.Hkv < max_hg ? p.Hkv : max_hg; h >= 1; --h)
    if (p.Hkv % h == 0) {
      hg = h;
      break;
    }
  const int ctas = (p.D == 64 ? 1 : 2) * (max_hg / hg);
  const int HB = p.D * 2;
  const int box = hg * 16 * HB, qb = hg * p.G * HB;
  const int stage = ((2 * box + qb + 1023) / 1024) * 1024;
  // a gathered output whose rows (here and on every peer) allow 16-byte
  // stores: each consumer warp stages its G x D output block in shared
  // memory and stores it in 16-byte pieces
  bool al16 = p.n_peers > 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 && (p.out_stride * 2) % 16 == 0;
  for (int r = 0; r < p.n_peers; ++r) al16 = al16 && (reinterpret_cast<uintptr_t>(p.peer_out[r]) & 15) == 0;
  const int stage_out = al16 ? (hg * p.G * p.D * 2 + 127) / 128 * 128 : 0;
  // per CTA: 1 KB reserved by the system, the header, 1 KB of alignment slack,
  // the static shared memory of finish_launch and the output staging
  const int budget = 228 * 1024 / ctas - 1024 - kTmaHeader - 1024 - 256 - stage_out;
  int stages = budget / stage;
  if (stages > kTmaMaxStages) stages = kTmaMaxStages;
  if (stages < 2) return NF_EUNSUPPORTED;
  CUtensorMap tk, tv;
  bool permuted = encode_pool_map(&tk, p.kp, dtype, p.D, p.Hkv, p.bs, p.num_blocks, hg, true) &&
                  encode_pool_map(&tv, p.vp, dtype, p.D, p.Hkv, p.bs, p.num_blocks, hg, true);
  if (!permuted && !(encode_pool_map(&tk, p.kp, dtype, p.D, p.Hkv, p.bs, p.num_blocks, hg, false) &&
                     encode_pool_map(&tv, p.vp, dtype, p.D, p.Hkv, p.bs, p.num_blocks, hg, false)))
    return NF_EUNSUPPORTED;
  p.HG = hg;
  p.n_hg = p.Hkv / hg;
  p.stages = stages;
  p.stage_bytes = stage;
  p.swz = permuted ? 1 : 0;  // reused as "one box covers all heads of the group"
  p.W = hg;
  p.stage_out = stage_out ? kTmaHeader + stages * stage : 0;
  const int smem = kTmaHeader + stages * stage + stage_out + 1024;  // + alignment slack
  auto kern = (dtype == NF_BF16) ? (p.D == 64 ? paged_attention_tma_kernel<__nv_bfloat16, 64>
                                              : paged_attention_tma_kernel<__nv_bfloat16, 128>)
                                 : (p.D == 64 ? paged_attention_tma_kernel<__half, 64>
                                              : paged_attention_tma_kernel<__half, 128>);
  if (hg == 1)
    kern = (dtype == NF_BF16) ? (p.D == 64 ? paged_attention_tma_kernel<__nv_bfloat16, 64, true>
                                           : paged_attention_tma_kernel<__nv_bfloat16, 128, true>)
                              : (p.D == 64 ? paged_attention_tma_kernel<__half, 64, true>
                                           : paged_attention_tma_kernel<__half, 128, true>);
  int per_sm = 1;
  const int threads = (hg + 1) * 32;
  cudaError_t e = prepare_launch(reinterpret_cast<const void*>(kern), smem, threads, &per_sm);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_paged_attention: smem attribute: %s", cudaGetErrorString(e));
  long long grid = (long long)sm_count() * per_sm;
  const long long need = (want + p.Hkv - 1) / p.Hkv * p.n_hg;  // work items: units x head groups
  if (need < grid) grid = need;
  if (grid < 1) grid = 1;
  // cooperative: the end-of-launch merge waits for every CTA
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  // programmatic stream serialization: the launch overlaps the kernel before
  // it (the KV append), whose writes the kernel waits for in pdl_wait()
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.pdl ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, kern, p, tk, tv);
  if (e != cudaSuccess) {  // not available with this launch: plain stream order
    (void)cudaGetLastError();
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p, tk, tv);
  }
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_paged_attention: launch: %s", cudaGetErrorString(e));
  *path = permuted ? 1 : 2;
  return check_launch("nf_paged_attention");
}

}  // namespace nf
