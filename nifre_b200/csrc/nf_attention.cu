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
// Work.  nf_pack_step emits one item per query token and cuts its keys into
// units of at most `split` keys, each described by one 32-byte record.  A
// work item of this kernel is (unit, KV head).  Every warp is an independent
// worker: it takes the next work item from a queue (one atomic in the
// caller's workspace), so fast warps simply take more items and the grid
// finishes together whatever the mix of context lengths.  The next item is
// requested two tiles before the current one's loads end and its record is
// prefetched, so taking work costs no stall.
//
// Staging.  Every warp runs its own pipeline: a ring of `stages` shared-memory
// slots, each holding the K rows and V rows (one head, head_dim elements each)
// of one tile of keys, filled with 16-byte cp.async copies.  A key tile is a
// gather: with 16-token blocks its rows come from blocks scattered over the
// pool and one head's row is only head_dim*2 bytes, so many small independent
// copies keep HBM busy where a few large copies issued by one thread cannot.
// The load cursor runs stages-1 tiles ahead of the compute cursor and crosses
// unit boundaries; unit records travel from the loader to the compute side
// through a small per-warp FIFO in shared memory.  Rows are XOR-swizzled in
// 16-byte chunks (chunk c of row r at c ^ (r & 7)) so the ldmatrix fragment
// loads are free of bank conflicts.  No warp ever waits on another warp: the
// only waits are cp.async.wait_group on the warp's own copies.
//
// Compute.  For 16-bit pools the scores S^T = K Q^T (keys x 8 query heads of
// the group) and the output O^T += V^T P^T (head_dim x 8) are mma.sync
// m16n8k16 tiles: a GQA group of up to 8 query heads shares one K/V read.
// Probabilities go from the S^T accumulator layout to the B-operand layout
// with movmatrix transposes.  Float32 pools use CUDA-core FMAs (the
// reference's float32 model keeps full precision).
//
// Split-K merge.  A unit whose item has more than one part writes (acc, m, l)
// to the caller's workspace; the last warp to finish an (item, KV head) --
// counted with one atomic -- merges all parts and writes the output.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <mutex>

#include "nf_attn_common.cuh"
#include "nf_internal.h"

namespace nf {

constexpr int kFifo = 8;        // unit records in flight between loader and compute
constexpr int kFifoInts = 16;   // ints per record
constexpr int kFifoBytes = kFifo * kFifoInts * 4;

// ---------------------------------------------------------------- load cursor
struct Loader {
  Work c;          // work item being loaded (c.w < 0: exhausted)
  int t;           // first key of the next tile to load
  int lb, off;     // its logical block and offset in that block
  int total;       // number of work items
  int pending;     // lane 0: queue ticket requested, not yet read
  int nstate;      // 0: next not requested yet, 1: ticket pending, 2: next record fetched
  int nw;          // next work item
  int4 na, nb;     // its unit record
  int fifo_w;      // FIFO write index
};

__device__ __forceinline__ void request_next(const AttnParams& p, Loader& L) {
  if ((threadIdx.x & 31) == 0) L.pending = atomicAdd(p.queue, 1);
  L.nstate = 1;
}

// Turn the pending ticket into the next item and start fetching its record.
__device__ __forceinline__ void resolve_next(const AttnParams& p, Loader& L) {
  L.nw = __shfl_sync(0xffffffffu, L.pending, 0);
  if (L.nw < L.total) {
    const int4* rec = reinterpret_cast<const int4*>(p.units) + 2 * (L.nw / p.Hkv);
    L.na = __ldg(rec);
    L.nb = __ldg(rec + 1);
  }
  L.nstate = 2;
}

__device__ __forceinline__ void fifo_push(unsigned char* fifo, Loader& L) {
  if ((threadIdx.x & 31) == 0) {
    int* e = reinterpret_cast<int*>(fifo) + (L.fifo_w % kFifo) * kFifoInts;
    const Work& c = L.c;
    e[0] = c.w; e[1] = c.u; e[2] = c.item; e[3] = c.slot; e[4] = c.q_row;
    e[5] = c.t0; e[6] = c.t1; e[7] = c.unit_base; e[8] = c.nparts; e[9] = c.kvh; e[10] = c.part;
  }
  ++L.fifo_w;
  __syncwarp();
}

// Make the prefetched item current (or mark the loader exhausted) and queue
// its record for the compute side.
__device__ __forceinline__ void loader_enter(const AttnParams& p, Loader& L, unsigned char* fifo) {
  if (L.nstate == 1) resolve_next(p, L);
  if (L.nw >= L.total) {
    L.c.w = -1;
    fifo_push(fifo, L);
    return;
  }
  Work& c = L.c;
  c.w = L.nw;
  c.u = L.nw / p.Hkv;
  c.kvh = L.nw - c.u * p.Hkv;
  c.item = L.na.x;
  c.slot = L.na.y;
  c.q_row = L.na.z;
  c.part = L.na.w;
  c.t0 = L.nb.x;
  c.t1 = L.nb.y;
  c.unit_base = L.nb.z;
  c.nparts = rec_parts(L.nb.w);
  L.t = c.t0;
  L.lb = c.t0 / p.bs;
  L.off = c.t0 - L.lb * p.bs;
  // pull the unit's block-table entries into L1 ahead of the tile loads
  {
    const int* btrow = p.bt + (long long)c.slot * p.max_blocks;
    const int lb_end = min((c.t1 - 1) / p.bs, p.max_blocks - 1);
    const int lane = threadIdx.x & 31;
    for (int lbx = L.lb + 32 * lane; lbx <= lb_end; lbx += 32 * 32)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(btrow + lbx));
  }
  fifo_push(fifo, L);
  L.nstate = 0;
  // a one- or two-tile unit needs its successor right away
  if (c.t1 - c.t0 <= 2 * p.tile) request_next(p, L);
}

__device__ __forceinline__ void loader_init(const AttnParams& p, Loader& L, unsigned char* fifo, int total) {
  L.total = total;
  L.fifo_w = 0;
  L.pending = 0;
  request_next(p, L);
  resolve_next(p, L);
  loader_enter(p, L, fifo);
}

// Advance by one tile.  The next work item is requested two tiles before the
// current unit's loads end (late enough that a warp never holds work another
// warp could start, early enough to hide the atomic) and its ticket is read
// one tile later.
__device__ __forceinline__ void loader_next(const AttnParams& p, Loader& L, unsigned char* fifo) {
  L.t += p.tile;
  L.off += p.tile;
  while (L.off >= p.bs) {
    L.off -= p.bs;
    ++L.lb;
  }
  if (L.nstate == 1) resolve_next(p, L);
  if (L.nstate == 0 && L.t + 2 * p.tile >= L.c.t1) request_next(p, L);
  if (L.t >= L.c.t1) loader_enter(p, L, fifo);
}

__device__ __forceinline__ Work fifo_pop(const unsigned char* fifo, int& r) {
  __syncwarp();
  const int* e = reinterpret_cast<const int*>(fifo) + (r % kFifo) * kFifoInts;
  ++r;
  Work c;
  c.w = e[0]; c.u = e[1]; c.item = e[2]; c.slot = e[3]; c.q_row = e[4];
  c.t0 = e[5]; c.t1 = e[6]; c.unit_base = e[7]; c.nparts = e[8]; c.kvh = e[9]; c.part = e[10];
  return c;
}

// With the first tile of a unit, bring the group's query rows along (G rows
// of head_bytes after the K and V tiles of the slot).
template <typename T>
__device__ __forceinline__ void stage_query(const AttnParams& p, const Loader& L, uint32_t slot_base) {
  if (!p.q_smem || L.t != L.c.t0) return;
  const int lane = threadIdx.x & 31;
  const char* qrow = p.q + ((long long)L.c.q_row * p.q_stride + (long long)L.c.kvh * p.G * p.D) * (long long)sizeof(T);
  const uint32_t qs = slot_base + 2 * p.tile * p.head_bytes;
  for (int idx = lane; idx < p.G * (p.head_bytes >> 4); idx += 32) cp_async16(qs + idx * 16, qrow + idx * 16);
}

// Copies of the loader's current tile into ring slot `slot_base`: any block
// size and row length, one block-table read per row.
template <typename T>
__device__ __forceinline__ void issue_tile(const AttnParams& p, const Loader& L, uint32_t slot_base) {
  const int lane = threadIdx.x & 31;
  const int cpr = p.head_bytes >> 4;  // 16-byte chunks per row
  const int* btrow = p.bt + (long long)L.c.slot * p.max_blocks;
  const int last = L.c.t1 - 1 - L.t;  // rows past the end repeat the last key (masked later)
  const size_t head_off = (size_t)L.c.kvh * p.D;
  for (int idx = lane; idx < p.tile * cpr; idx += 32) {
    const int r = idx / cpr, ch = idx - r * cpr;
    int off = L.off + min(r, last), lb = L.lb;
    while (off >= p.bs) {
      off -= p.bs;
      ++lb;
    }
    const int phys = checked_block(p, btrow, lb);
    const size_t row = ((size_t)phys * p.bs + off) * p.Hkv * p.D + head_off;
    const uint32_t dst = slot_base + tile_off(r, ch, p.head_bytes, p.swz);
    cp_async16(dst, reinterpret_cast<const char*>(reinterpret_cast<const T*>(p.kp) + row) + ch * 16);
    cp_async16(dst + p.tile * p.head_bytes, reinterpret_cast<const char*>(reinterpret_cast<const T*>(p.vp) + row) + ch * 16);
  }
  stage_query<T>(p, L, slot_base);
}

// Per-lane constants of the fast tile copy: the lane's 16-byte chunk of a
// row, its first row, and the swizzled destination offsets, which repeat
// every 8/RP rows.
template <int TILE, int HB>
struct LaneCopy {
  static constexpr int CPR = HB / 16;              // 16-byte chunks per row
  static constexpr int LPR = CPR < 32 ? CPR : 32;  // lanes per row
  static constexpr int RP = 32 / LPR;              // rows per pass
  static constexpr int CPL = CPR / LPR;            // chunks per lane per row
  static constexpr int NPAT = RP >= 8 ? 1 : 8 / RP;
  int src;          // byte offset within a pool row run: rg * row_stride + chunk * 16
  int dst[NPAT][CPL];
  __device__ __forceinline__ void init(int row_stride) {
    const int lane = threadIdx.x & 31;
    const int c0 = lane % LPR, rg = lane / LPR;
    src = rg * row_stride + c0 * 16;
#pragma unroll
    for (int q = 0; q < NPAT; ++q)
#pragma unroll
      for (int cc = 0; cc < CPL; ++cc) dst[q][cc] = tile_off(rg + RP * q, c0 + LPR * cc, HB, 1) - (RP * q) * HB;
  }
};

// Same copies with compile-time geometry: TILE keys, HB-byte head rows.  When
// the block size is a multiple of 16 each 16-key half of the tile is one run
// of consecutive pool rows: a full tile costs at most two block-table reads
// (L1 hits, prefetched when the unit was entered) and one add per copy.
template <typename T, int TILE, int HB>
__device__ __forceinline__ void issue_tile_fast(const AttnParams& p, const Loader& L, const LaneCopy<TILE, HB>& lc,
                                                uint32_t slot_base) {
  using LC = LaneCopy<TILE, HB>;
  if (!p.bs16 || L.c.t1 - L.t < TILE) {  // other block sizes and the tail tile of a unit
    issue_tile<T>(p, L, slot_base);
    return;
  }
  const int* btrow = p.bt + (long long)L.c.slot * p.max_blocks;
  const long long rs = (long long)p.Hkv * HB;  // pool row stride, bytes
  const char* kbase[TILE / 16];
  const char* vbase[TILE / 16];
#pragma unroll
  for (int h = 0; h < TILE / 16; ++h) {
    int off = L.off + 16 * h, lb = L.lb;
    if (off >= p.bs) {  // off and bs are multiples of 16: at most one block further
      off -= p.bs;
      ++lb;
    }
    const long long o = ((long long)checked_block(p, btrow, lb) * p.bs + off) * rs + (long long)L.c.kvh * HB + lc.src;
    kbase[h] = p.kp + o;
    vbase[h] = p.vp + o;
  }
#pragma unroll
  for (int j = 0; j < TILE / LC::RP; ++j) {
    const int r0 = LC::RP * j;  // first row of this pass (compile time)
    const int h = r0 >> 4;
    const int rrow = (r0 & 15) * (int)rs;
#pragma unroll
    for (int cc = 0; cc < LC::CPL; ++cc) {
      const uint32_t dst = slot_base + lc.dst[j % LC::NPAT][cc] + r0 * HB;
      cp_async16(dst, kbase[h] + rrow + LC::LPR * cc * 16);
      cp_async16(dst + TILE * HB, vbase[h] + rrow + LC::LPR * cc * 16);
    }
  }
  stage_query<T>(p, L, slot_base);
}

// ---------------------------------------------------------------- 16-bit pools: tensor-core tiles
// D_: head dim (64 or 128).  MT: 16-key m-tiles per warp tile (TILE = 16*MT keys).
// Both warp loops return the number of work items the warp finished.
template <typename T, int D_, int MT>
__device__ int warp_mma(const AttnParams& p, uint32_t ring, unsigned char* fifo, int total) {
  constexpr int KS = D_ / 16;  // k-steps of S^T and m-tiles of O^T
  constexpr int HB = D_ * 2;   // bytes of one head row
  constexpr int TILE = 16 * MT;
  const int lane = threadIdx.x & 31;
  const int n0 = 2 * (lane & 3);  // query heads of this lane's accumulator columns
  const int tq = lane >> 2;       // key row / d row of this lane in a fragment
  const bool has = tq < p.G;      // lane's B-operand column is a real query head
  const int S = p.stages;
  LaneCopy<TILE, HB> lc;
  lc.init(p.Hkv * HB);
  Loader L;
  loader_init(p, L, fifo, total);
  for (int s = 0; s < S - 1; ++s) {
    if (L.c.w >= 0) {
      issue_tile_fast<T, TILE, HB>(p, L, lc, ring + s * p.stage_bytes);
      loader_next(p, L, fifo);
    }
    cp_async_commit();
  }
  // fragment addressing (rows this lane supplies to ldmatrix, before the swizzle)
  const int kr = (lane & 7) + ((lane >> 3) & 1) * 8, kc = lane >> 4;        // K: row, chunk parity
  const int vr = (lane & 7) + ((lane >> 4) & 1) * 8, vc = (lane >> 3) & 1;  // V: row, chunk parity
  int k = 0, fr = 0, done = 0;
  while (true) {
    const Work c = fifo_pop(fifo, fr);
    if (c.w < 0) break;
    ++done;
    uint32_t qf[KS][2];
    if (!p.q_smem) {
      const T* qp = reinterpret_cast<const T*>(p.q) + (long long)c.q_row * p.q_stride +
                    (long long)(c.kvh * p.G + tq) * D_ + n0;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qf[ks][0] = has ? __ldg(reinterpret_cast<const uint32_t*>(qp + ks * 16)) : 0u;
        qf[ks][1] = has ? __ldg(reinterpret_cast<const uint32_t*>(qp + ks * 16 + 8)) : 0u;
      }
    }
    float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;
    float o[KS][4];
#pragma unroll
    for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    for (int tb = c.t0; tb < c.t1; tb += TILE, ++k) {
      cp_async_wait(S - 2);
      __syncwarp();
      if (L.c.w >= 0) {
        issue_tile_fast<T, TILE, HB>(p, L, lc, ring + ((k + S - 1) % S) * p.stage_bytes);
        loader_next(p, L, fifo);
      }
      cp_async_commit();
      const uint32_t kb = ring + (k % S) * p.stage_bytes;
      const uint32_t vb = kb + TILE * HB;
      if (p.q_smem && tb == c.t0) {
        // Q^T as the B operand, staged with this unit's first tile: column n = query head tq
        const uint32_t qs = kb + 2 * TILE * HB + tq * HB + n0 * 2;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          qf[ks][0] = has ? lds32(qs + ks * 32) : 0u;
          qf[ks][1] = has ? lds32(qs + ks * 32 + 16) : 0u;
        }
      }
      // S^T = K Q^T : TILE keys x 8 query heads (MT independent accumulator chains)
      float sc[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(kb + tile_off(16 * mt + kr, 2 * ks + kc, HB, 1), a0, a1, a2, a3);
          mma16816<T>(sc[mt], a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
        }
      }
      float x[MT][4];
      float mx0 = kNegInf, mx1 = kNegInf;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const bool v0 = tb + 16 * mt + tq < c.t1, v1 = tb + 16 * mt + tq + 8 < c.t1;
        x[mt][0] = v0 ? sc[mt][0] * p.scale_log2 : kNegInf;
        x[mt][1] = v0 ? sc[mt][1] * p.scale_log2 : kNegInf;
        x[mt][2] = v1 ? sc[mt][2] * p.scale_log2 : kNegInf;
        x[mt][3] = v1 ? sc[mt][3] * p.scale_log2 : kNegInf;
        mx0 = fmaxf(mx0, fmaxf(x[mt][0], x[mt][2]));
        mx1 = fmaxf(mx1, fmaxf(x[mt][1], x[mt][3]));
      }
#pragma unroll
      for (int o_ = 4; o_ < 32; o_ <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o_));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o_));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float b0 = mn0 == kNegInf ? 0.f : mn0, b1 = mn1 == kNegInf ? 0.f : mn1;
      const float al0 = ex2(m0 - b0), al1 = ex2(m1 - b1);
      m0 = mn0;
      m1 = mn1;
      l0 *= al0;
      l1 *= al1;
      uint32_t pb[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const float p0 = ex2(x[mt][0] - b0), p1 = ex2(x[mt][1] - b1);
        const float p2 = ex2(x[mt][2] - b0), p3 = ex2(x[mt][3] - b1);
        l0 += p0 + p2;
        l1 += p1 + p3;
        // P^T (keys x heads) as the B operand: transpose the two 8x8 halves
        pb[mt][0] = movmatrix_t(pack2<T>(p0, p1));
        pb[mt][1] = movmatrix_t(pack2<T>(p2, p3));
      }
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        o[i][0] *= al0;
        o[i][1] *= al1;
        o[i][2] *= al0;
        o[i][3] *= al1;
      }
      // O^T += V^T P^T
#pragma unroll
      for (int i = 0; i < KS; ++i) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(vb + tile_off(16 * mt + vr, 2 * i + vc, HB, 1), a0, a1, a2, a3);
          mma16816<T>(o[i], a0, a1, a2, a3, pb[mt][0], pb[mt][1]);
        }
      }
    }
    // row sums: lanes sharing lane&3 hold the same query heads
#pragma unroll
    for (int o_ = 4; o_ < 32; o_ <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o_);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o_);
    }
    mma_epilogue<T, D_>(p, c, o, m0, m1, l0, l1);
  }
  cp_async_wait(0);
  return done;
}

// ---------------------------------------------------------------- any dtype: CUDA-core path
// Any head_dim <= 32*DPL, up to 8 query heads per KV head; lanes split the
// head dimension.  Same pipeline and queue as the tensor-core path.
// One staged 16-key tile of the CUDA-core path for heads of up to 64
// dimensions (lane l holds dimensions l and l + 32).  Each lane's partial
// dot products for the 16 keys are summed over the warp by a reduce-scatter
// (one butterfly stage over the lane halves, then four halving stages), so
// that lane l ends with the full score of key l % 16 after 31 shuffles for
// the whole tile; the softmax statistics reduce over 16 lanes once per tile
// and the probabilities are broadcast back for O += P V.
template <typename T, int DPL>
__device__ __forceinline__ void simt_tile16(const AttnParams& p, const unsigned char* kb, const unsigned char* vb,
                                            int nv, const float (&qv)[8][DPL], float (&acc)[8][DPL], float (&m)[8],
                                            float (&l)[8]) {
  constexpr int TK = 16;
  const int lane = threadIdx.x & 31;
  const int HB = p.head_bytes;
  float kk[TK][DPL], vv[TK][DPL];
#pragma unroll
  for (int j = 0; j < TK; ++j) {
    const bool live = j < nv;  // rows past the unit hold whatever the block holds: not read
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane + 32 * i;
      const int byte = d * (int)sizeof(T);
      const int off = tile_off(j, byte >> 4, HB, p.swz) + (byte & 15);
      kk[j][i] = live && d < p.D ? Elem<T>::to_f(*reinterpret_cast<const T*>(kb + off)) : 0.f;
      vv[j][i] = live && d < p.D ? Elem<T>::to_f(*reinterpret_cast<const T*>(vb + off)) : 0.f;
    }
  }
  const int key = lane & (TK - 1);
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    if (n < p.G) {
      float s[TK];
#pragma unroll
      for (int j = 0; j < TK; ++j) {
        s[j] = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) s[j] = fmaf(qv[n][i], kk[j][i], s[j]);
      }
#pragma unroll
      for (int j = 0; j < TK; ++j) s[j] += __shfl_xor_sync(0xffffffffu, s[j], 16);
#pragma unroll
      for (int o = TK / 2; o >= 1; o >>= 1) {
        const bool up = lane & o;
#pragma unroll
        for (int j = 0; j < o; ++j) {
          const float send = up ? s[j] : s[j + o];
          const float keep = up ? s[j + o] : s[j];
          s[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      const float sc = key < nv ? s[0] : kNegInf;  // the score of key `key` (scale folded into q)
      float mx = sc;
#pragma unroll
      for (int o = TK / 2; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m[n], mx);  // finite: key 0 of the tile is live
      const float al = ex2(m[n] - mn);
      const float pk = ex2(sc - mn);
      float ps = pk;
#pragma unroll
      for (int o = TK / 2; o >= 1; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[n] = l[n] * al + ps;
      m[n] = mn;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[n][i] *= al;
#pragma unroll
      for (int j = 0; j < TK; ++j) {
        const float pj = __shfl_sync(0xffffffffu, pk, j);
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[n][i] = fmaf(pj, vv[j][i], acc[n][i]);
      }
    }
  }
}

template <typename T, int DPL>
__device__ int warp_simt(const AttnParams& p, uint32_t ring, unsigned char* ring_ptr, unsigned char* fifo,
                         int total) {
  const int lane = threadIdx.x & 31;
  const int S = p.stages;
  const int HB = p.head_bytes;
  Loader L;
  loader_init(p, L, fifo, total);
  for (int s = 0; s < S - 1; ++s) {
    if (L.c.w >= 0) {
      issue_tile<T>(p, L, ring + s * p.stage_bytes);
      loader_next(p, L, fifo);
    }
    cp_async_commit();
  }
  int k = 0, fr = 0, done = 0;
  while (true) {
    const Work c = fifo_pop(fifo, fr);
    if (c.w < 0) break;
    ++done;
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
    for (int tb = c.t0; tb < c.t1; tb += p.tile, ++k) {
      cp_async_wait(S - 2);
      __syncwarp();
      if (L.c.w >= 0) {
        issue_tile<T>(p, L, ring + ((k + S - 1) % S) * p.stage_bytes);
        loader_next(p, L, fifo);
      }
      cp_async_commit();
      const unsigned char* kb = ring_ptr + (k % S) * p.stage_bytes;
      const unsigned char* vb = kb + p.tile * HB;
      const int nv = min(p.tile, c.t1 - tb);
      if constexpr (DPL <= 2) {
        if (p.tile == 16) {  // the tile of this kernel (make_plan)
          simt_tile16<T, DPL>(p, kb, vb, nv, qv, acc, m, l);
          continue;
        }
      }
      // KB keys per softmax update: their dot products reduce across the warp side by side, so the
      // shuffle latency is paid once per KB keys instead of once per key (fewer for wide heads, whose
      // registers hold more of each row)
      constexpr int KB = DPL <= 2 ? 4 : (DPL <= 4 ? 2 : 1);
      for (int j0 = 0; j0 < nv; j0 += KB) {
        float kk[KB][DPL], vv[KB][DPL];
#pragma unroll
        for (int u = 0; u < KB; ++u) {
          const bool live = j0 + u < nv;  // rows past the unit hold whatever the block holds: not read
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            const int byte = d * (int)sizeof(T);
            const int off = tile_off(j0 + u, byte >> 4, HB, p.swz) + (byte & 15);
            kk[u][i] = live && d < p.D ? Elem<T>::to_f(*reinterpret_cast<const T*>(kb + off)) : 0.f;
            vv[u][i] = live && d < p.D ? Elem<T>::to_f(*reinterpret_cast<const T*>(vb + off)) : 0.f;
          }
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          if (n < p.G) {
            float s[KB];
#pragma unroll
            for (int u = 0; u < KB; ++u) {
              s[u] = 0.f;
#pragma unroll
              for (int i = 0; i < DPL; ++i) s[u] = fmaf(qv[n][i], kk[u][i], s[u]);
            }
#pragma unroll
            for (int o_ = 16; o_ > 0; o_ >>= 1) {
#pragma unroll
              for (int u = 0; u < KB; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o_);
            }
            float mn = m[n];
#pragma unroll
            for (int u = 0; u < KB; ++u) {
              if (j0 + u >= nv) s[u] = kNegInf;
              mn = fmaxf(mn, s[u]);  // finite: the first key of the group is live
            }
            const float al = ex2(m[n] - mn);
            float pu[KB], ps = 0.f;
#pragma unroll
            for (int u = 0; u < KB; ++u) {
              pu[u] = ex2(s[u] - mn);
              ps += pu[u];
            }
            l[n] = l[n] * al + ps;
            m[n] = mn;
#pragma unroll
            for (int i = 0; i < DPL; ++i) {
              float a = acc[n][i] * al;
#pragma unroll
              for (int u = 0; u < KB; ++u) a = fmaf(pu[u], vv[u][i], a);
              acc[n][i] = a;
            }
          }
        }
      }
    }
    if (c.nparts == 1) {
      const long long ob = (long long)c.q_row * p.out_stride + (long long)(c.kvh * p.G) * p.D;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        if (n < p.G) {
          const float inv = l[n] > 0.f ? 1.f / l[n] : 0.f;
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            if (d < p.D) store_out<T>(p, ob + n * p.D + d, Elem<T>::from_f(acc[n][i] * inv));
          }
        }
      }
    } else {
      const int DP = p.D + 4;
      float* wb = p.ws + ((long long)part_index(p, c) * p.Hq + c.kvh * p.G) * DP;
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
    }
  }
  cp_async_wait(0);
  return done;
}

// ---------------------------------------------------------------- kernel
template <typename T, int D_, int MT, bool MMA, int DPL>
__global__ void __launch_bounds__(256) paged_attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int cta_done;
  if (threadIdx.x == 0) cta_done = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int n_units = launch_units(p);
  const int total = n_units * p.Hkv;
  unsigned char* ring_ptr = smem + (size_t)warp * p.stages * p.stage_bytes;
  unsigned char* fifo = smem + (size_t)p.W * p.stages * p.stage_bytes + warp * kFifoBytes;
  const uint32_t ring = smem_u32(ring_ptr);
  int done;
  if constexpr (MMA) done = warp_mma<T, D_, MT>(p, ring, fifo, total);
  else done = warp_simt<T, DPL>(p, ring, ring_ptr, fifo, total);
  if ((threadIdx.x & 31) == 0 && done) atomicAdd(&cta_done, done);
  finish_launch<T, 8>(p, &cta_done, total, 1);
}

// ---------------------------------------------------------------- host plan
// Tensor-map staging (nf_attention_tma.cu); NF_EUNSUPPORTED means "use this file's kernel".
int launch_attention_tma(AttnParams p, int dtype, long long want, cudaStream_t st, int* path);

// Largest head count the entry points accept (keeps every size product in int64).
constexpr int kMaxHeads = 1 << 16;

struct Plan {
  int W, stages, head_bytes, stage_bytes, smem, swz, tile;
  bool mma, q_smem;
  int dpl;
};

static int make_plan(int dtype, int Hq, int Hkv, int D, bool q_smem_ok, Plan& pl) {
  const size_t es = dtype_size(dtype);
  if (!es) return fail(NF_EINVAL, "nf_paged_attention: bad dtype %d", dtype);
  if (Hq <= 0 || Hkv <= 0 || D <= 0 || Hq % Hkv != 0)
    return fail(NF_EINVAL, "nf_paged_attention: num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)", Hq, Hkv);
  const int G = Hq / Hkv;
  if (G > 8) return fail(NF_EUNSUPPORTED, "nf_paged_attention: more than 8 query heads per KV head (%d)", G);
  if (D > 256) return fail(NF_EUNSUPPORTED, "nf_paged_attention: head_dim %d > 256", D);
  pl.head_bytes = D * (int)es;
  if (pl.head_bytes % 16) return fail(NF_EUNSUPPORTED, "nf_paged_attention: a head row of %d bytes is not a multiple of 16", pl.head_bytes);
  if (D % 4) return fail(NF_EUNSUPPORTED, "nf_paged_attention: head_dim %d is not a multiple of 4", D);
  pl.mma = (dtype != NF_F32) && (D == 64 || D == 128);
  pl.q_smem = pl.mma && q_smem_ok;
  pl.dpl = D <= 32 ? 1 : D <= 64 ? 2 : D <= 128 ? 4 : 8;
  pl.swz = pl.head_bytes % 128 == 0;
  // warp tiles of about 4 KB of keys: 32 keys of 128-byte rows, else 16
  pl.tile = (pl.mma && D == 64) ? 32 : 16;
  pl.stage_bytes = (2 * pl.tile + (pl.q_smem ? G : 0)) * pl.head_bytes;  // K tile, V tile, query rows
  // Warps per CTA and ring depth: the most warps resident per SM with >= 3
  // slots per warp (each warp keeps two tiles in flight); ties go to fewer,
  // larger CTAs.  Two slots only as a last resort.
  // per CTA: 1 KB the system reserves and up to 256 B of the kernel's static
  // shared memory (finish_launch) besides the dynamic buffer
  const int kSmemSM = 228 * 1024, kSmemCTA = 227 * 1024 - 256, kReserve = 1024 + 256;
  int best = 0;
  pl.W = 0;
  for (int min_st = 3; min_st >= 2 && !pl.W; --min_st) {
    for (int w = 8; w >= 1; w >>= 1) {
      const int per_warp = min_st * pl.stage_bytes + kFifoBytes;
      if (w * per_warp > kSmemCTA) continue;
      int ctas = kSmemSM / (w * per_warp + kReserve);
      if (ctas * w > 64) ctas = 64 / w;
      if (ctas < 1 || ctas * w <= best) continue;
      best = ctas * w;
      pl.W = w;
      int st = ((kSmemSM / ctas - kReserve) / w - kFifoBytes) / pl.stage_bytes;
      if (w * (st * pl.stage_bytes + kFifoBytes) > kSmemCTA) st = (kSmemCTA / w - kFifoBytes) / pl.stage_bytes;
      pl.stages = st > 8 ? 8 : st;
    }
  }
  if (!pl.W) return fail(NF_EUNSUPPORTED, "nf_paged_attention: head rows of %d bytes do not fit the pipeline", pl.head_bytes);
  pl.smem = pl.W * (pl.stages * pl.stage_bytes + kFifoBytes);
  return ok();
}

template <typename T, int D_, int MT, bool MMA, int DPL>
static int launch_attn(const AttnParams& p, const Plan& pl, long long want, cudaStream_t st) {
  auto kern = paged_attention_kernel<T, D_, MT, MMA, DPL>;
  int per_sm = 1;
  cudaError_t e = prepare_launch(reinterpret_cast<const void*>(kern), pl.smem, pl.W * 32, &per_sm);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_paged_attention: smem attribute: %s", cudaGetErrorString(e));
  long long grid = (long long)sm_count() * per_sm;
  const long long need = (want + pl.W - 1) / pl.W;  // no more warps than work items
  if (need < grid) grid = need;
  if (grid < 1) grid = 1;
  // cooperative: the end-of-launch merge waits for every CTA
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(pl.W * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_paged_attention: launch: %s", cudaGetErrorString(e));
  return check_launch("nf_paged_attention");
}

template <typename T>
static int dispatch_attn(const AttnParams& p, const Plan& pl, long long want, cudaStream_t st) {
  if constexpr (!std::is_same<T, float>::value) {
    if (pl.mma && p.D == 64)
      return pl.tile == 32 ? launch_attn<T, 64, 2, true, 2>(p, pl, want, st) : launch_attn<T, 64, 1, true, 2>(p, pl, want, st);
    if (pl.mma && p.D == 128)
      return pl.tile == 32 ? launch_attn<T, 128, 2, true, 4>(p, pl, want, st) : launch_attn<T, 128, 1, true, 4>(p, pl, want, st);
  }
  switch (pl.dpl) {
    case 1: return launch_attn<T, 0, 1, false, 1>(p, pl, want, st);
    case 2: return launch_attn<T, 0, 1, false, 2>(p, pl, want, st);
    case 4: return launch_attn<T, 0, 1, false, 4>(p, pl, want, st);
    default: return launch_attn<T, 0, 1, false, 8>(p, pl, want, st);
  }
}

}  // namespace nf

extern "C" int nf_attention_workspace(int32_t max_units, int32_t max_items, int32_t num_q_heads,
                                      int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                                      int64_t* partial_floats, int64_t* counter_ints) {
  using namespace nf;
  Plan pl;
  int rc = make_plan(dtype, num_q_heads, num_kv_heads, head_dim, true, pl);
  if (rc) return rc;
  if (max_units <= 0 || max_items <= 0 || !partial_floats || !counter_ints)
    return fail(NF_EINVAL, "nf_attention_workspace: bad arguments");
  *partial_floats = (int64_t)max_units * num_q_heads * (head_dim + 4);
  *counter_ints = (int64_t)max_items * num_kv_heads + 4;
  return ok();
}

namespace nf {

// Checks the arguments of nf_paged_attention and fills the launch parameters;
// nothing is launched or queued.  The split-K workspace is checked against
// the step's sizes here, so a caller that supplies its own scratch
// (nf_paged_attention_noalloc) learns of every refusal before it queues work.
static int prepare_attention(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                             const void* k_pool, const void* v_pool, int32_t dtype, int32_t num_q_heads,
                             int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_blocks,
                             const int32_t* block_tables, int32_t max_blocks_per_seq, const int32_t* items,
                             const int32_t* units, const int32_t* counts, int32_t max_items, int32_t max_units,
                             int32_t split_tokens, float scale, float* ws_partials, int64_t ws_partial_floats,
                             int32_t* ws_counters, int64_t ws_counter_ints, int32_t* status, AttnParams& p,
                             Plan& pl) {
  const size_t es = dtype_size(dtype);
  auto al = [](const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
  const bool q_smem_ok = es && al(q, 16) && (q_row_stride * (int64_t)es) % 16 == 0;
  int rc = make_plan(dtype, num_q_heads, num_kv_heads, head_dim, q_smem_ok, pl);
  if (rc) return rc;
  if (!out || !q || !k_pool || !v_pool || !block_tables || !items || !units || !counts || !status)
    return fail(NF_EINVAL, "nf_paged_attention: null pointer argument");
  if (block_size <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0 || max_units <= 0 || max_items <= 0)
    return fail(NF_EINVAL, "nf_paged_attention: sizes must be positive");
  if (split_tokens <= 0 || split_tokens % 16 != 0)
    return fail(NF_EINVAL, "nf_paged_attention: split_tokens (%d) must be a positive multiple of 16", split_tokens);
  if (num_q_heads > kMaxHeads)
    return fail(NF_EUNSUPPORTED, "nf_paged_attention: %d query heads (at most %d)", num_q_heads, kMaxHeads);
  // every factor is bounded (units and items < 2^31, heads <= 2^16, head_dim <= 256): no product overflows
  const int64_t need_p = (int64_t)max_units * num_q_heads * (head_dim + 4);
  const int64_t need_c = (int64_t)max_items * num_kv_heads + 4;
  if (!ws_partials || ws_partial_floats < need_p || !ws_counters || ws_counter_ints < need_c)
    return fail(NF_EINVAL, "nf_paged_attention: workspace too small (need %lld floats, %lld counters)",
                (long long)need_p, (long long)need_c);
  if (!al(k_pool, 16) || !al(v_pool, 16)) return fail(NF_EINVAL, "nf_paged_attention: pools must be 16-byte aligned");
  if (!al(units, 16) || !al(items, 16))
    return fail(NF_EINVAL, "nf_paged_attention: items and units must be 16-byte aligned");
  if (!al(ws_partials, 16)) return fail(NF_EINVAL, "nf_paged_attention: partials must be 16-byte aligned");
  if (pl.mma && (!al(q, 4) || (q_row_stride * (int64_t)es) % 4 != 0))
    return fail(NF_EINVAL, "nf_paged_attention: q rows must be 4-byte aligned");
  p = AttnParams{};
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
  p.units = units;
  p.counts = counts;
  p.max_units = max_units;
  p.split = split_tokens;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.ws = ws_partials;
  p.cnt = ws_counters;
  p.queue = ws_counters + (int64_t)max_items * num_kv_heads;
  p.items = items;
  p.max_items = max_items;
  p.status = status;
  p.W = pl.W;
  p.stages = pl.stages;
  p.head_bytes = pl.head_bytes;
  p.stage_bytes = pl.stage_bytes;
  p.swz = pl.swz;
  p.tile = pl.tile;
  p.bs16 = block_size % 16 == 0;
  p.q_smem = pl.q_smem;
  p.pdl = 1;
  p.own_parts_only = 0;
  const size_t vb = es == 2 ? 8 : 16;  // bytes of four output elements
  p.vec_out = al(out, vb) && (out_row_stride * (int64_t)es) % (int64_t)vb == 0 && head_dim % 4 == 0;
  p.n_peers = 0;
  p.n_ranks = 1;
  p.rank = 0;
  p.epoch = 0;
  p.epoch_counter = nullptr;
  return ok();
}

// Fills the gathered-output fields of p from an NfGather (checked); nothing is launched.
static int apply_gather(AttnParams& p, const NfGather* g, size_t es) {
  if (!g) return ok();
  if (g->n_ranks < 1 || g->n_ranks > kMaxRanks || g->rank < 0 || g->rank >= g->n_ranks)
    return fail(NF_EINVAL, "gathered output: %d ranks (1..%d), rank %d", g->n_ranks, kMaxRanks, g->rank);
  if (g->n_ranks == 1) return ok();
  auto al = [](const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
  const size_t vb = es == 2 ? 8 : 16;
  for (int r = 0; r < g->n_ranks - 1; ++r) {
    if (!g->peer_out[r]) return fail(NF_EINVAL, "gathered output: peer_out[%d] is null", r);
    if (!al(g->peer_out[r], vb)) p.vec_out = 0;
    p.peer_out[r] = static_cast<char*>(g->peer_out[r]);
  }
  for (int r = 0; r < g->n_ranks; ++r) {
    if (!g->flags[r] || !al(g->flags[r], 4)) return fail(NF_EINVAL, "gathered output: flags[%d] is null or unaligned", r);
    p.rank_flags[r] = g->flags[r];
  }
  p.n_peers = g->n_ranks - 1;
  p.n_ranks = g->n_ranks;
  p.rank = g->rank;
  p.epoch = g->epoch;
  p.epoch_counter = g->epoch_counter;
  return ok();
}

static int launch_prepared(const AttnParams& p, const Plan& pl, int dtype, cudaStream_t st) {
  const long long want = (long long)p.max_units * p.Hkv;
  int arc = NF_EUNSUPPORTED;
  if (pl.mma) {
    int path = 0;
    arc = launch_attention_tma(p, dtype, want, st, &path);
    if (arc != NF_EUNSUPPORTED) set_attention_path(path);
  }
  if (arc == NF_EUNSUPPORTED) {
    set_attention_path(0);
    switch (dtype) {
      case NF_F32: arc = dispatch_attn<float>(p, pl, want, st); break;
      case NF_F16: arc = dispatch_attn<__half>(p, pl, want, st); break;
      case NF_BF16: arc = dispatch_attn<__nv_bfloat16>(p, pl, want, st); break;
      default: return fail(NF_EINVAL, "nf_paged_attention: bad dtype %d", dtype);
    }
  }
  return arc;
}

}  // namespace nf

extern "C" int nf_paged_attention(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                  const void* k_pool, const void* v_pool, int32_t dtype, int32_t num_q_heads,
                                  int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                  const int32_t* block_tables, int32_t max_blocks_per_seq, const int32_t* items,
                                  const int32_t* units, const int32_t* counts, int32_t max_items, int32_t max_units,
                                  int32_t split_tokens, float scale, float* ws_partials, int64_t ws_partial_floats,
                                  int32_t* ws_counters, int64_t ws_counter_ints, int32_t* status, void* stream) {
  using namespace nf;
  AttnParams p;
  Plan pl;
  const int rc = prepare_attention(out, out_row_stride, q, q_row_stride, k_pool, v_pool, dtype, num_q_heads,
                                   num_kv_heads, head_dim, block_size, num_blocks, block_tables, max_blocks_per_seq,
                                   items, units, counts, max_items, max_units, split_tokens, scale, ws_partials,
                                   ws_partial_floats, ws_counters, ws_counter_ints, status, p, pl);
  if (rc) return rc;
  return launch_prepared(p, pl, dtype, static_cast<cudaStream_t>(stream));
}

extern "C" int nf_paged_attention_gather(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                         const void* k_pool, const void* v_pool, int32_t dtype, int32_t num_q_heads,
                                         int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                         int32_t num_blocks, const int32_t* block_tables, int32_t max_blocks_per_seq,
                                         const int32_t* items, const int32_t* units, const int32_t* counts,
                                         int32_t max_items, int32_t max_units, int32_t split_tokens, float scale,
                                         float* ws_partials, int64_t ws_partial_floats, int32_t* ws_counters,
                                         int64_t ws_counter_ints, const NfGather* gather, int32_t* status,
                                         void* stream) {
  using namespace nf;
  AttnParams p;
  Plan pl;
  int rc = prepare_attention(out, out_row_stride, q, q_row_stride, k_pool, v_pool, dtype, num_q_heads, num_kv_heads,
                             head_dim, block_size, num_blocks, block_tables, max_blocks_per_seq, items, units, counts,
                             max_items, max_units, split_tokens, scale, ws_partials, ws_partial_floats, ws_counters,
                             ws_counter_ints, status, p, pl);
  if (rc) return rc;
  rc = apply_gather(p, gather, dtype_size(dtype));
  if (rc) return rc;
  return launch_prepared(p, pl, dtype, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- allocation-free variant
// Scratch for nf_paged_attention_noalloc: split-K partials followed by the
// part counters and the work queue.  It lives in this library's image, so
// every GPU that loads the library keeps these bytes until the process ends.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NF_NOALLOC_SCRATCH_BYTES];

namespace nf {
// Device address of g_noalloc_scratch in each CUDA context, looked up on the
// first call made with that context current (host code cannot use the symbol
// itself: on the host it names a stand-in, not device memory).  Keyed by the
// context rather than the device, so a caller that runs in a context of its
// own (not the device's primary context), or one created after a device
// reset, gets the address of its own module's copy.
struct ScratchAddr {
  CUcontext ctx;
  void* ptr;
};
static ScratchAddr g_noalloc_addr[64];
static int g_noalloc_n = 0;
static std::mutex g_noalloc_mu;

static PFN_cuCtxGetCurrent_v4000 ctx_get_fn() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 4000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
  }
  return fn;
}

// The scratch address in the current context (set up on first use).
static int noalloc_scratch(unsigned char** out) {
  // make sure a context is current (the runtime creates the primary one on first use)
  cudaError_t e = cudaFree(nullptr);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_paged_attention_noalloc: no CUDA context: %s", cudaGetErrorString(e));
  auto get_ctx = ctx_get_fn();
  CUcontext ctx = nullptr;
  if (!get_ctx || get_ctx(&ctx) != CUDA_SUCCESS || !ctx)
    return fail(NF_ECUDA, "nf_paged_attention_noalloc: cannot identify the current CUDA context");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  for (int i = 0; i < g_noalloc_n; ++i)
    if (g_noalloc_addr[i].ctx == ctx) {
      *out = static_cast<unsigned char*>(g_noalloc_addr[i].ptr);
      return ok();
    }
  void* ptr = nullptr;
  e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess || !ptr)
    return fail(NF_ECUDA, "nf_paged_attention_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  if (g_noalloc_n < 64) g_noalloc_addr[g_noalloc_n++] = ScratchAddr{ctx, ptr};
  *out = static_cast<unsigned char*>(ptr);
  return ok();
}
}  // namespace nf

extern "C" int nf_paged_attention_noalloc(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                          const void* k_pool, const void* v_pool, int32_t dtype,
                                          int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                          int32_t block_size, int32_t num_blocks, const int32_t* block_tables,
                                          int32_t max_blocks_per_seq, const int32_t* items, const int32_t* units,
                                          const int32_t* counts, int32_t max_items, int32_t max_units,
                                          int32_t split_tokens, float scale, int32_t* status, void* stream) {
  using namespace nf;
  if (max_units <= 0 || max_items <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return fail(NF_EINVAL, "nf_paged_attention_noalloc: sizes must be positive");
  if (num_q_heads > kMaxHeads || num_kv_heads > num_q_heads || head_dim > 256)
    return fail(NF_EINVAL, "nf_paged_attention_noalloc: head counts or head_dim out of range");
  // each factor is bounded above, so no product overflows; each part is checked against the buffer on its own
  const int64_t cap = (int64_t)NF_NOALLOC_SCRATCH_BYTES;
  const int64_t part_floats = (int64_t)max_units * num_q_heads * (head_dim + 4);
  const int64_t cnt_ints = (int64_t)max_items * num_kv_heads + 4;
  const int64_t part_bytes = ((part_floats * 4 + 255) / 256) * 256;
  if (part_bytes > cap || cnt_ints * 4 > cap || part_bytes + cnt_ints * 4 > cap)
    return fail(NF_EINVAL,
                "nf_paged_attention_noalloc: this step needs %lld bytes of scratch, the built-in buffer holds %lld "
                "(use nf_paged_attention with a caller-owned workspace, or a larger split_tokens)",
                (long long)(part_bytes + cnt_ints * 4), (long long)cap);
  unsigned char* base = nullptr;
  int rc = noalloc_scratch(&base);
  if (rc) return rc;
  float* partials = reinterpret_cast<float*>(base);
  int32_t* counters = reinterpret_cast<int32_t*>(base + part_bytes);
  AttnParams p;
  Plan pl;
  rc = prepare_attention(out, out_row_stride, q, q_row_stride, k_pool, v_pool, dtype, num_q_heads, num_kv_heads,
                         head_dim, block_size, num_blocks, block_tables, max_blocks_per_seq, items, units, counts,
                         max_items, max_units, split_tokens, scale, partials, part_floats, counters, cnt_ints, status,
                         p, pl);
  if (rc) return rc;  // refused before anything is queued
  // The buffer is shared by every call and keeps the last call's contents:
  // the counters and the work queue must start at zero (the partials need no
  // clearing).  The launch then goes in plain stream order behind the clear,
  // and refuses plans with cascade parts, whose slots this buffer never holds.
  p.pdl = 0;
  p.own_parts_only = 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(counters, 0, cnt_ints * 4, st);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_paged_attention_noalloc: clearing counters: %s", cudaGetErrorString(e));
  return launch_prepared(p, pl, dtype, st);
}

extern "C" int nf_noalloc_scratch_fill(int32_t byte, void* stream) {
  using namespace nf;
  unsigned char* base = nullptr;
  const int rc = noalloc_scratch(&base);
  if (rc) return rc;
  const cudaError_t e = cudaMemsetAsync(base, byte & 0xff, NF_NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_noalloc_scratch_fill: %s", cudaGetErrorString(e));
  return ok();
}

extern "C" int nf_paged_attention_args(const NfAttentionArgs* a, void* stream) {
  if (!a) return nf::fail(NF_EINVAL, "nf_paged_attention_args: null argument struct");
  return nf_paged_attention_gather(a->out, a->out_row_stride, a->q, a->q_row_stride, a->k_pool, a->v_pool, a->dtype,
                                   a->num_q_heads, a->num_kv_heads, a->head_dim, a->block_size, a->num_blocks,
                                   a->block_tables, a->max_blocks_per_seq, a->items, a->units, a->counts,
                                   a->max_items, a->max_units, a->split_tokens, a->scale, a->ws_partials,
                                   a->ws_partial_floats, a->ws_counters, a->ws_counter_ints, a->gather, a->status,
                                   stream);
}
