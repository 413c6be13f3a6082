// Chunked-prefill attention on fifth-generation tensor cores (tcgen05/TMEM).
//
// The reference computes a prefill chunk per row as get -> cat -> q @ k^T ->
// causal mask (query i at position past + i sees keys <= past + i) ->
// softmax(scores / sqrt(D)) -> @ v (src/inference/attention.py:106-152).
// Here a work item is a tile of 128 query rows -- 128/G tokens of one
// sequence times the G query heads that share a KV head -- against all keys
// up to its last token, for one KV head.  A CTA runs NP independent
// pipelines (two for head_dim 64, one for 128), each with its own work list,
// shared-memory region and tensor-memory columns:
//
//   producer lane: TMA copies of 128-key K and V tiles from the paged pools
//     (one 16-token box per block and 64-element half of a head, landing as
//     128-byte-swizzled rows), a ring of stages; the next tile's block ids
//     are loaded while the current tile's copies are in flight;
//   MMA lane: S = Q K^T (M=128, N=128, K=D) into tensor memory, then
//     O += P V (N=D, K=128) into O in tensor memory, each completion
//     committed to an mbarrier;
//   softmax warpgroup (thread = row): reads S from tensor memory twice, 64
//     columns at a time (the tile max, then the exponents), causal mask only
//     on tiles that cross the diagonal, exp2 with the scale folded into one
//     FMA, a reference max that moves only when a row's max grows by more
//     than 2^8 (O and the row sum rescaled then), P written as bfloat16/half
//     into the swizzled shared-memory A operand of P V; at the end it divides
//     by the row sum and stores the row.
//
// With two pipelines the SM holds two softmax warps per scheduler, so one
// pipeline's exponentials and waits overlap the other's.  Every wait is an
// mbarrier wait with a time limit (NF_STATUS_WAIT_TIMEOUT).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <math.h>

#include <type_traits>

#include "nf_common.cuh"
#include "nf_internal.h"
#include "nf_tma.cuh"
#include "nf_umma.cuh"

namespace nf {

struct PrefillParams {
  char* out;
  long long out_stride;
  const char* q;
  long long q_stride;
  int Hq, Hkv, G, bs, num_blocks;
  const int* bt;
  int max_blocks;
  const int* tiles;  // [n_tiles] x {slot, q_row0, ntok, pos0}
  int n_tiles;
  const int* sched;  // optional: [n_lists + 1] offsets, then the items (tile * Hkv + kv head) of each list
  int n_lists;
  float scale_log2;
  int* status;
};

constexpr float kPfNegInf = -INFINITY;

// Resources of one pipeline, per head_dim and pipelines per CTA.
template <int D_, int NP>
struct PfCfg {
  static constexpr uint32_t TILE = 128 * D_ * 2;         // a 128-row Q tile, or a 128-key K or V tile
  static constexpr uint32_t PB = 128 * 128 * 2;          // P: 128 rows x 128 keys
  static constexpr int NSB = NP == 1 ? 2 : 1;            // S buffers in tensor memory
  static constexpr int STAGES = NP == 1 ? (D_ == 64 ? 4 : 2) : 2;
  static constexpr uint32_t PIPE = TILE + PB + STAGES * 2 * TILE;  // Q, P, K/V stages
  static constexpr uint32_t SMEM = 1024 + 1024 + NP * PIPE;        // alignment slack, barriers, pipelines
  static constexpr uint32_t TM_PIPE = 256;               // tensor-memory columns per pipeline
  static constexpr uint32_t O_COL = NSB * 128;           // O after the S buffers
  static constexpr int THREADS = (4 + 4 * NP) * 32;      // warps 0..NP-1 producers, 2..2+NP-1 MMA, softmax from 4
};
constexpr uint32_t kTmemCols = 512;

// Barriers of pipeline pi, 128 bytes each at the start of the header:
// kv_full[4] 0, kv_empty[4] 32, s_full[2] 64, s_empty[2] 80, p_full 96,
// o_done 104, q_full 112; tensor-memory base at header + 512.
struct PfBars {
  uint32_t base;
  __device__ PfBars(uint32_t hdr, int pi) : base(hdr + 128 * pi) {}
  __device__ uint32_t kv_full(int s) const { return base + 8 * s; }
  __device__ uint32_t kv_empty(int s) const { return base + 32 + 8 * s; }
  __device__ uint32_t s_full(int b) const { return base + 64 + 8 * b; }
  __device__ uint32_t s_empty(int b) const { return base + 80 + 8 * b; }
  __device__ uint32_t p_full() const { return base + 96; }
  __device__ uint32_t o_done() const { return base + 104; }
  __device__ uint32_t q_full() const { return base + 112; }
};
constexpr uint32_t kPfTmemPtr = 512;

// The work items of pipeline `worker`: its list in the schedule, or every
// n_workers-th item.
struct PfItems {
  int i, end, step;
  const int* list;
  __device__ PfItems(const PrefillParams& p, int worker, int n_workers) {
    if (p.sched) {
      if (worker < p.n_lists) {
        i = __ldg(p.sched + worker);
        end = __ldg(p.sched + worker + 1);
      } else {
        i = end = 0;
      }
      step = 1;
      list = p.sched + p.n_lists + 1;
    } else {
      i = worker;
      end = p.n_tiles * p.Hkv;
      step = n_workers;
      list = nullptr;
    }
  }
  __device__ bool next(int& item) {
    if (i >= end) return false;
    item = list ? __ldg(list + i) : i;
    i += step;
    return true;
  }
};

// Block ids of the eight 16-key blocks of key tile j (keys >= nkeys: 0, not
// loaded).  The eight loads are independent, so they cost one round trip.
__device__ __forceinline__ void pf_tile_blocks(const PrefillParams& p, const int* btrow, int j, int nkeys,
                                               int (&ph)[8]) {
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const int key = (j * 8 + b) * 16, lb = key / p.bs;
    ph[b] = (key < nkeys && lb < p.max_blocks) ? __ldg(btrow + lb) : (key < nkeys ? -1 : 0);
  }
}

template <int D_, int NP>
__device__ void pf_producer(const PrefillParams& p, const CUtensorMap* tk, const CUtensorMap* tv, const PfBars& bar,
                            uint32_t kv_s, int worker, int n_workers) {
  using C = PfCfg<D_, NP>;
  constexpr int NDH = D_ / 64;
  const uint64_t pol = l2_evict_last();  // every query tile of a chunk reads the same keys
  int st = 0;
  uint32_t pe = 1;
  PfItems items(p, worker, n_workers);
  for (int item; items.next(item);) {
    const int t = item / p.Hkv, kvh = item - t * p.Hkv;
    const int4 tl = __ldg(reinterpret_cast<const int4*>(p.tiles) + t);
    const int nkeys = tl.w + tl.z, nkt = (nkeys + 127) >> 7;
    const int* btrow = p.bt + (long long)tl.x * p.max_blocks;
    int cur[8], nxt[8];
    pf_tile_blocks(p, btrow, 0, nkeys, cur);
    for (int j = 0; j < nkt; ++j) {
      if (!mbar_wait(bar.kv_empty(st), pe, p.status)) return;
      const int nb = min(8, (nkeys - j * 128 + 15) >> 4);
      const uint32_t full = bar.kv_full(st);
      mbar_arrive_expect_tx(full, nb * NDH * 2 * 2048);
      const uint32_t ks = kv_s + st * 2 * C::TILE, vs = ks + C::TILE;
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        if (b >= nb) break;
        const int off = ((j * 8 + b) * 16) % p.bs;
        int phys = cur[b];
        if (phys < 0 || phys >= p.num_blocks) {
          atomicOr(p.status, NF_STATUS_BAD_BLOCK);
          phys = 0;
        }
#pragma unroll
        for (int dh = 0; dh < NDH; ++dh) {
          const uint32_t dst = dh * 128 * 128 + b * 2048;
          if constexpr (D_ == 64) {
            tma_load_4d(ks + dst, tk, 0, kvh, off, phys, full, pol);
            tma_load_4d(vs + dst, tv, 0, kvh, off, phys, full, pol);
          } else {
            tma_load_5d(ks + dst, tk, 0, dh, kvh, off, phys, full, pol);
            tma_load_5d(vs + dst, tv, 0, dh, kvh, off, phys, full, pol);
          }
        }
      }
      if (j + 1 < nkt) {
        pf_tile_blocks(p, btrow, j + 1, nkeys, nxt);
#pragma unroll
        for (int b = 0; b < 8; ++b) cur[b] = nxt[b];
      }
      if (++st == C::STAGES) {
        st = 0;
        pe ^= 1;
      }
    }
  }
}

template <int D_, int NP>
__device__ void pf_mma(const PrefillParams& p, const PfBars& bar, uint32_t tmem, uint32_t q_s, uint32_t p_s,
                       uint32_t kv_s, bool bf, int worker, int n_workers) {
  using C = PfCfg<D_, NP>;
  constexpr uint32_t REG = 128 * 128;  // one 64-element region of a 128-row operand
  const uint32_t idesc_s = umma_idesc_f16(bf, 128, 128, false, false);
  const uint32_t idesc_o = umma_idesc_f16(bf, 128, D_, false, true);
  int st = 0, tc = 0, npv = 0, nq = 0;
  uint32_t pf = 0;
  auto issue_pv = [&](int stage, bool first) -> bool {
    if (!mbar_wait(bar.p_full(), npv & 1, p.status)) return false;
    ++npv;
    tc_fence_after();
    const uint32_t vs = kv_s + stage * 2 * C::TILE + C::TILE;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint64_t a = umma_sdesc_sw128(p_s + (kk >> 2) * REG + (kk & 3) * 32, 16, 1024);
      const uint64_t b = umma_sdesc_sw128(vs + kk * 16 * 128, REG, 1024);
      umma_f16_ss(tmem + C::O_COL, a, b, idesc_o, (first && kk == 0) ? 0u : 1u);
    }
    umma_commit(bar.o_done());
    umma_commit(bar.kv_empty(stage));
    return true;
  };
  PfItems items(p, worker, n_workers);
  for (int item; items.next(item);) {
    const int t = item / p.Hkv;
    const int4 tl = __ldg(reinterpret_cast<const int4*>(p.tiles) + t);
    const int nkt = (tl.w + tl.z + 127) >> 7;
    if (!mbar_wait(bar.q_full(), nq & 1, p.status)) return;
    ++nq;
    tc_fence_after();
    int prev = -1;
    for (int j = 0; j < nkt; ++j) {
      if (!mbar_wait(bar.kv_full(st), pf, p.status)) return;
      const int b = C::NSB == 2 ? (tc & 1) : 0;
      const int use = C::NSB == 2 ? (tc >> 1) : tc;  // uses of this S buffer so far
      if (!mbar_wait(bar.s_empty(b), (use & 1) ^ 1, p.status)) return;
      ++tc;
      tc_fence_after();
      const uint32_t ks = kv_s + st * 2 * C::TILE;
#pragma unroll
      for (int k = 0; k < D_ / 16; ++k) {
        const uint64_t a = umma_sdesc_sw128(q_s + (k >> 2) * REG + (k & 3) * 32, 16, 1024);
        const uint64_t bd = umma_sdesc_sw128(ks + (k >> 2) * REG + (k & 3) * 32, 16, 1024);
        umma_f16_ss(tmem + b * 128, a, bd, idesc_s, k > 0 ? 1u : 0u);
      }
      umma_commit(bar.s_full(b));
      if (prev >= 0 && !issue_pv(prev, j == 1)) return;
      prev = st;
      if (++st == C::STAGES) {
        st = 0;
        pf ^= 1;
      }
    }
    if (!issue_pv(prev, nkt == 1)) return;
  }
}

template <typename T, int D_, int NP>
__device__ void pf_softmax(const PrefillParams& p, const PfBars& bar, uint32_t tmem, uint32_t q_s, uint32_t p_s,
                           uint32_t kv_s, int worker, int n_workers) {
  using C = PfCfg<D_, NP>;
  constexpr int NDH = D_ / 64;
  constexpr uint32_t REG = 128 * 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3, row = quad * 32 + lane;
  const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
  const int G = p.G;
  int tc = 0, nod = 0, st = 0;
  PfItems items(p, worker, n_workers);
  for (int item; items.next(item);) {
    const int t = item / p.Hkv, kvh = item - t * p.Hkv;
    const int4 tl = __ldg(reinterpret_cast<const int4*>(p.tiles) + t);
    const int nkeys = tl.w + tl.z, nkt = (nkeys + 127) >> 7;
    const int tok = row / G, h = row - tok * G;
    const bool valid = tok < tl.z;
    const int qpos = tl.w + tok;
    // this row of Q into the swizzled A operand
    {
      const char* src = p.q + ((long long)(tl.y + tok) * p.q_stride + (long long)(kvh * G + h) * D_) * 2;
#pragma unroll
      for (int c = 0; c < NDH * 8; ++c) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (valid) v = __ldg(reinterpret_cast<const uint4*>(src) + c);
        const uint32_t a = q_s + (c >> 3) * REG + row * 128 + (((c & 7) ^ (row & 7)) << 4);
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(bar.q_full());
    float m = kPfNegInf, l = 0.f;
    for (int j = 0; j < nkt; ++j) {
      const int b = C::NSB == 2 ? (tc & 1) : 0;
      const int use = C::NSB == 2 ? (tc >> 1) : tc;
      if (!mbar_wait(bar.s_full(b), use & 1, p.status)) return;
      ++tc;
      tc_fence_after();
      const uint32_t s_addr = tmem + lane_addr + b * 128;
      const int k0 = j * 128;
      const int lim = valid ? qpos - k0 : -1;  // columns <= lim are visible (key k <= qpos)
      const bool full = __all_sync(0xffffffffu, lim >= 127);  // no row of the warp crosses the diagonal
      // pass 1: tile max of the raw scores, 64 columns at a time, 8 chains;
      // the causal mask only where some row of the warp crosses the diagonal
      float acc[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) acc[a] = kPfNegInf;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t x[64];
        tmem_ld32(s_addr + h2 * 64, *reinterpret_cast<uint32_t(*)[32]>(x));
        tmem_ld32(s_addr + h2 * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(x + 32));
        tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (h2 * 64 + i > lim) x[i] = __float_as_uint(kPfNegInf);
        }
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i & 7] = fmaxf(acc[i & 7], __uint_as_float(x[i]));
      }
      const float mt = fmaxf(fmaxf(fmaxf(acc[0], acc[1]), fmaxf(acc[2], acc[3])),
                             fmaxf(fmaxf(acc[4], acc[5]), fmaxf(acc[6], acc[7]))) * p.scale_log2;
      // lazy rescaling: the reference max moves (O and l rescaled) only when
      // the tile's max exceeds it by more than 8, so exponents stay <= 2^8
      const bool grow = mt > m + 8.f;
      const float mn = grow ? mt : m;
      const float alpha = grow ? ex2(m - mn) : 1.f;  // 0 on the first visible tile
      const float nbase = mn == kPfNegInf ? 0.f : -mn;
      // P and V of the previous tile must be consumed before P is rewritten:
      // wait for O += P V of tile j-1 (and rescale O if a row's max moved)
      if (j > 0) {
        if (!mbar_wait(bar.o_done(), nod & 1, p.status)) return;
        ++nod;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < D_ / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_addr + C::O_COL + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tmem + lane_addr + C::O_COL + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      // pass 2: exponents, row sum, P (16 chunks of 8 keys; keys 64r.. in region r)
      float sa[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) sa[a] = 0.f;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t x[64];
        tmem_ld32(s_addr + h2 * 64, *reinterpret_cast<uint32_t(*)[32]>(x));
        tmem_ld32(s_addr + h2 * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(x + 32));
        tmem_wait_ld();
        if (h2 == 1) {  // S fully read: the MMA may overwrite this buffer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar.s_empty(b));
        }
        if (!full) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (h2 * 64 + i > lim) x[i] = __float_as_uint(kPfNegInf);
        }
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          const float p0 = ex2(fmaf(__uint_as_float(x[i]), p.scale_log2, nbase));
          const float p1 = ex2(fmaf(__uint_as_float(x[i + 1]), p.scale_log2, nbase));
          sa[(i >> 1) & 7] += p0 + p1;
          x[i >> 1] = pack2<T>(p0, p1);  // packed P reuses the low half of x
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t a = p_s + h2 * REG + row * 128 + ((c ^ (row & 7)) << 4);
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x[4 * c]), "r"(x[4 * c + 1]),
                       "r"(x[4 * c + 2]), "r"(x[4 * c + 3])
                       : "memory");
        }
      }
      l = l * alpha + (((sa[0] + sa[1]) + (sa[2] + sa[3])) + ((sa[4] + sa[5]) + (sa[6] + sa[7])));
      m = mn;
      if (j == nkt - 1 && k0 + row >= nkeys) {
        // V rows past the tile's last visible key (their P is 0) may hold
        // anything: zero them so that 0 * NaN cannot reach O
        const uint32_t vs = kv_s + st * 2 * C::TILE + C::TILE;
#pragma unroll
        for (int dh = 0; dh < NDH; ++dh)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(vs + dh * REG + row * 128 + c * 16), "r"(0)
                         : "memory");
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar.p_full());
      if (++st == C::STAGES) st = 0;
    }
    // epilogue: O / l for the valid rows
    if (!mbar_wait(bar.o_done(), nod & 1, p.status)) return;
    ++nod;
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    T* dst = reinterpret_cast<T*>(p.out) + (long long)(tl.y + tok) * p.out_stride + (long long)(kvh * G + h) * D_;
#pragma unroll
    for (int c = 0; c < D_ / 32; ++c) {
      uint32_t o[32];
      tmem_ld32(tmem + lane_addr + C::O_COL + c * 32, o);
      tmem_wait_ld();
      if (valid) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack2<T>(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      }
    }
    tc_fence_before();
  }
}

template <typename T, int D_, int NP>
__global__ void __launch_bounds__(PfCfg<D_, NP>::THREADS, 1)
    prefill_attention_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tk,
                             const __grid_constant__ CUtensorMap tv) {
  using C = PfCfg<D_, NP>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t hdr = smem_u32(base);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int pi = 0; pi < NP; ++pi) {
      const PfBars bar(hdr, pi);
      for (int s = 0; s < C::STAGES; ++s) {
        mbar_init(bar.kv_full(s), 1);
        mbar_init(bar.kv_empty(s), 1);
      }
      for (int b = 0; b < C::NSB; ++b) {
        mbar_init(bar.s_full(b), 1);
        mbar_init(bar.s_empty(b), 4);
      }
      mbar_init(bar.p_full(), 4);
      mbar_init(bar.o_done(), 1);
      mbar_init(bar.q_full(), 4);
    }
    fence_mbar_init();
  }
  if (warp == 2) tmem_alloc(hdr + kPfTmemPtr, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem0 = *reinterpret_cast<volatile uint32_t*>(base + kPfTmemPtr);
  const int n_workers = gridDim.x * NP;
  // role and pipeline of this warp: producers 0..NP-1, MMA 2..2+NP-1, softmax warpgroups from warp 4
  int pi = -1, role = -1;
  if (warp < NP) {
    pi = warp;
    role = 0;
  } else if (warp >= 2 && warp < 2 + NP) {
    pi = warp - 2;
    role = 1;
  } else if (warp >= 4) {
    pi = (warp - 4) >> 2;
    role = 2;
  }
  if (role >= 0) {
    const PfBars bar(hdr, pi);
    const uint32_t q_s = hdr + 1024 + pi * C::PIPE, p_s = q_s + C::TILE, kv_s = p_s + C::PB;
    const uint32_t tmem = tmem0 + pi * C::TM_PIPE;
    const int worker = blockIdx.x * NP + pi;
    if (role == 0) {
      if ((threadIdx.x & 31) == 0) pf_producer<D_, NP>(p, &tk, &tv, bar, kv_s, worker, n_workers);
    } else if (role == 1) {
      if ((threadIdx.x & 31) == 0)
        pf_mma<D_, NP>(p, bar, tmem, q_s, p_s, kv_s, std::is_same<T, __nv_bfloat16>::value, worker, n_workers);
    } else {
      pf_softmax<T, D_, NP>(p, bar, tmem, q_s, p_s, kv_s, worker, n_workers);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem0, kTmemCols);
}

template <typename T, int D_>
static int launch_prefill(const PrefillParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int n_items,
                          cudaStream_t st) {
  constexpr int NP = D_ == 64 ? 2 : 1;
  using C = PfCfg<D_, NP>;
  auto kern = prefill_attention_kernel<T, D_, NP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_prefill_attention: smem attribute: %s", cudaGetErrorString(e));
  long long grid = p.sched ? (p.n_lists + NP - 1) / NP : ((long long)n_items + NP - 1) / NP;
  if (grid > sm_count()) grid = sm_count();
  kern<<<(int)grid, C::THREADS, C::SMEM, st>>>(p, tk, tv);
  return check_launch("nf_prefill_attention");
}

}  // namespace nf

extern "C" int nf_prefill_pipelines(int32_t head_dim) { return head_dim == 64 ? 2 : 1; }

extern "C" int nf_prefill_attention(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                    const void* k_pool, const void* v_pool, int32_t dtype, int32_t num_q_heads,
                                    int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                    const int32_t* block_tables, int32_t max_blocks_per_seq, const int32_t* tiles,
                                    int32_t n_tiles, const int32_t* schedule, int32_t n_lists, float scale,
                                    int32_t* status, void* stream) {
  using namespace nf;
  if (dtype != NF_BF16 && dtype != NF_F16)
    return fail(NF_EUNSUPPORTED, "nf_prefill_attention: 16-bit pools only (dtype %d)", dtype);
  if (head_dim != 64 && head_dim != 128)
    return fail(NF_EUNSUPPORTED, "nf_prefill_attention: head_dim %d (64 or 128)", head_dim);
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads)
    return fail(NF_EINVAL, "nf_prefill_attention: num_q_heads must be a multiple of num_kv_heads");
  const int G = num_q_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return fail(NF_EUNSUPPORTED, "nf_prefill_attention: %d query heads per KV head (1, 2, 4 or 8)", G);
  if (block_size <= 0 || block_size % 16)
    return fail(NF_EUNSUPPORTED, "nf_prefill_attention: block_size %d is not a multiple of 16", block_size);
  if (n_tiles < 0 || num_blocks <= 0 || max_blocks_per_seq <= 0)
    return fail(NF_EINVAL, "nf_prefill_attention: sizes must be positive");
  if (n_tiles == 0) return ok();
  if (!out || !q || !k_pool || !v_pool || !block_tables || !tiles || !status)
    return fail(NF_EINVAL, "nf_prefill_attention: null pointer argument");
  const int np = nf_prefill_pipelines(head_dim);
  if (schedule && (n_lists <= 0 || n_lists > sm_count() * np))
    return fail(NF_EINVAL, "nf_prefill_attention: a schedule needs 1..%d lists (got %d)", sm_count() * np, n_lists);
  auto al = [](const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
  if (!al(q, 16) || !al(out, 16) || (q_row_stride * 2) % 16 || (out_row_stride * 2) % 16 || !al(tiles, 16) ||
      !al(k_pool, 16) || !al(v_pool, 16))
    return fail(NF_EINVAL, "nf_prefill_attention: q/out rows, pools and tiles must be 16-byte aligned");
  CUtensorMap tk, tv;
  if (!encode_pool_map(&tk, k_pool, dtype, head_dim, num_kv_heads, block_size, num_blocks, 1, false) ||
      !encode_pool_map(&tv, v_pool, dtype, head_dim, num_kv_heads, block_size, num_blocks, 1, false))
    return fail(NF_ECUDA, "nf_prefill_attention: tensor map encoding failed");
  PrefillParams p;
  p.out = static_cast<char*>(out);
  p.out_stride = out_row_stride;
  p.q = static_cast<const char*>(q);
  p.q_stride = q_row_stride;
  p.Hq = num_q_heads;
  p.Hkv = num_kv_heads;
  p.G = G;
  p.bs = block_size;
  p.num_blocks = num_blocks;
  p.bt = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  p.sched = schedule;
  p.n_lists = n_lists;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  const int n_items = n_tiles * num_kv_heads;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == NF_BF16)
    return head_dim == 64 ? launch_prefill<__nv_bfloat16, 64>(p, tk, tv, n_items, st)
                          : launch_prefill<__nv_bfloat16, 128>(p, tk, tv, n_items, st);
  return head_dim == 64 ? launch_prefill<__half, 64>(p, tk, tv, n_items, st)
                        : launch_prefill<__half, 128>(p, tk, tv, n_items, st);
}
