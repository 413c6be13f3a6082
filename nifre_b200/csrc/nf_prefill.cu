// Chunked-prefill attention on fifth-generation tensor cores (tcgen05/TMEM).
//
// The reference computes a prefill chunk per row as get -> cat -> q @ k^T ->
// causal mask (query i at position past + i sees keys <= past + i) ->
// softmax(scores / sqrt(D)) -> @ v (src/inference/attention.py:106-152).
// Here a work item is a tile of 128 query rows -- 128/G tokens of one
// sequence times the G query heads that share a KV head -- against all keys
// up to its last token, for one KV head:
//
//   producer lane (warp 0): TMA copies of 128-key K and V tiles from the
//     paged pools (one 16-token box per block and 64-element half of a head,
//     landing as 128-byte-swizzled rows), a ring of stages;
//   MMA lane (warp 1): S = Q K^T (M=128, N=128, K=D) into one of two S
//     buffers in tensor memory, then O += P V (N=D, K=128) into O in tensor
//     memory, each completion committed to an mbarrier;
//   softmax warpgroup (warps 2-5, thread = row): reads S from tensor memory,
//     causal mask, running max and exp2 (scale folded in), rescales its O row
//     in tensor memory when the max grows, writes P as bfloat16/half into the
//     swizzled shared-memory A operand of the P V product, and at the end
//     divides by the row sum and stores the row.
//
// Every wait is an mbarrier wait with a time limit (NF_STATUS_WAIT_TIMEOUT).
// Tensor memory: S0 columns [0,128), S1 [128,256), O [256, 256+D).
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
  const int* sched;  // optional: [n_ctas + 1] offsets, then the items (tile * Hkv + kv head) of each CTA
  int n_ctas;
  float scale_log2;
  int* status;
  int stages;
};

constexpr int kPfThreads = 192;  // warp 0 producer, warp 1 MMA, warps 2-5 softmax
constexpr float kPfNegInf = -INFINITY;
constexpr int kPfHdr = 1024;     // mbarriers and the tensor-memory base
constexpr uint32_t kTmemCols = 512;

// header offsets: kv_full[4] 0, kv_empty[4] 32, s_full[2] 64, s_empty[2] 80,
// p_full 96, o_done 104, q_full 112, tensor-memory base 128
__device__ __forceinline__ uint32_t pf_off_kvfull(int s) { return 8 * s; }
__device__ __forceinline__ uint32_t pf_off_kvempty(int s) { return 32 + 8 * s; }
__device__ __forceinline__ uint32_t pf_off_sfull(int b) { return 64 + 8 * b; }
__device__ __forceinline__ uint32_t pf_off_sempty(int b) { return 80 + 8 * b; }
constexpr uint32_t kPfPfull = 96, kPfOdone = 104, kPfQfull = 112, kPfTmem = 128;

// The work items of this CTA: its list in the schedule, or every gridDim.x-th item.
struct PfItems {
  int i, end, step;
  const int* list;
  __device__ PfItems(const PrefillParams& p) {
    if (p.sched) {
      i = __ldg(p.sched + blockIdx.x);
      end = __ldg(p.sched + blockIdx.x + 1);
      step = 1;
      list = p.sched + p.n_ctas + 1;
    } else {
      i = blockIdx.x;
      end = p.n_tiles * p.Hkv;
      step = gridDim.x;
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

template <int D_>
__device__ void pf_producer(const PrefillParams& p, const CUtensorMap* tk, const CUtensorMap* tv, uint32_t hdr,
                            uint32_t kv_s) {
  constexpr int NDH = D_ / 64;
  constexpr uint32_t TILE = 128 * D_ * 2;  // bytes of a 128-key K or V tile
  const int S = p.stages;
  const uint64_t pol = l2_evict_last();  // every query tile of a chunk reads the same keys
  int st = 0;
  uint32_t pe = 1;
  PfItems items(p);
  for (int item; items.next(item);) {
    const int t = item / p.Hkv, kvh = item - t * p.Hkv;
    const int4 tl = __ldg(reinterpret_cast<const int4*>(p.tiles) + t);
    const int nkeys = tl.w + tl.z, nkt = (nkeys + 127) >> 7;
    const int* btrow = p.bt + (long long)tl.x * p.max_blocks;
    // the next tile's block ids are loaded while this tile's copies are in
    // flight and the next stage is awaited: a tile's copies never wait on
    // the block table
    int cur[8], nxt[8];
    pf_tile_blocks(p, btrow, 0, nkeys, cur);
    for (int j = 0; j < nkt; ++j) {
      if (!mbar_wait(hdr + pf_off_kvempty(st), pe, p.status)) return;
      const int nb = min(8, (nkeys - j * 128 + 15) >> 4);
      const uint32_t full = hdr + pf_off_kvfull(st);
      mbar_arrive_expect_tx(full, nb * NDH * 2 * 2048);
      const uint32_t ks = kv_s + st * 2 * TILE, vs = ks + TILE;
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        if (b >= nb) break;
        const int key = (j * 8 + b) * 16, off = key % p.bs;
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
      if (++st == S) {
        st = 0;
        pe ^= 1;
      }
    }
  }
}

template <int D_>
__device__ void pf_mma(const PrefillParams& p, uint32_t hdr, uint32_t tmem, uint32_t q_s, uint32_t p_s,
                       uint32_t kv_s, bool bf) {
  constexpr uint32_t TILE = 128 * D_ * 2;
  constexpr uint32_t REG = 128 * 128;  // one 64-element region of a 128-row operand
  const uint32_t idesc_s = umma_idesc_f16(bf, 128, 128, false, false);
  const uint32_t idesc_o = umma_idesc_f16(bf, 128, D_, false, true);
  const int S = p.stages;
  int st = 0, tc = 0, npv = 0, nq = 0;
  uint32_t pf = 0;
  auto issue_pv = [&](int stage, bool first) -> bool {
    if (!mbar_wait(hdr + kPfPfull, npv & 1, p.status)) return false;
    ++npv;
    tc_fence_after();
    const uint32_t vs = kv_s + stage * 2 * TILE + TILE;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint64_t a = umma_sdesc_sw128(p_s + (kk >> 2) * REG + (kk & 3) * 32, 16, 1024);
      const uint64_t b = umma_sdesc_sw128(vs + kk * 16 * 128, REG, 1024);
      umma_f16_ss(tmem + 256, a, b, idesc_o, (first && kk == 0) ? 0u : 1u);
    }
    umma_commit(hdr + kPfOdone);
    umma_commit(hdr + pf_off_kvempty(stage));
    return true;
  };
  PfItems items(p);
  for (int item; items.next(item);) {
    const int t = item / p.Hkv;
    const int4 tl = __ldg(reinterpret_cast<const int4*>(p.tiles) + t);
    const int nkt = (tl.w + tl.z + 127) >> 7;
    if (!mbar_wait(hdr + kPfQfull, nq & 1, p.status)) return;
    ++nq;
    tc_fence_after();
    int prev = -1;
    for (int j = 0; j < nkt; ++j) {
      if (!mbar_wait(hdr + pf_off_kvfull(st), pf, p.status)) return;
      const int b = tc & 1;
      if (!mbar_wait(hdr + pf_off_sempty(b), ((tc >> 1) & 1) ^ 1, p.status)) return;
      ++tc;
      tc_fence_after();
      const uint32_t ks = kv_s + st * 2 * TILE;
#pragma unroll
      for (int k = 0; k < D_ / 16; ++k) {
        const uint64_t a = umma_sdesc_sw128(q_s + (k >> 2) * REG + (k & 3) * 32, 16, 1024);
        const uint64_t bd = umma_sdesc_sw128(ks + (k >> 2) * REG + (k & 3) * 32, 16, 1024);
        umma_f16_ss(tmem + b * 128, a, bd, idesc_s, k > 0 ? 1u : 0u);
      }
      umma_commit(hdr + pf_off_sfull(b));
      if (prev >= 0 && !issue_pv(prev, j == 1)) return;
      prev = st;
      if (++st == S) {
        st = 0;
        pf ^= 1;
      }
    }
    if (!issue_pv(prev, nkt == 1)) return;
  }
}

template <typename T, int D_>
__device__ void pf_softmax(const PrefillParams& p, uint32_t hdr, uint32_t tmem, uint32_t q_s, uint32_t p_s,
                           uint32_t kv_s) {
  constexpr int NDH = D_ / 64;
  constexpr uint32_t TILE = 128 * D_ * 2;
  constexpr uint32_t REG = 128 * 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3, row = quad * 32 + lane;
  const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
  const int S = p.stages;
  const int G = p.G;
  int tc = 0, nod = 0, st = 0, nq = 0;
  PfItems items(p);
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
    if (lane == 0) mbar_arrive(hdr + kPfQfull);
    ++nq;
    float m = kPfNegInf, l = 0.f;
    for (int j = 0; j < nkt; ++j) {
      const int b = tc & 1;
      if (!mbar_wait(hdr + pf_off_sfull(b), (tc >> 1) & 1, p.status)) return;
      ++tc;
      tc_fence_after();
      uint32_t x[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_addr + b * 128 + c * 32, x[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(hdr + pf_off_sempty(b));
      // causal mask (key k visible to the query at qpos iff k <= qpos), only
      // on tiles that cross some row's diagonal; tile max of the raw scores
      // over 8 independent chains
      const int k0 = j * 128;
      const int lim = valid ? qpos - k0 : -1;  // columns <= lim are visible
      if (!__all_sync(0xffffffffu, lim >= 127)) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i > lim) x[c][i] = __float_as_uint(kPfNegInf);
      }
      float acc[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) acc[a] = kPfNegInf;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i & 7] = fmaxf(acc[i & 7], __uint_as_float(x[c][i]));
      const float mt = fmaxf(fmaxf(fmaxf(acc[0], acc[1]), fmaxf(acc[2], acc[3])),
                             fmaxf(fmaxf(acc[4], acc[5]), fmaxf(acc[6], acc[7]))) * p.scale_log2;
      // lazy rescaling: the reference max moves (and O and l are rescaled)
      // only when the tile's max exceeds it by more than 8, so exponents stay
      // <= 2^8 and most tiles need no O round trip through registers
      const bool grow = mt > m + 8.f;
      const float mn = grow ? mt : m;
      const float alpha = grow ? ex2(m - mn) : 1.f;  // 0 on the first visible tile
      const float nbase = mn == kPfNegInf ? 0.f : -mn;
      float sa[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) sa[a] = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = ex2(fmaf(__uint_as_float(x[c][i]), p.scale_log2, nbase));
          const float p1 = ex2(fmaf(__uint_as_float(x[c][i + 1]), p.scale_log2, nbase));
          sa[(i >> 1) & 7] += p0 + p1;
          pk[c * 16 + i / 2] = pack2<T>(p0, p1);
        }
      l = l * alpha + (((sa[0] + sa[1]) + (sa[2] + sa[3])) + ((sa[4] + sa[5]) + (sa[6] + sa[7])));
      m = mn;
      if (j > 0) {
        // O += P V of the previous tile must be done: rescale O, then P is free
        if (!mbar_wait(hdr + kPfOdone, nod & 1, p.status)) return;
        ++nod;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < D_ / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_addr + 256 + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tmem + lane_addr + 256 + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      // P row: 16 chunks of 8 keys, keys 64r.. in region r
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint32_t a = p_s + (c >> 3) * REG + row * 128 + (((c & 7) ^ (row & 7)) << 4);
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(pk[4 * c]), "r"(pk[4 * c + 1]),
                     "r"(pk[4 * c + 2]), "r"(pk[4 * c + 3])
                     : "memory");
      }
      if (j == nkt - 1 && k0 + row >= nkeys) {
        // V rows past the tile's last visible key (their P is 0) may hold
        // anything: zero them so that 0 * NaN cannot reach O
        const uint32_t vs = kv_s + st * 2 * TILE + TILE;
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
      if (lane == 0) mbar_arrive(hdr + kPfPfull);
      if (++st == S) st = 0;
    }
    // epilogue: O / l for the valid rows
    if (!mbar_wait(hdr + kPfOdone, nod & 1, p.status)) return;
    ++nod;
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    T* dst = reinterpret_cast<T*>(p.out) + (long long)(tl.y + tok) * p.out_stride + (long long)(kvh * G + h) * D_;
#pragma unroll
    for (int c = 0; c < D_ / 32; ++c) {
      uint32_t o[32];
      tmem_ld32(tmem + lane_addr + 256 + c * 32, o);
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

template <typename T, int D_>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_attention_kernel(const PrefillParams p,
                                                                          const __grid_constant__ CUtensorMap tk,
                                                                          const __grid_constant__ CUtensorMap tv) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t hdr = smem_u32(base);
  constexpr uint32_t QB = 128 * D_ * 2, PB = 128 * 128 * 2;
  const uint32_t q_s = hdr + kPfHdr, p_s = q_s + QB, kv_s = p_s + PB;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(hdr + pf_off_kvfull(s), 1);
      mbar_init(hdr + pf_off_kvempty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(hdr + pf_off_sfull(b), 1);
      mbar_init(hdr + pf_off_sempty(b), 4);
    }
    mbar_init(hdr + kPfPfull, 4);
    mbar_init(hdr + kPfOdone, 1);
    mbar_init(hdr + kPfQfull, 4);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(hdr + kPfTmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(base + kPfTmem);
  if (warp == 0) {
    if ((threadIdx.x & 31) == 0) pf_producer<D_>(p, &tk, &tv, hdr, kv_s);
  } else if (warp == 1) {
    if ((threadIdx.x & 31) == 0) pf_mma<D_>(p, hdr, tmem, q_s, p_s, kv_s, std::is_same<T, __nv_bfloat16>::value);
  } else {
    pf_softmax<T, D_>(p, hdr, tmem, q_s, p_s, kv_s);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace nf

extern "C" int nf_prefill_attention(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                    const void* k_pool, const void* v_pool, int32_t dtype, int32_t num_q_heads,
                                    int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                    const int32_t* block_tables, int32_t max_blocks_per_seq, const int32_t* tiles,
                                    int32_t n_tiles, const int32_t* schedule, int32_t n_ctas, float scale,
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
  p.n_ctas = n_ctas;
  if (schedule && (n_ctas <= 0 || n_ctas > sm_count()))
    return fail(NF_EINVAL, "nf_prefill_attention: a schedule needs 1..%d CTAs (got %d)", sm_count(), n_ctas);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  p.stages = head_dim == 64 ? 4 : 2;
  const int tile = 128 * head_dim * 2;
  const int smem = 1024 + kPfHdr + tile + 128 * 128 * 2 + p.stages * 2 * tile;
  auto kern = dtype == NF_BF16 ? (head_dim == 64 ? prefill_attention_kernel<__nv_bfloat16, 64>
                                                 : prefill_attention_kernel<__nv_bfloat16, 128>)
                               : (head_dim == 64 ? prefill_attention_kernel<__half, 64>
                                                 : prefill_attention_kernel<__half, 128>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_prefill_attention: smem attribute: %s", cudaGetErrorString(e));
  long long grid = (long long)n_tiles * num_kv_heads;
  if (grid > sm_count()) grid = sm_count();
  if (schedule) grid = n_ctas;
  kern<<<(int)grid, kPfThreads, smem, static_cast<cudaStream_t>(stream)>>>(p, tk, tv);
  return check_launch("nf_prefill_attention");
}
