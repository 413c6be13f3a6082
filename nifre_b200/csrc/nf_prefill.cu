// Chunked-prefill attention on fifth-generation tensor cores (tcgen05/TMEM).
//
// The reference computes a prefill chunk per row as get -> cat -> q @ k^T ->
// causal mask (query i at position past + i sees keys <= past + i) ->
// softmax(scores / sqrt(D)) -> @ v (src/inference/attention.py:106-152).
// Here a work item is 256 query rows -- 256/G consecutive tokens of one
// sequence times the G query heads that share a KV head -- against all keys
// up to its last token, for one KV head.  The rows form two 128-row halves
// that share one stream of K and V tiles; each CTA is persistent over its
// list of items:
//
//   producer warp: TMA copies of 128-key K and V tiles from the paged pools
//     (one 16-token box per block and 64-element part of a head, landing as
//     128-byte-swizzled rows) into separate K and V rings, so that a K stage
//     is refilled as soon as both halves' S = Q K^T have read it; the next
//     tile's block ids are loaded while the current tile's copies fly;
//   MMA warp (one lane issues): per key tile, S_h = Q_h K^T (M=128, N=128, K=D) into tensor
//     memory for each half h, then O_h += P_h V (N=D, K=128) with P_h read
//     from tensor memory (the TS form: A in tensor memory, V in shared);
//   two softmax warpgroups, one per half (thread = row, 216 registers), which alternate on
//     the tensor core: each reads its S_h tile from tensor memory once into
//     registers (for head_dim 64 the S buffer is released right away, so the
//     next S_h overlaps the exponentials), applies the causal mask only on
//     tiles that cross the diagonal, keeps a reference max that moves only
//     when a row's max grows by more than 2^8 (O_h and the row sum rescaled
//     then), computes exp2 with the scale folded into one packed FMA on the
//     special-function unit (a polynomial on the FMA pipe is a build option,
//     NF_PF_POLY: with two warps per scheduler the FMA pipe saturates first,
//     so it gains nothing at head_dim 64), and stores P_h
//     as bfloat16/half pairs into tensor memory; at the end it divides by the
//     row sum and stores the row.
//
// Tensor memory (512 columns): S_0, S_1 at 0 and 128, O_0, O_1 from 256; P_h
// has its own 64 columns from 384 for head_dim 64 and overwrites the first
// half of S_h for head_dim 128 (no room left), where the MMA warp then issues
// P_h V before the next S_h.  Every wait is an mbarrier wait with a time
// limit (NF_STATUS_WAIT_TIMEOUT).
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
  int rows;                             // rows of q and out
  int Hq, Hkv, G, TT, NH, bs, num_blocks;  // TT: tokens per 128-row half; NH: halves per item
  const int* bt;
  int max_blocks;
  const int* tiles;  // [n_tiles] x {slot, q_row0, ntok, pos0}
  int n_tiles;
  const int* order;  // optional: the items (tile * Hkv + kv head) in the order CTAs take them
  int* queue;        // [2]: next position in the order, CTAs finished (zero on entry and on exit)
  float scale_log2;
  int* status;
  // gathered output over several GPUs: rows also stored at peer_out[r] (same layout as out), r < n_peers
  int n_peers;
  char* peer_out[kMaxRanks - 1];
  // cascade mode (nf_cascade_attention on the tensor cores): an item is (task, KV head); its rows are the
  // decode queries of a group of sequences, its keys the range [key_begin, key_end) of their shared blocks,
  // and it writes split-K partial records instead of output rows
  const int* tasks;   // [n_tiles][8]: slot, first, count, part, key_begin, key_end, 0, 0
  const int* toks;    // [n_toks][2]: item of nf_pack_step, q row
  int n_toks;
  const int* items;   // nf_pack_step's work items (unit_base at [3])
  const int* counts;  // nf_pack_step's counts ([3]: partial slots)
  float* ws;          // partials [slots][Hq][D + 4]: acc[D], m, l, pad
  int max_items, max_units;
};

constexpr float kPfNegInf = -INFINITY;
#ifndef NF_PF_HALVES_64
#define NF_PF_HALVES_64 2
#endif
// 128-row query halves per work item (and CTA): head_dim 64 runs one half per
// CTA and two CTAs per SM, whose softmax warps then drift out of step and
// overlap one another's exponentials with their loads and stores; head_dim
// 128 (tensor work per tile doubled, tensor memory full) runs two halves that
// share one K/V stream.
__host__ __device__ constexpr int pf_halves(int d) { return d == 64 ? NF_PF_HALVES_64 : 2; }

template <int D_, int NH = pf_halves(D_)>
struct PfCfg {
  static constexpr uint32_t TILE = 128 * D_ * 2;  // a 128-row Q half, or a 128-key K or V tile
  static constexpr int NH_ = NH;
  static constexpr int MINB = NH == 1 ? 2 : 1;    // CTAs per SM
  static constexpr int QST = (D_ == 64 || NH == 1) ? 2 : 1;           // Q ring (an item's halves per stage)
  static constexpr int KST = NH == 1 ? 2 : (D_ == 64 ? 4 : 2);        // K ring
  static constexpr int VST = NH == 1 ? 2 : (D_ == 64 ? 5 : 3);        // V ring (held one tile longer than K)
  static constexpr bool P_ALIAS = D_ == 128;      // P_h over the first 64 columns of S_h
  static constexpr uint32_t Q_OFF = 1024;         // after the barrier header
  static constexpr uint32_t K_OFF = Q_OFF + QST * NH * TILE;
  static constexpr uint32_t V_OFF = K_OFF + KST * TILE;
  static constexpr uint32_t SMEM = 1024 + V_OFF + VST * TILE;  // + alignment slack
  static constexpr int THREADS = 128 * (1 + NH);  // warp 0 producer, 1 MMA, 4-7 half 0, 8-11 half 1
  // registers per thread at launch: 64K / (threads x CTAs per SM), rounded
  // to 8 (168 for two halves, 128 for one); the first warpgroup gives back
  // to REGS_CTRL and the softmax warpgroups take REGS_SOFTMAX, adding up to
  // the launch total (checked against the compiled count before a launch)
  static constexpr int LAUNCH_REGS = (65536 / (THREADS * MINB)) / 8 * 8;
  static constexpr int REGS_CTRL = NH == 1 ? 64 : 72, REGS_SOFTMAX = NH == 1 ? 192 : 216;
  static_assert(REGS_CTRL * 128 + REGS_SOFTMAX * 128 * NH <= LAUNCH_REGS * THREADS, "register split exceeds the launch");
  static constexpr uint32_t TMEM_COLS = NH == 1 ? 256 : 512;
  static __device__ __forceinline__ uint32_t s_col(int h) { return h * 128; }
  static __device__ __forceinline__ uint32_t o_col(int h) { return NH * 128 + h * D_; }
  static __device__ __forceinline__ uint32_t p_col(int h) { return P_ALIAS ? h * 128 : NH * (128 + D_) + h * 64; }
};

// Barriers at the start of the header: k_full[8] 0, k_empty[8] 64,
// v_full[8] 128, v_empty[8] 192, then per half s_full 256, s_free 272,
// p_full 288, o_done 304, per Q stage q_full 320, q_empty 336, per item
// slot item_full 384, item_empty 416, and per (half, quad) of softmax warps
// the exponent-pass turn 448; tensor-memory base at 512, item slots (8 ints
// each) from 640.
struct PfBars {
  uint32_t hdr;
  __device__ explicit PfBars(uint32_t h) : hdr(h) {}
  __device__ uint32_t k_full(int s) const { return hdr + 8 * s; }
  __device__ uint32_t k_empty(int s) const { return hdr + 64 + 8 * s; }
  __device__ uint32_t v_full(int s) const { return hdr + 128 + 8 * s; }
  __device__ uint32_t v_empty(int s) const { return hdr + 192 + 8 * s; }
  __device__ uint32_t s_full(int h) const { return hdr + 256 + 8 * h; }
  __device__ uint32_t s_free(int h) const { return hdr + 272 + 8 * h; }
  __device__ uint32_t p_full(int h) const { return hdr + 288 + 8 * h; }
  __device__ uint32_t o_done(int h) const { return hdr + 304 + 8 * h; }
  __device__ uint32_t q_full(int s) const { return hdr + 320 + 8 * s; }
  __device__ uint32_t q_empty(int s) const { return hdr + 336 + 8 * s; }
  __device__ uint32_t item_full(int s) const { return hdr + 384 + 8 * s; }
  __device__ uint32_t item_empty(int s) const { return hdr + 416 + 8 * s; }
  __device__ uint32_t turn(int h, int quad) const { return hdr + 448 + 8 * (h * 4 + quad); }
};
constexpr uint32_t kPfTmemPtr = 512;
constexpr uint32_t kPfItemSlots = 640;
constexpr int kPfItemRing = 4;


// ---------------------------------------------------------------- softmax arithmetic
// Pairs of fp32 values in one 64-bit register, for the packed fp32x2
// instructions of sm_100 (two FMAs or adds per issue).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^y for a pair y <= 8 on the FMA pipe instead of the special-function
// unit: y = j + f with j = round(y) (adding and subtracting 1.5 * 2^23), 2^f
// on [-1/2, 1/2] by 1 + c1 f + c2 f^2 + c3 f^3 fitted for minimum relative
// error (Lawson-weighted least squares; error 1.0e-4, far below the 2^-8 step
// of a 16-bit P), and j added to the exponent field.  y is clamped at -127;
// with the constant term exactly 1 the result there is exactly +0 and never
// negative or NaN above it.
__device__ __forceinline__ void exp2_poly2(uint64_t y2, float& r0, float& r1) {
  float y0, y1;
  f2_unpack(y2, y0, y1);
  const uint64_t y = f2_pack(fmaxf(y0, -127.f), fmaxf(y1, -127.f));
  const uint64_t t = f2_add(y, f2_pack(12582912.f, 12582912.f));
  const uint64_t j = f2_add(t, f2_pack(-12582912.f, -12582912.f));
  const uint64_t fr = f2_fma(j, f2_pack(-1.f, -1.f), y);  // y - j, exact
  uint64_t q = f2_fma(f2_pack(0.0550089292f, 0.0550089292f), fr, f2_pack(0.242210954f, 0.242210954f));
  q = f2_fma(q, fr, f2_pack(0.693282902f, 0.693282902f));
  q = f2_fma(q, fr, f2_pack(1.f, 1.f));
  float q0, q1, t0, t1;
  f2_unpack(q, q0, q1);
  f2_unpack(t, t0, t1);
  // t's low mantissa bits hold j (two's complement): shifted, they add j to the exponent
  r0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  r1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

#ifndef NF_PF_POLY
#define NF_PF_POLY 0
#endif
// Of every 8 pairs of exponentials, this many go to the polynomial (FMA
// pipe) and the rest to ex2 (special-function unit, 16 per clock per SM).
constexpr int kPfPolyPairs = NF_PF_POLY;

#ifndef NF_PF_TURNS
#define NF_PF_TURNS 0
#endif
// 1: the two halves' softmax warps on one scheduler take turns on the
// special-function unit (see pf_softmax).  Measured slower on B200 (59.4 vs
// 55.3 us on the mixed-step layer): the mbarrier hand-off costs ~300 cycles
// per turn and each warp's non-exponent work grows once the halves are out
// of step, so by default the halves share the unit in step.
constexpr bool kPfTurns = NF_PF_TURNS != 0;

// A ring position: stage index and the parity of its current fill.
struct Ring {
  int st = 0;
  uint32_t ph = 0;
  __device__ void next(int n) {
    if (++st == n) {
      st = 0;
      ph ^= 1;
    }
  }
  __device__ Ring ahead(int k, int n) const {  // the position k fills later
    Ring r;
    const int t = st + k;
    r.st = t % n;
    r.ph = ph ^ ((uint32_t)(t / n) & 1u);
    return r;
  }
};

// Work items come from one queue shared by all CTAs: the producer warp of
// a CTA claims the next position in the order (longest items first) when it
// starts loading an item, so CTAs that finish early take more, and passes
// the item with its tile descriptor to the CTA's other warps through a ring
// of shared-memory slots.  A slot holding -1 ends the CTA's work.
struct PfItemRing {
  const PfBars& bar;
  unsigned char* slots;
  Ring r;
  __device__ PfItemRing(const PfBars& b, unsigned char* base) : bar(b), slots(base + kPfItemSlots) {}
  __device__ int* slot(int st) const { return reinterpret_cast<int*>(slots + 32 * st); }
  // a reader warp: the next item (false at the end)
  __device__ bool next(int& item, int4& tl, int2& kr, int* status) {
    if (!mbar_wait(bar.item_full(r.st), r.ph, status)) return false;
    const volatile int* sl = slot(r.st);
    item = sl[0];
    tl = make_int4(sl[1], sl[2], sl[3], sl[4]);
    kr = make_int2(sl[5], sl[6]);
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar.item_empty(r.st));
    r.next(kPfItemRing);
    return item >= 0;
  }
};

// The producer warp's side of the queue: claim the next item, publish it.
// Cascade items are dealt in a fixed round-robin (claim k of CTA b is item
// b + k * gridDim.x): they are alike in size, and the cascade entry point
// has no queue buffer.
template <bool CASC>
__device__ __forceinline__ bool pf_claim_item(const PrefillParams& p, PfItemRing& ring, int& item, int4& tl, int2& kr,
                                              int& claims) {
  const int lane = threadIdx.x & 31;
  int pos = 0;
  if (CASC) {
    pos = blockIdx.x + claims * gridDim.x;
  } else {
    if (lane == 0) pos = atomicAdd(p.queue, 1);
    pos = __shfl_sync(0xffffffffu, pos, 0);
  }
  ++claims;
  const int n_items = p.n_tiles * p.Hkv;
  item = pos < n_items ? (p.order ? __ldg(p.order + pos) : pos) : -1;
  kr = make_int2(0, 0);
  if (item < 0) {
    tl = make_int4(0, 0, 0, 0);
  } else if (CASC) {
    tl = __ldg(reinterpret_cast<const int4*>(p.tasks) + 2 * (item / p.Hkv));
    const int4 tb = __ldg(reinterpret_cast<const int4*>(p.tasks) + 2 * (item / p.Hkv) + 1);
    kr = make_int2(tb.x, tb.y);
  } else {
    tl = __ldg(reinterpret_cast<const int4*>(p.tiles) + item / p.Hkv);
  }
  if (!mbar_wait(ring.bar.item_empty(ring.r.st), ring.r.ph ^ 1, p.status)) return false;
  if (lane == 0) {
    volatile int* sl = ring.slot(ring.r.st);
    sl[0] = item;
    sl[1] = tl.x;
    sl[2] = tl.y;
    sl[3] = tl.z;
    sl[4] = tl.w;
    sl[5] = kr.x;
    sl[6] = kr.y;
    mbar_arrive(ring.bar.item_full(ring.r.st));
  }
  __syncwarp();
  ring.r.next(kPfItemRing);
  return item >= 0;
}

// Shape of one work item: its key tiles, the halves that hold rows and
// each half's key tiles.  Prefill: tl = (slot, q_row0, ntok, pos0), keys
// [0, pos0 + ntok) with the causal limit (half 0 ends up to 128/G tokens
// earlier).  Cascade: tl = (slot, first query record, count, part), keys
// [k0, k1) all visible to every row; a malformed task is flagged and
// skipped by every role alike (bad).
template <bool CASC>
struct PfItem {
  int4 tl;
  int kvh, k0, nkeys, nkt, n_half, nkt_h[2];
  bool bad;
  __device__ PfItem(const PrefillParams& p, int item, int4 t, int2 kr) : tl(t) {
    kvh = item % p.Hkv;
    if (CASC) {
      k0 = kr.x;
      nkeys = kr.y - kr.x;
      bad = tl.x < 0 || tl.y < 0 || tl.z <= 0 || tl.y + tl.z > p.n_toks || tl.z > p.NH * p.TT || tl.w < 0 || k0 < 0 ||
            nkeys <= 0 || (k0 & 15) || (nkeys & 15) || kr.y > p.max_blocks * p.bs;
      nkt = bad ? 0 : (nkeys + 127) >> 7;
      n_half = tl.z > p.TT ? 2 : 1;
      nkt_h[0] = nkt_h[1] = nkt;
    } else {
      k0 = 0;
      bad = false;
      const int ntok = min(tl.z, p.NH * p.TT);
      nkeys = tl.w + ntok;
      nkt = (nkeys + 127) >> 7;
      n_half = ntok > p.TT ? 2 : 1;
      nkt_h[0] = (tl.w + min(ntok, p.TT) + 127) >> 7;
      nkt_h[1] = nkt;
    }
  }
  __device__ bool active(int h, int j) const { return h < n_half && j >= 0 && j < nkt_h[h]; }
};

// Block id of 16-key block `lane` (< 8) of key tile j (keys >= nkeys: 0,
// not loaded); lanes 0..7 load theirs together, one round trip per tile.
__device__ __forceinline__ int pf_block_id(const PrefillParams& p, const int* btrow, int j, int nkeys, int k0,
                                           int lane) {
  const int key = (j * 8 + lane) * 16, lb = (k0 + key) / p.bs;
  if (lane >= 8 || key >= nkeys) return 0;
  return lb < p.max_blocks ? __ldg(btrow + lb) : -1;
}

// Copies of one 128-key K or V tile: lane b < nb copies 16-key block b
// (both 64-element parts of a head for head_dim 128) after lane 0 has
// armed the stage's barrier with the tile's bytes.
template <int D_>
__device__ __forceinline__ void pf_load_tile(const PrefillParams& p, const CUtensorMap* tm, uint32_t dst0,
                                             uint32_t full, int blk, int j, int nb, int kvh, int k0, uint64_t pol,
                                             int lane) {
  constexpr int NDH = D_ / 64;
  if (lane == 0) mbar_arrive_expect_tx(full, nb * NDH * 2048);
  __syncwarp();
  if (lane < nb) {
    const int off = (k0 + (j * 8 + lane) * 16) % p.bs;
    int phys = blk;
    if (phys < 0 || phys >= p.num_blocks) {
      atomicOr(p.status, NF_STATUS_BAD_BLOCK);
      phys = 0;
    }
#pragma unroll
    for (int dh = 0; dh < NDH; ++dh) {
      const uint32_t dst = dst0 + dh * 128 * 128 + lane * 2048;
      if constexpr (D_ == 64)
        tma_load_4d(dst, tm, 0, kvh, off, phys, full, pol);
      else
        tma_load_5d(dst, tm, 0, dh, kvh, off, phys, full, pol);
    }
  }
}

// The cascade item's query rows, gathered by tensor copies: row i * G + g
// of half h is query head kvh * G + g of the group's (h * TT + i)-th query
// (toks[first + ...]).  One copy per query (and 64-element part of a head)
// brings its G heads -- G consecutive 128-byte rows of the tile, swizzled
// by their shared-memory address exactly as a whole-tile copy would be.
// The query rows come first, 32 per register and all in one round trip;
// rows of the active halves past the group's last query are zeroed.  A row
// outside [0, rows) is flagged (the tensor copy would read zeros there).
template <int D_>
__device__ __forceinline__ void pf_gather_queries(const PrefillParams& p, const PfItem<true>& w, const CUtensorMap* tq,
                                                  uint32_t dst0, uint32_t full, uint64_t pol, int lane) {
  using C = PfCfg<D_>;
  constexpr int NDH = D_ / 64;
  const int G = p.G, lg = __ffs(G) - 1;  // G is a power of two
  const int nq = w.n_half * p.TT;        // query slots of the active halves
  const int n = min(w.tl.z, nq);
  int rowv[C::NH_ * 4];
#pragma unroll
  for (int s = 0; s < C::NH_ * 4; ++s) {
    const int i = s * 32 + lane;
    rowv[s] = i < n ? __ldg(p.toks + 2 * (w.tl.y + i) + 1) : 0;
  }
  const int zrow0 = n << lg, zrows = (nq - n) << lg;  // tile rows R = i * G + g over the active halves
  for (int c = lane; c < zrows * NDH * 8; c += 32) {
    const int R = zrow0 + c / (NDH * 8), rest = c % (NDH * 8);
    const uint32_t dst = dst0 + (R >> 7) * C::TILE + (rest >> 3) * 128 * 128 + (R & 127) * 128 + ((rest & 7) << 4);
    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0) : "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) mbar_arrive_expect_tx(full, n * G * 128 * NDH);
  __syncwarp();
#pragma unroll
  for (int s = 0; s < C::NH_ * 4; ++s) {
    const int i = s * 32 + lane;
    if (i < n) {
      const int row = rowv[s];
      if (row < 0 || row >= p.rows) atomicOr(p.status, NF_STATUS_BAD_SHARED);
      const int R = i << lg;
      const uint32_t d = dst0 + (R >> 7) * C::TILE + (R & 127) * 128;
#pragma unroll
      for (int dh = 0; dh < NDH; ++dh) {
        if constexpr (D_ == 64)
          tma_load_3d(d, tq, 0, w.kvh * G, row, full, pol);
        else
          tma_load_4d(d + dh * 128 * 128, tq, 0, dh, w.kvh * G, row, full, pol);
      }
    }
  }
}

// The producer warp: every lane runs the loop (waits included), lanes 0..7
// load block ids and issue the tensor copies.
template <int D_, bool CASC>
__device__ void pf_producer(const PrefillParams& p, const CUtensorMap* tq, const CUtensorMap* tk,
                            const CUtensorMap* tv, const PfBars& bar, uint32_t q_s, uint32_t k_s, uint32_t v_s,
                            PfItemRing& ring) {
  using C = PfCfg<D_>;
  constexpr int NDH = D_ / 64;
  const int lane = threadIdx.x & 31;
  const uint64_t pol = l2_evict_last();  // every query tile of a chunk reads the same keys
  const uint64_t pol_q = l2_evict_first();  // queries are read once
  Ring qr, kr, vr;
  int it, claims = 0;
  int4 itl;
  int2 ikr;
  while (pf_claim_item<CASC>(p, ring, it, itl, ikr, claims)) {
    const PfItem<CASC> w(p, it, itl, ikr);
    if (w.bad) {
      if (lane == 0) atomicOr(p.status, NF_STATUS_BAD_SHARED);
      continue;
    }
    // the item's query rows, both halves (one copy per half and 64-element part)
    if (!mbar_wait(bar.q_empty(qr.st), qr.ph ^ 1, p.status)) return;
    const uint32_t q_full = bar.q_full(qr.st);
    // block ids of key tile 0, requested before the query copies
    const int* btrow = p.bt + (long long)w.tl.x * p.max_blocks;
    int cur = pf_block_id(p, btrow, 0, w.nkeys, w.k0, lane);
    if constexpr (CASC) {
      // q may come from the launch before this one on the stream (a projection
      // launched ahead with programmatic serialization): wait for it here,
      // after the setup and the first records, before the first query copy
      if (claims == 1) pdl_wait();
      pf_gather_queries<D_>(p, w, tq, q_s + qr.st * C::NH_ * C::TILE, q_full, pol_q, lane);
    } else {
      const int nq = w.n_half * NDH;
      if (lane == 0) mbar_arrive_expect_tx(q_full, nq * 128 * 128);
      __syncwarp();
      if (lane < nq) {
        const int h = lane / NDH, dh = lane - h * NDH;
        const uint32_t dst = q_s + (qr.st * C::NH_ + h) * C::TILE + dh * 128 * 128;
        const int row0 = w.tl.y + h * p.TT;
        if constexpr (D_ == 64)
          tma_load_3d(dst, tq, 0, w.kvh * p.G, row0, q_full, pol_q);
        else
          tma_load_4d(dst, tq, 0, dh, w.kvh * p.G, row0, q_full, pol_q);
      }
    }
    qr.next(C::QST);
    for (int j = 0; j < w.nkt; ++j) {
      const int nb = min(8, (w.nkeys - j * 128 + 15) >> 4);
      if (!mbar_wait(bar.k_empty(kr.st), kr.ph ^ 1, p.status)) return;
      pf_load_tile<D_>(p, tk, k_s + kr.st * C::TILE, bar.k_full(kr.st), cur, j, nb, w.kvh, w.k0, pol, lane);
      kr.next(C::KST);
      if (!mbar_wait(bar.v_empty(vr.st), vr.ph ^ 1, p.status)) return;
      pf_load_tile<D_>(p, tv, v_s + vr.st * C::TILE, bar.v_full(vr.st), cur, j, nb, w.kvh, w.k0, pol, lane);
      vr.next(C::VST);
      if (j + 1 < w.nkt) cur = pf_block_id(p, btrow, j + 1, w.nkeys, w.k0, lane);
    }
  }
}

// The MMA warp: every lane runs the loop and its waits; lane 0 issues the
// MMAs and the commits that track them.
template <int D_, bool CASC>
__device__ void pf_mma(const PrefillParams& p, const PfBars& bar, uint32_t tmem, uint32_t q_s, uint32_t k_s,
                       uint32_t v_s, bool bf, PfItemRing& ring) {
  using C = PfCfg<D_>;
  const bool leader = elect_one();
  constexpr uint32_t REG = 128 * 128;  // one 64-element region of a 128-row operand
  const uint32_t idesc_s = umma_idesc_f16(bf, 128, 128, false, false);
  const uint32_t idesc_o = umma_idesc_f16(bf, 128, D_, false, true);
  Ring qr, kr, vr;
  int n_s[2] = {0, 0}, n_p[2] = {0, 0};
  auto wait_p = [&](int h) -> bool {
    if (!mbar_wait(bar.p_full(h), n_p[h] & 1, p.status)) return false;
    ++n_p[h];
    return true;
  };
  // Operands of tcgen05.mma live in warp-uniform registers: the tensor-memory
  // and shared-memory bases are broadcast from lane 0 so that the compiler
  // knows them uniform, and the descriptors of Q half 0, K stage 0 and V
  // stage 0 are built once; other stages, halves and k-steps are constant
  // offsets in the 16-byte address field (all below 2^18 bytes, so no carry
  // leaves it).  Lane 0 issues.
  tmem = __shfl_sync(0xffffffffu, tmem, 0);
  const uint64_t dq = umma_sdesc_sw128(__shfl_sync(0xffffffffu, q_s, 0), 16, 1024);
  const uint64_t dk = umma_sdesc_sw128(__shfl_sync(0xffffffffu, k_s, 0), 16, 1024);
  const uint64_t dv = umma_sdesc_sw128(__shfl_sync(0xffffffffu, v_s, 0), REG, 1024);
  // O_h += P_h V of the tile in V stage vst (first: overwrite O_h)
  auto issue_pv = [&](int h, int vst, bool first) {
    tc_fence_after();
    const uint64_t b0 = dv + (uint64_t)(vst * (C::TILE >> 4));
    const uint32_t d = tmem + C::o_col(h), a0 = tmem + C::p_col(h);
    if (leader) {
      umma_f16_ts(d, a0, b0, idesc_o, first ? 0u : 1u);
#pragma unroll
      for (int kk = 1; kk < 8; ++kk) umma_f16_ts(d, a0 + kk * 8, b0 + (uint64_t)(kk * 16 * 128 >> 4), idesc_o, 1u);
      umma_commit(bar.o_done(h));
    }
    __syncwarp();
  };
  auto issue_s = [&](int h, int kst) {
    const uint64_t a0 = dq + (uint64_t)((qr.st * C::NH_ + h) * (C::TILE >> 4)), b0 = dk + (uint64_t)(kst * (C::TILE >> 4));
    const uint32_t d = tmem + C::s_col(h);
    if (leader) {
#pragma unroll
      for (int k = 0; k < D_ / 16; ++k) {
        const uint64_t off = (uint64_t)(((k >> 2) * REG + (k & 3) * 32) >> 4);
        umma_f16_ss(d, a0 + off, b0 + off, idesc_s, k > 0 ? 1u : 0u);
      }
      umma_commit(bar.s_full(h));
    }
    __syncwarp();
  };
  int it;
  int4 itl;
  int2 ikr;
  while (ring.next(it, itl, ikr, p.status)) {
    const PfItem<CASC> w(p, it, itl, ikr);
    if (w.bad) continue;
    int vprev = -1;  // V stage of tile j-1
    if (!mbar_wait(bar.q_full(qr.st), qr.ph, p.status)) return;
    for (int j = 0; j < w.nkt; ++j) {
      if (!mbar_wait(bar.k_full(kr.st), kr.ph, p.status)) return;
#pragma unroll
      for (int h = 0; h < C::NH_; ++h) {
        if (C::P_ALIAS && w.active(h, j - 1)) {
          // P_h of tile j-1 sits in S_h: consume it before S_h is rewritten
          if (!wait_p(h)) return;
          issue_pv(h, vprev, j == 1);
        }
        if (!w.active(h, j)) continue;
        if (!C::P_ALIAS) {
          if (!mbar_wait(bar.s_free(h), (n_s[h] & 1) ^ 1, p.status)) return;
        }
        ++n_s[h];
        tc_fence_after();
        issue_s(h, kr.st);
      }
      if (leader) umma_commit(bar.k_empty(kr.st));
      kr.next(C::KST);
      if (j > 0) {
        if (!C::P_ALIAS) {
#pragma unroll
          for (int h = 0; h < C::NH_; ++h) {
            if (!w.active(h, j - 1)) continue;
            if (!wait_p(h)) return;
            issue_pv(h, vprev, j == 1);
          }
        }
        if (leader) umma_commit(bar.v_empty(vprev));
      }
      if (!mbar_wait(bar.v_full(vr.st), vr.ph, p.status)) return;
      vprev = vr.st;
      vr.next(C::VST);
    }
    // every S of the item is issued: the Q stage is free once they complete
    if (leader) umma_commit(bar.q_empty(qr.st));
    qr.next(C::QST);
    // the last tile: rows of V past the last key are zeroed by the last
    // half's warpgroup, so both halves' P must be in before either P V
    const int jl = w.nkt - 1;
#pragma unroll
    for (int h = 0; h < C::NH_; ++h)
      if (w.active(h, jl) && !wait_p(h)) return;
#pragma unroll
    for (int h = 0; h < C::NH_; ++h)
      if (w.active(h, jl)) issue_pv(h, vprev, jl == 0);
    if (leader) umma_commit(bar.v_empty(vprev));
  }
}

template <typename T, int D_, bool CASC>
__device__ void pf_softmax(const PrefillParams& p, const PfBars& bar, uint32_t tmem, uint32_t v_s, int h,
                           PfItemRing& ring) {
  using C = PfCfg<D_>;
  constexpr int NDH = D_ / 64;
  constexpr uint32_t REG = 128 * 128;
  constexpr bool kTurns = C::NH_ == 2 && kPfTurns;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3, row = quad * 32 + lane;  // tensor-memory lanes of this warp: quad*32..
  const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
  const uint32_t s_addr = tmem + lane_addr + C::s_col(h), o_addr = tmem + lane_addr + C::o_col(h);
  const uint32_t p_addr = tmem + lane_addr + C::p_col(h);
  const int G = p.G;
  int n_s = 0, n_o = 0;
  // Turns on the special-function unit: this warp and the other half's warp
  // on the same scheduler (same quad) take their exponent passes in turn,
  // half 0 first, so that one's loads, maxima and stores overlap the other's
  // exponentials.  turns counts the passes taken since the CTA started; a
  // pass waits on the other warp's previous one (mbarrier, time-limited).
  int turns = 0;
  const uint32_t my_turn = bar.turn(h, quad), other_turn = bar.turn(h ^ 1, quad);
  Ring vr;  // V ring position of this CTA's current tile (every item advances it)
  int it;
  int4 itl;
  int2 ikr;
  while (ring.next(it, itl, ikr, p.status)) {
    const PfItem<CASC> w(p, it, itl, ikr);
    if (w.bad) continue;
    if (!CASC && h == 0 && w.tl.z > p.NH * p.TT && threadIdx.x == 128) atomicOr(p.status, NF_STATUS_BAD_TILE);
    const Ring vlast = vr.ahead(w.nkt - 1, C::VST);  // V stage of the item's last tile
    vr = vr.ahead(w.nkt, C::VST);
    const bool active = h < w.n_half;
    const int nkt = active ? w.nkt_h[h] : 0;
    // both warps of a quad take one turn per key tile of the item's longer half
    const int rounds = kTurns ? w.nkt_h[w.n_half - 1] : nkt;
    const int tok = h * p.TT + row / G, hd = row % G;  // cascade: tok = the query's index in the group
    const bool valid = CASC ? tok < w.tl.z : (tok < min(w.tl.z, p.NH * p.TT) && w.tl.y + tok < p.rows);
    // the last visible key of the row, counted from the item's first key
    const int qpos = CASC ? w.nkeys - 1 : w.tl.w + tok;
    // cascade: the row's partial record, its three dependent loads issued now
    // so that they complete while the item's tiles stream
    float* rec = nullptr;
    if (CASC && valid) {
      const int item = __ldg(p.toks + 2 * (w.tl.y + tok));
      const int n_items = min(__ldg(p.counts), p.max_items);
      const int n_slots = min(__ldg(p.counts + 3), p.max_units);
      const int slot = item >= 0 && item < n_items ? __ldg(p.items + 4 * item + 3) + w.tl.w : -1;
      if (slot < 0 || slot >= n_slots)
        atomicOr(p.status, NF_STATUS_UNIT_OVERFLOW);
      else
        rec = p.ws + ((long long)slot * p.Hq + (long long)w.kvh * G + hd) * (D_ + 4);
    }
    float m = kPfNegInf, l = 0.f;
    for (int j = 0; j < rounds; ++j) {
      const bool has = j < nkt;
      uint32_t x[128];
      float mn = 0.f, alpha = 1.f, nbase = 0.f;
      uint64_t sum2[4];
      if (has) {
        if (!mbar_wait(bar.s_full(h), n_s & 1, p.status)) return;
        ++n_s;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(x + 32 * c));
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_reg_fence(*reinterpret_cast<uint32_t(*)[32]>(x + 32 * c));
        if (!C::P_ALIAS) {  // S_h is in registers: the next S_h may be computed
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar.s_free(h));
        }
        const int k0 = j * 128;
        const int lim = valid ? qpos - k0 : -1;  // columns <= lim are visible (key k <= qpos)
        if (!__all_sync(0xffffffffu, lim >= 127)) {  // some row of the warp crosses the diagonal
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i > lim) x[i] = __float_as_uint(kPfNegInf);
        }
        float acc[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) acc[a] = fmaxf(__uint_as_float(x[a]), __uint_as_float(x[a + 8]));
#pragma unroll
        for (int i = 16; i < 128; i += 16)
#pragma unroll
          for (int a = 0; a < 8; ++a) acc[a] = fmax3(acc[a], __uint_as_float(x[i + a]), __uint_as_float(x[i + 8 + a]));
        const float mt = fmaxf(fmaxf(fmaxf(acc[0], acc[1]), fmaxf(acc[2], acc[3])),
                               fmaxf(fmaxf(acc[4], acc[5]), fmaxf(acc[6], acc[7]))) * p.scale_log2;
        // lazy rescaling: the reference max moves (O and l rescaled) only when
        // the tile's max exceeds it by more than 8, so exponents stay <= 2^8
        const bool grow = mt > m + 8.f;
        mn = grow ? mt : m;
        alpha = grow ? ex2(m - mn) : 1.f;  // 0 on the first visible tile
        nbase = mn == kPfNegInf ? 0.f : -mn;
      }
      if (kTurns && (h == 1 || turns > 0)) {  // the other warp's previous exponent pass is done
        if (!mbar_wait(other_turn, (uint32_t)((turns - (h == 0 ? 1 : 0)) & 1), p.status)) return;
      }
      if (has) {
        // exponents (packed pairs: scale and offset in one fp32x2 FMA), row
        // sum, P packed in pairs into the low half of x
        const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2), nb2 = f2_pack(nbase, nbase);
#pragma unroll
        for (int a = 0; a < 4; ++a) sum2[a] = 0ull;
#pragma unroll
        for (int i = 0; i < 128; i += 2) {
          const uint64_t y2 = f2_fma(f2_pack(__uint_as_float(x[i]), __uint_as_float(x[i + 1])), sc2, nb2);
          float p0, p1;
          if (((i >> 1) & 7) < kPfPolyPairs) {
            exp2_poly2(y2, p0, p1);
          } else {
            float y0, y1;
            f2_unpack(y2, y0, y1);
            p0 = ex2(y0);
            p1 = ex2(y1);
          }
          sum2[(i >> 1) & 3] = f2_add(sum2[(i >> 1) & 3], f2_pack(p0, p1));
          x[i >> 1] = pack2<T>(p0, p1);
        }
      }
      if (kTurns) {  // this warp's exponent pass is done: the other warp's turn
        __syncwarp();
        if (lane == 0) mbar_arrive(my_turn);
        ++turns;
      }
      if (!has) continue;
      // O_h += P_h V of tile j-1 must be done before P_h is rewritten and
      // before O_h is rescaled (when a row's max moved)
      if (j > 0) {
        if (!mbar_wait(bar.o_done(h), n_o & 1, p.status)) return;
        ++n_o;
        tc_fence_after();
      }
      tmem_st32(p_addr, *reinterpret_cast<uint32_t(*)[32]>(x));
      tmem_st32(p_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(x + 32));
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int c = 0; c < D_ / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + c * 32, o);
          tmem_wait_ld();
          tmem_reg_fence(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(o_addr + c * 32, o);
        }
      }
      float sa[8];
#pragma unroll
      for (int a = 0; a < 4; ++a) f2_unpack(sum2[a], sa[2 * a], sa[2 * a + 1]);
      l = l * alpha + (((sa[0] + sa[1]) + (sa[2] + sa[3])) + ((sa[4] + sa[5]) + (sa[6] + sa[7])));
      m = mn;
      if (h == w.n_half - 1 && j == nkt - 1 && j * 128 + row >= w.nkeys) {
        // V rows past the item's last key (their P is 0) may hold anything:
        // zero them so that 0 * NaN cannot reach O
        if (!mbar_wait(bar.v_full(vlast.st), vlast.ph, p.status)) return;
        const uint32_t vs = v_s + vlast.st * C::TILE;
#pragma unroll
        for (int dh = 0; dh < NDH; ++dh)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(vs + dh * REG + row * 128 + c * 16), "r"(0)
                         : "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar.p_full(h));
    }
    if (!active) continue;
    // epilogue: O_h / l for the valid rows (cascade: the row's split-K part record)
    if (!mbar_wait(bar.o_done(h), n_o & 1, p.status)) return;
    ++n_o;
    tc_fence_after();
    if constexpr (CASC) {
#pragma unroll
      for (int c = 0; c < D_ / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_addr + c * 32, o);
        tmem_wait_ld();
        tmem_reg_fence(o);
        if (rec) {
          float4* r4 = reinterpret_cast<float4*>(rec + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            __stcg(r4 + i, make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                       __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3])));
        }
      }
      if (rec) __stcg(reinterpret_cast<float2*>(rec + D_), make_float2(m, l));
      tc_fence_before();
      continue;
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    T* dst = reinterpret_cast<T*>(p.out) + (long long)(w.tl.y + tok) * p.out_stride + (long long)(w.kvh * G + hd) * D_;
#pragma unroll
    for (int c = 0; c < D_ / 32; ++c) {
      uint32_t o[32];
      tmem_ld32(o_addr + c * 32, o);
      tmem_wait_ld();
      tmem_reg_fence(o);
      if (valid) {
        uint32_t wv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          wv[i] = pack2<T>(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) d4[i] = make_uint4(wv[4 * i], wv[4 * i + 1], wv[4 * i + 2], wv[4 * i + 3]);
        const long long off = reinterpret_cast<char*>(dst + c * 32) - p.out;
        for (int r = 0; r < p.n_peers; ++r) {
          uint4* e4 = reinterpret_cast<uint4*>(p.peer_out[r] + off);
#pragma unroll
          for (int i = 0; i < 4; ++i) e4[i] = make_uint4(wv[4 * i], wv[4 * i + 1], wv[4 * i + 2], wv[4 * i + 3]);
        }
      }
    }
    tc_fence_before();
  }
  // a gathered output: the rows stored to other GPUs are visible system-wide
  // before this warp is done (the launch that signals the peers follows)
  if (p.n_peers) __threadfence_system();
}

template <typename T, int D_, bool CASC>
__global__ void __launch_bounds__(PfCfg<D_>::THREADS, PfCfg<D_>::MINB)
    prefill_attention_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tq,
                             const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv) {
  using C = PfCfg<D_>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t hdr = smem_u32(base);
  const PfBars bar(hdr);
  const int warp = threadIdx.x >> 5;
  // cascade: the decode launch that follows may start as this grid's CTAs leave
  if (CASC) pdl_launch_dependents();
  // the tensor maps' descriptors, and (cascade: the first item of this CTA is
  // item blockIdx.x) its task record, are fetched during the setup
  if (threadIdx.x == 32) {
    tma_prefetch_map(&tk);
    tma_prefetch_map(&tv);
    tma_prefetch_map(&tq);
    if (CASC && (int)blockIdx.x < p.n_tiles * p.Hkv)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(p.tasks + 8 * (blockIdx.x / p.Hkv)));
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::KST; ++s) {
      mbar_init(bar.k_full(s), 1);
      mbar_init(bar.k_empty(s), 1);
    }
    for (int s = 0; s < C::VST; ++s) {
      mbar_init(bar.v_full(s), 1);
      mbar_init(bar.v_empty(s), 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(bar.s_full(h), 1);
      mbar_init(bar.s_free(h), 4);
      mbar_init(bar.p_full(h), 4);
      mbar_init(bar.o_done(h), 1);
    }
    for (int s = 0; s < C::QST; ++s) {
      mbar_init(bar.q_full(s), 1);
      mbar_init(bar.q_empty(s), 1);
    }
    for (int t = 0; t < 8; ++t) mbar_init(bar.turn(t >> 2, t & 3), 1);
    for (int s = 0; s < kPfItemRing; ++s) {
      mbar_init(bar.item_full(s), 1);
      mbar_init(bar.item_empty(s), 1 + 4 * C::NH_);  // the MMA warp and the softmax warps
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(hdr + kPfTmemPtr, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(base + kPfTmemPtr);
  const uint32_t q_s = hdr + C::Q_OFF, k_s = hdr + C::K_OFF, v_s = hdr + C::V_OFF;
  PfItemRing ring(bar, base);
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REGS_CTRL));
    if (warp == 0)
      pf_producer<D_, CASC>(p, &tq, &tk, &tv, bar, q_s, k_s, v_s, ring);
    else if (warp == 1)
      pf_mma<D_, CASC>(p, bar, tmem, q_s, k_s, v_s, std::is_same<T, __nv_bfloat16>::value, ring);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::REGS_SOFTMAX));
    pf_softmax<T, D_, CASC>(p, bar, tmem, v_s, (warp - 4) >> 2, ring);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
  // cascade: the grid ends after the launch before it, so that a launch waiting for this grid sees that one's
  // writes too
  if (CASC && threadIdx.x == 0) pdl_wait();
  // every claim of this CTA is made; the last CTA out rewinds the queue for the next launch
  if (!CASC && threadIdx.x == 0 && atomicAdd(p.queue + 1, 1) == (int)gridDim.x - 1) {
    atomicExch(p.queue, 0);
    atomicExch(p.queue + 1, 0);
  }
}

template <typename T, int D_, bool CASC = false>
static int launch_prefill(const PrefillParams& p, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          int n_items, cudaStream_t st) {
  using C = PfCfg<D_>;
  auto kern = prefill_attention_kernel<T, D_, CASC>;
  cudaError_t e = prepare_launch(reinterpret_cast<const void*>(kern), (int)C::SMEM, C::THREADS, nullptr);
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_prefill_attention: smem attribute: %s", cudaGetErrorString(e));
  // setmaxnreg moves registers between warpgroups within the launch total:
  // refuse a build whose register count would not cover the split
  // (the count is a property of the binary: queried once)
  static int regs = -1;
  if (regs < 0) {
    cudaFuncAttributes fa;
    regs = cudaFuncGetAttributes(&fa, kern) == cudaSuccess ? fa.numRegs : 0;
  }
  if (C::REGS_CTRL * 128 + C::REGS_SOFTMAX * 128 * C::NH_ > regs * C::THREADS)
    return fail(NF_EUNSUPPORTED, "nf_prefill_attention: kernel built with %d registers per thread, the warpgroup "
                "split needs %d", regs, C::LAUNCH_REGS);
  long long grid = n_items;
  if (grid > (long long)sm_count() * C::MINB) grid = (long long)sm_count() * C::MINB;
  if (!CASC) {
    kern<<<(int)grid, C::THREADS, C::SMEM, st>>>(p, tq, tk, tv);
    return check_launch("nf_prefill_attention");
  }
  // the cascade: programmatic stream serialization (the kernel waits for the
  // launch before it ahead of its first read of q), plain stream order where
  // the launch refuses the attribute
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p, tq, tk, tv);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    cfg.numAttrs = 0;
    e = cudaLaunchKernelEx(&cfg, kern, p, tq, tk, tv);
  }
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_cascade_attention: %s", cudaGetErrorString(e));
  return check_launch("nf_cascade_attention");
}

// nf_cascade_attention on the tensor cores: 16-bit pools, head_dim 64/128,
// 1/2/4/8 query heads per KV head, block size a multiple of 16; a task
// holds up to 256 / G queries and any whole number of 16-key groups.
int cascade_tensor_core(const CascTcArgs& a) {
  if (a.dtype != NF_BF16 && a.dtype != NF_F16) return NF_EUNSUPPORTED;
  if ((a.D != 64 && a.D != 128) || a.bs % 16) return NF_EUNSUPPORTED;
  const int G = a.Hq / a.Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return NF_EUNSUPPORTED;
  if (a.n_tasks == 0) return ok();
  // tq: boxes of one query row's G heads (the rows are gathered one copy per query)
  CUtensorMap tq, tk, tv;
  if (!encode_rows_map(&tq, a.q, a.dtype, a.D, a.Hq, a.q_rows, a.q_stride, G, 1) ||
      !encode_pool_map(&tk, a.kp, a.dtype, a.D, a.Hkv, a.bs, a.num_blocks, 1, false) ||
      !encode_pool_map(&tv, a.vp, a.dtype, a.D, a.Hkv, a.bs, a.num_blocks, 1, false))
    return fail(NF_ECUDA, "nf_cascade_attention: tensor map encoding failed");
  PrefillParams p = {};
  p.out = nullptr;
  p.q = static_cast<const char*>(a.q);
  p.q_stride = a.q_stride;
  p.rows = a.q_rows;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.G = G;
  p.TT = 128 / G;
  p.NH = pf_halves(a.D);
  p.bs = a.bs;
  p.num_blocks = a.num_blocks;
  p.bt = a.bt;
  p.max_blocks = a.max_blocks;
  p.n_tiles = a.n_tasks;
  p.order = nullptr;
  p.queue = nullptr;
  p.scale_log2 = a.scale_log2;
  p.status = a.status;
  p.n_peers = 0;
  p.tasks = a.tasks;
  p.toks = a.toks;
  p.n_toks = a.n_toks;
  p.items = a.items;
  p.counts = a.counts;
  p.ws = a.ws;
  p.max_items = a.max_items;
  p.max_units = a.max_units;
  const int n_items = a.n_tasks * a.Hkv;
  cudaStream_t st = static_cast<cudaStream_t>(a.stream);
  if (a.dtype == NF_BF16)
    return a.D == 64 ? launch_prefill<__nv_bfloat16, 64, true>(p, tq, tk, tv, n_items, st)
                     : launch_prefill<__nv_bfloat16, 128, true>(p, tq, tk, tv, n_items, st);
  return a.D == 64 ? launch_prefill<__half, 64, true>(p, tq, tk, tv, n_items, st)
                   : launch_prefill<__half, 128, true>(p, tq, tk, tv, n_items, st);
}

}  // namespace nf

extern "C" int nf_prefill_tile_rows(int32_t head_dim) { return 128 * nf::pf_halves(head_dim); }

extern "C" int nf_prefill_attention_gather(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                           int32_t num_rows, const void* k_pool, const void* v_pool, int32_t dtype,
                                           int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                           int32_t block_size, int32_t num_blocks, const int32_t* block_tables,
                                           int32_t max_blocks_per_seq, const int32_t* tiles, int32_t n_tiles,
                                           const int32_t* order, int32_t* queue, float scale, const NfGather* gather,
                                           int32_t* status, void* stream) {
  using namespace nf;
  int n_peers = 0;
  if (gather) {
    if (gather->n_ranks < 1 || gather->n_ranks > kMaxRanks || gather->rank < 0 || gather->rank >= gather->n_ranks)
      return fail(NF_EINVAL, "nf_prefill_attention: gathered output of %d ranks (1..%d), rank %d", gather->n_ranks,
                  kMaxRanks, gather->rank);
    n_peers = gather->n_ranks - 1;
    for (int r = 0; r < n_peers; ++r)
      if (!gather->peer_out[r] || (reinterpret_cast<uintptr_t>(gather->peer_out[r]) & 15))
        return fail(NF_EINVAL, "nf_prefill_attention: peer_out[%d] is null or not 16-byte aligned", r);
  }
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
  if (n_tiles < 0 || num_blocks <= 0 || max_blocks_per_seq <= 0 || num_rows <= 0)
    return fail(NF_EINVAL, "nf_prefill_attention: sizes must be positive");
  if (n_tiles == 0) return ok();
  if (!out || !q || !k_pool || !v_pool || !block_tables || !tiles || !status)
    return fail(NF_EINVAL, "nf_prefill_attention: null pointer argument");
  if (!queue) return fail(NF_EINVAL, "nf_prefill_attention: null work queue");
  auto al = [](const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
  if (!al(q, 16) || !al(out, 16) || (q_row_stride * 2) % 16 || (out_row_stride * 2) % 16 || !al(tiles, 16) ||
      !al(k_pool, 16) || !al(v_pool, 16))
    return fail(NF_EINVAL, "nf_prefill_attention: q/out rows, pools and tiles must be 16-byte aligned");
  CUtensorMap tq, tk, tv;
  if (!encode_rows_map(&tq, q, dtype, head_dim, num_q_heads, num_rows, q_row_stride, G, 128 / G) ||
      !encode_pool_map(&tk, k_pool, dtype, head_dim, num_kv_heads, block_size, num_blocks, 1, false) ||
      !encode_pool_map(&tv, v_pool, dtype, head_dim, num_kv_heads, block_size, num_blocks, 1, false))
    return fail(NF_ECUDA, "nf_prefill_attention: tensor map encoding failed");
  PrefillParams p;
  p.out = static_cast<char*>(out);
  p.out_stride = out_row_stride;
  p.q = static_cast<const char*>(q);
  p.q_stride = q_row_stride;
  p.rows = num_rows;
  p.Hq = num_q_heads;
  p.Hkv = num_kv_heads;
  p.G = G;
  p.TT = 128 / G;
  p.NH = pf_halves(head_dim);
  p.bs = block_size;
  p.num_blocks = num_blocks;
  p.bt = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  p.order = order;
  p.queue = queue;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  p.n_peers = n_peers;
  for (int r = 0; r < n_peers; ++r) p.peer_out[r] = static_cast<char*>(gather->peer_out[r]);
  const int n_items = n_tiles * num_kv_heads;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == NF_BF16)
    return head_dim == 64 ? launch_prefill<__nv_bfloat16, 64>(p, tq, tk, tv, n_items, st)
                          : launch_prefill<__nv_bfloat16, 128>(p, tq, tk, tv, n_items, st);
  return head_dim == 64 ? launch_prefill<__half, 64>(p, tq, tk, tv, n_items, st)
                        : launch_prefill<__half, 128>(p, tq, tk, tv, n_items, st);
}

extern "C" int nf_prefill_attention(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                    int32_t num_rows, const void* k_pool, const void* v_pool, int32_t dtype,
                                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                    int32_t num_blocks, const int32_t* block_tables, int32_t max_blocks_per_seq,
                                    const int32_t* tiles, int32_t n_tiles, const int32_t* order, int32_t* queue,
                                    float scale, int32_t* status, void* stream) {
  return nf_prefill_attention_gather(out, out_row_stride, q, q_row_stride, num_rows, k_pool, v_pool, dtype,
                                     num_q_heads, num_kv_heads, head_dim, block_size, num_blocks, block_tables,
                                     max_blocks_per_seq, tiles, n_tiles, order, queue, scale, nullptr, status, stream);
}
