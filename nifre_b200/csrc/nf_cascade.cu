// Cascade attention over keys that several decode queries share.
//
// When sequences of a step start with the same physical blocks (prompt
// prefixes imported from the prefix index, jyotilakra92/nifre
// src/inference/prefix_cache.py:33-81 and paged_kv_cache.py:87-105), the
// split-K decode kernel would stream those blocks once per sequence.  With
// 1, 2, 4 or 8 query heads per KV head (G) the tasks run on the tensor cores,
// in the cascade mode of the prefill kernel (nf_prefill.cu,
// cascade_tensor_core); this file holds the entry point, the task limits
// and, for other group sizes, an mma.sync kernel: a CTA takes the queries of
// up to 128 / G of those sequences for one KV head (G query heads each: up
// to 128 query rows) and one range of the shared keys (at most 256), stages
// its K and V in shared memory once, and computes for every row the partial
// softmax state over that range: the
// unnormalised sum of 2^(s - m) v, its maximum m and its weight l, with s
// the score times scale * log2(e) -- the same partial record the decode
// kernel writes for a key range of an item, in the item's partial slot
// unit_base + part.  The decode launch that follows covers each query's own
// keys as its later parts and merges all of them (nf_attn_common.cuh).
//
// Layout of the work: one CTA per (task, KV head), 8 warps of 16 query rows
// (row = sequence * G + head).  The range's block ids are read once into
// shared memory, then every 64-key slice of the range is requested at once
// by 16-byte asynchronous copies, so the copies' latency is paid once per
// CTA and each slice is consumed as it lands: S = Q K^T and O += P V on the
// tensor cores (m16n8k16), online softmax in registers.  The work is small next to the
// bytes it saves (128 rows x a few thousand keys per prefix and head), so a
// simple kernel that reads each shared block once per (group of sequences,
// KV head) is enough.
#include "nf_common.cuh"
#include "nf_internal.h"

namespace nf {

struct CascadeParams {
  float* ws;  // partials [slots][Hq][D + 4]: acc[D], m, l, pad
  const char* q;
  long long q_stride;  // elements between query rows
  int q_rows;          // rows of q: a query row outside [0, q_rows) is flagged
  const char* kp;
  const char* vp;
  int Hq, Hkv, D, G, bs, num_blocks;
  const int* bt;
  int max_blocks;
  const int* items;   // per query token: slot, q_row, kv_len, unit_base
  const int* counts;  // of nf_pack_step: [0] tokens, [3] partial slots
  int max_items, max_units;
  const int* tasks;   // [n_tasks][8]: slot, first, count, part, key_begin, key_end, 0, 0
  int n_tasks;
  const int* toks;    // [n_toks][2]: item (query token), q row
  int n_toks;
  float scale_log2;
  int* status;
};

constexpr int kCascRows = 128;     // query rows per CTA (8 warps x 16)
constexpr int kCascThreads = 256;
constexpr int kCascKeys = 64;      // keys per staged slice
constexpr int kCascStages = 4;     // slices per CTA: key ranges of at most 256 keys

__host__ __device__ constexpr int casc_pitch(int D) { return D * 2 + 16; }  // padded row: conflict-free ldmatrix

template <typename T, int D_>
__device__ __forceinline__ void cascade_body(const CascadeParams& p, unsigned char* casc_smem) {
  constexpr int PITCH = casc_pitch(D_);
  constexpr int SLICE = kCascKeys * PITCH;  // bytes of one slice of K (or V)
  constexpr int KS = D_ / 16;               // k-steps of Q K^T
  constexpr int NO = D_ / 8;                // n-tiles of the output
  constexpr int CHUNKS = D_ / 8;            // 16-byte chunks per key row
  const int task = blockIdx.x, kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // the task: ta = (slot whose table holds the shared blocks, first query, queries, part), tb.x/y = keys
  const int4 ta = __ldg(reinterpret_cast<const int4*>(p.tasks) + 2 * task);
  const int4 tb = __ldg(reinterpret_cast<const int4*>(p.tasks) + 2 * task + 1);
  const int k0 = tb.x, k1 = tb.y;
  if (ta.x < 0 || ta.y < 0 || ta.z <= 0 || ta.y + ta.z > p.n_toks || ta.z > kCascRows / p.G || ta.w < 0 ||
      k0 < 0 || k1 <= k0 || (k0 & 15) || (k1 & 15) || k1 > p.max_blocks * p.bs ||
      k1 - k0 > kCascStages * kCascKeys) {
    if (tid == 0) atomicOr(p.status, NF_STATUS_BAD_SHARED);
    return;
  }
  // this thread's rows: r0 = 16 warp + lane / 4 and r0 + 8 (row = query * G + head); their
  // records are requested now, beside the block ids
  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8;
  const int rows = ta.z * p.G;
  const bool live = warp * 16 < rows;  // warps past the last row only stage
  int2 tq0 = make_int2(-1, 0), tq1 = make_int2(-1, 0);
  if (r0 < rows) tq0 = __ldg(reinterpret_cast<const int2*>(p.toks) + ta.y + r0 / p.G);
  if (r1 < rows) tq1 = __ldg(reinterpret_cast<const int2*>(p.toks) + ta.y + r1 / p.G);
  const int n_items = min(__ldg(p.counts), p.max_items);
  const int n_slots = min(__ldg(p.counts + 3), p.max_units);
  const int* btrow = p.bt + (long long)ta.x * p.max_blocks;
  const uint32_t sK = smem_u32(casc_smem), sV = sK + kCascStages * SLICE;

  // pool row of the first key of each 16-key group of the range (-1: a bad block id)
  __shared__ long long grp_row[kCascStages * kCascKeys / 16];
  const int n_grp = (k1 - k0) >> 4;
  if (tid < n_grp) {
    const int key = k0 + 16 * tid;
    const int blk = __ldg(btrow + key / p.bs);
    if (blk < 0 || blk >= p.num_blocks) {
      atomicOr(p.status, NF_STATUS_BAD_BLOCK);
      grp_row[tid] = -1;
    } else {
      grp_row[tid] = (long long)blk * p.bs + key % p.bs;
    }
  }
  __syncthreads();
  // every slice of the range in flight at once, one copy group per slice;
  // rows past the range are zeros (their scores are masked; 0 * P stays 0)
  const int n_slices = (k1 - k0 + kCascKeys - 1) / kCascKeys;
  for (int i = 0; i < n_slices; ++i) {
    for (int c = tid; c < kCascKeys * CHUNKS; c += kCascThreads) {
      const int r = c / CHUNKS, ch = c - r * CHUNKS;
      const int g = i * (kCascKeys / 16) + (r >> 4);
      const uint32_t dk = sK + i * SLICE + r * PITCH + ch * 16, dv = sV + i * SLICE + r * PITCH + ch * 16;
      const long long row0 = g < n_grp ? grp_row[g] : -1;
      if (row0 >= 0) {
        const long long row = (row0 + (r & 15)) * p.Hkv + kvh;
        cp_async16(dk, p.kp + (row * D_ + ch * 8) * 2);
        cp_async16(dv, p.vp + (row * D_ + ch * 8) * 2);
      } else {
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dk), "r"(0) : "memory");
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dv), "r"(0) : "memory");
      }
    }
    cp_async_commit();
  }

  const bool row0_ok = tq0.y >= 0 && tq0.y < p.q_rows, row1_ok = tq1.y >= 0 && tq1.y < p.q_rows;
  if ((tq0.x >= 0 && !row0_ok) || (tq1.x >= 0 && !row1_ok)) atomicOr(p.status, NF_STATUS_BAD_SHARED);
  const int tok0 = tq0.x >= 0 && tq0.x < n_items && row0_ok ? tq0.x : -1;
  const int tok1 = tq1.x >= 0 && tq1.x < n_items && row1_ok ? tq1.x : -1;
  // partial slots of the rows' items (checked at the store), requested beside the query rows
  int base0 = -1, next0 = 0, base1 = -1, next1 = 0;
  if (tok0 >= 0) {
    base0 = __ldg(p.items + 4 * tok0 + 3);
    next0 = tok0 + 1 < n_items ? __ldg(p.items + 4 * (tok0 + 1) + 3) : n_slots;
  }
  if (tok1 >= 0) {
    base1 = __ldg(p.items + 4 * tok1 + 3);
    next1 = tok1 + 1 < n_items ? __ldg(p.items + 4 * (tok1 + 1) + 3) : n_slots;
  }
  // Q fragments (A operand, rows r0/r1, columns 16 ks + 2 (lane % 4) (+1, +8, +9)); the q rows
  // come with the query records (the rows nf_pack_step gives these items)
  uint32_t qa[KS][4];
  {
    const T* q0 = nullptr;
    const T* q1 = nullptr;
    if (tok0 >= 0)
      q0 = reinterpret_cast<const T*>(p.q) + (long long)tq0.y * p.q_stride + (long long)(kvh * p.G + r0 % p.G) * D_;
    if (tok1 >= 0)
      q1 = reinterpret_cast<const T*>(p.q) + (long long)tq1.y * p.q_stride + (long long)(kvh * p.G + r1 % p.G) * D_;
    const int c = 2 * (lane & 3);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qa[ks][0] = q0 ? __ldg(reinterpret_cast<const uint32_t*>(q0 + 16 * ks + c)) : 0u;
      qa[ks][1] = q1 ? __ldg(reinterpret_cast<const uint32_t*>(q1 + 16 * ks + c)) : 0u;
      qa[ks][2] = q0 ? __ldg(reinterpret_cast<const uint32_t*>(q0 + 16 * ks + c + 8)) : 0u;
      qa[ks][3] = q1 ? __ldg(reinterpret_cast<const uint32_t*>(q1 + 16 * ks + c + 8)) : 0u;
    }
  }
  float o[NO][4];
#pragma unroll
  for (int i = 0; i < NO; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  // ldmatrix lane addresses: K rows (keys) for B of Q K^T, V rows (keys) for B of P V
  const int mk = lane >> 3, rk = lane & 7;
  const int k_key = (mk >> 1) * 8 + rk, k_col = (mk & 1) * 8;  // non-transposed: (keys, d) quadrants
  const int v_key = (mk & 1) * 8 + rk, v_col = (mk >> 1) * 8;  // transposed
  for (int i = 0; i < n_slices; ++i) {
    cp_async_wait(n_slices - 1 - i);  // slice i has landed (this thread's copies)
    __syncthreads();                  // ... and every thread's
    if (live) {
      const uint32_t kb = sK + i * SLICE, vb = sV + i * SLICE;
      float s[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kb + (16 * j2 + k_key) * PITCH + (16 * ks + k_col) * 2, b0, b1, b2, b3);
          mma16816<T>(s[2 * j2], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
          mma16816<T>(s[2 * j2 + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
        }
      }
      // scale, mask keys past the range, running maximum per row
      const int kbase = k0 + i * kCascKeys + 2 * (lane & 3);
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const bool v0 = kbase + 8 * j < k1, v1 = kbase + 8 * j + 1 < k1;
        s[j][0] = v0 ? s[j][0] * p.scale_log2 : -INFINITY;
        s[j][1] = v1 ? s[j][1] * p.scale_log2 : -INFINITY;
        s[j][2] = v0 ? s[j][2] * p.scale_log2 : -INFINITY;
        s[j][3] = v1 ? s[j][3] * p.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
        mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float b0 = mn0 == -INFINITY ? 0.f : mn0, b1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = ex2(m0 - b0), al1 = ex2(m1 - b1);
      m0 = mn0;
      m1 = mn1;
      l0 *= al0;
      l1 *= al1;
#pragma unroll
      for (int n = 0; n < NO; ++n) {
        o[n][0] *= al0;
        o[n][1] *= al0;
        o[n][2] *= al1;
        o[n][3] *= al1;
      }
      uint32_t pa[4][4];  // P as the A operand of P V, 16 keys per k-step
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float e0 = ex2(s[j][0] - b0), e1 = ex2(s[j][1] - b0);
        const float e2 = ex2(s[j][2] - b1), e3 = ex2(s[j][3] - b1);
        l0 += e0 + e1;
        l1 += e2 + e3;
        pa[j >> 1][(j & 1) * 2] = pack2<T>(e0, e1);
        pa[j >> 1][(j & 1) * 2 + 1] = pack2<T>(e2, e3);
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int dd = 0; dd < D_ / 16; ++dd) {
          uint32_t v0, v1, v2, v3;
          ldsm_x4_t(vb + (16 * kk + v_key) * PITCH + (16 * dd + v_col) * 2, v0, v1, v2, v3);
          mma16816<T>(o[2 * dd], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], v0, v1);
          mma16816<T>(o[2 * dd + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], v2, v3);
        }
      }
    }
  }
  if (!live) return;
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  // partial records: slot unit_base + part of each row's item, inside that item's slots
  auto store = [&](int tok, int base, int next, int r, float (&acc)[NO][4], int h, float m, float l) {
    if (tok < 0) return;
    const int slot = base + ta.w;
    if (base < 0 || slot >= next || slot >= p.max_units) {
      if ((lane & 3) == 0) atomicOr(p.status, NF_STATUS_UNIT_OVERFLOW);
      return;
    }
    float* w = p.ws + ((long long)slot * p.Hq + kvh * p.G + r % p.G) * (D_ + 4);
    const int c = 2 * (lane & 3);
#pragma unroll
    for (int n = 0; n < NO; ++n)
      __stcg(reinterpret_cast<float2*>(w + 8 * n + c), make_float2(acc[n][h], acc[n][h + 1]));
    if ((lane & 3) == 0) __stcg(reinterpret_cast<float2*>(w + D_), make_float2(m, l));
  };
  store(tok0, base0, next0, r0, o, 0, m0, l0);
  store(tok1, base1, next1, r1, o, 2, m1, l1);
}

// Launched with programmatic stream serialization behind the step's KV
// append (or prefill), whose writes it does not read: the shared blocks are
// full and the append fills only each sequence's own last block.  So the
// launch starts while that kernel runs, lets the decode launch that follows
// start as its CTAs free SMs (the decode waits for this grid before reading
// the pools), and ends only after the kernel before it has ended, so that
// whatever waits for this grid also sees that kernel's writes.
template <typename T, int D_>
__global__ void __launch_bounds__(kCascThreads, D_ == 64 ? 2 : 1) cascade_kernel(const CascadeParams p) {
  extern __shared__ __align__(128) unsigned char casc_smem[];
  pdl_launch_dependents();
  cascade_body<T, D_>(p, casc_smem);
  if (threadIdx.x == 0) pdl_wait();
}

}  // namespace nf

namespace nf {
// The tensor-core path (the prefill kernel's pipeline, nf_prefill.cu) serves
// 16-bit pools with head_dim 64/128, 1, 2, 4 or 8 query heads per KV head and
// block sizes that are multiples of 16; other shapes use this file's kernel.
static bool cascade_on_tensor_cores(int dtype, int Hq, int Hkv, int D, int bs) {
  if ((dtype != NF_BF16 && dtype != NF_F16) || (D != 64 && D != 128) || bs % 16 || Hkv <= 0 || Hq % Hkv) return false;
  const int G = Hq / Hkv;
  return G == 1 || G == 2 || G == 4 || G == 8;
}
}  // namespace nf

extern "C" int nf_cascade_limits(int32_t dtype, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                 int32_t block_size, int32_t* max_rows, int32_t* max_keys) {
  using namespace nf;
  if (!max_rows || !max_keys) return fail(NF_EINVAL, "nf_cascade_limits: null pointer argument");
  if (cascade_on_tensor_cores(dtype, num_q_heads, num_kv_heads, head_dim, block_size)) {
    *max_rows = 256;       // two 128-row halves sharing the task's K/V stream
    *max_keys = 1 << 30;   // any whole number of 16-key groups
  } else {
    *max_rows = kCascRows;
    *max_keys = kCascStages * kCascKeys;
  }
  return ok();
}

extern "C" int nf_cascade_attention(float* ws_partials, int64_t ws_partial_floats, const void* q, int64_t q_row_stride,
                                    int32_t num_q_rows,
                                    const void* k_pool, const void* v_pool, int32_t dtype, int32_t num_q_heads,
                                    int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                    const int32_t* block_tables, int32_t max_blocks_per_seq, const int32_t* items,
                                    const int32_t* counts, int32_t max_items, int32_t max_units,
                                    const int32_t* tasks, int32_t n_tasks, const int32_t* toks, int32_t n_toks,
                                    float scale, int32_t* status, void* stream) {
  using namespace nf;
  if (n_tasks == 0) return ok();
  if (dtype != NF_BF16 && dtype != NF_F16)
    return fail(NF_EUNSUPPORTED, "nf_cascade_attention: 16-bit pools only (dtype %d)", dtype);
  if (head_dim != 64 && head_dim != 128)
    return fail(NF_EUNSUPPORTED, "nf_cascade_attention: head_dim %d (64 or 128)", head_dim);
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads)
    return fail(NF_EINVAL, "nf_cascade_attention: %d query heads over %d KV heads", num_q_heads, num_kv_heads);
  const int G = num_q_heads / num_kv_heads;
  if (G > kCascRows) return fail(NF_EUNSUPPORTED, "nf_cascade_attention: %d query heads per KV head", G);
  if (block_size <= 0 || block_size % 16)
    return fail(NF_EUNSUPPORTED, "nf_cascade_attention: block_size %d is not a multiple of 16", block_size);
  if (!ws_partials || !q || !k_pool || !v_pool || !block_tables || !items || !counts || !tasks || !toks || !status)
    return fail(NF_EINVAL, "nf_cascade_attention: null pointer argument");
  if (n_tasks < 0 || n_toks <= 0 || num_q_rows <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0 || max_items <= 0 ||
      max_units <= 0)
    return fail(NF_EINVAL, "nf_cascade_attention: sizes must be positive");
  if ((int64_t)max_units * num_q_heads * (head_dim + 4) > ws_partial_floats)
    return fail(NF_EINVAL, "nf_cascade_attention: workspace holds fewer than max_units partial slots");
  auto al = [](const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
  if (!al(k_pool, 16) || !al(v_pool, 16) || !al(q, 4) || (q_row_stride * 2) % 4 != 0)
    return fail(NF_EINVAL, "nf_cascade_attention: pools must be 16-byte and q rows 4-byte aligned");
  if (!al(ws_partials, 8) || !al(items, 16) || !al(tasks, 16) || !al(toks, 8))
    return fail(NF_EINVAL, "nf_cascade_attention: items and tasks must be 16-byte, toks 8-byte aligned");
  if (n_tasks > 65535 * 1024) return fail(NF_EINVAL, "nf_cascade_attention: too many tasks (%d)", n_tasks);
  if (cascade_on_tensor_cores(dtype, num_q_heads, num_kv_heads, head_dim, block_size)) {
    if (!al(q, 16) || (q_row_stride * 2) % 16 != 0)
      return fail(NF_EINVAL, "nf_cascade_attention: q rows must be 16-byte aligned");
    CascTcArgs a;
    a.ws = ws_partials;
    a.q = q;
    a.q_stride = q_row_stride;
    a.q_rows = num_q_rows;
    a.kp = k_pool;
    a.vp = v_pool;
    a.dtype = dtype;
    a.Hq = num_q_heads;
    a.Hkv = num_kv_heads;
    a.D = head_dim;
    a.bs = block_size;
    a.num_blocks = num_blocks;
    a.bt = block_tables;
    a.max_blocks = max_blocks_per_seq;
    a.items = items;
    a.counts = counts;
    a.max_items = max_items;
    a.max_units = max_units;
    a.tasks = tasks;
    a.n_tasks = n_tasks;
    a.toks = toks;
    a.n_toks = n_toks;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.status = status;
    a.stream = stream;
    return cascade_tensor_core(a);
  }
  CascadeParams p;
  p.ws = ws_partials;
  p.q = static_cast<const char*>(q);
  p.q_stride = q_row_stride;
  p.q_rows = num_q_rows;
  p.kp = static_cast<const char*>(k_pool);
  p.vp = static_cast<const char*>(v_pool);
  p.Hq = num_q_heads;
  p.Hkv = num_kv_heads;
  p.D = head_dim;
  p.G = G;
  p.bs = block_size;
  p.num_blocks = num_blocks;
  p.bt = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.items = items;
  p.counts = counts;
  p.max_items = max_items;
  p.max_units = max_units;
  p.tasks = tasks;
  p.n_tasks = n_tasks;
  p.toks = toks;
  p.n_toks = n_toks;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  const int smem = 2 * kCascStages * kCascKeys * casc_pitch(head_dim);
  const dim3 grid((unsigned)n_tasks, (unsigned)num_kv_heads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kCascThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // programmatic serialization where the launch accepts it, else plain stream order
#define NF_CASC_LAUNCH(T, D)                                                                               \
  do {                                                                                                     \
    e = cudaFuncSetAttribute(cascade_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);     \
    if (e == cudaSuccess) {                                                                                \
      e = cudaLaunchKernelEx(&cfg, cascade_kernel<T, D>, p);                                               \
      if (e != cudaSuccess) {                                                                              \
        (void)cudaGetLastError();                                                                          \
        cfg.numAttrs = 0;                                                                                  \
        e = cudaLaunchKernelEx(&cfg, cascade_kernel<T, D>, p);                                             \
      }                                                                                                    \
    }                                                                                                      \
  } while (0)
  if (dtype == NF_BF16) {
    if (head_dim == 64) NF_CASC_LAUNCH(__nv_bfloat16, 64); else NF_CASC_LAUNCH(__nv_bfloat16, 128);
  } else {
    if (head_dim == 64) NF_CASC_LAUNCH(__half, 64); else NF_CASC_LAUNCH(__half, 128);
  }
#undef NF_CASC_LAUNCH
  if (e != cudaSuccess) return fail(NF_ECUDA, "nf_cascade_attention: %s", cudaGetErrorString(e));
  return check_launch("nf_cascade_attention");
}
