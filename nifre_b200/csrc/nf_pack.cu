// GPU-side packing of one step's ragged batch.
//
// Replaces the per-row / per-token host loops of the reference step
// (jyotilakra92/nifre src/inference/): batching.py:8-19 (left padding),
// model_runner.py:39-50,73-75 (chunk slicing and slot lists),
// models/gpt.py:108-126 (positions read back from kv_cache.pos),
// paged_kv_cache.py:107-121 + block_table.py:36-40 (per-token resolve).
// One CTA does the whole step: a step holds at most a few thousand tokens
// (the reference token budget is 2048 by default, 4096 at most in the
// auto-tuner's range), which one CTA scans in a few microseconds, and a
// single launch keeps the per-step host work to one upload.
#include "nf_common.cuh"
#include "nf_internal.h"

namespace nf {

struct PackParams {
  const int* seqs;
  int n_seqs;
  const int* patches;
  int n_patches;
  int* bt;
  int num_slots, max_blocks, bs, num_blocks, split;
  const int* seq_split;  // per-sequence unit size (NULL: split for all)
  const int* seq_shared; // per sequence: keys [0, shared) served by cascade parts, their count (NULL: none)
  int* slot_mapping;
  int* src_rows;
  long long* positions;
  int* items;
  int* units;
  int* counts;
  int n_tokens, max_units;
  int* status;
};

constexpr int kPackThreads = 1024;

// One round of a CTA-wide exclusive scan: returns carry + the sum of x over
// the threads before this one, and advances every thread's carry by the
// round's total.  Every thread of the CTA calls it.
__device__ int cta_scan_round(int x, int& carry) {
  __shared__ int warp_tot[32];
  __shared__ int round_tot;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = warp_tot[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    warp_tot[lane] = wi - w;  // exclusive prefix of the warp totals
    if (lane == 31) round_tot = wi;
  }
  __syncthreads();
  const int excl = carry + warp_tot[warp] + incl - x;
  carry += round_tot;
  __syncthreads();  // warp_tot and round_tot are rewritten by the next round
  return excl;
}

// Exclusive scan, in place, of a[i * stride] for i < n by one CTA.
// Returns the total to every thread.
__device__ int cta_exclusive_scan(int* a, int n, int stride) {
  int carry = 0;
  for (int base = 0; base < n; base += kPackThreads) {
    const int i = base + threadIdx.x;
    const int x = (i < n) ? a[(long long)i * stride] : 0;
    const int e = cta_scan_round(x, carry);
    if (i < n) a[(long long)i * stride] = e;
  }
  return carry;
}

// Sequence of token t: the last s with cu[s] <= t (cu = query offsets).
__device__ __forceinline__ int seq_of(const int* cu, int n_seqs, int t) {
  int lo = 0, hi = n_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Unit size of sequence s: its seq_split entry when that is a positive
// multiple of 16, 0 when the entry is 0 (the sequence's queries are left to
// another kernel: no units), else the step's split.
__device__ __forceinline__ int unit_size(const PackParams& p, int s) {
  if (!p.seq_split) return p.split;
  const int v = p.seq_split[s];
  if (v == 0) return 0;
  return (v > 0 && (v & 15) == 0) ? v : p.split;
}

__device__ __forceinline__ int parts_of(int kv_len, int us) { return us > 0 ? (kv_len + us - 1) / us : 0; }

// Keys [0, shared) of sequence s and the number nc of cascade parts that
// hold their partial results (both 0 without a record).  A record must leave
// the query at least one key of its own (0 < shared < kv_len) and belong to
// a sequence with units; otherwise the sequence is flagged, its cascade
// slots are kept (nf_cascade_attention may write them) and its own keys
// are skipped.
__device__ __forceinline__ void shared_of(const PackParams& p, int s, int kv_len, int& shared, int& nc) {
  shared = nc = 0;
  if (!p.seq_shared) return;
  const int sh = p.seq_shared[2 * s], n = p.seq_shared[2 * s + 1];
  if (sh == 0 && n == 0) return;
  nc = min(max(n, 0), 1 << 16);
  if (sh > 0 && sh < kv_len && n > 0 && unit_size(p, s) > 0) {
    shared = sh;
  } else {
    shared = kv_len;
    atomicOr(p.status, NF_STATUS_BAD_SHARED);
  }
}

__global__ void __launch_bounds__(kPackThreads) pack_kernel(const PackParams p) {
  extern __shared__ int cu[];  // n_seqs + 1 query offsets
  const int tid = threadIdx.x;

  // 1. block-table writes recorded by the host allocator for this step.
  for (int i = tid; i < p.n_patches; i += kPackThreads) {
    const int slot = p.patches[3 * i], lb = p.patches[3 * i + 1], phys = p.patches[3 * i + 2];
    if (slot < 0 || slot >= p.num_slots || lb < 0 || lb >= p.max_blocks || phys < 0 || phys >= p.num_blocks) {
      atomicOr(p.status, NF_STATUS_BAD_BLOCK);
      continue;
    }
    p.bt[(long long)slot * p.max_blocks + lb] = phys;
  }
  __shared__ int multi_sh, cross_sh, max_parts_sh, first_sh;
  if (tid == 0) {
    multi_sh = cross_sh = max_parts_sh = 0;
    first_sh = 1 << 29;
  }
  // 2. query offsets: scan of q_len.
  for (int s = tid; s < p.n_seqs; s += kPackThreads) cu[s] = p.seqs[4 * s + 2];
  __syncthreads();
  const int total = cta_exclusive_scan(cu, p.n_seqs, 1);
  if (tid == 0) cu[p.n_seqs] = total;
  __syncthreads();
  const int T = min(total, p.n_tokens);
  if (total != p.n_tokens && tid == 0) atomicOr(p.status, NF_STATUS_UNIT_OVERFLOW);

  // 3. per-token expansion: slot mapping, source row, position, work item.
  for (int t = tid; t < T; t += kPackThreads) {
    const int s = seq_of(cu, p.n_seqs, t), i = t - cu[s];
    int slot = p.seqs[4 * s];
    const int q_start = p.seqs[4 * s + 1], ctx_before = p.seqs[4 * s + 3];
    if (slot < 0 || slot >= p.num_slots) {
      atomicOr(p.status, NF_STATUS_BAD_SLOT);
      slot = 0;
    }
    const int pos = ctx_before + i;
    const int lb = pos / p.bs;
    int phys = (lb < p.max_blocks) ? p.bt[(long long)slot * p.max_blocks + lb] : -1;
    if (phys < 0 || phys >= p.num_blocks) {
      atomicOr(p.status, NF_STATUS_BAD_BLOCK);
      phys = 0;
    }
    p.slot_mapping[t] = phys * p.bs + pos % p.bs;
    p.src_rows[t] = q_start + i;
    if (p.positions) p.positions[t] = pos;
    const int kv_len = pos + 1;  // query at pos sees keys 0..pos (attention.py:144-152)
    int4 it;
    it.x = slot;
    it.y = q_start + i;
    it.z = kv_len;
    const int us = unit_size(p, s);
    int shared = 0, nc = 0;
    shared_of(p, s, kv_len, shared, nc);
    const int own = parts_of(kv_len - shared, us);
    it.w = nc + own;  // number of parts; scanned below
    if (it.w > 1) multi_sh = 1;
    if (own > 1) cross_sh = 1;
    if (us > 0) atomicMin(&first_sh, t);
    if (it.w > kMaxParts) atomicMax(&max_parts_sh, it.w);
    reinterpret_cast<int4*>(p.items)[t] = it;
  }
  __syncthreads();
  // 4. unit base of each item: scan of the split counts.
  const int n_units = cta_exclusive_scan(p.items + 3, T, 4);
  // The first nc parts of an item whose sequence shares its first keys with
  // others (cascade parts, written by nf_cascade_attention) have partial
  // slots but no record in the list; its own keys follow them as parts
  // nc, nc+1, ...
  // 5. the unit list, one self-contained record per key range of an item:
  // (item, slot, q_row, part, key_begin, key_end, unit_base, n_parts).  The
  // parts of an item are contiguous from its unit_base in key order (that is
  // where the kernels put their split-K partials); the list itself holds the
  // units of sequences with the step's split first and the units of
  // sequences given a smaller unit size after them, each class in item
  // order.  Workers that take units in list order so end on short units and
  // finish close together, and the items of the first class complete, and
  // merge, while the bulk of the keys still streams.
  __shared__ int n_fine_sh, n_casc_sh;
  if (tid == 0) n_fine_sh = n_casc_sh = 0;
  __syncthreads();
  int my_fine = 0, my_casc = 0;
  for (int t = tid; t < T; t += kPackThreads) {
    const int s = seq_of(cu, p.n_seqs, t), kv_len = p.items[4 * t + 2];
    const int us = unit_size(p, s);
    int shared = 0, nc = 0;
    shared_of(p, s, kv_len, shared, nc);
    if (us < p.split) my_fine += parts_of(kv_len - shared, us);
    my_casc += nc;
  }
  if (my_fine) atomicAdd(&n_fine_sh, my_fine);
  if (my_casc) atomicAdd(&n_casc_sh, my_casc);
  __syncthreads();
  const int n_list = n_units - n_casc_sh;  // units in the list: every part but the cascade ones
  const int n_bulk = n_list - n_fine_sh;
  int fine_carry = 0, casc_carry = 0;
  for (int base = 0; base < T; base += kPackThreads) {
    const int t = base + tid;
    int4 it = make_int4(0, 0, 0, 0);
    int us = p.split, n = 0, shared = 0, nc = 0;
    if (t < T) {
      const int s = seq_of(cu, p.n_seqs, t);
      it = reinterpret_cast<const int4*>(p.items)[t];
      us = unit_size(p, s);
      shared_of(p, s, it.z, shared, nc);
      n = parts_of(it.z - shared, us);
    }
    const bool fine = us < p.split;
    const int fb = cta_scan_round(fine ? n : 0, fine_carry);  // fine units of the items before t
    const int cb = cta_scan_round(nc, casc_carry);           // cascade parts of the items before t
    if (t < T) {
      const int first = fine ? n_bulk + fb : it.w - fb - cb;  // list position of the item's first unit
      for (int j = 0; j < n; ++j) {
        const int u = first + j;
        if (u < p.max_units) {
          int4* rec = reinterpret_cast<int4*>(p.units) + 2 * u;
          rec[0] = make_int4(t, it.x, it.y, nc + j);
          // low 16 bits: the item's parts; high: its units (the parts that are
          // not cascade parts), so that the last unit to finish can merge
          rec[1] = make_int4(shared + j * us, min(shared + (j + 1) * us, it.z), it.w,
                             (min(n, kMaxParts) << 16) | min(nc + n, kMaxParts));
        }
      }
    }
  }
  if (tid == 0) {
    if (n_units > p.max_units) atomicOr(p.status, NF_STATUS_UNIT_OVERFLOW);
    if (max_parts_sh > kMaxParts) atomicOr(p.status, NF_STATUS_UNIT_OVERFLOW);
    p.counts[0] = T;
    p.counts[1] = min(n_list, p.max_units);
    // bit 0: some item has more than one part; bit 1: some item has more than
    // one unit (its parts come from several workers of the attention launch);
    // from bit 2: the first item with units (the rows before it are the
    // prefill kernel's), where the end-of-launch merge starts looking
    p.counts[2] = multi_sh | (cross_sh << 1) | (min(first_sh, T) << 2);
    p.counts[3] = min(n_units, p.max_units);  // partial slots of all items, cascade parts included
  }
}

}  // namespace nf

extern "C" int nf_pack_step(const int32_t* seqs, int32_t n_seqs, const int32_t* patches, int32_t n_patches,
                            int32_t* block_tables, int32_t num_slots, int32_t max_blocks_per_seq,
                            int32_t block_size, int32_t num_blocks, int32_t split_tokens,
                            const int32_t* seq_split, const int32_t* seq_shared,
                            int32_t* slot_mapping, int32_t* src_rows, int64_t* positions, int32_t* items,
                            int32_t* units, int32_t* counts, int32_t n_tokens, int32_t max_units,
                            int32_t* status, void* stream) {
  using namespace nf;
  if (n_seqs <= 0 || n_tokens <= 0) return fail(NF_EINVAL, "nf_pack_step: empty step (n_seqs=%d, n_tokens=%d)", n_seqs, n_tokens);
  if (!seqs || !block_tables || !slot_mapping || !src_rows || !items || !units || !counts || !status)
    return fail(NF_EINVAL, "nf_pack_step: null pointer argument");
  if (n_patches > 0 && !patches) return fail(NF_EINVAL, "nf_pack_step: patches is null");
  if (block_size <= 0 || split_tokens <= 0 || num_slots <= 0 || max_blocks_per_seq <= 0 || num_blocks <= 0)
    return fail(NF_EINVAL, "nf_pack_step: sizes must be positive");
  if (max_units <= 0) return fail(NF_EINVAL, "nf_pack_step: max_units must be positive");
  if (split_tokens % 16 != 0)
    return fail(NF_EINVAL, "nf_pack_step: split_tokens (%d) must be a multiple of 16", split_tokens);
  if ((reinterpret_cast<uintptr_t>(items) & 15) != 0 || (reinterpret_cast<uintptr_t>(units) & 15) != 0)
    return fail(NF_EINVAL, "nf_pack_step: items and units must be 16-byte aligned");
  const size_t smem = sizeof(int) * (size_t)(n_seqs + 1);
  if (smem > 200 * 1024) return fail(NF_EINVAL, "nf_pack_step: too many sequences (%d)", n_seqs);
  if (smem > 48 * 1024) cudaFuncSetAttribute(pack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  PackParams p;
  p.seqs = seqs;
  p.n_seqs = n_seqs;
  p.patches = patches;
  p.n_patches = n_patches;
  p.bt = block_tables;
  p.num_slots = num_slots;
  p.max_blocks = max_blocks_per_seq;
  p.bs = block_size;
  p.num_blocks = num_blocks;
  p.split = split_tokens;
  p.seq_split = seq_split;
  p.seq_shared = seq_shared;
  p.slot_mapping = slot_mapping;
  p.src_rows = src_rows;
  p.positions = reinterpret_cast<long long*>(positions);
  p.items = items;
  p.units = units;
  p.counts = counts;
  p.n_tokens = n_tokens;
  p.max_units = max_units;
  p.status = status;
  pack_kernel<<<1, kPackThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("nf_pack_step");
}
