/*
 * nifre_b200 -- C ABI of the B200 (sm_100a) ragged paged-attention path.
 *
 * Everything here is plain C: raw device pointers borrowed from the caller,
 * sizes in elements unless a name says bytes, a CUDA stream passed as void*,
 * int status returns (0 = ok) with the message of the last failure of the
 * calling thread in nf_last_error().  The library allocates no device memory:
 * every buffer, workspace included, belongs to the caller.
 *
 * Reference interfaces replaced (jyotilakra92/nifre, src/inference/):
 *   nf_pack_step        -> the per-row host loops that build a step's batch:
 *                          batching.py:8-19 (left padding + input_lens),
 *                          model_runner.py:39-50,73-75 (chunk slicing, slots),
 *                          gpt.py:108-126 (positions from kv_cache.pos),
 *                          paged_kv_cache.py:107-121 (per-token resolve of the
 *                          destination slot), block_table.py:36-40 (resolve).
 *   nf_kv_append        -> PagedKVCache.append, paged_kv_cache.py:107-121
 *                          (scatter of the new K/V rows; pos advance on the
 *                          last layer, :120-121).
 *   nf_paged_attention  -> Attention._forward_with_cache(_row),
 *                          attention.py:77-142 (get -> cat -> q@k^T ->
 *                          causal mask -> softmax(/sqrt(D)) -> @v), reading K/V
 *                          in place from the block pool instead of the
 *                          PagedKVCache.get gather, paged_kv_cache.py:123-142.
 *
 * Pool layout (unchanged from paged_kv_cache.py:72-85): per layer one K and
 * one V tensor of shape (num_blocks, block_size, num_kv_heads, head_dim),
 * row-major.  Token t of a sequence lives in row
 *     slot = block_table[t / block_size] * block_size + t % block_size.
 */
#ifndef NIFRE_B200_H
#define NIFRE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define NF_F32 0
#define NF_F16 1
#define NF_BF16 2

/* return codes */
#define NF_OK 0
#define NF_EINVAL 1       /* bad argument (host-side check, nothing launched) */
#define NF_ECUDA 2        /* a CUDA runtime call failed */
#define NF_EUNSUPPORTED 3 /* shape/type combination without a kernel */

/* bits of the device status word kernels may set (never a trap) */
#define NF_STATUS_BAD_BLOCK 1   /* block id or logical block out of range: access skipped */
#define NF_STATUS_UNIT_OVERFLOW 2 /* more work units than the caller's workspace holds */
#define NF_STATUS_WAIT_TIMEOUT 4  /* a pipeline wait gave up after its time limit */
#define NF_STATUS_BAD_SLOT 8    /* cache slot out of range: entry skipped */
#define NF_STATUS_BAD_TILE 16   /* prefill tile longer than nf_prefill_tile_rows() rows: rest skipped */
#define NF_STATUS_BAD_SHARED 32 /* shared-key record that leaves a query no key of its own: its keys skipped */
#define NF_STATUS_FOREIGN_PARTS 64 /* plan with cascade parts given to nf_paged_attention_noalloc: nothing computed */

/* Record layouts (int32) of the step descriptor the host uploads. */
#define NF_SEQ_FIELDS 4   /* slot, q_start (row of the first new token), q_len, ctx_before */
#define NF_PATCH_FIELDS 3 /* slot, logical block index, physical block id */
#define NF_ITEM_FIELDS 4  /* slot, q_row, kv_len, unit_base */
#define NF_UNIT_FIELDS 8  /* item, slot, q_row, part, key_begin, key_end, unit_base, n_parts */

/*
 * Gathered output over several GPUs of one node (one process per GPU, KV
 * heads sharded over the ranks).  The attention output rows of this rank's
 * query heads go to `out` (this GPU's gathered buffer, at this rank's column
 * offset) and, through peer stores over NVLink, to the same place in every
 * other rank's gathered buffer: peer_out[i] is that address in the buffer of
 * the i-th other rank (rank order, this rank left out), as mapped into this
 * process by nf_ipc_open.  flags[r] is rank r's flag array (int32[n_ranks],
 * zero when allocated, mapped likewise; flags[rank] is this GPU's own).
 * epoch numbers the exchanges: the same value on every rank for the same
 * call, increasing from 1.  With epoch_counter (device int32, zero when
 * allocated, one per rank) the epoch is kept on the device instead: the
 * launch that signals adds one to *epoch_counter and uses the result, so
 * that a captured CUDA graph replays with a fresh epoch each time (every
 * rank must make the same exchanges in the same order; epoch is then
 * ignored).  n_ranks == 1 means no exchange.
 */
#define NF_MAX_RANKS 8
typedef struct NfGather {
  int32_t n_ranks;
  int32_t rank;
  int32_t epoch;
  int32_t pad;
  void* peer_out[NF_MAX_RANKS - 1];
  int32_t* flags[NF_MAX_RANKS];
  int32_t* epoch_counter;
} NfGather;

/* Message of the last failed call on this thread ("" if none). */
const char* nf_last_error(void);

/* ABI revision of this header; bumped on any signature change. */
int nf_abi_version(void);

/*
 * Which kernel the last nf_paged_attention call of this thread launched:
 * 0 = per-warp cp.async staging (any dtype and shape),
 * 1 = tensor-map (TMA) staging, one copy per 16-token block for all heads of
 *     a CTA, 2 = tensor-map staging with one copy per head; -1 = none yet.
 * A diagnostic with no counterpart in the reference.
 */
int nf_last_attention_path(void);

/*
 * Diagnostic, no counterpart in the reference: runs one of the bounded waits
 * that every kernel of this library uses on a wait that nothing satisfies,
 * with a limit of limit_cycles SM clock cycles (0 < limit <= the kernels' own
 * limit of about two seconds).  kind 0: an mbarrier wait (the pipeline
 * waits); kind 1: a wait until the device counter *counter reaches target
 * (the split-K kernels' end-of-launch wait).  The kernel must end, set
 * NF_STATUS_WAIT_TIMEOUT in *status and write 0 to *result (1 if the wait
 * was satisfied: kind 1 with *counter >= target).  Used by the tests of the
 * failure detection; nothing faults or hangs.
 */
int nf_selftest_wait(int32_t kind, int64_t limit_cycles, const int32_t* counter, int32_t target,
                     int32_t* status, int32_t* result, void* stream);

/*
 * Diagnostic, no counterpart in the reference: one 128 x N x K bfloat16
 * tensor-core (tcgen05) product from 128-byte-swizzled shared memory into
 * tensor memory, the building block of the prefill kernel.  A: 128 x K,
 * B: N x K (mode 0, C = A B^T) or K x N (mode 1 and 2, C = A B), row-major
 * device arrays; mode 2 stages A in tensor memory (the P V operand form of
 * the prefill kernel).  C: 128 x N float32.  N, K in {64, 128}.
 */
int nf_selftest_umma(const void* A, const void* B, float* C, int32_t N, int32_t K, int32_t mode,
                     int32_t* status, void* stream);

/*
 * nf_pack_step: expand one step's ragged batch on the device.
 *
 * seqs[n_seqs][4]      (device) slot, q_start, q_len, ctx_before of each
 *                      sequence in the step, in the order the reference
 *                      processes rows (prefill rows first, then decode rows).
 * patches[n_patches][3](device) block-table writes applied first:
 *                      block_tables[slot][logical] = physical.
 * block_tables         (device, in/out) int32 [num_slots][max_blocks_per_seq].
 * Outputs, one entry per new token t (n_tokens = sum of q_len):
 *   slot_mapping[t]    destination pool row of token t,
 *   src_rows[t]        row of token t in the caller's q/k/v tensors,
 *   positions[t]       absolute position (int64, may be NULL),
 *   items[t][4]        attention work item of the query at token t,
 * and the split-K work list units[max_units][8] (16-byte aligned): key
 * ranges [key_begin, key_end) of an item, each record self-contained so a
 * kernel needs one read per unit.  The queries of sequence s use units of
 * seq_split[s] keys (device, n_seqs entries; NULL, or an entry that is
 * negative or not a multiple of 16, means split_tokens; 0 means no units:
 * the sequence's queries are left to nf_prefill_attention).  An item's n_parts units are
 * its parts 0..n_parts-1 in key order, with split-K partial slots
 * unit_base + part; the list holds the units of sequences at split_tokens
 * first and those of sequences with a smaller unit size after them, each
 * class in item order, so that a dynamic queue over the list ends on short
 * units.  split_tokens must be a positive multiple of 16.
 * seq_shared[n_seqs][2] (device, may be NULL): per sequence the number of
 * leading keys it shares with other sequences of the step and the number nc
 * of cascade parts that nf_cascade_attention computes over them ({0, 0}:
 * none).  Such an item's parts 0..nc-1 are those cascade parts (partial
 * slots, no unit records); its units cover keys [shared, kv_len) as parts
 * nc, nc+1, ...  A unit record's last field holds its item's part count
 * (low 16 bits, at most 32767: more is flagged NF_STATUS_UNIT_OVERFLOW) and
 * unit count (high bits); when one unit covers an item's own keys, the
 * tensor-map decode kernel merges the item's cascade parts in that unit's
 * epilogue.
 * counts[4]: counts[0] = n_tokens, counts[1] = number of units in the list,
 * counts[2] = bit 0: some item has more than one part, bit 1: some item has
 * more than one unit (the attention launch then merges at its end), bits 2
 * and up: the first item with units (the items before it have none),
 * counts[3] = number of partial slots (units + cascade parts).
 */
int nf_pack_step(const int32_t* seqs, int32_t n_seqs,
                 const int32_t* patches, int32_t n_patches,
                 int32_t* block_tables, int32_t num_slots, int32_t max_blocks_per_seq,
                 int32_t block_size, int32_t num_blocks, int32_t split_tokens,
                 const int32_t* seq_split, const int32_t* seq_shared,
                 int32_t* slot_mapping, int32_t* src_rows, int64_t* positions,
                 int32_t* items, int32_t* units, int32_t* counts,
                 int32_t n_tokens, int32_t max_units,
                 int32_t* status, void* stream);

/*
 * nf_kv_append: pool[slot_mapping[t]] = new[src_rows[t]] for K and V.
 * pool_rows = num_blocks * block_size (rows outside it are skipped and flagged).
 * Each pool row holds num_kv_heads*head_dim elements of pool_dtype; source
 * rows start every src_row_stride elements (so a head slice of a wider
 * projection can be passed with an offset pointer).  Values are converted to
 * the pool dtype with round-to-nearest-even, as torch's copy does.
 * If pos_out (int64 [num_slots]) is not NULL the kernel also sets
 * pos_out[slot] = ctx_before + q_len for each of the n_seqs records in seqs:
 * the reference advances pos only on the last layer (paged_kv_cache.py:120-121).
 */
int nf_kv_append(void* k_pool, void* v_pool, int32_t pool_dtype, int64_t pool_rows,
                 const void* k_new, const void* v_new, int32_t src_dtype,
                 int64_t k_src_row_stride, int64_t v_src_row_stride,
                 const int32_t* slot_mapping, const int32_t* src_rows, int32_t n_tokens,
                 int32_t num_kv_heads, int32_t head_dim,
                 const int32_t* seqs, int32_t n_seqs, int64_t* pos_out,
                 int32_t* status, void* stream);

/*
 * nf_qkv_append: the attention input projection fused with the KV append
 * (replaces GptAttention.forward's three nn.Linear calls + the cache append,
 * models/gpt.py:38-51 and paged_kv_cache.py:107-121).  For the `rows` rows
 * of x (row r = token r of the step, whose pool row is slot_mapping[r]):
 *   y = x W^T (+ bias), W = weight (n_q + 2 n_kv rows of k_dim elements, the
 *   q, k and v projection weights stacked in nn.Linear layout),
 *   q_out[r] = y[r, 0:n_q], k_pool[slot] = y[r, n_q:n_q+n_kv],
 *   v_pool[slot] = y[r, n_q+n_kv:],
 * on the tensor cores (tcgen05, fp32 accumulation, rounded once to the
 * 16-bit dtype of x, weight, q_out and the pools).  n_q and n_kv multiples
 * of 64, k_dim of 8; pools hold pool_rows rows of n_kv elements; slots
 * outside them are skipped and flagged (NF_STATUS_BAD_SLOT).  If pos_out is
 * not NULL, pos_out[slot] = ctx_before + q_len for each of the n_seqs step
 * records of nf_pack_step (the last layer's append, paged_kv_cache.py:120-121).
 */
int nf_qkv_append(const void* x, int64_t x_row_stride, int32_t rows, const void* weight, const void* bias,
                  int32_t k_dim, int32_t n_q, int32_t n_kv, void* q_out, int64_t q_out_row_stride,
                  void* k_pool, void* v_pool, int64_t pool_rows, int32_t dtype,
                  const int32_t* slot_mapping, const int32_t* seqs, int32_t n_seqs, int64_t* pos_out,
                  int32_t* status, void* stream);

/*
 * nf_attention_workspace: sizes of the caller-owned split-K workspace for
 * nf_paged_attention (float partials and int32 counters).  Counters must be
 * zeroed once when allocated; the kernel leaves them zero when it returns.
 */
int nf_attention_workspace(int32_t max_units, int32_t max_items, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                           int64_t* partial_floats, int64_t* counter_ints);

/*
 * nf_paged_attention: out[q_row] = softmax(q[q_row] k^T * scale) v over keys
 * [0, kv_len) of the item's sequence, for every work item produced by
 * nf_pack_step, with query head j reading KV head j / (num_q_heads/num_kv_heads).
 * q/out rows hold num_q_heads*head_dim elements of `dtype` (the pool dtype);
 * rows start every q_row_stride / out_row_stride elements.  Work is the
 * unit list of nf_pack_step (split_tokens: the value given there, checked
 * again here); partial results go to ws_partials and are merged at the end
 * of the same launch, once every unit is done (the kernel is launched
 * cooperatively: all its CTAs are resident at once).  items (16-byte
 * aligned) locate each item's parts.
 */
int nf_paged_attention(void* out, int64_t out_row_stride,
                       const void* q, int64_t q_row_stride,
                       const void* k_pool, const void* v_pool, int32_t dtype,
                       int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                       int32_t block_size, int32_t num_blocks,
                       const int32_t* block_tables, int32_t max_blocks_per_seq,
                       const int32_t* items, const int32_t* units, const int32_t* counts,
                       int32_t max_items, int32_t max_units, int32_t split_tokens, float scale,
                       float* ws_partials, int64_t ws_partial_floats,
                       int32_t* ws_counters, int64_t ws_counter_ints,
                       int32_t* status, void* stream);

/*
 * nf_paged_attention_gather: nf_paged_attention whose output is gathered
 * over the ranks of `gather` (see NfGather) in the same launch, replacing
 * attention + an all-gather collective: every output row is stored on this
 * GPU and on each peer; once all of the launch's rows are stored, its last
 * CTA sets this rank's entry of every rank's flag array to gather->epoch
 * and waits (time-limited: NF_STATUS_WAIT_TIMEOUT) until every rank has
 * done the same, so the launch ends with the whole gathered output in this
 * GPU's buffer.  Outputs written earlier on the same stream by
 * nf_prefill_attention_gather are covered by the same signal.  Every rank
 * must make the matching call (same epoch); ranks run on different GPUs.
 * The shard-parallel form of reference attention.py:77-104 (one process per
 * GPU, KV heads split over the ranks); gather == NULL is nf_paged_attention.
 */
int nf_paged_attention_gather(void* out, int64_t out_row_stride,
                              const void* q, int64_t q_row_stride,
                              const void* k_pool, const void* v_pool, int32_t dtype,
                              int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                              int32_t block_size, int32_t num_blocks,
                              const int32_t* block_tables, int32_t max_blocks_per_seq,
                              const int32_t* items, const int32_t* units, const int32_t* counts,
                              int32_t max_items, int32_t max_units, int32_t split_tokens, float scale,
                              float* ws_partials, int64_t ws_partial_floats,
                              int32_t* ws_counters, int64_t ws_counter_ints,
                              const NfGather* gather, int32_t* status, void* stream);

/*
 * The per-layer calls with their arguments in one struct: a host binding
 * fills the step's constant fields once and changes only the per-layer
 * pointers between calls, so that a call marshals one pointer instead of
 * twenty to thirty arguments (the binding's per-call cost is then the
 * launch itself).  Fields and meaning are those of nf_paged_attention_gather
 * and nf_kv_append, in the same order.
 */
typedef struct NfAttentionArgs {
  void* out;
  int64_t out_row_stride;
  const void* q;
  int64_t q_row_stride;
  const void* k_pool;
  const void* v_pool;
  int32_t dtype, num_q_heads, num_kv_heads, head_dim, block_size, num_blocks;
  const int32_t* block_tables;
  int32_t max_blocks_per_seq, max_items, max_units, split_tokens;
  const int32_t* items;
  const int32_t* units;
  const int32_t* counts;
  float scale;
  int32_t pad;
  float* ws_partials;
  int64_t ws_partial_floats;
  int32_t* ws_counters;
  int64_t ws_counter_ints;
  const NfGather* gather;
  int32_t* status;
} NfAttentionArgs;

int nf_paged_attention_args(const NfAttentionArgs* args, void* stream);

typedef struct NfAppendArgs {
  void* k_pool;
  void* v_pool;
  int64_t pool_rows;
  const void* k_new;
  const void* v_new;
  int64_t k_src_row_stride, v_src_row_stride;
  int32_t pool_dtype, src_dtype, n_tokens, num_kv_heads, head_dim, n_seqs;
  const int32_t* slot_mapping;
  const int32_t* src_rows;
  const int32_t* seqs;
  int64_t* pos_out;
  int32_t* status;
} NfAppendArgs;

int nf_kv_append_args(const NfAppendArgs* args, void* stream);

/*
 * nf_exchange_barrier: the signal-and-wait of a gathered output on its own
 * (one thread): for a layer whose rows were all written by
 * nf_prefill_attention_gather (no decode launch follows to signal).
 */
int nf_exchange_barrier(const NfGather* gather, int32_t* status, void* stream);

/*
 * CUDA IPC mapping of a device buffer into the other processes of the node
 * (for NfGather).  nf_ipc_handle writes the 64-byte handle of the allocation
 * holding `ptr` and the offset of `ptr` inside it; nf_ipc_open maps another
 * process's handle and returns the address at `offset` in this process;
 * nf_ipc_close unmaps it (pass the address and offset nf_ipc_open gave).
 */
int nf_ipc_handle(const void* ptr, void* handle64, int64_t* offset);
int nf_ipc_open(const void* handle64, int64_t offset, void** ptr);
int nf_ipc_close(void* ptr, int64_t offset);

/*
 * nf_cascade_attention: partial attention of decode queries over keys that
 * several sequences share (leading blocks imported from the prefix index,
 * prefix_cache.py:33-81, paged_kv_cache.py:87-105), each shared block read
 * once per group of sequences and KV head instead of once per sequence.
 * tasks[n_tasks][8] (device, 16-byte aligned): slot (whose block table
 * holds the shared blocks), first, count, part, key_begin, key_end
 * (multiples of 16), 0, 0 -- the task's queries are toks[first ..
 * first+count), where toks[n_toks][2] (device, 8-byte aligned) holds (item
 * number of nf_pack_step, row of the query in q, below num_q_rows).  Each
 * task writes the partial softmax state of its queries over keys
 * [key_begin, key_end) into partial slot items[item].unit_base + part of
 * ws_partials (the layout of nf_attention_workspace), for every KV head.
 * The same step's nf_pack_step must have been given, through seq_shared,
 * the shared key count and cascade part count of each such sequence; the
 * following nf_paged_attention on the same stream and workspace then merges
 * these parts with the queries' own keys (nf_paged_attention_noalloc
 * cannot: its workspace is its own, so plans with cascade parts go to
 * nf_paged_attention).  16-bit pools, head_dim 64 or 128, block_size a
 * multiple of 16.  nf_cascade_limits gives the largest task: with 1, 2, 4
 * or 8 query heads per KV head (G) the tasks run on the tensor cores (the
 * prefill kernel's tcgen05 pipeline, one (task, KV head) item at a time per
 * CTA: up to 256 / G queries and any whole number of 16-key groups; q rows
 * 16-byte aligned);
 * other group sizes use an mma.sync kernel (one CTA per
 * task and KV head: up to 128 / G queries and 256 keys) launched with
 * programmatic stream serialization: the launch before it on the stream
 * must not write the shared blocks, q, items or counts (the step's KV
 * append writes none of them).  A malformed task, or a query row outside
 * [0, num_q_rows), sets NF_STATUS_BAD_SHARED and is skipped.
 */
int nf_cascade_attention(float* ws_partials, int64_t ws_partial_floats,
                         const void* q, int64_t q_row_stride, int32_t num_q_rows,
                         const void* k_pool, const void* v_pool, int32_t dtype,
                         int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                         int32_t block_size, int32_t num_blocks,
                         const int32_t* block_tables, int32_t max_blocks_per_seq,
                         const int32_t* items, const int32_t* counts, int32_t max_items, int32_t max_units,
                         const int32_t* tasks, int32_t n_tasks, const int32_t* toks, int32_t n_toks,
                         float scale,
                         int32_t* status, void* stream);

/*
 * nf_cascade_limits: the largest task nf_cascade_attention takes for this
 * shape -- query rows (queries x query heads per KV head) and keys.
 */
int nf_cascade_limits(int32_t dtype, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                      int32_t* max_rows, int32_t* max_keys);

/*
 * nf_prefill_attention: causal attention of prefill chunks on the tensor
 * cores (tcgen05, tensor memory), for 16-bit pools with head_dim 64 or 128,
 * 1, 2, 4 or 8 query heads per KV head and block_size a multiple of 16.
 * tiles[n_tiles][4] (device, 16-byte aligned): slot, q_row0, ntok, pos0 -- the
 * ntok (<= nf_prefill_tile_rows() / group size) consecutive query tokens of
 * one sequence whose rows in q/out start at q_row0 and whose absolute
 * positions start at pos0; query pos0 + i attends over keys [0, pos0 + i] of
 * the slot's block table (attention.py:144-152), all already appended.
 * Writes those rows of out (rows >= num_rows, the rows of q and out, are
 * neither read nor written).  Work items are (tile, KV head), numbered
 * tile * num_kv_heads + head.  One persistent CTA per SM takes items from a
 * queue shared by all CTAs, in the order given by `order` (device, n_tiles *
 * num_kv_heads item numbers, longest first for balance; NULL: item number
 * order).  queue (device, int32[2]) must be zero on entry; the kernel leaves
 * it zero, so one buffer serves every launch on a stream (launches that share
 * it must not overlap).
 */
int nf_prefill_attention(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                         int32_t num_rows, const void* k_pool, const void* v_pool, int32_t dtype,
                         int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                         int32_t block_size, int32_t num_blocks,
                         const int32_t* block_tables, int32_t max_blocks_per_seq,
                         const int32_t* tiles, int32_t n_tiles,
                         const int32_t* order, int32_t* queue, float scale,
                         int32_t* status, void* stream);

/*
 * nf_prefill_attention_gather: nf_prefill_attention whose output rows are
 * also stored into the other ranks' gathered buffers (gather->peer_out,
 * 16-byte aligned; see NfGather).  It sets no flag: the layer's
 * nf_paged_attention_gather (or nf_exchange_barrier) on the same stream
 * signals the peers for all of the layer's rows.
 */
int nf_prefill_attention_gather(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                int32_t num_rows, const void* k_pool, const void* v_pool, int32_t dtype,
                                int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                int32_t block_size, int32_t num_blocks,
                                const int32_t* block_tables, int32_t max_blocks_per_seq,
                                const int32_t* tiles, int32_t n_tiles,
                                const int32_t* order, int32_t* queue, float scale,
                                const NfGather* gather, int32_t* status, void* stream);

/* Query rows (tokens x query heads per KV head) of one nf_prefill_attention work item for this
 * head_dim: 256 (two 128-row halves sharing one stream of K/V tiles) for head_dim 64 and 128. */
int nf_prefill_tile_rows(int32_t head_dim);

/*
 * nf_paged_attention_noalloc: nf_paged_attention without a caller workspace.
 * This entry point has no counterpart in the reference.  It is for callers
 * that cannot allocate device memory themselves -- for example a host binding
 * that only borrows the tensors of another runtime, or a server whose device
 * memory is entirely reserved by its own pool -- and so cannot pass
 * ws_partials / ws_counters.  The split-K scratch is instead a buffer of
 * NF_NOALLOC_SCRATCH_BYTES compiled into this library (every GPU that loads
 * the library holds it until the process exits).  The call allocates
 * nothing: the first call in a CUDA context looks up that buffer's device
 * address in that context (so make that first call before any stream
 * capture), and every call clears the buffer's counters with cudaMemsetAsync
 * on `stream`, after every argument check has passed (a refused call queues
 * nothing).  A step whose scratch (max_units * num_q_heads * (head_dim + 4)
 * floats, rounded up to 256 bytes, plus max_items * num_kv_heads + 4 ints)
 * exceeds the buffer is rejected with NF_EINVAL.  All calls share the one
 * buffer: calls that overlap on the GPU (other streams, other threads) race
 * and give wrong results.  The buffer holds only this call's split-K parts,
 * so a plan with cascade parts (nf_pack_step given seq_shared; they belong to
 * nf_cascade_attention's workspace) is not computed: the kernel sets
 * NF_STATUS_FOREIGN_PARTS and leaves out untouched.  Arguments and results
 * are otherwise those of nf_paged_attention.
 */
#define NF_NOALLOC_SCRATCH_BYTES (16u << 20)

int nf_paged_attention_noalloc(void* out, int64_t out_row_stride,
                               const void* q, int64_t q_row_stride,
                               const void* k_pool, const void* v_pool, int32_t dtype,
                               int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                               int32_t block_size, int32_t num_blocks,
                               const int32_t* block_tables, int32_t max_blocks_per_seq,
                               const int32_t* items, const int32_t* units, const int32_t* counts,
                               int32_t max_items, int32_t max_units, int32_t split_tokens, float scale,
                               int32_t* status, void* stream);

/*
 * Test hook of nf_paged_attention_noalloc, no counterpart in the reference:
 * fills its built-in scratch buffer (in the current CUDA context) with the
 * byte `byte` on `stream`, so that a test can show that every call of
 * nf_paged_attention_noalloc clears what must start at zero itself.
 */
int nf_noalloc_scratch_fill(int32_t byte, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NIFRE_B200_H */
