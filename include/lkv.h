/*
 * lkv.h — C ABI of liblkv_sm100.so, the sm_100a kernels behind LazyKV's tiered decode path.
 *
 * Every entry point is `extern "C"`, takes plain pointers, sizes and a CUDA stream (as void*),
 * never synchronises, and returns an lkv_status. On a non-zero status, lkv_last_error() gives
 * the message of the calling thread's last failure. Device pointers may also be device views of
 * pinned, mapped host memory (the cold tier read through zero-copy loads).
 *
 * Reference interfaces are cited as file:line within PS12007/LazyKV; each entry point replaces
 * the torch calls made there.
 */
#ifndef LKV_H
#define LKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  LKV_OK = 0,
  LKV_ERR_ARG = 1,      /* a size, shape or dtype the kernels do not support */
  LKV_ERR_PTR = 2,      /* a null or misaligned pointer where one is required */
  LKV_ERR_CUDA = 3,     /* a CUDA launch or runtime error */
  LKV_ERR_WORKSPACE = 4 /* the workspace passed is smaller than the query function says */
} lkv_status;

/* Element types of KV, metadata and queries. */
typedef enum { LKV_F32 = 0, LKV_BF16 = 1 } lkv_dtype;

/* Order of a top-k list: descending bound then ascending id (top_blocks' order), or ascending id. */
typedef enum { LKV_ORDER_BOUND = 0, LKV_ORDER_BLOCK = 1 } lkv_order;

/* Cold-tier storage: int8 records (lazykv/quant.py:73-87) or whole pairs in the model dtype. */
typedef enum { LKV_COLD_INT8 = 0, LKV_COLD_PAIRS = 1 } lkv_cold_kind;

/* Library version string and the calling thread's last error message (copied into buf). */
const char* lkv_version(void);
size_t lkv_last_error(char* buf, size_t len);

/* Bytes of one packed (block, head) record. Replaces lazykv/quant.py:46-49 packed_pair_bytes. */
int64_t lkv_packed_pair_bytes(int bs, int d);

/*
 * Context-range sharding of one layer's sealed blocks over `world` GPUs (no reference
 * counterpart: the reference runs on one GPU). Host-only. Rank r holds sealed blocks [lo, hi), the
 * contiguous ranges of ceil(n_sealed / world) blocks; the sink (block 0) is on rank 0 and is never
 * a candidate, and the current block belongs to the last rank. The budget k_total is shared in
 * proportion to the candidates, the remainder one block each to the lowest ranks with room, so the
 * local budgets sum to k_total. out[5] = {lo, hi, first candidate, candidates, local budget}.
 */
int lkv_shard_plan(int n_sealed, int k_total, int world, int rank, int32_t* out);

/*
 * Channel-wise min/max of each block's keys. Replaces the amin/amax of
 * lazykv/selection.py:142-144, lazykv/tiered.py:173-175 and :369-370.
 * Key element (head j, block b, token t, channel c) is keys[j*s_head + b*s_block + t*s_tok + c];
 * kmin/kmax [h, cap, d] (same dtype as keys) are written at [j, first_block + b, :] with
 * m_head = cap * d.
 */
int lkv_block_minmax(const void* keys, int dtype, int h, int n_blocks, int bs, int d,
                     int64_t s_head, int64_t s_block, int64_t s_tok, void* kmin, void* kmax,
                     int64_t m_head, int first_block, void* stream);

/*
 * int8 quantise-on-write. Replaces lazykv/quant.py:73-87 pack (and, fused, the dequantise and
 * metadata of lazykv/tiered.py:187-197 and :365-370). pairs [n_blocks, h, 2, bs, d] in `dtype`
 * -> records [n_blocks, h, W] (W = lkv_packed_pair_bytes), bit-exact with the reference.
 * Optional outputs (NULL to skip): kmin/kmax over the dequantised keys in `dtype`, written like
 * lkv_block_minmax; deq [n_blocks, h, 2, bs, d] the dequantised pairs in `dtype`.
 */
int lkv_pack_int8(const void* pairs, int dtype, int n_blocks, int h, int bs, int d,
                  uint8_t* records, void* kmin, void* kmax, int64_t m_head, int first_block,
                  void* deq, void* stream);

/* int8 dequantise-on-read. Replaces lazykv/quant.py:90-105 unpack: records [n, W] -> out
 * [n, 2, bs, d] in out_dtype, bit-exact. */
int lkv_unpack_int8(const uint8_t* records, int64_t n, int bs, int d, void* out, int out_dtype,
                    void* stream);

/*
 * Gather-scatter fetch of (block, head) pairs from the host store into the slot pool. Replaces
 * the staged gather of lazykv/tiered.py:429-447 (index_select, H2D, unpack, index_copy_).
 * src: int8 records [rows, W] (LKV_COLD_INT8, dequantised into `dtype`) or pairs
 * [rows, 2, bs, d] in `dtype` (LKV_COLD_PAIRS). dst: pairs [rows, 2, bs, d] in `dtype`.
 * Row i of the fetch copies src row src_rows[i] to dst row dst_rows[i].
 */
int lkv_fetch_pairs(const void* src, int src_kind, const int64_t* src_rows, void* dst,
                    const int64_t* dst_rows, int64_t n, int bs, int d, int dtype, void* stream);

/*
 * Quest bound and device-side top-k. Replaces lazykv/selection.py:38-62 quest_bound/top_blocks
 * and the host round trip of lazykv/tiered.py:383-387 rank.
 * q [hq, d] (q_dtype); kmin/kmax [h, cap, d] (meta_dtype, row stride m_head per head);
 * candidates are blocks [first_block, first_block + n_cand). bound_mode LKV_BF16 rounds as the
 * reference's bf16 matmuls do, LKV_F32 keeps float32. Output: out_blocks [h, k] (row stride
 * out_ld >= k) block ids; with LKV_ORDER_BOUND in descending bound order, ties by ascending block
 * id (the selected set is the same either way; ties at the k-th bound go to the lower ids), with
 * LKV_ORDER_BLOCK in ascending block id (no sort). Optional: out_bound [h, n_cand] float32;
 * bitmap [h, bitmap_words] set exactly at the selected block ids (the words are cleared first).
 * Workspace: lkv_quest_topk_workspace(h, n_cand) bytes, zero-filled once when allocated: its first
 * 64 KiB + 256 bytes hold per-head counters that the LKV_ORDER_BLOCK paths expect at zero and
 * leave so (calls on one workspace must not overlap on the GPU; re-zero them after a call that
 * returned an error). With bf16 query and metadata at head_dim 64 in LKV_ORDER_BLOCK (G in
 * {1, 2, 4, 8}, n_cand <= 16,384, h <= 64) the selection is a TMA scoring kernel (CTAs of 128
 * candidates) followed, by programmatic dependent launch, by a select kernel of one 8-CTA cluster
 * per head; no CTA waits for a CTA outside its cluster. The scoring's tile loads are bounded waits:
 * a wait that runs out records status 1 (lkv_device_status, lkv_status_poll) and the head's output
 * becomes every listed id -1 and an empty bitmap, so an exact pass over the complement still
 * covers every candidate.
 */
size_t lkv_quest_topk_workspace(int h, int n_cand);
int lkv_quest_topk(const void* q, int q_dtype, int hq, int h, int d, const void* kmin,
                   const void* kmax, int meta_dtype, int64_t m_head, int first_block, int n_cand,
                   int k, int bound_mode, int order, int32_t* out_blocks, int out_ld,
                   float* out_bound, uint32_t* bitmap, int bitmap_words, void* workspace,
                   size_t workspace_bytes, void* stream);

/*
 * lkv_quest_topk without a workspace argument, for callers that cannot allocate device memory
 * when they select (an allocator-free runtime, an allocator callback, a process that reserved all
 * device memory up front). No counterpart in the reference. Same arguments, results and errors
 * as lkv_quest_topk; its scratch is a fixed device array inside the library (4 MiB of keys after
 * 64 KiB + 256 bytes of counters), so it takes h * n_cand <= 524,288 and returns LKV_ERR_ARG above
 * that. It allocates nothing. The first call on a device looks up that array's device address
 * (make it before any stream capture); calls must run with the stream's device current. All calls
 * share the array: calls that overlap on the GPU race, so serialise them (one stream, or events).
 * The counters must read zero when a call starts: the array starts zeroed, every complete call
 * leaves them zero, and a call that returns an error clears them (an asynchronous memset on the
 * stream, which allocates nothing).
 */
int lkv_quest_topk_noalloc(const void* q, int q_dtype, int hq, int h, int d, const void* kmin,
                           const void* kmax, int meta_dtype, int64_t m_head, int first_block,
                           int n_cand, int k, int bound_mode, int order, int32_t* out_blocks,
                           int out_ld, float* out_bound, uint32_t* bitmap, int bitmap_words,
                           void* stream);

/*
 * Global top-k over candidates gathered from the shards (no reference counterpart): for KV head j
 * the candidates are (bounds[j*ld + i], ids[j*ld + i]), i < n, listed in ascending id (as the
 * shards' LKV_ORDER_BLOCK selections concatenate in rank order); the k with the highest bound,
 * ties at the k-th bound to the lower ids, as lkv_quest_topk orders them. k <= 16384.
 * Workspace: lkv_topk_merge_workspace(h, n) bytes (same contract as lkv_quest_topk's).
 */
size_t lkv_topk_merge_workspace(int h, int n);
int lkv_topk_merge(const float* bounds, const int32_t* ids, int h, int n, int64_t ld, int k,
                   int bound_mode, int order, int32_t* out_blocks, int out_ld, uint32_t* bitmap,
                   int bitmap_words, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The Quest bound of every candidate, and nothing else (the scoring half of lkv_quest_topk;
 * lazykv/selection.py:38-53, quest_bound, computes the same scores): bounds[j*bounds_ld + i] is
 * candidate first_block + i's bound for KV head j, computed and rounded exactly as lkv_quest_topk
 * ranks it (bound_mode), stored as bounds_dtype (bf16 only in the bf16 bound mode, where it is
 * exact; or float32). One launch, no workspace. A shard's input to lkv_topk_gathered.
 */
int lkv_quest_bounds(const void* q, int q_dtype, int hq, int h, int d, const void* kmin,
                     const void* kmax, int meta_dtype, int64_t m_head, int first_block, int n_cand,
                     int bound_mode, void* bounds, int bounds_dtype, int64_t bounds_ld,
                     void* stream);

/*
 * Global top-k of a context-sharded layer from every shard's bounds (no reference counterpart;
 * the reference is single-device): bounds [world][h][ld] as all-gathered from lkv_quest_bounds,
 * rank r holding seg_n[r] candidates that follow rank r-1's in block order. The selection is the
 * k highest bounds over all ranks, ties at the k-th bound to the lower block ids: the set
 * lkv_quest_topk picks over the unsharded candidates. Every rank computes it from the same
 * gathered bounds; this call writes rank `rank`'s part: out_local [h, out_ld] gets, per head, the
 * chosen candidates of that rank as local ids (out_base + index within the rank) in ascending
 * order, then -1 up to out_cols (out_cols >= min(k, seg_n[rank])); the bitmap (optional) is
 * cleared and set at those local ids. world <= 64. One launch of one CTA per head, no workspace.
 */
int lkv_topk_gathered(const void* bounds, int bounds_dtype, int world, int h, int64_t ld,
                      const int32_t* seg_n, int k, int rank, int out_base, int32_t* out_local,
                      int out_ld, int out_cols, uint32_t* bitmap, int bitmap_words, void* stream);

/*
 * lkv_topk_gathered for an attention before the admit (as lkv_quest_topk_resident): for each chosen
 * local id b written at column c, hot[h * hot_ld + c] = block_slot[h * cap + b] when that is a slot
 * (>= 1), else -1 (and -1 in the padding columns); the bitmap marks only the resident ones.
 */
int lkv_topk_gathered_resident(const void* bounds, int bounds_dtype, int world, int h, int64_t ld,
                               const int32_t* seg_n, int k, int rank, int out_base,
                               int32_t* out_local, int out_ld, int out_cols, uint32_t* bitmap,
                               int bitmap_words, const int32_t* block_slot, int cap, int32_t* hot,
                               int64_t hot_ld, void* stream);

/*
 * Split decode attention over listed blocks, emitting (normalised out, lse). Replaces the gather
 * + SDPA + GPU log-sum-exp of lazykv/tiered.py:465-487, lazykv/attention.py:97-136 and
 * lazykv/exact.py:380-393.
 * Per KV head j the key sequence is the n_list blocks blocks[j*n_list + i] in order; the last one
 * holds `last_fill` live tokens (the current block, lazykv/selection.py:65-69), the others bs.
 * A listed id b maps to storage row r = slot_of ? slot_of[j*slot_stride + b] : b, and key element
 * (t, c) of that row is k_base[r*s_row + j*s_head + t*s_tok + c] (values at v_base, same strides).
 * n_rows: how many storage rows those strides address (rows 0..n_rows-1 of every head lie inside
 * the buffers); it bounds the tensor-map loads of the bf16 d-64 path, and 0 ("unknown") keeps the
 * call on the CUDA-core kernels.
 * q [hq, d] in `dtype`; out [hq, d] float32 (divided by its normaliser) and lse [hq] float32.
 * Workspace: lkv_attention_workspace(h, hq, d, n_list) bytes.
 */
size_t lkv_attention_workspace(int h, int hq, int d, int n_items);
int lkv_hot_attention(const void* q, int hq, int h, int d, int bs, const void* k_base,
                      const void* v_base, int dtype, int64_t s_row, int64_t s_head, int64_t s_tok,
                      int64_t n_rows, const int32_t* blocks, int n_list, const int32_t* slot_of,
                      int64_t slot_stride, int last_fill, float scale, float* out, float* lse,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * Exact pass over the cold blocks. Replaces lazykv/exact.py:88-127 cpu_partial_attention (and
 * the float32 mirror it reads, lazykv/exact.py:130-152) with a GPU pass over the complement only.
 * Attends blocks [first_block, first_block + n_blocks) of every KV head j, skipping those whose
 * bit is set in excluded[j*bitmap_words + b/32]; the store is cold [blocks, h, W] int8 records
 * (dequantised as lazykv/quant.py:unpack to `dtype`, fused: each block is attended as a fetch
 * would put it in a slot) or cold [blocks, h, 2, bs, d] pairs in `dtype` (LKV_COLD_PAIRS). A head
 * with no block left returns lse = -inf and out = 0.
 * Workspace: lkv_attention_workspace(h, hq, d, n_blocks) bytes.
 */
int lkv_cold_attention(const void* q, int hq, int h, int d, int bs, const void* cold,
                       int cold_kind, int dtype, int first_block, int n_blocks,
                       const uint32_t* excluded, int bitmap_words, float scale, float* out,
                       float* lse, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The hot set of lkv_exact_attention: the arguments of lkv_hot_attention, as a struct.
 */
typedef struct {
  const void* k_base;
  const void* v_base;
  int dtype;
  int64_t s_row, s_head, s_tok;
  const int32_t* blocks;
  int n_list;
  const int32_t* slot_of;
  int64_t slot_stride;
  int last_fill;
  int64_t n_rows;
} lkv_hot_set;

/* The cold set of lkv_exact_attention: the arguments of lkv_cold_attention, as a struct. */
typedef struct {
  const void* store;
  int kind;
  int first_block;
  int n_blocks;
  const uint32_t* excluded;
  int bitmap_words;
} lkv_cold_set;

/*
 * Both passes and their merge in one launch (plus one small combine): replaces the GPU attention,
 * the CPU pass and the blend of lazykv/exact.py:225-264 (ExactTieredCache.merge). The hot and cold
 * partials are computed by one grid whose CTAs take chunks of either set; the combine writes the
 * merged out [hq, d] in out_dtype and lse [hq] (both optional), and optionally the per-set
 * partials part_out [2, hq, d] / part_lse [2, hq] (hot first), float32. q is in hot->dtype.
 * Workspace: lkv_exact_attention_workspace(h, hq, d, n_list, n_blocks) bytes.
 */
size_t lkv_exact_attention_workspace(int h, int hq, int d, int n_list, int n_blocks);
int lkv_exact_attention(const void* q, int hq, int h, int d, int bs, const lkv_hot_set* hot,
                        const lkv_cold_set* cold, float scale, void* out, int out_dtype,
                        float* lse, float* part_out, float* part_lse, void* workspace,
                        size_t workspace_bytes, void* stream);

/*
 * Ragged rows: many sequences of different lengths in one decode step (continuous batching). The
 * reference is batch-1 only; per sequence these calls compute what lkv_quest_topk and
 * lkv_exact_attention compute for one (lazykv/selection.py:38-62 top_blocks over the Quest bound,
 * lazykv/exact.py:225-264 with the int8 cold tier), over all sequences in one launch each.
 * Row r = seq * heads + head. A sequence's blocks live anywhere in a paged store: its block table
 * table[seq * table_stride + b] gives the store row of its logical block b. Candidates of row r are
 * logical blocks 1 .. n_cand(r).
 *
 * lkv_ragged_quest_topk: q [rows * g, d]; kmin / kmax [heads][store rows][d] (row stride m_head per
 * head) in q's dtype; row_sel [rows][2] = (n_cand, k), n_cand <= max_cand <= 16384; work
 * [n_work][2] = (row, first candidate) chunks of 256 candidates covering every row's candidates
 * (a row with n candidates has ceil(n / 256) chunks at 0, 256, ...). out_blocks [rows][out_stride]
 * receives each row's k kept logical blocks in ascending order (the top k by bound, ties to the
 * lowest ids) and bitmap [rows][bitmap_words] (optional) their bits. Workspace:
 * lkv_ragged_topk_workspace(rows, max_cand) bytes.
 */
size_t lkv_ragged_topk_workspace(int rows, int max_cand);
int lkv_ragged_quest_topk(const void* q, int q_dtype, int rows, int g, int d, int heads,
                          const void* kmin, const void* kmax, int meta_dtype, int64_t m_head,
                          int64_t n_store, const int32_t* table, int64_t table_stride,
                          const int32_t* row_sel, int max_cand, const int32_t* work, int n_work,
                          int bound_mode, int32_t* out_blocks, int64_t out_stride,
                          uint32_t* bitmap, int bitmap_words, void* workspace,
                          size_t workspace_bytes, void* stream);

/*
 * lkv_ragged_schedule (host memory, no device work): the CTAs of one ragged attention launch.
 * row_items [rows] = a row's hot items plus an upper bound of its cold items; writes sched
 * [n][4] = (row, index in the row, the row's CTAs, the row's first partial) and *n_parts, and
 * returns n (the CTA count; at most max_ctas) or a negative status.
 */
int lkv_ragged_schedule(const int32_t* row_items, int rows, int n_sms, int32_t* sched, int max_ctas,
                        int* n_parts);
size_t lkv_ragged_attention_workspace(int g, int n_parts);

/*
 * lkv_ragged_exact_attention: every row's hot set and int8 cold set with their merge, in one
 * launch of the tensor-core stream kernel (bf16, d 64, bs 16, g in {1, 2, 4, 8}, device-resident
 * stores). hot: the pool of bf16 pairs as in lkv_exact_attention, `blocks` [rows][n_list] holding
 * pool rows directly (slot_of NULL; n_list is the row stride), each row's count in row_info.
 * records [n_records, heads, W] int8 records read through the block tables; excluded [rows]
 * [bitmap_words] the blocks of each row's hot set. row_info [rows][4] = (hot items, fill of the
 * current block, n_cand, 0): the hot list's last item is the current block, masked past its fill.
 * sched (device copy of lkv_ragged_schedule's output, n_ctas entries, n_parts partials). out
 * [rows * g, d] in out_dtype and lse [rows * g] (optional). Workspace:
 * lkv_ragged_attention_workspace(g, n_parts) bytes, zero-filled once (counters kept at zero).
 */
int lkv_ragged_exact_attention(const void* q, int rows, int g, int d, int bs, int heads,
                               const lkv_hot_set* hot, const uint8_t* records, int64_t n_records,
                               const int32_t* table, int64_t table_stride, const uint32_t* excluded,
                               int bitmap_words, const int32_t* row_info, const int32_t* sched,
                               int n_ctas, int n_parts, float scale, void* out, int out_dtype,
                               float* lse, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The cold tier of ragged rows in pinned host memory (lazykv/tiered.py:489-511 over
 * lazykv/pinned.py:73-92, the zero-copy read of the cold store): before the attention, the records
 * it will read are read over the link with mapped loads and staged in HBM. records [n_records,
 * heads, width] is the host store's device address (mapped, pinned); table [n][table_stride] the
 * batch's block tables; work [n_work][2] and row_info [rows][4] as lkv_ragged_quest_topk and
 * lkv_ragged_exact_attention take them; excluded (optional) the blocks the attention will skip,
 * which are not read. Candidate c (block 1 + c) of sequence i goes to staged row stage_first[i] + c
 * of stage [stage_rows, heads, width] (device memory), and stage_table [n][stage_stride] gets that
 * row (or -1 where the block table names no store row): lkv_ragged_exact_attention with
 * records = stage and table = stage_table then attends exactly what it would over a device store.
 * One launch of n_work CTAs; width a multiple of 16.
 */
int lkv_ragged_stage_records(const uint8_t* records, int64_t n_records, int heads, int width,
                             const int32_t* table, int64_t table_stride, const int32_t* work,
                             int n_work, const int32_t* row_info, const uint32_t* excluded,
                             int bitmap_words, uint8_t* stage, int64_t stage_rows,
                             const int32_t* stage_first, int32_t* stage_table,
                             int64_t stage_stride, void* stream);

/*
 * Residency admit on the device, fused with the fetch of the misses. Replaces the host side of
 * lazykv/tiered.py:383-487 (rank's device-to-host copy, the numpy LRU of admit, the staged H2D and
 * index_copy_, and the gather's last_used update), with the same LRU rule: for KV head j, chosen
 * [h, k] (row stride chosen_ld) block ids; a chosen block with block_slot -1 misses; victims are the
 * slots not holding a chosen block, least recently used first (ties by slot), given to the misses
 * in chosen order; evicted blocks get block_slot -1 and evicted_at = step (evicted_at optional);
 * every chosen slot gets last_used = step. Tables: block_slot [h, cap] int32 (pool index
 * 1..n_slots or -1), slot_block [h, n_slots] int32, last_used [h, n_slots] int64, evicted_at [h, cap]
 * int64. Each miss is then copied from the store (rows block*h + head: int8 records dequantised as
 * lazykv/quant.py:unpack, or pairs in `dtype`) into pool [n_slots + 2, h, 2, bs, d] row slot*h + head.
 * miss_blk / miss_slot [h, k] receive the misses in chosen order and n_miss [h] their count;
 * slots_out [h, k] (row stride slots_ld, optional) the pool index of every chosen block afterwards.
 * miss_total (optional, int64): every head's miss count is added to it on the device, a running
 * count of fetched pairs that needs no per-step host work (the reference's fetch counters).
 */
int lkv_tier_admit(const int32_t* chosen, int h, int k, int64_t chosen_ld, int32_t* block_slot,
                   int cap, int32_t* slot_block, int64_t* last_used, int n_slots,
                   int64_t* evicted_at, int64_t step, const void* store, int store_kind, void* pool,
                   int bs, int d, int dtype, int32_t* miss_blk, int32_t* miss_slot, int32_t* n_miss,
                   int32_t* slots_out, int64_t slots_ld, int64_t* miss_total, void* stream);

/*
 * One decode step of an exact int8/bf16 tier in the resident-split order, as a single call: for a
 * host that issues every layer's step eagerly, the three calls and the stream hand-off below cost
 * it less in one than in five (no reference counterpart: the reference's step is host-driven).
 * In order, on `stream` unless said:
 *   1. wait for the previous step's admit of the same events object (its tables, slots, chosen ids);
 *   2. unless `selected` is set (a selection already in `chosen`, its hot list and bitmap written by
 *      the caller), lkv_quest_topk_resident with the q / kmin / kmax / chosen / block_slot / hot /
 *      bitmap fields and the selection workspace;
 *   3. lkv_exact_attention over hot_set and cold_set into out / lse with the attention workspace;
 *   4. on `admit_stream`, after step 2: lkv_tier_admit of `chosen` (no slots_out), the misses fetched
 *      from `store` into `pool`, miss_total (optional) counting them; then the events object
 *      records this admit's completion.
 * The attention therefore runs while the admit does; its victims are never slots the hot list
 * names. Field meanings, limits and errors are those of the three entry points; the first failure
 * is returned (later parts are not issued). Events: lkv_split_events_create (two CUDA events,
 * no device memory; make it with the tier's device current), lkv_split_events_destroy;
 * lkv_split_join makes `stream` wait for the last admit, lkv_split_wait makes the host wait for it.
 */
typedef struct {
  const void* q;
  int q_dtype, hq, h, d;
  const void* kmin;
  const void* kmax;
  int meta_dtype;
  int64_t m_head;
  int first_block, n_cand, k, bound_mode;
  int32_t* chosen;
  int chosen_ld;
  int32_t* block_slot;
  int cap;
  int32_t* hot;
  int64_t hot_ld;
  uint32_t* bitmap;
  int bitmap_words;
  void* sel_workspace;
  size_t sel_workspace_bytes;
  int bs;
  const lkv_hot_set* hot_set;
  const lkv_cold_set* cold_set;
  float scale;
  void* out;
  int out_dtype;
  float* lse;
  void* att_workspace;
  size_t att_workspace_bytes;
  int32_t* slot_block;
  int64_t* last_used;
  int n_slots;
  int64_t* evicted_at;
  int64_t step;
  const void* store;
  int store_kind;
  void* pool;
  int pool_dtype;
  int32_t* miss_blk;
  int32_t* miss_slot;
  int32_t* n_miss;
  int64_t* miss_total;
  int selected;
} lkv_split_step_args;

typedef struct lkv_split_events lkv_split_events;
int lkv_split_events_create(lkv_split_events** out);
int lkv_split_events_destroy(lkv_split_events* ev);
int lkv_split_step(const lkv_split_step_args* a, lkv_split_events* ev, void* stream, void* admit_stream);
int lkv_split_join(lkv_split_events* ev, void* stream);
int lkv_split_wait(lkv_split_events* ev);

/*
 * Decode-time append (lazykv/tiered.py:306-334, the write of a new token into the block being
 * filled): T tokens of keys k and values v (element (head, token, channel) at head * s_head + token *
 * s_tok + channel, in elements of `dtype`) into slot [h, 2, bs, d] of the pool at token positions
 * fill .. fill + T - 1 (fill + T <= bs). One launch for both halves.
 */
int lkv_append_tokens(const void* k, int64_t k_s_head, int64_t k_s_tok, const void* v,
                      int64_t v_s_head, int64_t v_s_tok, int h, int t, int d, int dtype, void* slot,
                      int bs, int fill, void* stream);

/*
 * The bitmap of a selection made elsewhere (a recorded one replayed, lazykv/tiered.py:715-724):
 * for head j, bitmap [h, bitmap_words] row j is cleared, then the bit of every id in ids [h, k]
 * (row stride ids_ld) is set, as lkv_quest_topk sets it for its own selection; -1 entries and ids
 * at or past 32 * bitmap_words are skipped. An exact pass then skips exactly those blocks
 * (lazykv/exact.py:371-378). One launch of h CTAs.
 */
int lkv_mark_blocks(const int32_t* ids, int h, int k, int64_t ids_ld, uint32_t* bitmap,
                    int bitmap_words, void* stream);

/*
 * The selection for an attention that runs before (or beside) the step's admit: lkv_quest_topk in
 * LKV_ORDER_BLOCK, plus, for the j-th chosen block b of head h, hot[h * hot_ld + j] =
 * block_slot[h * cap + b] when that is a slot (>= 1), else -1, and a bitmap that marks only those
 * resident blocks. An exact pass over the bitmap's complement then covers the chosen blocks that
 * are not resident yet (from their records: the values a fetch would put in a slot), so the
 * output equals the admit-first order's, and lkv_tier_admit (with slots_out null) can run after
 * the attention or on another stream: its victims are never slots this hot list names. Same
 * selection paths and workspace as lkv_quest_topk (block order, h <= 64). The reference admits
 * before it attends (lazykv/tiered.py:389-487); no counterpart for the split.
 */
int lkv_quest_topk_resident(const void* q, int q_dtype, int hq, int h, int d, const void* kmin,
                            const void* kmax, int meta_dtype, int64_t m_head, int first_block,
                            int n_cand, int k, int bound_mode, int32_t* out_blocks, int out_ld,
                            const int32_t* block_slot, int cap, int32_t* hot, int64_t hot_ld,
                            uint32_t* bitmap, int bitmap_words, void* workspace,
                            size_t workspace_bytes, void* stream);

/*
 * lkv_quest_topk in block order followed by lkv_tier_admit of its selection, in one call: the
 * selection written to out_blocks (and the bitmap) is made resident (LRU victims, misses fetched and
 * dequantised into their slots, slots_out = the slots of the selected blocks). Replaces
 * lazykv/tiered.py:383-463 (rank, then admit). Same arguments and results as the two calls (the
 * selection's chosen_ld is out_ld, its k the admit's k, miss_total as lkv_tier_admit's); the admit's
 * arguments are checked before anything runs, so an invalid call launches nothing.
 * No reference counterpart as one call (the reference ranks on the device, then admits on the host).
 */
int lkv_quest_topk_admit(const void* q, int q_dtype, int hq, int h, int d, const void* kmin,
                         const void* kmax, int meta_dtype, int64_t m_head, int first_block,
                         int n_cand, int k, int bound_mode, int32_t* out_blocks, int out_ld,
                         float* out_bound, uint32_t* bitmap, int bitmap_words, void* workspace,
                         size_t workspace_bytes, int32_t* block_slot, int cap, int32_t* slot_block,
                         int64_t* last_used, int n_slots, int64_t* evicted_at, int64_t step,
                         const void* store, int store_kind, void* pool, int bs, int dtype,
                         int32_t* miss_blk, int32_t* miss_slot, int32_t* n_miss, int32_t* slots_out,
                         int64_t slots_ld, int64_t* miss_total, void* stream);

/*
 * Status word of the kernels that wait on shared-memory barriers (bounded waits): 0 when no wait
 * ran out, else the first code recorded (1 = a wait timed out; 2 = an attention CTA's item list
 * overflowed its shared memory, a sizing error that leaves that call's output empty). Synchronous;
 * clears it if asked.
 * No reference counterpart (the reference has no device-side waits).
 */
int lkv_device_status(int* status, int clear);

/*
 * A mirror of the status word in pinned, mapped host memory: after lkv_status_attach() (once per
 * device, with that device current; allocates the host word on the first call in the process),
 * every kernel that records a status also sets the mirror with a system-scope atomic, and
 * lkv_status_poll() reads it without synchronising (it sees a kernel's status once that kernel has
 * run), clearing it if asked. A decode loop polls it once per step to turn a bounded wait that ran
 * out into an error on the host without a device synchronisation per step.
 * No reference counterpart (the reference has no device-side waits).
 */
int lkv_status_attach(void);
int lkv_status_poll(int* status, int clear);

/*
 * Test hooks of the bounded waits (no reference counterpart). key LKV_DEBUG_SELECT_WAIT_ITERS sets
 * the bound (tries, 1 .. 2^21) of the TMA-scored selection's tile waits, for every later call in
 * the process; LKV_DEBUG_SELECT_STALL_NEXT = 1 makes every scoring CTA of the next TMA-scored
 * selection first wait on a barrier that nothing completes, so that the wait runs out and the
 * failure path runs (status 1, poisoned output) with the GPU left usable.
 * LKV_DEBUG_EXCHANGE_WAIT_ITERS sets the bound (polls, 1 .. 2^22) of lkv_exchange_merge's wait for
 * its peers. Not for production use; not thread-safe.
 */
enum { LKV_DEBUG_SELECT_WAIT_ITERS = 1, LKV_DEBUG_SELECT_STALL_NEXT = 2, LKV_DEBUG_EXCHANGE_WAIT_ITERS = 3 };
int lkv_debug_set(int key, int64_t value);

/*
 * The cross-GPU exchange of a context-sharded layer's partials by peer stores over NVLink, merged
 * by log-sum-exp (the n-way merge_lse of lazykv/exact.py:69-85; the reference is single-device and
 * has no counterpart). Each rank allocates one region (lkv_exchange_alloc: cudaMalloc'd, zeroed,
 * lkv_exchange_region_bytes(rows, d, world) bytes) and gets its 64-byte CUDA IPC handle; the ranks
 * swap handles (any host channel) and open their peers' regions (lkv_exchange_open; closed with
 * lkv_exchange_close, freed with lkv_exchange_free). lkv_exchange_merge, one launch per layer and
 * step, takes this rank's partial (out [rows, d] float32, lse [rows]) and the regions of every rank
 * in rank order (bases[rank] its own): it stores the rank's rows into every region, adds one to a
 * per-row-group arrival counter there, waits until every rank's rows of this exchange have
 * arrived (a bounded wait: on timeout the status word gets 1 and the rows become this rank's own
 * partial), and writes the merge (merged [rows, d] in out_dtype, merged_lse [rows] optional).
 * Every rank calls it the same number of times per region, with the same rows and d; consecutive
 * calls alternate between two halves of the inbox, so one rank may run one exchange ahead of
 * another. d % 4 == 0; world <= 64; rows <= 4,096. Graph-capturable (no host state per call).
 */
size_t lkv_exchange_region_bytes(int rows, int d, int world);
int lkv_exchange_alloc(int rows, int d, int world, void** base, void* ipc_handle);
int lkv_exchange_open(const void* ipc_handle, void** peer_base);
int lkv_exchange_close(void* peer_base);
int lkv_exchange_free(void* base);
int lkv_exchange_merge(const float* out, const float* lse, int rows, int d, int world, int rank,
                       void* const* bases, void* merged, int out_dtype, float* merged_lse,
                       void* stream);

/*
 * Log-sum-exp merge of n_parts partials. Replaces lazykv/exact.py:69-85 merge_lse (n_parts = 2)
 * and is the cross-GPU merge of all-gathered shard partials. outs [n_parts, rows, d] and lses
 * [n_parts, rows] float32 -> out [rows, d] in out_dtype, lse_out [rows] float32 (optional).
 * Parts with lse = -inf contribute nothing; all parts empty gives out = 0, lse = -inf.
 */
int lkv_lse_merge(const float* outs, const float* lses, int n_parts, int64_t rows, int d,
                  void* out, int out_dtype, float* lse_out, void* stream);

/*
 * lkv_lse_merge over partials packed as each rank sends them in one collective: part k at
 * parts + k * rows * (d + 1) holds out [rows, d] then lse [rows] (the per-rank partials of a
 * context-sharded step after an all-gather; no reference counterpart).
 */
int lkv_lse_merge_packed(const float* parts, int n_parts, int64_t rows, int d, void* out, int out_dtype,
                         float* lse_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LKV_H */
