/*
 * snapmind_b200 — C ABI of the B200 (sm_100a) KV-cache hot path of snapmind.
 *
 * Plain C: device pointers, element strides, sizes, a cudaStream_t passed as
 * `void *`.  Every entry point returns an int status; on failure the message
 * of the calling host thread's last error is returned by snapmind_last_error().
 * No entry point allocates device memory; callers own every buffer.
 *
 * Paged pool layout (one pool for K, one for V):
 *     pool[layer][block][head][slot][dim]      (dim contiguous)
 * A (block, head) tile of block_size x head_dim elements is contiguous, so a
 * gather moves whole tiles and the decode kernel stages one tile per TMA copy.
 * `pool_layer_stride` is the element distance between consecutive layers
 * (0 when a call covers a single layer).
 *
 * Block tables are int32 rows of physical block ids: entry j of sequence b
 * (layer l when tables are per layer) lives at
 *     block_tables[l * table_stride_layer + b * table_stride_seq + j].
 *
 * Device error word: kernels never trap.  An out-of-range block id, table
 * entry or split skips the access and ORs a SNAPMIND_DEVERR_* bit into
 * `*err_word` (a device int32 the caller owns and may pass as NULL).
 */
#ifndef SNAPMIND_B200_H_
#define SNAPMIND_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define SNAPMIND_API __attribute__((visibility("default")))
#else
#define SNAPMIND_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define SNAPMIND_OK 0
#define SNAPMIND_ERR_OUT_OF_BLOCKS 1 /* "PagedKVCache: out of blocks" */
#define SNAPMIND_ERR_BAD_ARGUMENT 2
#define SNAPMIND_ERR_CUDA 3
#define SNAPMIND_ERR_TIMEOUT 4
#define SNAPMIND_ERR_UNSUPPORTED 5

/* element types */
#define SNAPMIND_DTYPE_F32 0
#define SNAPMIND_DTYPE_BF16 1
#define SNAPMIND_DTYPE_F16 2

/* device error word bits */
#define SNAPMIND_DEVERR_BLOCK_ID 1      /* physical block id outside [0, num_blocks) */
#define SNAPMIND_DEVERR_TABLE 2         /* logical block index outside the table row */
#define SNAPMIND_DEVERR_SPLIT 4         /* sequence longer than the split plan covers */
#define SNAPMIND_DEVERR_OUT_OF_BLOCKS 8 /* reserve found too few free blocks */
#define SNAPMIND_DEVERR_TIMEOUT 16      /* a bounded device wait gave up */
#define SNAPMIND_DEVERR_POSITION 32     /* rotary position outside the cos/sin tables */

/* decode flags */
#define SNAPMIND_DECODE_FORCE_GENERIC 1 /* use the CUDA-core kernel even where the tensor-core one applies */

SNAPMIND_API int snapmind_abi_version(void);
SNAPMIND_API const char *snapmind_last_error(void);

/*
 * Append n_tokens K/V rows per sequence into the paged pools.
 * Replaces the per-token slice writes of PagedKVCache.store
 * (snapmind/kv_cache/paged.py:34-54): token t of sequence b goes to slot
 * s = slot_start(b) + t, block table entry s / block_size, row s % block_size.
 * slot_start(b) = slot_starts[b] + slot_start0 when slot_starts != NULL, else
 * slot_start0.  Input element (layer, b, head, t, d) is read at
 * k_new + layer*in_stride_layer + b*in_stride_seq + head*in_stride_head
 *       + t*in_stride_tok + d.
 * Input and pool dtypes may differ (values are converted, round to nearest even).
 * Table entries must already exist (the host or snapmind_kv_reserve grows them).
 * v_pool and v_new may both be NULL: a single-pool cache (the MLA latent rows).
 */
SNAPMIND_API int snapmind_kv_append(void *k_pool, void *v_pool, int pool_dtype, int64_t pool_layer_stride,
                       const void *k_new, const void *v_new, int in_dtype,
                       int64_t in_stride_layer, int64_t in_stride_seq, int64_t in_stride_head,
                       int64_t in_stride_tok,
                       const int32_t *block_tables, int64_t table_stride_seq,
                       int64_t table_stride_layer, int32_t table_width,
                       const int32_t *slot_starts, int32_t slot_start0,
                       int32_t n_layers, int32_t batch, int32_t n_tokens, int32_t n_heads,
                       int32_t head_dim, int32_t block_size, int32_t num_blocks,
                       int32_t *err_word, void *stream);

/*
 * Gather the first seq_len(b) tokens of every sequence out of the paged pools.
 * Replaces PagedKVCache.fetch (snapmind/kv_cache/paged.py:56-78): the output of
 * each layer is the concatenation over b of (n_heads, seq_len(b), head_dim)
 * blocks — for one sequence exactly the (1, H, T, D) tensor fetch returns.
 * seq_len(b) = seq_lens[b] when seq_lens != NULL, else seq_len0.
 * Output layer l starts at k_out + l*out_layer_stride and holds
 * out_layer_capacity elements; when the lengths need more, nothing is written
 * and SNAPMIND_DEVERR_TABLE is set.  batch <= 8192.  v_pool and v_out may both
 * be NULL (single-pool cache).
 */
SNAPMIND_API int snapmind_kv_gather(const void *k_pool, const void *v_pool, int dtype, int64_t pool_layer_stride,
                       void *k_out, void *v_out, int64_t out_layer_stride,
                       int64_t out_layer_capacity,
                       const int32_t *block_tables, int64_t table_stride_seq,
                       int64_t table_stride_layer, int32_t table_width,
                       const int32_t *seq_lens, int32_t seq_len0,
                       int32_t n_layers, int32_t batch, int32_t n_heads, int32_t head_dim,
                       int32_t block_size, int32_t num_blocks, int32_t *err_word, void *stream);

/*
 * Move n token rows (all heads, K and V) inside one layer's pools, reading
 * every source row before writing any destination row.  Replaces the
 * clone-then-assign compaction loop of PagedKVCache.evict
 * (snapmind/kv_cache/paged.py:96-113).  The four index arrays are HOST arrays
 * of n entries (copied into the launch parameters); n <= 64.
 */
SNAPMIND_API int snapmind_kv_copy_slots(void *k_pool, void *v_pool, int dtype,
                           const int32_t *src_blocks, const int32_t *src_rows,
                           const int32_t *dst_blocks, const int32_t *dst_rows, int32_t n,
                           int32_t n_heads, int32_t head_dim, int32_t block_size,
                           int32_t num_blocks, int32_t *err_word, void *stream);

/*
 * Reserve room for n_new tokens in each of `batch` sequences sharing one pool
 * (the batched form of the block growth in PagedKVCache.store,
 * snapmind/kv_cache/paged.py:38-42).  Sequences that cross a block boundary
 * take blocks from the top of the device free stack in ascending sequence
 * order; seq_lens[b] += n_new.  All or nothing: when the stack holds too few
 * blocks or a table row is too short, nothing changes and the matching
 * SNAPMIND_DEVERR_* bit is set.
 */
SNAPMIND_API int snapmind_kv_reserve(int32_t *block_tables, int64_t table_stride_seq, int32_t table_width,
                        int32_t *seq_lens, int32_t batch, int32_t n_new, int32_t block_size,
                        int32_t *free_stack, int32_t *free_top, int32_t num_blocks,
                        int32_t *err_word, void *stream);

/*
 * Return the blocks of the listed sequences to the device free stack (in
 * list order, each sequence's blocks in table order) and set their length to 0.
 * seq_ids is a device array of n_release sequence indices.
 */
SNAPMIND_API int snapmind_kv_release(int32_t *block_tables, int64_t table_stride_seq, int32_t table_width,
                        int32_t *seq_lens, const int32_t *seq_ids, int32_t n_release,
                        int32_t block_size, int32_t *free_stack, int32_t *free_top,
                        int32_t num_blocks, int32_t *err_word, void *stream);

/*
 * One segment of a token-dimension concatenation: `rows` rows (the leading
 * dims of a (..., T, D) tensor, flattened) of n_tokens x head_dim elements,
 * row r starting row_stride tokens (row_stride*head_dim elements) after row
 * r-1 at k (likewise v).
 */
typedef struct snapmind_segment {
  const void *k;
  const void *v;
  int64_t row_stride;
  int32_t n_tokens;
  int32_t pad_;
} snapmind_segment;

/*
 * Concatenate segments along the token dimension into (rows, sum n, D)
 * outputs — the torch.cat(k_parts, dim=-2) of the tiered cache's live view
 * (snapmind/kv_cache/tiered.py:156-182) in one launch per 256 segments.
 * `segs` is a HOST array of n_segs descriptors.  Output row r starts
 * out_row_stride tokens after row r-1 (out_row_stride >= sum n).
 */
SNAPMIND_API int snapmind_kv_concat(const snapmind_segment *segs, int32_t n_segs, int32_t rows,
                       int32_t head_dim, int dtype, void *k_out, void *v_out,
                       int64_t out_row_stride, void *stream);

/*
 * Batched tiered pool, placement step (the device-side form of the tiered
 * cache's residency policy, snapmind/kv_cache/tiered.py:95-154, with the
 * LRU + sink/window pinning of the many-sequence pool).  One CTA: every
 * sequence grows by n_new tokens (a new chunk gets a slot; the chunk just
 * completed is copied to outbound staging slot stage_out_base + b), then each
 * request (req_seq[i], req_chunk[i]) that is not resident is admitted from
 * inbound staging slot stage_in_base + i.  Slots come free ones first (by id),
 * then least recently used by (slot_last, slot id) among unpinned chunks;
 * chunk 0, chunks overlapping the last `window` tokens and the active chunk
 * are pinned.  Rebuilds tables [batch][max_chunks] (resident slots in chunk
 * order) and table_lens, and writes the copy plan [max_plan][2] (src, dst
 * slot) and its length.  req_* are HOST arrays of n_req <= 64 entries;
 * n_slots <= 8192.  Pool exhaustion sets SNAPMIND_DEVERR_OUT_OF_BLOCKS.
 */
SNAPMIND_API int snapmind_tiered_plan(int32_t *slot_owner, int32_t *slot_last, int32_t *chunk_slot,
                         int32_t *seq_lens, int32_t *tables, int32_t *table_lens, int32_t *plan,
                         int32_t *plan_count, int32_t batch, int32_t max_chunks, int32_t n_slots,
                         int32_t chunk, int32_t sink, int32_t window, int32_t step, int32_t n_new,
                         int32_t stage_in_base, int32_t stage_out_base, int32_t max_plan,
                         const int32_t *req_seq, const int32_t *req_chunk, int32_t n_req,
                         int32_t *err_word, void *stream);

/*
 * Execute a tiered plan: copy slot src -> dst for every plan entry, every
 * layer, K and V (slot_bytes bytes per slot and layer, layer_stride_bytes
 * between layers).
 */
SNAPMIND_API int snapmind_tiered_move(void *k_pool, void *v_pool, int64_t layer_stride_bytes, int64_t slot_bytes,
                         int32_t n_layers, const int32_t *plan, const int32_t *plan_count,
                         int32_t max_plan, void *stream);

/*
 * Strided copy between host-pinned backing and device slots (height rows of
 * width bytes; direction inferred from the pointers), issued with
 * cudaMemcpy2DAsync on `stream` — one call moves a chunk's K (or V) rows of
 * every layer.  Replaces the chunk `.to(device)` / `.to("cpu")` moves of the
 * tiered cache (snapmind/kv_cache/tiered.py:108-118, 142-151).
 */
SNAPMIND_API int snapmind_copy_2d(void *dst, int64_t dst_pitch, const void *src, int64_t src_pitch, int64_t width,
                     int64_t height, void *stream);

/*
 * Rotary position encoding of q and k in place, one launch for both — the
 * rotate-half RoPE of RotaryPositionalEncoding.apply_to_qk
 * (snapmind/layers/positional/rope.py:47-61), bit-identical to it on the same
 * device: cos/sin rows cast to the tensor's dtype, x*cos and
 * rotate_half(x)*sin and their sum each rounded to the dtype.  q is
 * [batch][n_q_heads][n_tok][head_dim] and k [batch][n_kv_heads][n_tok][head_dim]
 * with the given element strides (head_dim contiguous), both of `dtype`;
 * cos_table / sin_table are fp32 [n_pos][head_dim].  Token t of sequence b
 * uses row positions[b * pos_stride_b + t] (int64, device; pos_stride_b = 0
 * shares one position list across the batch), or row t when positions is
 * NULL.  A position outside [0, n_pos) leaves its row unchanged and sets
 * SNAPMIND_DEVERR_POSITION.
 */
SNAPMIND_API int snapmind_rope_qk(void *q, int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_t,
                                  int32_t n_q_heads, void *k, int64_t k_stride_b, int64_t k_stride_h,
                                  int64_t k_stride_t, int32_t n_kv_heads, int dtype, int32_t batch, int32_t n_tok,
                                  int32_t head_dim, const float *cos_table, const float *sin_table, int64_t n_pos,
                                  const int64_t *positions, int64_t pos_stride_b, int32_t *err_word, void *stream);

/*
 * Frozen chunk keys of the lookahead indexer: for chunks
 * [chunk_begin, chunk_begin + chunk_count) of every sequence, the mean of the
 * chunk's rows (the first `width` columns of each pool row of row_width
 * elements) — LookaheadSparseIndexer.build_frozen_keys
 * (snapmind/layers/indexer/lookahead.py:40-50), with chunk c = block c of the
 * sequence's table (block_size = chunk size).  When `proj` is not NULL the mean
 * is also projected: out = proj . mean, proj row-major [out_dim][width] of
 * proj_dtype.  out is fp32 [batch][max_chunks][out_dim or width]; chunks past
 * a sequence's length are written as zeros.  seq_lens may be NULL: every
 * chunk then holds block_size rows.
 */
SNAPMIND_API int snapmind_indexer_pool_chunks(const void *pool, int dtype, int64_t row_width, int32_t width,
                                 const int32_t *block_tables, int64_t table_stride, int32_t table_width,
                                 const int32_t *seq_lens, int32_t batch, int32_t block_size,
                                 int32_t num_blocks, int32_t chunk_begin, int32_t chunk_count,
                                 int32_t max_chunks, const void *proj, int proj_dtype, int32_t out_dim,
                                 float *out, void *workspace, int64_t workspace_bytes, int32_t *err_word,
                                 void *stream);

/*
 * Bytes of workspace (fp32 chunk means) that lets snapmind_indexer_pool_chunks
 * pool many chunks and project them in two kernels (a streaming mean over
 * many chunks in flight, then a tiled projection).  Without it, or for a few
 * chunks, one fused kernel does both (same result up to fp32 rounding).
 */
SNAPMIND_API int64_t snapmind_indexer_pool_workspace_bytes(int32_t batch, int32_t chunk_count, int32_t width);

/*
 * The reference chunk score for every chunk at once (lookahead.py:82-106):
 * scores[c] = mean_n sigmoid(sum_h relu(q[n,h,:] . keys[c,:]) * w[n,h]);
 * q fp32 [n_rows][n_heads][dim], w fp32 [n_rows][n_heads], keys fp32
 * [n_chunks][dim].
 */
SNAPMIND_API int snapmind_indexer_score_ref(const float *q, const float *w, int32_t n_rows, int32_t n_heads,
                               const float *keys, int32_t n_chunks, int32_t dim, float *scores,
                               void *stream);

/*
 * The query of the chunk selector, out[b][o] = sum_d w[o][d] * hidden[b][d]
 * with fp32 accumulation and fp32 output: hidden [batch][d_model] and w
 * [out_dim][d_model] in `dtype`.  One launch that reads w once (the selector's
 * W_q projection; the reference indexer projects its query with nn.Linear
 * layers, snapmind/layers/indexer/lookahead.py:32-35).
 */
SNAPMIND_API int snapmind_indexer_query(const void *hidden, const void *w, int dtype, float *out, int32_t batch,
                                        int32_t d_model, int32_t out_dim, void *stream);

/*
 * Sigmoid-gated chunk scores sigmoid(q . k * scale + bias) and the k best
 * chunks per sequence (no reference counterpart: IndexerConfig.score_k exists
 * but is never read, snapmind/core/config.py:92).  Order: score descending,
 * then chunk id ascending (a stable descending sort).  q [batch][dim], keys
 * [batch][max_chunks][dim] (dtype), n_chunks[b] (device, or n_chunks0 for all)
 * chunks valid per sequence; out_idx int32 [batch][k] (-1 past the valid
 * chunks), optional out_score [batch][k] and all_scores [batch][max_chunks].
 * max_chunks <= 16384.
 */
SNAPMIND_API int snapmind_indexer_topk(const void *q, const void *keys, int dtype, const int32_t *n_chunks,
                          int32_t n_chunks0, int32_t batch, int32_t max_chunks, int32_t dim, float scale,
                          float bias, int32_t k, int32_t *out_idx, float *out_score, float *all_scores,
                          void *workspace, int64_t workspace_bytes, void *stream);

/*
 * Bytes of device workspace snapmind_indexer_topk uses for its many-CTA form
 * (chunks scored and pre-selected 128 per CTA, the last CTA of a sequence
 * merging the candidates); 0 for invalid sizes.  The workspace must be
 * zero-filled before its first use and is left zeroed by every call; calls
 * sharing one workspace must not overlap on the GPU.  With workspace NULL the
 * call uses one CTA per sequence instead (same result).
 */
SNAPMIND_API int64_t snapmind_indexer_topk_workspace_bytes(int32_t batch, int32_t max_chunks, int32_t k);

/*
 * Sparse MLA decode attention over the positions of an attention sink
 * (< sink), a recent window (>= len - window) and the selected chunks
 * (selected [batch][k] chunk ids, -1 = unused), read from the paged latent
 * pools (latent [blocks][block_size][kv_lora_rank], rope
 * [blocks][block_size][rope_dim]) through the block tables.  Computes, per
 * head, softmax(scale * (q_lat . c_t + q_pe . k_pe_t)) over those positions
 * and the latent output sum_t p_t c_t into out [batch][n_heads][kv_lora_rank]
 * — the attention of MultiHeadLatentAttention.forward
 * (snapmind/layers/attention/mla.py:217-245) with the query absorbed into the
 * latent space (q_lat = W_uk^T q_nope) and restricted to the selection.
 * n_heads is a multiple of 16; splits > 1 need a zero-filled workspace of
 * snapmind_sparse_mla_workspace_bytes(...) bytes.
 */
/*
 * Split count the sparse MLA kernels run best with for this batch (CTAs per
 * sequence along the attended positions): the tcgen05 kernel (128 heads,
 * kv_lora_rank 512, rope 64, block 64, bf16/f16, k <= 256) fills the SMs with
 * (split, head half) CTAs; the other shapes with (split, 32-head group) CTAs.
 * No reference counterpart (the reference has no GPU path).
 */
SNAPMIND_API int32_t snapmind_sparse_mla_default_splits(int32_t batch, int32_t n_heads, int32_t kv_lora_rank,
                                                       int32_t rope_dim, int32_t block_size, int32_t dtype);
SNAPMIND_API int64_t snapmind_sparse_mla_workspace_bytes(int32_t batch, int32_t n_heads, int32_t kv_lora_rank,
                                                         int32_t n_splits);
SNAPMIND_API int snapmind_sparse_mla_decode(const void *q_lat, const void *q_pe, int dtype, const void *latent_pool,
                               const void *rope_pool, const int32_t *block_tables, int64_t table_stride,
                               int32_t table_width, const int32_t *seq_lens, const int32_t *selected,
                               int32_t k, int32_t sink, int32_t window, float scale, int32_t batch,
                               int32_t n_heads, int32_t kv_lora_rank, int32_t rope_dim, int32_t block_size,
                               int32_t num_blocks, int32_t n_splits, void *out, void *workspace,
                               int64_t workspace_bytes, int32_t *err_word, void *stream);

/*
 * Paged GQA decode attention: one query token per sequence against the
 * seq_lens[b] cached tokens reached through the block table.  Computes
 * softmax(q k^T * scale) v per query head, query head h reading kv head
 * h / (n_q_heads / n_kv_heads) — the math of GroupedQueryAttention.forward
 * (snapmind/layers/attention/gqa.py:69-82: repeat_interleave, matmul, softmax,
 * matmul) over the tokens PagedKVCache.fetch would return, without
 * materialising either.  q, pools and out share `dtype`; accumulation is fp32.
 *
 * Long sequences are split into chunks of split_tokens tokens (a multiple of
 * block_size; <= 0 picks snapmind_paged_gqa_decode_split_tokens) processed by
 * separate CTAs; the last CTA of a sequence merges the partial softmax states.
 * `workspace` must hold snapmind_paged_gqa_decode_workspace_bytes(...) bytes.
 * It starts with the split tickets, one int32 per (sequence, kv head), which
 * must be zero when a call starts and are zero again when it ends; the
 * partial states follow at the next 256-byte boundary.  A zero-filled
 * workspace is reusable by calls over the same or fewer sequences; a call over
 * more sequences than an earlier one needs the bytes of its extra tickets
 * cleared first (the earlier call may have put partials there).  Calls
 * sharing one workspace must not overlap on the GPU.
 */
SNAPMIND_API int32_t snapmind_paged_gqa_decode_split_tokens(int32_t batch, int32_t n_kv_heads,
                                               int32_t max_seq_len, int32_t block_size);
SNAPMIND_API int64_t snapmind_paged_gqa_decode_workspace_bytes(int32_t batch, int32_t n_q_heads,
                                                  int32_t n_kv_heads, int32_t head_dim,
                                                  int32_t max_seq_len, int32_t split_tokens);
SNAPMIND_API int snapmind_paged_gqa_decode(const void *q, int64_t q_stride_seq, int64_t q_stride_head,
                              const void *k_pool, const void *v_pool, int dtype,
                              const int32_t *block_tables, int64_t table_stride_seq,
                              int32_t table_width, const int32_t *seq_lens,
                              void *out, int64_t out_stride_seq, int64_t out_stride_head,
                              float scale, int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
                              int32_t head_dim, int32_t block_size, int32_t num_blocks,
                              int32_t max_seq_len, int32_t split_tokens, int32_t flags,
                              void *workspace, int64_t workspace_bytes, int32_t *err_word,
                              void *stream);

/*
 * snapmind_paged_gqa_decode with this step's token stored by the same launch:
 * replaces snapmind_kv_append of one token per sequence (PagedKVCache.store,
 * snapmind/kv_cache/paged.py:34-54) followed by snapmind_paged_gqa_decode
 * (the attention of snapmind/layers/attention/gqa.py:62-85, whose cache
 * concatenation the store stands for).  seq_lens already counts the token
 * (after the reserve that gave it a slot): k_new[b] / v_new[b]
 * ([batch][n_kv_heads][head_dim] in the pool's dtype, element strides
 * new_stride_seq / new_stride_head, head dim contiguous) are written at
 * position seq_lens[b] - 1 of sequence b, then every sequence attends over its
 * seq_lens[b] tokens.  On the tensor-core path the split holding that
 * position writes the rows before its loads; elsewhere the append kernel runs
 * first on the same stream.  The stored bytes equal snapmind_kv_append's.
 */
SNAPMIND_API int snapmind_paged_gqa_decode_append(const void *q, int64_t q_stride_seq, int64_t q_stride_head,
                                     void *k_pool, void *v_pool, int dtype,
                                     const int32_t *block_tables, int64_t table_stride_seq,
                                     int32_t table_width, const int32_t *seq_lens,
                                     const void *k_new, const void *v_new, int64_t new_stride_seq,
                                     int64_t new_stride_head, void *out, int64_t out_stride_seq,
                                     int64_t out_stride_head, float scale, int32_t batch, int32_t n_q_heads,
                                     int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                                     int32_t num_blocks, int32_t max_seq_len, int32_t split_tokens,
                                     int32_t flags, void *workspace, int64_t workspace_bytes,
                                     int32_t *err_word, void *stream);

/*
 * snapmind_paged_gqa_decode over a window of each sequence: sequence b attends
 * to tokens [seq_starts[b], seq_lens[b]) of its table row (seq_starts: int32,
 * device, one entry per sequence; a start at or past the length gives a zero
 * output).  For a sliding window kept as a ring of blocks the start is below
 * block_size: the blocks before the window are dropped from the table and the
 * first block's leading tokens are masked.  No reference counterpart as one op:
 * the reference trims the concatenated K/V to the window
 * (snapmind/kv_cache/sliding_window.py:31-38, snapmind/models/mistral.py:58-60).
 */
SNAPMIND_API int snapmind_paged_gqa_decode_window(const void *q, int64_t q_stride_seq, int64_t q_stride_head,
                                                 const void *k_pool, const void *v_pool, int dtype,
                                                 const int32_t *block_tables, int64_t table_stride_seq,
                                                 int32_t table_width, const int32_t *seq_lens,
                                                 const int32_t *seq_starts, void *out, int64_t out_stride_seq,
                                                 int64_t out_stride_head, float scale, int32_t batch,
                                                 int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                                                 int32_t block_size, int32_t num_blocks, int32_t max_seq_len,
                                                 int32_t split_tokens, int32_t flags, void *workspace,
                                                 int64_t workspace_bytes, int32_t *err_word, void *stream);

/*
 * snapmind_paged_gqa_decode for a rank of a KV-head-sharded decode: this rank
 * holds kv heads [head_offset / group, ...) of every sequence and its query
 * heads start at global head `head_offset`.  Instead of one local output, the
 * kernel stores every finished output row into the output buffer of each of
 * the n_peers ranks (peer_out: device array of n_peers 16-byte-aligned device
 * pointers, in rank order, this rank's own buffer included; peers are reached
 * by plain 16-byte NVLink stores through CUDA IPC mappings), at the global
 * head offset, with out_stride_seq / out_stride_head of the full
 * [batch][heads][head_dim] buffer (head_dim and both strides multiples of 16
 * bytes).  seq_starts may be NULL (whole sequences) or as in
 * snapmind_paged_gqa_decode_window.  The workspace is that of
 * snapmind_paged_gqa_decode.  Follow it on the same stream with
 * snapmind_peer_sync (SIGNAL | WAIT).  No reference counterpart: snapmind runs
 * on one device; this replaces the all-gather of the per-rank head slices.
 */
SNAPMIND_API int snapmind_paged_gqa_decode_peers(const void *q, int64_t q_stride_seq, int64_t q_stride_head,
                                                const void *k_pool, const void *v_pool, int dtype,
                                                const int32_t *block_tables, int64_t table_stride_seq,
                                                int32_t table_width, const int32_t *seq_lens,
                                                const int32_t *seq_starts, void *const *peer_out,
                                                int32_t n_peers, int32_t head_offset, int64_t out_stride_seq,
                                                int64_t out_stride_head, float scale, int32_t batch,
                                                int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                                                int32_t block_size, int32_t num_blocks, int32_t max_seq_len,
                                                int32_t split_tokens, int32_t flags, void *workspace,
                                                int64_t workspace_bytes, int32_t *err_word, void *stream);

/*
 * One warp on `stream`.  SNAPMIND_PEER_SIGNAL: after a system-scope fence
 * (the peer stores of the work before it on the stream are complete), write
 * `epoch` (> 0, growing from call to call) into element `rank` of every rank's
 * flag array (peer_flags: device array of n_peers pointers to int32[n_peers]).
 * SNAPMIND_PEER_WAIT: wait until flags[r] >= epoch for every r < n_peers
 * (this rank's own flag array); the wait gives up after 2 s and then ORs
 * SNAPMIND_DEVERR_TIMEOUT into *err_word.  Work enqueued after it on the
 * stream sees every rank's output rows.
 */
#define SNAPMIND_PEER_SIGNAL 1
#define SNAPMIND_PEER_WAIT 2
SNAPMIND_API int snapmind_peer_sync(int32_t *const *peer_flags, const int32_t *flags, int32_t n_peers,
                                    int32_t rank, int32_t epoch, int32_t what, int32_t *err_word, void *stream);

/*
 * CUDA IPC for the peer buffers.  snapmind_ipc_export writes the
 * SNAPMIND_IPC_HANDLE_BYTES-byte handle of the device allocation holding `ptr`
 * and ptr's offset inside it; another process on the same node opens it with
 * snapmind_ipc_open (peer access enabled) and gets the matching pointer of its
 * own address space, to be released with snapmind_ipc_close(ptr, offset).  An
 * allocation can be opened once per process.
 */
#define SNAPMIND_IPC_HANDLE_BYTES 64
SNAPMIND_API int snapmind_ipc_export(const void *ptr, void *handle_out, int64_t *offset_out);
SNAPMIND_API int snapmind_ipc_open(const void *handle, int64_t offset, void **ptr_out);
SNAPMIND_API int snapmind_ipc_close(void *ptr, int64_t offset);

/*
 * The same paged GQA decode for callers that cannot allocate device memory:
 * a host bound through this C ABI with no CUDA allocator of its own (or whose
 * device memory belongs to another allocator it cannot reach), or a serving
 * loop that must not call cudaMalloc between steps because it can synchronise
 * the device.  No counterpart exists in the reference (snapmind has no GPU
 * path); it takes the arguments of snapmind_paged_gqa_decode minus the
 * workspace and allocates nothing.
 *
 * Its scratch is a static device array of SNAPMIND_NOALLOC_DECODE_SCRATCH_BYTES
 * that every GPU loading the library holds until exit; a call that would need
 * more is rejected (SNAPMIND_ERR_BAD_ARGUMENT, with the sizes in the message).
 * The first call on a device looks up the array's address — make it before
 * any stream capture.  All calls on a device share the array: each clears the
 * ticket counters it needs on its stream, and calls that overlap on the GPU
 * race on the shared scratch and must not be issued.
 */
#define SNAPMIND_NOALLOC_DECODE_SCRATCH_BYTES (16u << 20)
SNAPMIND_API int snapmind_paged_gqa_decode_noalloc(const void *q, int64_t q_stride_seq, int64_t q_stride_head,
                                      const void *k_pool, const void *v_pool, int dtype,
                                      const int32_t *block_tables, int64_t table_stride_seq,
                                      int32_t table_width, const int32_t *seq_lens,
                                      void *out, int64_t out_stride_seq, int64_t out_stride_head,
                                      float scale, int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
                                      int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                      int32_t max_seq_len, int32_t split_tokens, int32_t flags,
                                      int32_t *err_word, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SNAPMIND_B200_H_ */
