/*
 * linattn_b200 — C ABI of the B200 (sm_100a) sparse-attention hot path.
 *
 * Plain pointers and sizes only.  Every buffer is device memory owned by the
 * caller, workspaces included; the library allocates nothing on a call.  The one
 * exception is linattn_sparse_attention_noalloc, whose scratch is a fixed
 * library-owned device array (see its declaration).  Kernels are enqueued on the caller's
 * `stream` (a cudaStream_t passed as void*; NULL = legacy default stream).
 * Functions return LINATTN_OK or an error code; linattn_last_error() gives the
 * message (thread-local).  Device-side problems (a page id outside the page
 * table, a bounded wait that gave up) are OR-ed into the optional `status`
 * word (int32 in device memory) as LINATTN_DEV_* bits and never trap.
 *
 * Each entry point names the reference function it replaces (paths inside the
 * tongxin/linattn project).
 */
#ifndef LINATTN_B200_H
#define LINATTN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
enum {
  LINATTN_F32 = 0,
  LINATTN_F16 = 1,
  LINATTN_BF16 = 2,
  LINATTN_FP8E4M3 = 3, /* float8_e4m3fn codes + fp32 scales */
  LINATTN_I32 = 4,
  LINATTN_I64 = 5
};

/* host return codes */
enum { LINATTN_OK = 0, LINATTN_EINVAL = 1, LINATTN_EUNSUPPORTED = 2, LINATTN_ECUDA = 3 };

/* device status bits */
enum { LINATTN_DEV_BAD_ID = 1, LINATTN_DEV_TIMEOUT = 2, LINATTN_DEV_OVERFLOW = 4 };

/*
 * KV pages.  Page `p` of (batch b, kv head h) holds `page_size` contiguous rows of
 * `head_dim` elements at
 *     base + b*stride_b + phys*stride_page + h*stride_head        (elements)
 * with phys = page_table[b*page_table_stride + p] (paged pool, stride_b = 0) or
 * phys = p (no page table).  The reference's contiguous cache (B, H_kv, T, D) is
 * stride_b = H_kv*T*D, stride_page = page_size*D, stride_head = T*D; the paged pool
 * [N_phys, H_kv, P, D] is stride_page = H_kv*P*D, stride_head = P*D.
 * Rows at positions >= seq_lens[b] (or seq_len) are never read.
 * fp8: k_scale/v_scale hold one fp32 scale per (phys page, kv head).
 * The 16-bit tensor-core path reads K/V through TMA tensor maps over the 2-D view
 * [total_rows, head_dim] of each allocation, so every stride must be a multiple of
 * head_dim.
 */
typedef struct {
  const void* k;
  const void* v;
  int64_t stride_b;
  int64_t stride_page;
  int64_t stride_head;
  const int32_t* page_table; /* [B, page_table_stride] or NULL */
  int64_t page_table_stride;
  int64_t num_phys_pages; /* bound on page_table entries (device-checked) */
  const float* k_scale;
  const float* v_scale;
  int64_t scale_stride_page;
  int64_t scale_stride_head;
  const int32_t* seq_lens; /* [B] or NULL */
  int64_t seq_len;         /* used when seq_lens is NULL */
  int32_t dtype;
  int32_t page_size;
  int32_t head_dim;
  int32_t n_kv_heads;
  int64_t total_rows; /* D-element rows addressable from k (and from v); 0 = derive from the pool
                         (page table set) or from B * stride_b / head_dim */
} linattn_kv_t;

/*
 * Quest page metadata (channel-wise min and max of K per page and kv head).
 * Entry (b, page p, head h) at base + b*stride_b + phys*stride_page + h*stride_head
 * with the same page-table rule as linattn_kv_t.  The reference layout
 * (B, H, n_pages, D) is stride_b = H*n_pages*D, stride_page = D, stride_head = n_pages*D.
 */
typedef struct {
  const void* mins;
  const void* maxs;
  int64_t stride_b;
  int64_t stride_page;
  int64_t stride_head;
  const int32_t* page_table;
  int64_t page_table_stride;
  int64_t num_phys_pages;
  int32_t dtype;
  int32_t n_heads; /* metadata heads: H_kv (GQA) or H_q (one per query head) */
} linattn_meta_t;

/* Per-(batch, list head, query) id lists: entry j of list (b, h, t) at
 * ids[b*stride_b + h*stride_h + t*stride_t + j]; its length is
 * counts[b*cstride_b + h*cstride_h + t*cstride_t] (or max_len when counts is NULL).
 * Negative ids are padding and are skipped. */
typedef struct {
  const void* ids;
  int32_t ids_dtype; /* LINATTN_I32 or LINATTN_I64 */
  int32_t n_heads;   /* list heads; query heads [h*G, (h+1)*G) share list h, G = H_q / n_heads */
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_t;
  int64_t max_len;
  const int32_t* counts;
  int64_t cstride_b;
  int64_t cstride_h;
  int64_t cstride_t;
} linattn_lists_t;

const char* linattn_last_error(void);
int linattn_version(void);

/*
 * Page bounds of a (B, H, T, D) key tensor (any strides, unit stride on D) into
 * contiguous (B, H, ceil(T/P), D) mins/maxs of the same dtype; the tail page
 * ignores rows past T.
 * Replaces page_bounds_torch / page_update_triton,
 * src/linattn/kernels/triton/quest_pages.py:38-48 and :134-142.
 */
int linattn_page_bounds(const void* k, int32_t dtype, int64_t B, int64_t H, int64_t T, int64_t D,
                        const int64_t* k_strides /*[4] elements*/, int64_t page_size, void* mins, void* maxs,
                        void* stream);

/*
 * Refresh the metadata of a paged pool for the pages touched by an append: for
 * every batch b, pages [first_page[b], ceil(seq_len_b / P)) (first_page NULL = all).
 * Metadata is written to `meta` (mins/maxs through the same page table); for fp8
 * pools the bounds are taken over the dequantised keys and rounded outward when
 * the metadata dtype is narrower than fp32.
 * Replaces QuestAttention._refresh_pages, src/linattn/variants/selection.py:181-201,
 * and the paged form of _page_update_kernel, quest_pages.py:84-100.
 */
int linattn_paged_page_bounds(const linattn_kv_t* kv, int64_t B, const int32_t* first_page, int64_t max_pages,
                              const linattn_meta_t* meta, int32_t* status, void* stream);

/*
 * Decode / chunk append in one launch: rows t of k_new, v_new (B, H_kv, T_new, D),
 * any strides with unit stride on D, go to position start_pos[b] + t of sequence b
 * (logical page pos / page_size through kv->page_table, row pos % page_size), converted
 * to the pool's dtype, and the Quest bounds of every page the new rows touch become
 * min / max over the page's earlier rows (taken from the stored bounds) and the new
 * rows (outward-rounded to the metadata dtype), equal to a recomputation over all of
 * the page's rows.  start_pos: device int32 [B], the sequence lengths before the
 * append (e.g. kv->seq_lens, updated by the caller afterwards).  The page table must
 * already map the touched pages.  16/32-bit pools only (fp8 pools are quantised a
 * whole page at a time).
 * Replaces the KV write of QuestAttention.push_kv followed by _refresh_pages
 * (src/linattn/variants/selection.py:176-201; page_update_triton,
 * src/linattn/kernels/triton/quest_pages.py:84-100, 134-142).
 */
int linattn_paged_append(const linattn_kv_t* kv, const linattn_meta_t* meta, int64_t B, const void* k_new,
                         const void* v_new, int32_t new_dtype, const int64_t* new_strides /*[4] elements*/,
                         int64_t T_new, const int32_t* start_pos, int32_t* status, void* stream);

/*
 * Quest upper-bound scores s[b,h,t,p] = sum_d max(q_d*min_d, q_d*max_d) in fp32,
 * written to scores (B, H_q, T_q, n_pages) contiguous, with the selection masks of
 * the reference applied: pages starting after the query position (offset + t), or
 * past a ragged sequence end (n_pages_b[b]), are -inf; the query's own page and the
 * first `sink_pages` pages are +inf.  Query head h reads metadata head
 * h / (H_q / meta->n_heads).
 * Replaces page_scores_torch + the masking of page_select_torch,
 * src/linattn/kernels/triton/quest_pages.py:51-75 (own page per row as in
 * src/linattn/variants/selection.py:220-230), and _page_score_kernel :103-131.
 */
int linattn_quest_scores(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t Tq, int64_t D,
                         const int64_t* q_strides /*[4]*/, const linattn_meta_t* meta, int64_t page_size,
                         int64_t n_pages, int64_t offset, int32_t sink_pages, const int32_t* n_pages_b,
                         float* scores, int32_t* status, void* stream);

/*
 * Top-k of every score row (B, H_q, T_q, n_pages), sorted by descending score with
 * ties broken by the lowest page index, k_b = max(1, min(topk, n_pages_b)).
 * ids_i64 / ids_i32 (B, H_q, T_q, topk), slots >= k_b set to -1.  When union_ids is
 * given, also the sorted union of the selected pages (score > -inf) over each group
 * of `group` consecutive query heads: union_ids (B, H_q/group, T_q, max_union),
 * union_count (B, H_q/group, T_q), and optionally union_tokens = tokens of those
 * pages at positions <= offset + t and < seq_len (page_size, seq_lens needed).
 * Replaces torch.topk in page_select_torch (quest_pages.py:76-77), topk_blocks
 * (selection.py:51-59) and the GQA union (selection.py:232-235).
 */
int linattn_page_topk(const float* scores, int64_t B, int64_t Hq, int64_t Tq, int64_t n_pages, int64_t topk,
                      const int32_t* n_pages_b, int64_t* ids_i64, int32_t* ids_i32, int64_t group,
                      int32_t* union_ids, int32_t* union_count, int64_t max_union, int32_t* union_tokens,
                      int64_t page_size, int64_t offset, const int32_t* seq_lens, int64_t seq_len,
                      int32_t* status, void* stream);

/*
 * Fused Quest selection for one decode step of B sequences: page scores, top-k per
 * query head and the union per kv head in one kernel (one CTA per sequence and kv
 * head).  Metadata is [B, H_kv, max_pages, 2, D] (logical page order, min row then
 * max row, f16/bf16).  The query of sequence b sits at position seq_lens[b] - 1: pages
 * below n_pages_b[b] are visible; the first `sink_pages` and, with `force_last`, the last
 * one are forced in (a shard of a sequence-sharded cache that does not hold the query's
 * page passes force_last = 0).  ids (B, H_q, topk) int32 sorted by (score desc, page asc), -1 padded; scores
 * (B, H_q, max_pages) optional; union_ids (B, H_kv, max_union) ascending with counts
 * and token counts.  Group size H_q / H_kv in {1, 2, 4, 8}; D in {64, 128}.
 * Replaces, for T_q == 1, page_select_torch (src/linattn/kernels/triton/quest_pages.py:57-78)
 * followed by the GQA union of QuestAttention.page_selection
 * (src/linattn/variants/selection.py:214-237).
 */
int linattn_quest_decode_select(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t D,
                                const int64_t* q_strides /*[4]*/, const void* meta, int32_t meta_dtype,
                                int64_t n_kv_heads, int64_t max_pages, const int32_t* n_pages_b,
                                const int32_t* seq_lens, int64_t page_size, int64_t topk, int32_t sink_pages,
                                int32_t force_last, int32_t* ids, float* scores, int32_t* union_ids,
                                int32_t* union_count, int64_t max_union, int32_t* union_tokens, int32_t* status,
                                void* stream);

/*
 * The candidates form of linattn_quest_decode_select, for long sequences and the
 * sequence-sharded decode: the page axis is cut into chunks of chunk_pages pages, one
 * CTA per (sequence, kv head, chunk), and each writes, for every query head, the top
 * `topk` pages of its chunk as candidates: cand_scores / cand_ids at
 * [c * cand_stride + (b * H_q + h) * topk + r], sorted by (score desc, page asc), page
 * ids offset by page_base[b] (NULL = 0), padded with (-inf, -1).  Forced pages (the
 * last page when force_last, the first sink_pages) score +inf.  scores (B, H_q,
 * max_pages), when not NULL, receives every page score.  linattn_shard_merge over the
 * chunks (R = n_chunks, rank_stride = cand_stride) then gives the same top-k and GQA
 * union as linattn_quest_decode_select (page_select_torch,
 * src/linattn/kernels/triton/quest_pages.py:57-78): a page of the global top-k is in
 * its chunk's top-k.  No single reference counterpart (the reference scores and
 * selects in one pass over the whole sequence).
 */
int linattn_quest_decode_candidates(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t D,
                                    const int64_t* q_strides, const void* meta, int32_t meta_dtype,
                                    int64_t n_kv_heads, int64_t max_pages, const int32_t* n_pages_b, int64_t topk,
                                    int32_t sink_pages, int32_t force_last, int64_t chunk_pages,
                                    const int32_t* page_base, float* cand_scores, int32_t* cand_ids,
                                    int64_t cand_stride, float* scores, int32_t* status, void* stream);

/*
 * Exact softmax attention of each query over the KV rows of its list's pages.
 * q and out are (B, H_q, T_q, D) with element strides; out has q's dtype.  Rows at
 * positions >= seq_len_b are skipped; with `causal`, rows after offset + t too.
 * A page list may be split over `n_splits` CTAs (split-KV); the partial (o, lse)
 * then go to `workspace` (fp32, linattn_sparse_attention_workspace() bytes) and are
 * merged by the log-sum-exp combine.  lse_out (B, H_q, T_q) optional (natural log).
 * Replaces block_sparse_attention_torch / _block_sparse_fwd_kernel,
 * src/linattn/kernels/triton/block_sparse.py:40-163, the C paged decode
 * src/linattn/kernels/c/decode_attn.c:72-133, and the masked dense attention of
 * BlockSelectionAttention.attend, src/linattn/variants/selection.py:110-116.
 */
int linattn_sparse_attention(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t Tq,
                             const int64_t* q_strides /*[4]*/, const linattn_kv_t* kv,
                             const linattn_lists_t* lists, int32_t causal, int64_t offset, float scale,
                             void* out, const int64_t* out_strides /*[4]*/, float* lse_out, int32_t n_splits,
                             float* workspace, int64_t workspace_bytes, int32_t* status, void* stream);

/*
 * linattn_sparse_attention with an explicit output dtype (f32, f16 or bf16): f32 keeps
 * the partial results of a sequence-sharded decode at full precision until their
 * log-sum-exp merge (linattn_lse_combine).  No counterpart in the reference.
 */
int linattn_sparse_attention_out(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t Tq,
                                 const int64_t* q_strides /*[4]*/, const linattn_kv_t* kv,
                                 const linattn_lists_t* lists, int32_t causal, int64_t offset, float scale,
                                 void* out, int32_t out_dtype, const int64_t* out_strides /*[4]*/, float* lse_out,
                                 int32_t n_splits, float* workspace, int64_t workspace_bytes, int32_t* status,
                                 void* stream);

/* Workspace bytes linattn_sparse_attention needs for n_splits > 1. */
int64_t linattn_sparse_attention_workspace(int64_t B, int64_t Hq, int64_t Tq, int64_t D, int32_t n_splits);

/*
 * Split-KV merge: o = sum_s exp(lse_s - L) o_s, L = logsumexp_s lse_s, for `rows`
 * rows of D channels.  o_parts [S, rows, D] fp32, lse_parts [S, rows] (natural log,
 * -inf for an empty part).  out [rows, D] in out_dtype (f32/f16/bf16); lse_out
 * [rows] optional.  A row whose parts are all empty gives o = 0, L = -inf.
 * No reference counterpart (the reference never splits the KV axis); it merges the
 * per-GPU partials of the sequence-sharded decode after an NCCL all-gather.
 */
int linattn_lse_combine(const float* o_parts, const float* lse_parts, int64_t S, int64_t rows, int64_t D,
                        void* out, int32_t out_dtype, float* lse_out, void* stream);

/*
 * linattn_lse_combine over parts that are not packed densely: part s of o starts at
 * o_parts + s * o_part_stride floats and its lse at lse_parts + s * lse_part_stride
 * (0 = rows * D / rows, the dense layout).  Lets the sequence-sharded decode gather one
 * [o | lse] block per rank with a single all-gather and merge it in place.
 */
int linattn_lse_combine_strided(const float* o_parts, int64_t o_part_stride, const float* lse_parts,
                                int64_t lse_part_stride, int64_t S, int64_t rows, int64_t D, void* out,
                                int32_t out_dtype, float* lse_out, void* stream);

/*
 * linattn_sparse_attention without a workspace argument, for callers that cannot
 * allocate device memory where they run attention (an engine that owns all of HBM
 * through its own pool and forbids side allocations, or a latency-critical path
 * that cannot take cudaMalloc's implicit device synchronisation).  No counterpart in
 * the reference.  The split-KV scratch is a 64 MiB device array inside this library
 * (linattn_sparse_attention_noalloc_limit() bytes), held by every GPU that loads it
 * until exit; a call whose scratch need (linattn_sparse_attention_workspace) exceeds
 * it fails with LINATTN_EINVAL.  The first call on a device resolves the array's
 * device address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture.  All calls share the array: calls that overlap on
 * the GPU race.  Allocates nothing (no cudaMalloc / cudaFree).
 */
int linattn_sparse_attention_noalloc(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t Tq,
                                     const int64_t* q_strides, const linattn_kv_t* kv, const linattn_lists_t* lists,
                                     int32_t causal, int64_t offset, float scale, void* out,
                                     const int64_t* out_strides, float* lse_out, int32_t n_splits, int32_t* status,
                                     void* stream);
int64_t linattn_sparse_attention_noalloc_limit(void);

/*
 * Lightning-indexer scores of queries [t_begin, t_end):
 * I[b,t,s] = sum_h w[b,t,h] * ReLU(q_idx[b,t,h,:] . k_idx[b,s,h,:]) in fp32, written to
 * scores[(b * (t_end - t_begin) + t - t_begin) * row_stride + s] for s < Tk.
 * q_idx (B, Tq, H_I, D), k_idx (B, Tk, H_I, D), head_weights (B, Tq, H_I), element
 * strides.  fp8 e4m3 keys carry one fp32 scale per `scale_group` tokens
 * (k_scale[b * scale_batch_stride + s / scale_group]).  Key s covers positions
 * [s * key_block, (s + 1) * key_block) (1 for tokens; the pooling ratio for pooled
 * groups) and is visible from query t iff s * key_block <= offset + t.  causal = 1:
 * invisible keys score -inf; causal = 2: the same inside each 64-key tile that holds a
 * visible key, while tiles after every query of a 64-query block are left unwritten
 * (for a causal top-k, which never reads them).  H_I * D <= 512.  16-bit queries
 * with fp8 keys (or keys of the query's type) run on the tensor cores for
 * (H_I, D) in {(1|2|4, 64), (1|2, 128), (4|8, 32), (4|8, 16)} with contiguous
 * (B, T_k, H_I, D) keys.  status: device
 * status word (LINATTN_DEV_TIMEOUT if a tile copy never arrives), may be NULL.
 * Replaces indexer_scores_torch (src/linattn/kernels/triton/fused_indexer.py:52-60) and
 * the score pass of _indexer_block_max_kernel / _indexer_gather_kernel (:80-171).
 */
int linattn_indexer_scores(const void* q_idx, int32_t q_dtype, const int64_t* q_strides /*[4]*/,
                           const void* k_idx, int32_t k_dtype, const int64_t* k_strides /*[4]*/,
                           const float* k_scale, int64_t scale_group, int64_t scale_batch_stride,
                           const void* head_weights, int32_t w_dtype, const int64_t* w_strides /*[3]*/,
                           int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D, int32_t causal,
                           int64_t offset, int64_t key_block, int64_t t_begin, int64_t t_end, float* scores,
                           int64_t row_stride,
                           int32_t* status, void* stream);

/*
 * Top-k of each of `rows` fp32 rows of n scores (row r at scores + r * row_stride),
 * ties at the k-th value going to the lowest indices, k of each written at
 * (r / period) * out_batch_stride + (r % period) * out_stride: with `sorted`, values
 * descending (lowest index first among equal values); else in ascending index order.
 * With `causal`, row r only considers its first
 * min(n, (first_pos + r % period) / key_block + 1) entries and pads the remaining
 * slots with (-inf, -1).  The first `skip` entries of every row are never candidates
 * (indices stay those of the full row).  k <= 4096; rows of up to 32768 entries stay in registers,
 * longer ones are re-read from global memory.
 * Replaces the torch.topk of indexer_topk_torch
 * (src/linattn/kernels/triton/fused_indexer.py:63-73) and of DSAAttention.select
 * (src/linattn/variants/selection.py:744-749).
 */
int linattn_row_topk(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t k,
                     int32_t causal, int64_t first_pos, int64_t key_block, int64_t period, int64_t skip,
                     int32_t sorted, float* values,
                     int64_t* idx_i64, int32_t* idx_i32, int64_t out_stride, int64_t out_batch_stride,
                     void* stream);

/*
 * Token-sparse attention (DSA / CSA prefill and decode).  Each query (b, h, t) attends
 * to the union of: the tokens of its list (list head h / (H_q / lists->n_heads); each
 * entry id stands for tokens [id * block, id * block + block); negative ids are
 * padding), the first `sink` tokens, and the `window` tokens ending at position
 * offset + t; restricted to positions < Tk, and <= offset + t when `causal`.  A token
 * in several of these counts once.  q, out (B, H_q, T_q, D); K, V (B, H_kv, Tk, D)
 * with element strides kv_strides = {batch, head, token} (rows contiguous, 16-byte
 * aligned); q / K / V bf16 or f16 (one type), D in {64, 128}.  lse_out (B, H_q, T_q)
 * and reads_out (B, H_q, T_q, tokens read) optional.  A query with nothing to read
 * reads token min(offset + t, Tk - 1) with `diag_fallback` (the reference's empty-row
 * rule, selection.py:100-107), else gets o = 0, lse = -inf.  v_unscale (NULL for a V of
 * q's type): with bf16 q / K, `v` may instead be an f16 copy of V scaled by a power of
 * two per (b, kv head) (linattn_prefill_v_to_f16 writes it), v_unscale[b * Hkv + kvh]
 * the factor that undoes it; P V then takes one f16 P part.
 * Replaces the masked attention of BlockSelectionAttention.attend
 * (src/linattn/variants/selection.py:86-116) for the DSA selection
 * (DSAAttention.select, :738-763), and block_sparse_attention_torch with block_size 1
 * (src/linattn/kernels/triton/block_sparse.py:40-75).
 */
int linattn_token_attention(const void* q, int32_t dtype, int64_t B, int64_t Hq, int64_t Tq,
                            const int64_t* q_strides /*[4]*/, const void* k, const void* v, const float* v_unscale,
                            int64_t Hkv, int64_t Tk,
                            int64_t D, const int64_t* kv_strides /*[3]*/, const linattn_lists_t* lists, int64_t block,
                            int64_t sink, int64_t window, int32_t causal, int64_t offset, float scale,
                            int32_t diag_fallback, void* out, const int64_t* out_strides /*[4]*/, float* lse_out,
                            int32_t* reads_out, int32_t* status, void* stream);

/*
 * Mean of each `block` consecutive tokens of x (B, H, T, D) (element strides), the
 * tail block padded by repeating the last token: out (B, H, ceil(T / block), D) fp32,
 * contiguous.  Replaces block_reduce (src/linattn/core.py:103-120) for the pooled
 * queries / keys of MInferenceAttention._block_sparse and MoBAAttention.select
 * (src/linattn/variants/selection.py:339-353, 635-649).
 */
int linattn_block_mean(const void* x, int32_t dtype, int64_t B, int64_t H, int64_t T, int64_t D,
                       const int64_t* strides /*[4]*/, int64_t block, float* out, void* stream);

/*
 * CSA2 compressed KV: the mean of each `ratio` consecutive tokens of x (B, H, T, D)
 * (element strides, tail padded by repeating the last token) rounded to x's dtype, then,
 * for bits 4 or 8, stored through the group-wise codec (FP4 E2M1 with absmax / 6 scales,
 * or FP8 e4m3 with absmax / 448 scales, one scale per `group` = 32 channels, tail groups
 * zero-padded) and dequantised back to x's dtype; bits 16 is the rounded mean alone.
 * out (B, H, ceil(T / ratio), D) contiguous, x's dtype (bf16, f16 or f32), D <= 256.
 * Replaces CSA2Attention.compressed_kv (src/linattn/variants/csa2.py:73-81), i.e.
 * block_reduce (src/linattn/core.py:103-120) followed by quantize / dequantize
 * (src/linattn/kv/quant.py:76-109).
 */
int linattn_csa2_pool_quant(const void* x, int32_t dtype, int64_t B, int64_t H, int64_t T, int64_t D,
                            const int64_t* strides /*[4]*/, int64_t ratio, int32_t bits, int32_t group, void* out,
                            void* stream);

/*
 * Measurement utility: reads `bytes` (a multiple of 16, 16-byte aligned) of device
 * memory `reps` times with a persistent grid of up to min(2 x SMs, sink_words) CTAs,
 * folding the data into sink[0 .. grid) (uint32 device words, xor-accumulated) so the
 * loads cannot be elided.  Timed with events, bytes * reps / time is the read roof of a
 * buffer that stays in L2 (<= ~100 MB) or of HBM (larger).  No counterpart in the
 * reference: it gives the L2-gather roofline of linattn_token_attention its denominator.
 */
int linattn_read_bandwidth(const void* buf, int64_t bytes, int32_t reps, uint32_t* sink, int64_t sink_words,
                           void* stream);

/*
 * Block selection in one launch: scores, causal top-k and the forced-block merge.
 * Row r of (b, h) (a (B, H_q, R, D), element strides, f32 / f16 / bf16) is scored
 * against the candidates of its kv head h / (H_q / H_kv) (bm (B, H_kv, NC, D)):
 * s(r, c) = scale * sum_d a[r, d] * bm[c, d] in fp32, channel order 0 .. D-1.  Row r
 * takes candidates [skip, min(floor((first_pos + r) / key_block), NC - 1)] and keeps
 * the top k (1 <= k <= 32) by (score desc, index asc); these are merged as
 * linattn_merge_block_lists does with own = min(floor((merge_pos + r) / own_div),
 * NC - 1), sink and window, into out (B, H_q, R, n_max) ascending, -1 padded, and
 * counts (B, H_q, R).  Optional: topk_out (B, H_q, R, k), the top k in score order
 * (-1 padded); scores_out (B, H_q, R, NC), the fp32 scores the selection ranked
 * (entries outside a row's candidate range are left unwritten).  D <= 256.
 * Replaces the pooled block scores, torch.topk and the boolean unions of
 * MInferenceAttention._block_sparse (src/linattn/variants/selection.py:339-353),
 * MoBAAttention.select (:635-649) and NSAAttention's selection branch
 * (src/linattn/variants/native_sparse.py:78-92), and builds the sink + window +
 * top-k lists of the block-sparse prefill.
 */
int linattn_block_score_topk(const void* a, int32_t a_dtype, const int64_t* a_strides /*[4]*/, const void* bm,
                             int32_t b_dtype, const int64_t* b_strides /*[4]*/, int64_t B, int64_t Hq, int64_t Hkv,
                             int64_t R, int64_t NC, int64_t D, float scale, int64_t k, int64_t first_pos,
                             int64_t key_block, int64_t skip, int64_t merge_pos, int64_t own_div, int64_t sink,
                             int64_t window, int32_t force_own, int32_t* out, int64_t n_max, int32_t* counts,
                             int32_t* topk_out, float* scores_out, void* stream);

/*
 * Block lists from a top-k selection: for each of `rows` rows, the ascending union
 * (duplicates removed) of its top-k ids (int32, -1 padded, rows of k) with the forced
 * blocks [0, sink) and [own - window + 1, own], plus `own` itself with force_own, all
 * clipped to [0, own], where own = min((first_pos + r % period) / own_div, n_blocks - 1).
 * out (rows, n_max) -1 padded; counts (rows) optional.  Replaces the boolean unions of
 * MInferenceAttention._block_sparse (own block, selection.py:350-351) and
 * MoBAAttention.select (own block, :645-646), and builds the sink + window + top-k lists
 * of the block-sparse prefill.
 */
int linattn_merge_block_lists(const int32_t* topk, int64_t rows, int64_t k, int64_t period, int64_t first_pos,
                              int64_t own_div, int64_t n_blocks, int64_t sink, int64_t window, int32_t force_own,
                              int32_t* out, int64_t n_max, int32_t* counts, void* stream);

/*
 * Block-sparse causal prefill on the tcgen05 tensor cores.  Query t of head h reads the
 * 64-token key blocks of list ids[b, h, t / rows_per_list, :] (ascending, -1 padded,
 * counts optional; id_strides / count_strides = {batch, head, list row} in elements),
 * plus the tokens below `sink`, restricted to keys < Tk and, with `causal` = c >= 1, to
 * keys j with j * c <= offset + t + c - 1 (c = 1: j <= offset + t; c > 1: the keys are
 * pooled groups of c tokens, read once their group has started, the compression branch
 * of NSAAttention, src/linattn/variants/native_sparse.py:67-76); with `window` > 0
 * (no sink) also to keys >= offset + t - window + 1 (the window branch,
 * native_sparse.py:100-105).  q (B, H_q, T_q, 128), K / V (B, H_kv, Tk, 128): contiguous rows,
 * bf16 or f16 (one type); out with element strides, lse_out (B, H_q, T_q) optional.
 * Lists of at most 64 blocks, Tk <= 2^18.  A row that reads nothing gets o = 0,
 * lse = -inf.  Replaces the token mask + masked dense attention of
 * MInferenceAttention._block_sparse and MoBAAttention.select
 * (src/linattn/variants/selection.py:339-353, 635-649, 86-116) and
 * block_sparse_attention_torch for prefill (src/linattn/kernels/triton/block_sparse.py:40-75).
 * With bf16 inputs, v_f16 / v_scale (from linattn_prefill_v_to_f16, or NULL) let the
 * P V product run in f16 with a single P part: V is read from v_f16 and O multiplied
 * by v_scale[b * H_kv + kv head]; without them P is split into bf16 hi + lo parts.
 */
int linattn_block_sparse_prefill(const void* q, int32_t dtype, int64_t B, int64_t Hq, int64_t Tq, const void* k,
                                 const void* v, int64_t Hkv, int64_t Tk, int64_t D, const int32_t* ids,
                                 const int32_t* counts, const int64_t* id_strides /*[3]*/, int64_t n_max,
                                 int64_t rows_per_list, const int64_t* count_strides /*[3]*/, int64_t sink,
                                 int32_t causal, int64_t window, int64_t offset, float scale, void* out,
                                 const int64_t* out_strides /*[4]*/, float* lse_out, const void* v_f16,
                                 const float* v_scale, int32_t* status, void* stream);

/*
 * f16 copy of a contiguous bf16 V for linattn_block_sparse_prefill: `heads` blocks of
 * `per_head` elements (B * H_kv blocks of T_k * 128); per block a power-of-two scale
 * s >= 1 with max|V| / s <= 2^15 (s = 1 unless |V| exceeds 2^15), out = V / s rounded
 * to f16 (exact for every value in f16's normal range), scale[block] = s.
 * amax_scratch: `heads` uint32 of device scratch.  No reference counterpart.
 */
int linattn_prefill_v_to_f16(const void* v, int64_t heads, int64_t per_head, void* out, float* scale,
                             uint32_t* amax_scratch, void* stream);

/*
 * Sequence-sharded Quest decode, merge step.  scores / ids (R, B, H_q, K): the R
 * shards' (or chunks') local top-K candidates (fp32 scores, global page ids, -1 =
 * none), rank-major as an all-gather leaves them; each row of K sorted by (score desc,
 * page asc) with the -1 slots last, and no page in two blocks (as
 * linattn_quest_decode_candidates writes them).  Per (b, query head) the global top-`topk` by (score
 * desc, page asc) is taken (written to sel (B, H_q, topk), -1 padded, when sel is not
 * NULL); the pages of this shard, [page_lo[b], page_hi[b]), selected by any head of a
 * kv head's group go to union_ids (B, H_kv, max_union) as ascending LOCAL ids
 * (page - page_lo[b]), -1 padded, with union_count (B, H_kv).  R <= 64, R * K <= 4096.
 * No counterpart in the reference (which never shards the KV sequence); the selection
 * equals page_select_torch's (src/linattn/kernels/triton/quest_pages.py:57-78) over
 * the whole cache.  rank_stride: elements from one shard's (B, H_q, K) block to the
 * next in both scores and ids (0 = B * H_q * K, dense), so a gathered buffer holding
 * each rank's [scores | ids] pair is read in place.  union_tokens (B, H_kv), when not
 * NULL, receives the tokens of the union pages: sum over pages g of
 * clamp(seq_lens[b] - g * page_size, 0, page_size), g the global page.  sel_scores
 * (B, H_q, topk), when not NULL, receives the scores of sel (-inf past the last).  With
 * union_ids NULL no union is built (sel required): a shard merging its own chunks
 * before the exchange, so that it sends one sorted block of K instead of one per chunk.
 */
int linattn_shard_merge(const float* scores, const int32_t* ids, int64_t R, int64_t B, int64_t Hq, int64_t K,
                        int64_t rank_stride, int64_t topk, int64_t n_kv_heads, const int32_t* page_lo, const int32_t* page_hi,
                        int64_t max_local, int32_t* sel, float* sel_scores, int32_t* union_ids, int32_t* union_count,
                        int64_t max_union, const int32_t* seq_lens, int64_t page_size, int32_t* union_tokens,
                        void* stream);


#ifdef __cplusplus
}
#endif

#endif /* LINATTN_B200_H */
