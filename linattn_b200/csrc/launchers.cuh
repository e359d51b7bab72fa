// Host-side launcher declarations shared by the kernel units and the C ABI.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "sparse_attention.cuh"

namespace linattn {

struct TopkParams {
  const float* scores;
  int64_t B, Hq, Tq, n, topk;
  const int32_t* n_pages_b;
  int64_t* ids64;
  int32_t* ids32;
  int64_t group;
  int32_t* union_ids;
  int32_t* union_count;
  int64_t max_union;
  int32_t* union_tokens;
  int64_t P, offset;
  const int32_t* seq_lens;
  int64_t seq_len;
  int32_t* status;
};

int device_index();
// Record `msg` as linattn_last_error() and return `code` (host side).
int set_error(int code, const char* msg);

cudaError_t launch_page_bounds(const void* k, int dtype, int64_t B, int64_t H, int64_t T_, int64_t D,
                               const int64_t* s, int64_t P, void* mins, void* maxs, cudaStream_t stream);
cudaError_t launch_paged_append(const linattn_kv_t& kv, const linattn_meta_t& meta, int64_t B, const void* k_new,
                                const void* v_new, int new_dtype, const int64_t* s, int64_t T_new,
                                const int32_t* start_pos, int32_t* status, cudaStream_t stream);
cudaError_t launch_paged_page_bounds(const linattn_kv_t& kv, int64_t B, const int32_t* first_page,
                                     int64_t max_pages, const linattn_meta_t& meta, int32_t* status,
                                     cudaStream_t stream);
cudaError_t launch_quest_scores(const void* q, int q_dtype, int64_t B, int64_t Hq, int64_t Tq, int64_t D,
                                const int64_t* qs, const linattn_meta_t& meta, int64_t P, int64_t n_pages,
                                int64_t offset, int sink_pages, const int32_t* n_pages_b, float* scores,
                                int32_t* status, cudaStream_t stream);
size_t page_topk_smem_bytes(int64_t n, int64_t topk);
cudaError_t launch_page_topk(const TopkParams& p, cudaStream_t stream);
cudaError_t launch_lse_combine(const float* o_parts, const float* lse_parts, int64_t S, int64_t rows, int64_t D,
                               void* out, int out_dtype, int64_t H, int64_t Tq, const int64_t* os, float* lse_out,
                               cudaStream_t stream, int64_t o_part_stride = 0, int64_t lse_part_stride = 0);
// Zeroes `bytes` (a multiple of 16) at `words` as a programmatic-dependent kernel that
// ends after the stream's previous kernel (lse_combine.cu).
cudaError_t launch_attn_counters_clear(void* words, int64_t bytes, cudaStream_t stream);
cudaError_t launch_sparse_attention_f32(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream);
cudaError_t launch_sparse_attention_f16(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream);
cudaError_t launch_sparse_attention_bf16(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream);
cudaError_t launch_sparse_attention_fp8(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream);
cudaError_t launch_sparse_attention_mma_bf16(const AttnParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                                            int box_rows, int D, int* counter, int64_t n_items, cudaStream_t stream);
cudaError_t launch_sparse_attention_mma_f16(const AttnParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                                           int box_rows, int D, int* counter, int64_t n_items, cudaStream_t stream);
cudaError_t launch_sparse_attention_mma_fp8(const AttnParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                                           int box_rows, int D, int* counter, int64_t n_items, cudaStream_t stream);
int sm_count();
// Tensor-core indexer scores (indexer_mma.cu); false when the call is not eligible
// (nothing launched), else *err holds the launch status.
bool indexer_scores_mma(const void* q, int q_dtype, const int64_t* qs, const void* k, int k_dtype, const int64_t* ks,
                        const float* k_scale, int64_t group, int64_t ss, const void* w, int w_dtype, const int64_t* ws,
                        int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D, int causal, int64_t offset,
                        int64_t key_block, int64_t t_begin, int64_t t_end, float* scores, int64_t row_stride, int32_t* status,
                        cudaStream_t st, cudaError_t* err);
// 2-D TMA tensor map {inner, rows} (row stride in bytes) with box {box_inner, box_rows}
// and 128-byte swizzle, from a process-wide cache.  False if encoding fails.
bool tensor_map_2d(CUtensorMap* out, const void* base, CUtensorMapDataType cu_dtype, int64_t inner, int64_t rows,
                   int64_t stride_bytes, int box_inner, int box_rows);
int tile_rows_f32(int D);
int tile_rows_f16(int D);
int tile_rows_bf16(int D);
int tile_rows_fp8(int D);

}  // namespace linattn
