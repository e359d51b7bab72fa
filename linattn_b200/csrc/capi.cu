// extern "C" entry points: argument validation, template dispatch, launch.
// Nothing here allocates device memory; every buffer comes from the caller.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "launchers.cuh"

namespace linattn {
int device_index() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}
int sm_count() {
  static int cache[64] = {};
  const int d = device_index();
  if (d < 0 || d >= 64) return 1;
  if (cache[d] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0) n = 1;
    cache[d] = n;
  }
  return cache[d];
}
}  // namespace linattn

using namespace linattn;

namespace {
thread_local std::string g_err;
}  // namespace

namespace linattn {
int set_error(int code, const char* msg) {
  g_err = msg;
  return code;
}
}  // namespace linattn

namespace {

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LINATTN_OK;
  return fail(LINATTN_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

int elem_bytes(int dtype) {
  switch (dtype) {
    case LINATTN_F32: return 4;
    case LINATTN_F16: return 2;
    case LINATTN_BF16: return 2;
    case LINATTN_FP8E4M3: return 1;
    case LINATTN_I32: return 4;
    case LINATTN_I64: return 8;
    default: return 0;
  }
}

bool is_float16_32(int dtype) { return dtype == LINATTN_F32 || dtype == LINATTN_F16 || dtype == LINATTN_BF16; }

bool aligned(const void* p, int64_t a) { return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(a)) == 0; }

bool head_dim_ok(int64_t D) { return D == 8 || D == 16 || D == 32 || D == 64 || D == 128 || D == 256; }

int attn_tile_rows(int dtype, int D) {
  switch (dtype) {
    case LINATTN_F32: return tile_rows_f32(D);
    case LINATTN_F16: return tile_rows_f16(D);
    case LINATTN_BF16: return tile_rows_bf16(D);
    case LINATTN_FP8E4M3: return tile_rows_fp8(D);
    default: return 0;
  }
}

int check_kv(const linattn_kv_t* kv) {
  if (!kv) return fail(LINATTN_EINVAL, "kv descriptor is NULL");
  const int eb = elem_bytes(kv->dtype);
  if (!(is_float16_32(kv->dtype) || kv->dtype == LINATTN_FP8E4M3))
    return fail(LINATTN_EUNSUPPORTED, "kv dtype %d not supported", kv->dtype);
  if (!kv->k || !kv->v) return fail(LINATTN_EINVAL, "kv base pointers must be non-NULL");
  if (kv->page_size <= 0 || kv->n_kv_heads <= 0) return fail(LINATTN_EINVAL, "page_size and n_kv_heads must be > 0");
  if (!head_dim_ok(kv->head_dim)) return fail(LINATTN_EUNSUPPORTED, "head_dim %d not in {8,...,256}", kv->head_dim);
  if ((static_cast<int64_t>(kv->head_dim) * eb) % 16 != 0)
    return fail(LINATTN_EUNSUPPORTED, "head_dim*elem_bytes must be a multiple of 16 (got %d*%d)", kv->head_dim, eb);
  if (!aligned(kv->k, 16) || !aligned(kv->v, 16)) return fail(LINATTN_EINVAL, "K/V base pointers must be 16-byte aligned");
  if ((kv->stride_b * eb) % 16 || (kv->stride_page * eb) % 16 || (kv->stride_head * eb) % 16)
    return fail(LINATTN_EINVAL, "K/V strides must be multiples of 16 bytes");
  if (kv->page_table && (kv->page_table_stride <= 0 || kv->num_phys_pages <= 0))
    return fail(LINATTN_EINVAL, "page_table_stride and num_phys_pages must be > 0 with a page table");
  if (kv->dtype == LINATTN_FP8E4M3 && (!kv->k_scale || !kv->v_scale))
    return fail(LINATTN_EINVAL, "fp8 KV needs k_scale and v_scale");
  if (!kv->seq_lens && kv->seq_len < 0) return fail(LINATTN_EINVAL, "seq_len must be >= 0");
  return LINATTN_OK;
}

// ---- TMA tensor maps over the [rows, D] view of a K or V pool ----------------------
// 2-D map {D, rows} with 128-byte x box_rows boxes and 128-byte swizzle (16-bit: 64
// elements per box row; fp8 codes as bytes: 128).
bool kv_tensor_map(CUtensorMap* out, const void* base, int64_t rows, int d, int dtype, int box_rows) {
  if (dtype == LINATTN_FP8E4M3)
    return tensor_map_2d(out, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, d, rows, d, 128, box_rows);
  return tensor_map_2d(out, base, dtype == LINATTN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                       d, rows, static_cast<int64_t>(d) * 2, 64, box_rows);
}

}  // namespace

extern "C" {

const char* linattn_last_error(void) { return g_err.c_str(); }

int linattn_version(void) { return 1; }

int linattn_page_bounds(const void* k, int32_t dtype, int64_t B, int64_t H, int64_t T, int64_t D,
                        const int64_t* k_strides, int64_t page_size, void* mins, void* maxs, void* stream) {
  if (!is_float16_32(dtype)) return fail(LINATTN_EUNSUPPORTED, "page_bounds: dtype %d not supported", dtype);
  if (!k || !mins || !maxs || !k_strides) return fail(LINATTN_EINVAL, "page_bounds: NULL pointer");
  if (B < 0 || H < 0 || T < 0 || D <= 0 || page_size <= 0)
    return fail(LINATTN_EINVAL, "page_bounds: bad shape B=%lld H=%lld T=%lld D=%lld P=%lld", (long long)B,
                (long long)H, (long long)T, (long long)D, (long long)page_size);
  return cuda_status(launch_page_bounds(k, dtype, B, H, T, D, k_strides, page_size, mins, maxs,
                                        static_cast<cudaStream_t>(stream)),
                     "page_bounds");
}

int linattn_paged_page_bounds(const linattn_kv_t* kv, int64_t B, const int32_t* first_page, int64_t max_pages,
                              const linattn_meta_t* meta, int32_t* status, void* stream) {
  int rc = check_kv(kv);
  if (rc) return rc;
  if (!meta || !meta->mins || !meta->maxs) return fail(LINATTN_EINVAL, "paged_page_bounds: metadata pointers NULL");
  if (!is_float16_32(meta->dtype)) return fail(LINATTN_EUNSUPPORTED, "metadata dtype %d not supported", meta->dtype);
  if (meta->page_table && (meta->page_table_stride <= 0 || meta->num_phys_pages <= 0))
    return fail(LINATTN_EINVAL, "metadata page table needs a stride and num_phys_pages");
  if (B < 0 || max_pages < 0) return fail(LINATTN_EINVAL, "paged_page_bounds: B and max_pages must be >= 0");
  return cuda_status(launch_paged_page_bounds(*kv, B, first_page, max_pages, *meta, status,
                                              static_cast<cudaStream_t>(stream)),
                     "paged_page_bounds");
}

int linattn_paged_append(const linattn_kv_t* kv, const linattn_meta_t* meta, int64_t B, const void* k_new,
                         const void* v_new, int32_t new_dtype, const int64_t* new_strides, int64_t T_new,
                         const int32_t* start_pos, int32_t* status, void* stream) {
  int rc = check_kv(kv);
  if (rc) return rc;
  if (kv->dtype != LINATTN_F32 && kv->dtype != LINATTN_F16 && kv->dtype != LINATTN_BF16)
    return fail(LINATTN_EUNSUPPORTED, "paged_append: 16/32-bit pools only (fp8 pools are quantised per page)");
  if (!meta || !meta->mins || !meta->maxs) return fail(LINATTN_EINVAL, "paged_append: metadata pointers NULL");
  if (!is_float16_32(meta->dtype)) return fail(LINATTN_EUNSUPPORTED, "metadata dtype %d not supported", meta->dtype);
  if (meta->page_table && (meta->page_table_stride <= 0 || meta->num_phys_pages <= 0))
    return fail(LINATTN_EINVAL, "metadata page table needs a stride and num_phys_pages");
  if (!is_float16_32(new_dtype)) return fail(LINATTN_EUNSUPPORTED, "paged_append: new rows dtype %d", new_dtype);
  if (!k_new || !v_new || !new_strides || !start_pos) return fail(LINATTN_EINVAL, "paged_append: NULL pointer");
  if (B < 0 || T_new < 0) return fail(LINATTN_EINVAL, "paged_append: B and T_new must be >= 0");
  if (new_strides[3] != 1) return fail(LINATTN_EINVAL, "paged_append: new rows need unit stride on D");
  return cuda_status(launch_paged_append(*kv, *meta, B, k_new, v_new, new_dtype, new_strides, T_new, start_pos,
                                         status, static_cast<cudaStream_t>(stream)),
                     "paged_append");
}

int linattn_quest_scores(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t Tq, int64_t D,
                         const int64_t* q_strides, const linattn_meta_t* meta, int64_t page_size, int64_t n_pages,
                         int64_t offset, int32_t sink_pages, const int32_t* n_pages_b, float* scores,
                         int32_t* status, void* stream) {
  if (!q || !q_strides || !meta || !scores) return fail(LINATTN_EINVAL, "quest_scores: NULL pointer");
  if (!is_float16_32(q_dtype)) return fail(LINATTN_EUNSUPPORTED, "quest_scores: q dtype %d not supported", q_dtype);
  if (!is_float16_32(meta->dtype))
    return fail(LINATTN_EUNSUPPORTED, "quest_scores: metadata dtype %d not supported", meta->dtype);
  if (!head_dim_ok(D)) return fail(LINATTN_EUNSUPPORTED, "quest_scores: head_dim %lld not in {8,...,256}", (long long)D);
  if (meta->n_heads <= 0 || Hq % meta->n_heads)
    return fail(LINATTN_EINVAL, "quest_scores: metadata heads (%d) must divide query heads (%lld)", meta->n_heads,
                (long long)Hq);
  const int eb = elem_bytes(meta->dtype);
  if (!aligned(meta->mins, 16) || !aligned(meta->maxs, 16) || (meta->stride_b * eb) % 16 ||
      (meta->stride_page * eb) % 16 || (meta->stride_head * eb) % 16)
    return fail(LINATTN_EINVAL, "quest_scores: metadata rows must be 16-byte aligned");
  if (meta->page_table && (meta->page_table_stride < n_pages || meta->num_phys_pages <= 0))
    return fail(LINATTN_EINVAL, "quest_scores: page table stride must cover n_pages");
  if (page_size <= 0 || n_pages < 0 || B < 0 || Tq < 0 || offset < 0)
    return fail(LINATTN_EINVAL, "quest_scores: bad sizes");
  return cuda_status(launch_quest_scores(q, q_dtype, B, Hq, Tq, D, q_strides, *meta, page_size, n_pages, offset,
                                         sink_pages, n_pages_b, scores, status, static_cast<cudaStream_t>(stream)),
                     "quest_scores");
}

int linattn_page_topk(const float* scores, int64_t B, int64_t Hq, int64_t Tq, int64_t n_pages, int64_t topk,
                      const int32_t* n_pages_b, int64_t* ids_i64, int32_t* ids_i32, int64_t group,
                      int32_t* union_ids, int32_t* union_count, int64_t max_union, int32_t* union_tokens,
                      int64_t page_size, int64_t offset, const int32_t* seq_lens, int64_t seq_len, int32_t* status,
                      void* stream) {
  if (!scores) return fail(LINATTN_EINVAL, "page_topk: scores is NULL");
  if (n_pages <= 0 || n_pages > 32768)
    return fail(LINATTN_EUNSUPPORTED, "page_topk: n_pages %lld outside [1, 32768]", (long long)n_pages);
  if (topk < 1 || topk > 4096) return fail(LINATTN_EUNSUPPORTED, "page_topk: topk %lld outside [1, 4096]", (long long)topk);
  if (group < 1 || Hq % group) return fail(LINATTN_EINVAL, "page_topk: group must divide Hq");
  if (union_ids && (!union_count || max_union < 1))
    return fail(LINATTN_EINVAL, "page_topk: union needs union_count and max_union >= 1");
  if (union_tokens && page_size <= 0) return fail(LINATTN_EINVAL, "page_topk: union_tokens needs page_size");
  const size_t smem = page_topk_smem_bytes(n_pages, topk);
  if (smem > 200 * 1024) return fail(LINATTN_EUNSUPPORTED, "page_topk: n_pages/topk too large for shared memory");
  TopkParams p;
  p.scores = scores; p.B = B; p.Hq = Hq; p.Tq = Tq; p.n = n_pages; p.topk = topk; p.n_pages_b = n_pages_b;
  p.ids64 = ids_i64; p.ids32 = ids_i32; p.group = group; p.union_ids = union_ids; p.union_count = union_count;
  p.max_union = max_union; p.union_tokens = union_tokens; p.P = page_size > 0 ? page_size : 1; p.offset = offset;
  p.seq_lens = seq_lens; p.seq_len = seq_len; p.status = status;
  return cuda_status(launch_page_topk(p, static_cast<cudaStream_t>(stream)), "page_topk");
}

// workspace: [256-byte header: the work counter of the tensor-core path]
//            [n_splits > 1: o partials fp32 (S, rows, D)][lse partials fp32 (S, rows)]
static constexpr int64_t kWsHeader = 256;

int64_t linattn_sparse_attention_workspace(int64_t B, int64_t Hq, int64_t Tq, int64_t D, int32_t n_splits) {
  if (n_splits <= 1) return kWsHeader;
  return kWsHeader + static_cast<int64_t>(n_splits) * B * Hq * Tq * (D + 1) * static_cast<int64_t>(sizeof(float));
}

int linattn_sparse_attention(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t Tq,
                             const int64_t* q_strides, const linattn_kv_t* kv, const linattn_lists_t* lists,
                             int32_t causal, int64_t offset, float scale, void* out, const int64_t* out_strides,
                             float* lse_out, int32_t n_splits, float* workspace, int64_t workspace_bytes,
                             int32_t* status, void* stream) {
  return linattn_sparse_attention_out(q, q_dtype, B, Hq, Tq, q_strides, kv, lists, causal, offset, scale, out,
                                      q_dtype, out_strides, lse_out, n_splits, workspace, workspace_bytes, status,
                                      stream);
}

int linattn_sparse_attention_out(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t Tq,
                                 const int64_t* q_strides, const linattn_kv_t* kv, const linattn_lists_t* lists,
                                 int32_t causal, int64_t offset, float scale, void* out, int32_t out_dtype,
                                 const int64_t* out_strides, float* lse_out, int32_t n_splits, float* workspace,
                                 int64_t workspace_bytes, int32_t* status, void* stream) {
  int rc = check_kv(kv);
  if (!is_float16_32(out_dtype)) return fail(LINATTN_EUNSUPPORTED, "sparse_attention: out dtype %d", out_dtype);
  if (rc) return rc;
  if (!q || !q_strides || !out || !out_strides || !lists || !lists->ids)
    return fail(LINATTN_EINVAL, "sparse_attention: NULL pointer");
  if (!is_float16_32(q_dtype)) return fail(LINATTN_EUNSUPPORTED, "sparse_attention: q dtype %d not supported", q_dtype);
  if (lists->ids_dtype != LINATTN_I32 && lists->ids_dtype != LINATTN_I64)
    return fail(LINATTN_EINVAL, "sparse_attention: list ids must be int32 or int64");
  if (B < 0 || Tq < 0 || Hq <= 0) return fail(LINATTN_EINVAL, "sparse_attention: bad sizes");
  if (Hq % kv->n_kv_heads) return fail(LINATTN_EINVAL, "sparse_attention: H_kv must divide H_q");
  if (lists->n_heads <= 0 || Hq % lists->n_heads || lists->n_heads % kv->n_kv_heads)
    return fail(LINATTN_EINVAL,
                "sparse_attention: list heads (%d) must divide H_q (%lld) and be a multiple of H_kv (%d)",
                lists->n_heads, (long long)Hq, kv->n_kv_heads);
  if (lists->max_len < 0) return fail(LINATTN_EINVAL, "sparse_attention: max_len < 0");
  const int D = kv->head_dim;
  const int TR = attn_tile_rows(kv->dtype, D);
  if (kv->page_size > TR && kv->page_size % TR)
    return fail(LINATTN_EUNSUPPORTED, "sparse_attention: page_size %d > %d must be a multiple of %d", kv->page_size,
                TR, TR);
  if (n_splits < 1) return fail(LINATTN_EINVAL, "sparse_attention: n_splits must be >= 1");
  const int64_t rows = B * Hq * Tq;
  if (rows == 0) return LINATTN_OK;
  AttnParams p;
  p.q = q; p.q_dtype = q_dtype; p.out_dtype = out_dtype; p.B = B; p.Hq = Hq; p.Tq = Tq;
  for (int i = 0; i < 4; ++i) { p.qs[i] = q_strides[i]; p.os[i] = out_strides[i]; }
  p.kv = *kv; p.lists = *lists; p.causal = causal; p.offset = offset;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out; p.lse_out = lse_out; p.n_splits = n_splits; p.status = status;
  const int64_t g_total = Hq / lists->n_heads;
  // tensor-core path: 16-bit KV with q of the same dtype and D in {64, 128}, or fp8 KV
  // with a 16-bit q (exact in f16 after a power-of-two factor; an fp32 q stays on the
  // fp32 CUDA-core path), D = 128 and pages of at least one 32-row tile (so that a tile
  // has one pair of scales); at most 128 list entries per split (the producer's
  // per-item table), and K/V describable as TMA tensor maps over their [rows, D] views:
  // strides multiples of D, pages either at least one tile (4096 bytes of rows) or a
  // power of two >= 8 rows (box starts stay 1024-byte aligned for the 128-byte
  // swizzle), rows below 2^31 (32-bit coordinates).
  const bool f8_mma = kv->dtype == LINATTN_FP8E4M3 && (q_dtype == LINATTN_BF16 || q_dtype == LINATTN_F16) &&
                      D == 128 && kv->page_size >= 32;
  bool mma_path = (((kv->dtype == LINATTN_BF16 || kv->dtype == LINATTN_F16) && q_dtype == kv->dtype &&
                    (D == 64 || D == 128)) ||
                   f8_mma) &&
                  (lists->max_len + n_splits - 1) / n_splits <= 128;
  const int tile_rows_mma = f8_mma ? 32 : 2048 / D;
  const int64_t P = kv->page_size;
  const int box_rows = static_cast<int>(P >= tile_rows_mma ? tile_rows_mma : P);
  mma_path = mma_path && (P >= tile_rows_mma || (P >= 8 && (P & (P - 1)) == 0)) && kv->stride_b % D == 0 &&
             kv->stride_page % D == 0 && kv->stride_head % D == 0;
  int64_t total_rows = kv->total_rows;
  if (total_rows <= 0) {
    if (kv->page_table)
      total_rows = ((kv->num_phys_pages - 1) * kv->stride_page + (kv->n_kv_heads - 1) * kv->stride_head) / D + P;
    else if (kv->stride_b > 0)
      total_rows = B * kv->stride_b / D;
  }
  mma_path = mma_path && total_rows > 0 && total_rows < (1ll << 31) - 4096;
  CUtensorMap tmk, tmv;
  if (mma_path)
    mma_path = kv_tensor_map(&tmk, kv->k, total_rows, D, kv->dtype, box_rows) &&
               kv_tensor_map(&tmv, kv->v, total_rows, D, kv->dtype, box_rows);
  int G = 1;
  while (G < g_total && G < 8) G <<= 1;
  const int head_chunk = mma_path ? 8 : G;
  p.heads_per_list = static_cast<int>(g_total);
  p.n_head_chunks = static_cast<int>((g_total + head_chunk - 1) / head_chunk);
  const int64_t need = linattn_sparse_attention_workspace(B, Hq, Tq, D, n_splits);
  if (!workspace || workspace_bytes < need)
    return fail(LINATTN_EINVAL, "sparse_attention: workspace of %lld bytes needed", (long long)need);
  if (!aligned(workspace, 256)) return fail(LINATTN_EINVAL, "sparse_attention: workspace must be 256-byte aligned");
  int* counter = reinterpret_cast<int*>(workspace);
  p.ws_o = nullptr;
  p.ws_lse = nullptr;
  if (n_splits > 1) {
    p.ws_o = workspace + kWsHeader / 4;
    p.ws_lse = p.ws_o + static_cast<int64_t>(n_splits) * rows * D;
  }
  const int64_t units = B * static_cast<int64_t>(lists->n_heads) * Tq;
  const int64_t blocks = units * p.n_head_chunks * n_splits;
  if (blocks > 0x7fffffffLL) return fail(LINATTN_EUNSUPPORTED, "sparse_attention: too many work items");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (mma_path) {
    // a kernel, not a memset node, so that the chain selection -> clear -> attention
    // stays kernel to kernel (programmatic dependent launches)
    e = launch_attn_counters_clear(counter, kWsHeader, st);
    if (e == cudaSuccess)
      e = kv->dtype == LINATTN_BF16  ? launch_sparse_attention_mma_bf16(p, tmk, tmv, box_rows, D, counter, blocks, st)
          : kv->dtype == LINATTN_F16 ? launch_sparse_attention_mma_f16(p, tmk, tmv, box_rows, D, counter, blocks, st)
                                     : launch_sparse_attention_mma_fp8(p, tmk, tmv, box_rows, D, counter, blocks, st);
  } else {
    const unsigned grid = static_cast<unsigned>(blocks);
    switch (kv->dtype) {
      case LINATTN_F32: e = launch_sparse_attention_f32(p, D, G, grid, st); break;
      case LINATTN_F16: e = launch_sparse_attention_f16(p, D, G, grid, st); break;
      case LINATTN_BF16: e = launch_sparse_attention_bf16(p, D, G, grid, st); break;
      case LINATTN_FP8E4M3: e = launch_sparse_attention_fp8(p, D, G, grid, st); break;
      default: return fail(LINATTN_EUNSUPPORTED, "sparse_attention: kv dtype");
    }
  }
  rc = cuda_status(e, "sparse_attention");
  if (rc || n_splits == 1) return rc;
  return cuda_status(launch_lse_combine(p.ws_o, p.ws_lse, n_splits, rows, D, out, out_dtype, Hq, Tq, out_strides,
                                        lse_out, st),
                     "sparse_attention combine");
}

int linattn_lse_combine_strided(const float* o_parts, int64_t o_part_stride, const float* lse_parts,
                                int64_t lse_part_stride, int64_t S, int64_t rows, int64_t D, void* out,
                                int32_t out_dtype, float* lse_out, void* stream) {
  if (!o_parts || !lse_parts || !out) return fail(LINATTN_EINVAL, "lse_combine: NULL pointer");
  if (!is_float16_32(out_dtype)) return fail(LINATTN_EUNSUPPORTED, "lse_combine: out dtype %d", out_dtype);
  if (S < 1 || rows < 0 || D < 1 || D > 256) return fail(LINATTN_EINVAL, "lse_combine: bad sizes (D <= 256)");
  if ((o_part_stride != 0 && o_part_stride < rows * D) || (lse_part_stride != 0 && lse_part_stride < rows))
    return fail(LINATTN_EINVAL, "lse_combine: part strides overlap");
  const int64_t os[4] = {0, 0, D, 1};
  return cuda_status(launch_lse_combine(o_parts, lse_parts, S, rows, D, out, out_dtype, 1, rows > 0 ? rows : 1, os,
                                        lse_out, static_cast<cudaStream_t>(stream), o_part_stride, lse_part_stride),
                     "lse_combine");
}

int linattn_lse_combine(const float* o_parts, const float* lse_parts, int64_t S, int64_t rows, int64_t D, void* out,
                        int32_t out_dtype, float* lse_out, void* stream) {
  return linattn_lse_combine_strided(o_parts, 0, lse_parts, 0, S, rows, D, out, out_dtype, lse_out, stream);
}

}  // extern "C"
