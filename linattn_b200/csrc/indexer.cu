// Lightning-indexer scores and row top-k (DSA / CSA token selection).
//
// indexer_scores_kernel: I[b,t,s] = sum_h w[b,t,h] * ReLU(q[b,t,h,:] . k[b,s,h,:] * scale_s)
//   in fp32 (src/linattn/kernels/triton/fused_indexer.py:52-60).  fp8 keys carry one
//   fp32 scale per `group` tokens (scale > 0, so it commutes with the ReLU).  One CTA
//   computes a 32-query x 64-key tile for a range of queries: the tiles of q and k
//   are staged in shared memory as fp32 (k rows padded so the 32 lanes of a warp,
//   one key each, hit 32 different banks); warp w owns 4 queries, lane l keys l and
//   l + 32.  With `causal`, keys after the query position (offset + t) are -inf.
// row_topk_kernel: the k largest values of each score row, sorted by (value desc,
//   index asc): a 4-pass 8-bit radix select over order-preserving keys in shared
//   memory (ties at the k-th value -> lowest index; rows longer than 32768 are
//   re-read from global memory on each pass), then a bitonic sort of the k winners.  Rows shorter than k (causal) pad with (-inf, -1).
#include <cstdio>

#include "launchers.cuh"

namespace linattn {

namespace {

constexpr int IQ = 32;  // queries per tile
constexpr int IK = 64;  // keys per tile

template <typename T>
__device__ __forceinline__ float elem(const T* p, int64_t i);
template <> __device__ __forceinline__ float elem<float>(const float* p, int64_t i) { return p[i]; }
template <> __device__ __forceinline__ float elem<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <> __device__ __forceinline__ float elem<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <> __device__ __forceinline__ float elem<fp8e4m3>(const fp8e4m3* p, int64_t i) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(p[i].x), __NV_E4M3);
  return __half2float(*reinterpret_cast<const __half*>(&h));
}

struct IndexerParams {
  const void* q;
  int q_dtype;
  const void* k;
  const float* k_scale;  // (B, ceil(Tk / group)) or NULL
  int64_t group;
  const void* w;
  int w_dtype;
  int64_t B, Tq, Tk, H, D;
  int64_t qs[4], ks[4], ws[3], ss;  // element strides; ss = batch stride of k_scale
  int causal;
  int64_t offset;
  int64_t t_begin;  // first query of this launch; rows of `scores` are t - t_begin
  float* scores;
  int64_t row_stride;
};

}  // namespace

template <typename KT>
__global__ void __launch_bounds__(256) indexer_scores_kernel(const IndexerParams p) {
  extern __shared__ float ismem[];
  const int64_t HD = p.H * p.D;
  const int64_t kpad = HD + 1;  // odd row stride: lanes (one key each) hit distinct banks
  float* qs = ismem;                 // [IQ][HD]
  float* ks = qs + IQ * HD;          // [IK][kpad]
  float* wsm = ks + IK * kpad;       // [IQ][H]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t b = blockIdx.z;
  const int64_t t0 = p.t_begin + static_cast<int64_t>(blockIdx.y) * IQ;
  const int64_t s0 = static_cast<int64_t>(blockIdx.x) * IK;
  const int64_t t_last = lmin(p.Tq, t0 + IQ) - 1;
  if (p.causal && s0 > p.offset + t_last) {
    // whole tile after every query of the block: -inf
    for (int i = tid; i < IQ * IK; i += 256) {
      const int64_t t = t0 + i / IK, s = s0 + i % IK;
      if (t < p.Tq && s < p.Tk) p.scores[(b * (p.Tq - p.t_begin) + t - p.t_begin) * p.row_stride + s] = -INFINITY;
    }
    return;
  }
  for (int64_t i = tid; i < IQ * HD; i += 256) {
    const int64_t r = i / HD, c = i % HD, t = t0 + r;
    qs[i] = t < p.Tq ? load_any(p.q, b * p.qs[0] + t * p.qs[1] + (c / p.D) * p.qs[2] + (c % p.D) * p.qs[3], p.q_dtype)
                     : 0.f;
  }
  const KT* kb = static_cast<const KT*>(p.k);
  for (int64_t i = tid; i < IK * HD; i += 256) {
    const int64_t r = i / HD, c = i % HD, s = s0 + r;
    ks[r * kpad + c] = s < p.Tk ? elem<KT>(kb, b * p.ks[0] + s * p.ks[1] + (c / p.D) * p.ks[2] + (c % p.D) * p.ks[3])
                                : 0.f;
  }
  for (int64_t i = tid; i < IQ * p.H; i += 256) {
    const int64_t r = i / p.H, h = i % p.H, t = t0 + r;
    wsm[i] = t < p.Tq ? load_any(p.w, b * p.ws[0] + t * p.ws[1] + h * p.ws[2], p.w_dtype) : 0.f;
  }
  __syncthreads();
  // warp w: queries 4w..4w+3; lane: keys lane, lane + 32
  float acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = 0.f;
  for (int64_t h = 0; h < p.H; ++h) {
    float dot[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) dot[i][0] = dot[i][1] = 0.f;
    const float* k0 = ks + lane * kpad + h * p.D;
    const float* k1 = ks + (lane + 32) * kpad + h * p.D;
    for (int64_t d = 0; d < p.D; ++d) {
      const float a0 = k0[d], a1 = k1[d];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float qv = qs[(warp * 4 + i) * HD + h * p.D + d];
        dot[i][0] = fmaf(qv, a0, dot[i][0]);
        dot[i][1] = fmaf(qv, a1, dot[i][1]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float wv = wsm[(warp * 4 + i) * p.H + h];
      // fp8: ReLU(scale * dot) = scale * ReLU(dot) for scale > 0; applied below
      acc[i][0] = fmaf(wv, fmaxf(dot[i][0], 0.f), acc[i][0]);
      acc[i][1] = fmaf(wv, fmaxf(dot[i][1], 0.f), acc[i][1]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t t = t0 + warp * 4 + i;
    if (t >= p.Tq) continue;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int64_t s = s0 + lane + 32 * j;
      if (s >= p.Tk) continue;
      float v = acc[i][j];
      if (p.k_scale) v *= p.k_scale[b * p.ss + s / p.group];
      if (p.causal && s > p.offset + t) v = -INFINITY;
      p.scores[(b * (p.Tq - p.t_begin) + t - p.t_begin) * p.row_stride + s] = v;
    }
  }
}

// ---------------------------------------------------------------------------------
// row top-k
// ---------------------------------------------------------------------------------
constexpr int64_t kSmemKeys = 32768;

struct RowTopkParams {
  const float* scores;
  int64_t rows, n, row_stride;
  int64_t k;
  int64_t kpow2;
  int causal;
  int64_t first_pos;  // causal: row r keeps n_valid = min(n, first_pos + r % period + 1)
  int64_t period;     // rows per sequence
  float* values;      // row r -> (r / period) * out_bstride + (r % period) * out_stride
  int64_t* idx64;
  int32_t* idx32;
  int64_t out_stride, out_bstride;
};

__global__ void __launch_bounds__(512) row_topk_kernel(const RowTopkParams p) {
  extern __shared__ uint32_t tsm[];
  // rows of up to kSmemKeys entries are staged in shared memory as order-preserving
  // keys; longer rows are re-read from global memory (L2) on every pass
  const bool staged = p.n <= kSmemKeys;
  uint32_t* keys = tsm;                              // [n] when staged
  uint32_t* sk = tsm + (staged ? p.n : 0);           // [kpow2] selected keys
  uint32_t* si = sk + p.kpow2;                       // [kpow2] selected indices
  __shared__ uint32_t hist[256];
  __shared__ uint32_t scratch[17];
  __shared__ uint32_t sh_digit, sh_remaining, sh_count;
  const int tid = threadIdx.x;
  const int64_t r = blockIdx.x;
  const int64_t seg = r / p.period, j = r % p.period;
  const int64_t nv = p.causal ? lmax(0, lmin(p.n, p.first_pos + j + 1)) : p.n;
  const int64_t ob = seg * p.out_bstride + j * p.out_stride;
  const int64_t kb = lmin(p.k, nv);
  const float* row = p.scores + r * p.row_stride;
  if (staged)
    for (int64_t i = tid; i < nv; i += 512) keys[i] = float_key(row[i]);
  auto key_at = [&](int64_t i) { return staged ? keys[i] : float_key(row[i]); };
  if (tid == 0) sh_count = 0u;
  __syncthreads();
  uint32_t prefix = 0u, mask = 0u, remaining = static_cast<uint32_t>(kb);
  if (kb > 0) {
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (tid < 256) hist[tid] = 0u;
      __syncthreads();
      for (int64_t i = tid; i < nv; i += 512) {
        const uint32_t key = key_at(i);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      const uint32_t c = tid < 256 ? hist[255 - tid] : 0u;
      const uint32_t above = block_exclusive_scan<512>(c, scratch, nullptr);
      if (tid < 256 && above < remaining && above + c >= remaining) {
        sh_digit = 255u - static_cast<uint32_t>(tid);
        sh_remaining = remaining - above;
      }
      __syncthreads();
      prefix |= sh_digit << shift;
      mask |= 0xffu << shift;
      remaining = sh_remaining;
    }
  }
  const uint32_t kstar = prefix, need_eq = remaining;
  const int64_t chunk = (nv + 511) / 512;
  const int64_t i0 = lmin(nv, tid * chunk), i1 = lmin(nv, i0 + chunk);
  uint32_t n_eq = 0u;
  for (int64_t i = i0; i < i1; ++i) n_eq += key_at(i) == kstar ? 1u : 0u;
  uint32_t eq_seen = block_exclusive_scan<512>(n_eq, scratch, nullptr);
  if (kb > 0) {
    for (int64_t i = i0; i < i1; ++i) {
      const uint32_t key = key_at(i);
      bool take = key > kstar;
      if (key == kstar) {
        take = eq_seen < need_eq;
        ++eq_seen;
      }
      if (take) {
        const uint32_t pos = atomicAdd(&sh_count, 1u);
        if (pos < static_cast<uint32_t>(kb)) {
          sk[pos] = key;
          si[pos] = static_cast<uint32_t>(i);
        }
      }
    }
  }
  __syncthreads();
  // pad to a power of two with entries that sort last
  for (int64_t i = kb + tid; i < p.kpow2; i += 512) {
    sk[i] = 0u;
    si[i] = 0xffffffffu;
  }
  __syncthreads();
  // bitonic sort: descending by key, ascending by index among equal keys
  for (int64_t size = 2; size <= p.kpow2; size <<= 1) {
    for (int64_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (int64_t i = tid; i < p.kpow2; i += 512) {
        const int64_t j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const uint32_t ka = sk[i], kb2 = sk[j], ia = si[i], ib = si[j];
          const bool a_first = ka > kb2 || (ka == kb2 && ia < ib);  // a belongs before b
          if (a_first != desc) {
            sk[i] = kb2;
            sk[j] = ka;
            si[i] = ib;
            si[j] = ia;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int64_t i = tid; i < p.k; i += 512) {
    const bool ok = i < kb;
    if (p.values) p.values[ob + i] = ok ? key_float(sk[i]) : -INFINITY;
    if (p.idx64) p.idx64[ob + i] = ok ? static_cast<int64_t>(si[i]) : -1;
    if (p.idx32) p.idx32[ob + i] = ok ? static_cast<int32_t>(si[i]) : -1;
  }
}

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_indexer_scores(const void* q_idx, int32_t q_dtype, const int64_t* q_strides,
                                      const void* k_idx, int32_t k_dtype, const int64_t* k_strides,
                                      const float* k_scale, int64_t scale_group, int64_t scale_batch_stride,
                                      const void* head_weights, int32_t w_dtype, const int64_t* w_strides,
                                      int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D, int32_t causal,
                                      int64_t offset, int64_t t_begin, int64_t t_end, float* scores,
                                      int64_t row_stride, void* stream) {
  if (!q_idx || !k_idx || !head_weights || !scores || !q_strides || !k_strides || !w_strides)
    return set_error(LINATTN_EINVAL, "indexer_scores: NULL pointer");
  const bool qok = q_dtype == LINATTN_F32 || q_dtype == LINATTN_F16 || q_dtype == LINATTN_BF16;
  if (!qok || !(w_dtype == LINATTN_F32 || w_dtype == LINATTN_F16 || w_dtype == LINATTN_BF16))
    return set_error(LINATTN_EUNSUPPORTED, "indexer_scores: q / weights dtype");
  if (k_dtype == LINATTN_FP8E4M3 && (!k_scale || scale_group < 1))
    return set_error(LINATTN_EINVAL, "indexer_scores: fp8 keys need k_scale and scale_group");
  if (H < 1 || D < 1 || H * D > 512) return set_error(LINATTN_EUNSUPPORTED, "indexer_scores: H * D must be <= 512");
  if (t_begin < 0 || t_end > Tq || t_begin > t_end || row_stride < Tk)
    return set_error(LINATTN_EINVAL, "indexer_scores: bad query range or row stride");
  if (B == 0 || t_end == t_begin || Tk == 0) return LINATTN_OK;
  IndexerParams p;
  p.q = q_idx; p.q_dtype = q_dtype; p.k = k_idx; p.k_scale = k_scale; p.group = scale_group > 0 ? scale_group : 1;
  p.w = head_weights; p.w_dtype = w_dtype; p.B = B; p.Tq = t_end; p.Tk = Tk; p.H = H; p.D = D;
  for (int i = 0; i < 4; ++i) { p.qs[i] = q_strides[i]; p.ks[i] = k_strides[i]; }
  for (int i = 0; i < 3; ++i) p.ws[i] = w_strides[i];
  p.ss = scale_batch_stride; p.causal = causal; p.offset = offset; p.t_begin = t_begin; p.scores = scores;
  p.row_stride = row_stride;
  const size_t smem = (static_cast<size_t>(IQ) * H * D + static_cast<size_t>(IK) * (H * D + 1) +
                       static_cast<size_t>(IQ) * H) * sizeof(float);
  dim3 grid(static_cast<unsigned>((Tk + IK - 1) / IK), static_cast<unsigned>((t_end - t_begin + IQ - 1) / IQ),
            static_cast<unsigned>(B));
  if (B > 65535 || grid.y > 65535) return set_error(LINATTN_EUNSUPPORTED, "indexer_scores: too many query tiles");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  auto go = [&](auto kernel) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess) kernel<<<grid, 256, smem, st>>>(p);
    if (e == cudaSuccess) e = cudaGetLastError();
  };
  switch (k_dtype) {
    case LINATTN_F32: go(indexer_scores_kernel<float>); break;
    case LINATTN_F16: go(indexer_scores_kernel<__half>); break;
    case LINATTN_BF16: go(indexer_scores_kernel<__nv_bfloat16>); break;
    case LINATTN_FP8E4M3: go(indexer_scores_kernel<fp8e4m3>); break;
    default: return set_error(LINATTN_EUNSUPPORTED, "indexer_scores: k dtype");
  }
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "indexer_scores: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}

extern "C" int linattn_row_topk(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t k,
                                int32_t causal, int64_t first_pos, int64_t period, float* values,
                                int64_t* idx_i64, int32_t* idx_i32, int64_t out_stride, int64_t out_batch_stride,
                                void* stream) {
  if (!scores) return set_error(LINATTN_EINVAL, "row_topk: scores is NULL");
  if (n < 1 || n >= (int64_t(1) << 31)) return set_error(LINATTN_EUNSUPPORTED, "row_topk: row length must be in [1, 2^31)");
  if (k < 1 || k > 4096) return set_error(LINATTN_EUNSUPPORTED, "row_topk: k must be in [1, 4096]");
  if (row_stride < n || out_stride < k || period < 1) return set_error(LINATTN_EINVAL, "row_topk: bad strides");
  if (rows == 0) return LINATTN_OK;
  int64_t kp = 1;
  while (kp < k) kp <<= 1;
  RowTopkParams p;
  p.scores = scores; p.rows = rows; p.n = n; p.row_stride = row_stride; p.k = k; p.kpow2 = kp; p.causal = causal;
  p.first_pos = first_pos; p.period = period; p.values = values; p.idx64 = idx_i64; p.idx32 = idx_i32;
  p.out_stride = out_stride; p.out_bstride = out_batch_stride;
  const size_t smem = static_cast<size_t>((n <= kSmemKeys ? n : 0) + 2 * kp) * sizeof(uint32_t);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaFuncSetAttribute(row_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e == cudaSuccess) {
    row_topk_kernel<<<static_cast<unsigned>(rows), 512, smem, st>>>(p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "row_topk: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
