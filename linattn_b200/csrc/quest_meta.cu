// Quest page metadata: channel-wise min / max of the keys of every (page, kv head).
//
// Bandwidth-bound reduction: one warp per (batch, head, page); the lanes stride over
// the channels so every row read is a coalesced 32-lane access.  Min/max is exact, so
// for 16-bit and fp32 keys the metadata equals the reference bit for bit
// (src/linattn/kernels/triton/quest_pages.py:38-48).
#include "common.cuh"

namespace linattn {

template <typename T>
__device__ __forceinline__ float elem_to_float(const T* p, int64_t i);
template <> __device__ __forceinline__ float elem_to_float<float>(const float* p, int64_t i) { return p[i]; }
template <> __device__ __forceinline__ float elem_to_float<__half>(const __half* p, int64_t i) {
  return __half2float(p[i]);
}
template <> __device__ __forceinline__ float elem_to_float<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <> __device__ __forceinline__ float elem_to_float<fp8e4m3>(const fp8e4m3* p, int64_t i) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(p[i].x), __NV_E4M3);
  return __half2float(*reinterpret_cast<const __half*>(&h));
}

// Store min rounded toward -inf and max toward +inf, so that narrowing keeps the
// metadata a valid (outward) bound.  Exact whenever the value is representable.
__device__ __forceinline__ void store_bound(void* base, int64_t idx, int dtype, float v, bool is_min) {
  switch (dtype) {
    case LINATTN_F32: static_cast<float*>(base)[idx] = v; break;
    case LINATTN_F16:
      static_cast<__half*>(base)[idx] = is_min ? __float2half_rd(v) : __float2half_ru(v);
      break;
    case LINATTN_BF16:
      static_cast<__nv_bfloat16*>(base)[idx] = is_min ? __float2bfloat16_rd(v) : __float2bfloat16_ru(v);
      break;
    default: break;
  }
}

// Contiguous (B, H, T, D) keys -> (B, H, n_pages, D) bounds of the same dtype.
template <typename T>
__global__ void __launch_bounds__(256) page_bounds_kernel(const T* __restrict__ k, int64_t B, int64_t H, int64_t T_,
                                                          int64_t D, int64_t sb, int64_t sh, int64_t st, int64_t sd,
                                                          int64_t P, int64_t n_pages, T* __restrict__ mins,
                                                          T* __restrict__ maxs) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = B * H * n_pages;
  if (warp >= total) return;
  const int64_t p = warp % n_pages;
  const int64_t bh = warp / n_pages;
  const int64_t h = bh % H, b = bh / H;
  const int64_t r0 = p * P;
  const int64_t r1 = min(r0 + P, T_);
  const T* base = k + b * sb + h * sh;
  T* omin = mins + (bh * n_pages + p) * D;
  T* omax = maxs + (bh * n_pages + p) * D;
  for (int64_t c = lane; c < D; c += 32) {
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t r = r0; r < r1; ++r) {
      const float v = elem_to_float<T>(base, r * st + c * sd);
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    // exact: the value came from a T
    if constexpr (sizeof(T) == 4) {
      omin[c] = mn;
      omax[c] = mx;
    } else if constexpr (std::is_same<T, __half>::value) {
      omin[c] = __float2half_rn(mn);
      omax[c] = __float2half_rn(mx);
    } else {
      omin[c] = __float2bfloat16_rn(mn);
      omax[c] = __float2bfloat16_rn(mx);
    }
  }
}

// Paged pool: refresh pages [first_page[b], ceil(seq_len_b / P)) of every batch.
template <typename T>
__global__ void __launch_bounds__(256) paged_page_bounds_kernel(linattn_kv_t kv, int64_t B,
                                                                const int32_t* __restrict__ first_page,
                                                                int64_t max_pages, linattn_meta_t meta,
                                                                int32_t* status) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t H = kv.n_kv_heads;
  if (warp >= B * max_pages * H) return;
  const int64_t h = warp % H;
  const int64_t p = (warp / H) % max_pages;
  const int64_t b = warp / (H * max_pages);
  const int64_t P = kv.page_size, D = kv.head_dim;
  const int64_t len = kv.seq_lens ? kv.seq_lens[b] : kv.seq_len;
  const int64_t n_pages = (len + P - 1) / P;
  const int64_t p0 = first_page ? first_page[b] : 0;
  if (p < p0 || p >= n_pages) return;
  int64_t phys = p;
  if (kv.page_table) {
    phys = kv.page_table[b * kv.page_table_stride + p];
    if (phys < 0 || phys >= kv.num_phys_pages) {
      if (lane == 0) report(status, LINATTN_DEV_BAD_ID);
      return;
    }
  }
  int64_t mphys = p;
  if (meta.page_table) {
    mphys = meta.page_table[b * meta.page_table_stride + p];
    if (mphys < 0 || mphys >= meta.num_phys_pages) {
      if (lane == 0) report(status, LINATTN_DEV_BAD_ID);
      return;
    }
  }
  const int64_t rows = min(P, len - p * P);
  const T* base = static_cast<const T*>(kv.k) + b * kv.stride_b + phys * kv.stride_page + h * kv.stride_head;
  float scale = 1.f;
  if (kv.k_scale) scale = kv.k_scale[phys * kv.scale_stride_page + h * kv.scale_stride_head];
  const int64_t mo = b * meta.stride_b + mphys * meta.stride_page + h * meta.stride_head;
  for (int64_t c = lane; c < D; c += 32) {
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t r = 0; r < rows; ++r) {
      const float v = elem_to_float<T>(base, r * D + c) * scale;
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    store_bound(const_cast<void*>(meta.mins), mo + c, meta.dtype, mn, true);
    store_bound(const_cast<void*>(meta.maxs), mo + c, meta.dtype, mx, false);
  }
}

// Append: new rows of every sequence into the paged pool, and their pages' bounds.
// One CTA per (batch, kv head, page touched by the new rows), one thread per channel:
// the thread writes its channel of every new row of the page (K and V, converted to
// the pool's dtype; rows are coalesced across the threads) and folds the stored keys
// into the page's bounds, starting from the stored bounds when the page already held
// rows.  Min / max are exact and the outward rounding of narrower metadata commutes
// with them, so the result equals a recomputation over all of the page's rows.
template <typename T>
__device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_float<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename T>
__global__ void __launch_bounds__(256) paged_append_kernel(linattn_kv_t kv, linattn_meta_t meta,
                                                           const void* __restrict__ k_new,
                                                           const void* __restrict__ v_new, int new_dtype,
                                                           int64_t sb, int64_t sh, int64_t st, int64_t T_new,
                                                           const int32_t* __restrict__ start_pos, int32_t* status) {
  const int64_t H = kv.n_kv_heads, P = kv.page_size, D = kv.head_dim;
  const int64_t h = blockIdx.x % H, b = blockIdx.x / H;
  const int64_t start = start_pos[b];
  const int64_t lp = start / P + blockIdx.y;  // logical page
  const int64_t r0 = lmax(start, lp * P), r1 = lmin(start + T_new, (lp + 1) * P);
  if (r0 >= r1 || start < 0) return;
  int64_t phys = lp;
  if (kv.page_table) {
    phys = lp < kv.page_table_stride ? kv.page_table[b * kv.page_table_stride + lp] : -1;
    if (phys < 0 || phys >= kv.num_phys_pages) {
      if (threadIdx.x == 0) report(status, LINATTN_DEV_BAD_ID);
      return;
    }
  }
  int64_t mphys = lp;
  if (meta.page_table) {
    mphys = lp < meta.page_table_stride ? meta.page_table[b * meta.page_table_stride + lp] : -1;
    if (mphys < 0 || mphys >= meta.num_phys_pages) {
      if (threadIdx.x == 0) report(status, LINATTN_DEV_BAD_ID);
      return;
    }
  }
  const int64_t pool0 = b * kv.stride_b + phys * kv.stride_page + h * kv.stride_head;
  T* kp = static_cast<T*>(const_cast<void*>(kv.k)) + pool0;
  T* vp = static_cast<T*>(const_cast<void*>(kv.v)) + pool0;
  const int64_t mo = b * meta.stride_b + mphys * meta.stride_page + h * meta.stride_head;
  const bool had_rows = lp * P < start;
  for (int64_t c = threadIdx.x; c < D; c += blockDim.x) {
    float mn = INFINITY, mx = -INFINITY;
    if (had_rows) {
      mn = load_any(meta.mins, mo + c, meta.dtype);
      mx = load_any(meta.maxs, mo + c, meta.dtype);
    }
    for (int64_t r = r0; r < r1; ++r) {
      const int64_t src = b * sb + h * sh + (r - start) * st + c;
      const T kv_k = from_float<T>(load_any(k_new, src, new_dtype));
      const T kv_v = from_float<T>(load_any(v_new, src, new_dtype));
      kp[(r - lp * P) * D + c] = kv_k;
      vp[(r - lp * P) * D + c] = kv_v;
      const float stored = elem_to_float<T>(&kv_k, 0);
      mn = fminf(mn, stored);
      mx = fmaxf(mx, stored);
    }
    store_bound(const_cast<void*>(meta.mins), mo + c, meta.dtype, mn, true);
    store_bound(const_cast<void*>(meta.maxs), mo + c, meta.dtype, mx, false);
  }
}

// ---------------------------------------------------------------------------------
// launchers (called from capi.cu)
// ---------------------------------------------------------------------------------
cudaError_t launch_page_bounds(const void* k, int dtype, int64_t B, int64_t H, int64_t T_, int64_t D,
                               const int64_t* s, int64_t P, void* mins, void* maxs, cudaStream_t stream) {
  const int64_t n_pages = (T_ + P - 1) / P;
  const int64_t warps = B * H * n_pages;
  if (warps == 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
  switch (dtype) {
    case LINATTN_F32:
      page_bounds_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(k), B, H, T_, D, s[0], s[1],
                                                          s[2], s[3], P, n_pages, static_cast<float*>(mins),
                                                          static_cast<float*>(maxs));
      break;
    case LINATTN_F16:
      page_bounds_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(k), B, H, T_, D, s[0], s[1],
                                                           s[2], s[3], P, n_pages, static_cast<__half*>(mins),
                                                           static_cast<__half*>(maxs));
      break;
    case LINATTN_BF16:
      page_bounds_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(k), B, H, T_, D, s[0], s[1], s[2], s[3], P, n_pages,
          static_cast<__nv_bfloat16*>(mins), static_cast<__nv_bfloat16*>(maxs));
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_paged_page_bounds(const linattn_kv_t& kv, int64_t B, const int32_t* first_page,
                                     int64_t max_pages, const linattn_meta_t& meta, int32_t* status,
                                     cudaStream_t stream) {
  const int64_t warps = B * max_pages * kv.n_kv_heads;
  if (warps == 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
  switch (kv.dtype) {
    case LINATTN_F32:
      paged_page_bounds_kernel<float><<<grid, 256, 0, stream>>>(kv, B, first_page, max_pages, meta, status);
      break;
    case LINATTN_F16:
      paged_page_bounds_kernel<__half><<<grid, 256, 0, stream>>>(kv, B, first_page, max_pages, meta, status);
      break;
    case LINATTN_BF16:
      paged_page_bounds_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(kv, B, first_page, max_pages, meta,
                                                                        status);
      break;
    case LINATTN_FP8E4M3:
      paged_page_bounds_kernel<fp8e4m3><<<grid, 256, 0, stream>>>(kv, B, first_page, max_pages, meta, status);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_paged_append(const linattn_kv_t& kv, const linattn_meta_t& meta, int64_t B, const void* k_new,
                                const void* v_new, int new_dtype, const int64_t* s, int64_t T_new,
                                const int32_t* start_pos, int32_t* status, cudaStream_t stream) {
  if (B == 0 || T_new == 0) return cudaSuccess;
  const int64_t P = kv.page_size;
  const dim3 grid(static_cast<unsigned>(B * kv.n_kv_heads), static_cast<unsigned>((T_new + P - 1 + P - 1) / P));
  const unsigned threads = static_cast<unsigned>(lmin(256, (kv.head_dim + 31) / 32 * 32));
  switch (kv.dtype) {
    case LINATTN_F32:
      paged_append_kernel<float><<<grid, threads, 0, stream>>>(kv, meta, k_new, v_new, new_dtype, s[0], s[1], s[2],
                                                               T_new, start_pos, status);
      break;
    case LINATTN_F16:
      paged_append_kernel<__half><<<grid, threads, 0, stream>>>(kv, meta, k_new, v_new, new_dtype, s[0], s[1], s[2],
                                                                T_new, start_pos, status);
      break;
    case LINATTN_BF16:
      paged_append_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>(kv, meta, k_new, v_new, new_dtype, s[0],
                                                                       s[1], s[2], T_new, start_pos, status);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace linattn
