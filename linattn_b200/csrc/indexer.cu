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
  int64_t kb;       // key s covers positions [s * kb, (s + 1) * kb): visible iff s * kb <= offset + t
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
  if (p.causal && s0 * p.kb > p.offset + t_last) {
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
      if (p.causal && s * p.kb > p.offset + t) v = -INFINITY;
      p.scores[(b * (p.Tq - p.t_begin) + t - p.t_begin) * p.row_stride + s] = v;
    }
  }
}

// ---------------------------------------------------------------------------------
// row top-k
// ---------------------------------------------------------------------------------
constexpr int64_t kSmemKeys = 32768;

// Keys visible from position pos when key s covers [s * kb, (s + 1) * kb): s * kb <= pos.
__device__ __forceinline__ int64_t visible_keys(int64_t n, int64_t pos, int64_t kb) {
  return pos < 0 ? 0 : lmin(n, pos / kb + 1);
}

struct RowTopkParams {
  const float* scores;
  int64_t rows, n, row_stride;
  int64_t k;
  int64_t kpow2;
  int causal;
  int64_t first_pos;  // causal: row r keeps n_valid = min(n, (first_pos + r % period) / kb + 1)
  int64_t kb;
  int64_t period;     // rows per sequence
  float* values;      // row r -> (r / period) * out_bstride + (r % period) * out_stride
  int64_t* idx64;
  int32_t* idx32;
  int64_t out_stride, out_bstride;
  int sorted;  // 1: by (value desc, index asc); 0: ascending index
  int64_t skip;  // entries [0, skip) of every row are not candidates
};

// Rows of up to NT * ITEMS entries: each thread keeps ITEMS order-preserving keys in
// registers (entry i = it * NT + tid).  The first digit is one of 4096 bins linear in
// the value over the row's finite range (monotone in the key, so it is a valid radix
// digit, and it spreads the shared-memory atomics); 12-bit digits of the key relative
// to the chosen bin's smallest key follow, for entries of that bin only.
template <int NT, int ITEMS>
__global__ void __launch_bounds__(NT, 1024 / NT) row_topk_reg_kernel(const RowTopkParams p) {
  constexpr int BPT = 4096 / NT;  // first-pass bins per thread
  extern __shared__ uint32_t rsm[];  // sorted: keys[kpow2] + idx[kpow2]; index order: bitmap
  __shared__ uint32_t hist[4096];
  __shared__ uint32_t scratch[NT / 32 + 1];
  __shared__ uint32_t sh_min[NT / 32], sh_max[NT / 32];
  __shared__ uint32_t sh_digit, sh_remaining, sh_bin_count, sh_count;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t r = blockIdx.x;
  const int64_t seg = r / p.period, j = r % p.period;
  const int nv_all = static_cast<int>(p.causal ? visible_keys(p.n, p.first_pos + j, p.kb) : p.n);
  const int skip = static_cast<int>(lmin(p.skip, nv_all));
  const int nv = nv_all - skip;  // candidates: entries skip .. nv_all - 1, indexed from 0 here
  const int64_t ob = seg * p.out_bstride + j * p.out_stride;
  const int kb = static_cast<int>(lmin(p.k, nv));
  const float* row = p.scores + r * p.row_stride + skip;

  uint32_t u[ITEMS];
  // range of the finite entries, as order-preserving keys (for the first digit)
  uint32_t fmin_k = 0xffffffffu, fmax_k = 0u;
  const int my_n = nv > tid ? (nv - tid + NT - 1) / NT : 0;  // entries it < my_n are valid
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const float f = it < my_n ? __ldg(row + it * NT + tid) : 0.f;
    u[it] = float_key(f);
    if (it < my_n && isfinite(f)) {
      fmin_k = min(fmin_k, u[it]);
      fmax_k = max(fmax_k, u[it]);
    }
  }
  // block-wide min / max of two keys (all threads get the result)
  auto block_min_max = [&](uint32_t& mn, uint32_t& mx) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) {
      sh_min[warp] = mn;
      sh_max[warp] = mx;
    }
    __syncthreads();
    mn = sh_min[0];
    mx = sh_max[0];
#pragma unroll
    for (int w = 1; w < NT / 32; ++w) {
      mn = min(mn, sh_min[w]);
      mx = max(mx, sh_max[w]);
    }
    __syncthreads();
  };
  // k-th largest digit over hist[0..4095] (descending): digit, count still needed in
  // it, and its population
  auto find_digit = [&](uint32_t remaining) {
    uint32_t cnt[BPT], loc = 0u;
#pragma unroll
    for (int e = 0; e < BPT; ++e) {
      cnt[e] = hist[4095 - BPT * tid - e];
      loc += cnt[e];
    }
    uint32_t above = block_exclusive_scan<NT>(loc, scratch, nullptr);
    if (above < remaining && above + loc >= remaining) {
#pragma unroll
      for (int e = 0; e < BPT; ++e) {
        if (above < remaining && above + cnt[e] >= remaining) {
          sh_digit = static_cast<uint32_t>(4095 - BPT * tid - e);
          sh_remaining = remaining - above;
          sh_bin_count = cnt[e];
        }
        above += cnt[e];
      }
    }
    __syncthreads();
  };
  if (tid == 0) sh_count = 0u;
  uint32_t kstar = 0u, need_eq = 0u, eq_total = 0u;
  if (kb > 0 && kb < nv) {
    block_min_max(fmin_k, fmax_k);
    // first digit: 4096 bins linear in the value over the finite range (monotone in
    // the key; non-finite entries go to the end bins)
    const bool any_finite = fmin_k <= fmax_k;
    const float lo = key_float(fmin_k), span = key_float(fmax_k) - lo;
    const bool linear = any_finite && span > 0.f && isfinite(span);
    const float bscale = linear ? 4096.f / span : 0.f;
    auto bin_of = [&](uint32_t key) -> uint32_t {
      if (!any_finite) return key >> 20;
      if (key < fmin_k) return 0u;
      if (key > fmax_k) return 4095u;
      if (!linear) return 0u;
      return static_cast<uint32_t>(min(static_cast<int>((key_float(key) - lo) * bscale), 4095));
    };
    for (int i = tid; i < 4096; i += NT) hist[i] = 0u;
    __syncthreads();
#pragma unroll
    for (int it = 0; it < ITEMS; ++it)
      if (it < my_n) atomicAdd(&hist[bin_of(u[it])], 1u);
    __syncthreads();
    find_digit(static_cast<uint32_t>(kb));
    const uint32_t d1 = sh_digit;
    uint32_t remaining = sh_remaining;
    eq_total = sh_bin_count;
    // entries in that bin, and their key range
    uint32_t inb = 0u, blo = 0xffffffffu, bhi = 0u;
#pragma unroll
    for (int it = 0; it < ITEMS; ++it)
      if (it < my_n && bin_of(u[it]) == d1) {
        inb |= 1u << it;
        blo = min(blo, u[it]);
        bhi = max(bhi, u[it]);
      }
    block_min_max(blo, bhi);
    // refine inside the bin: 12-bit digits of key - blo, entries with a matching prefix
    const uint32_t rng = bhi - blo;
    int bits_left = rng ? 32 - __clz(rng) : 0;
    uint32_t prefix = 0u;
    while (bits_left > 0) {
      const int width = bits_left < 12 ? bits_left : 12;
      const int shift = bits_left - width;
      for (int i = tid; i < 4096; i += NT) hist[i] = 0u;
      __syncthreads();
#pragma unroll
      for (int it = 0; it < ITEMS; ++it) {
        const uint32_t uk = u[it] - blo;
        if (((inb >> it) & 1u) && (static_cast<uint64_t>(uk) >> (shift + width)) == prefix)
          atomicAdd(&hist[(uk >> shift) & ((1u << width) - 1u)], 1u);
      }
      __syncthreads();
      find_digit(remaining);
      prefix = (prefix << width) | sh_digit;
      remaining = sh_remaining;
      eq_total = sh_bin_count;
      bits_left = shift;
    }
    kstar = blo + prefix;  // full key of the k-th largest entry
    need_eq = remaining;
  }
  // ---- which entries are taken: key > kstar, or key == kstar among the first need_eq
  uint64_t take = 0u;
  if (kb >= nv) {
#pragma unroll
    for (int it = 0; it < ITEMS; ++it)
      if (it < my_n) take |= 1ull << it;
  } else if (kb > 0) {
    const bool all_ties = need_eq == eq_total;
#pragma unroll
    for (int it = 0; it < ITEMS; ++it)
      if (it < my_n && (u[it] > kstar || (all_ties && u[it] == kstar))) take |= 1ull << it;
    if (!all_ties) {
      // ties at the k-th value go to the lowest indices: select the need_eq-th smallest
      // index among them by two radix passes over the index (high bits, then low bits)
      const int lo_bits = nv > 256 ? 32 - __clz(static_cast<uint32_t>(nv - 1)) - 8 : 0;
      uint32_t want = need_eq, hi = 0u;
      for (int pass = 0; pass < 2; ++pass) {
        if (tid < 256) hist[tid] = 0u;
        __syncthreads();
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
          const uint32_t i = static_cast<uint32_t>(it * NT + tid);
          if (it < my_n && u[it] == kstar) {
            if (pass == 0) atomicAdd(&hist[i >> lo_bits], 1u);
            else if ((i >> lo_bits) == hi) atomicAdd(&hist[i & ((1u << lo_bits) - 1u)], 1u);
          }
        }
        __syncthreads();
        const uint32_t cbin = tid < 256 ? hist[tid] : 0u;
        const uint32_t before = block_exclusive_scan<NT>(cbin, scratch, nullptr);  // ascending bins
        if (tid < 256 && before < want && before + cbin >= want) {
          sh_digit = static_cast<uint32_t>(tid);
          sh_remaining = want - before;
        }
        __syncthreads();
        if (pass == 0) hi = sh_digit;
        want = sh_remaining;
        if (lo_bits == 0) break;
      }
      // the last tie taken has index (hi << lo_bits) | low digit
      const uint32_t last = lo_bits ? ((hi << lo_bits) | sh_digit) : hi;
#pragma unroll
      for (int it = 0; it < ITEMS; ++it) {
        if (it < my_n && u[it] == kstar && static_cast<uint32_t>(it * NT + tid) <= last) take |= 1ull << it;
      }
    }
  }
  if (p.sorted) {
    uint32_t* sk = rsm;
    uint32_t* si = rsm + p.kpow2;
#pragma unroll
    for (int it = 0; it < ITEMS; ++it)
      if ((take >> it) & 1u) {
        const uint32_t pos = atomicAdd(&sh_count, 1u);
        if (pos < static_cast<uint32_t>(kb)) {
          sk[pos] = u[it];
          si[pos] = static_cast<uint32_t>(it * NT + tid);
        }
      }
    __syncthreads();
    for (int64_t i = kb + tid; i < p.kpow2; i += NT) {
      sk[i] = 0u;
      si[i] = 0xffffffffu;
    }
    __syncthreads();
    for (int64_t size = 2; size <= p.kpow2; size <<= 1) {
      for (int64_t stride = size >> 1; stride > 0; stride >>= 1) {
        for (int64_t i = tid; i < p.kpow2; i += NT) {
          const int64_t jj = i ^ stride;
          if (jj > i) {
            const bool desc = (i & size) == 0;
            const uint32_t ka = sk[i], kb2 = sk[jj], ia = si[i], ib = si[jj];
            const bool a_first = ka > kb2 || (ka == kb2 && ia < ib);
            if (a_first != desc) {
              sk[i] = kb2;
              sk[jj] = ka;
              si[i] = ib;
              si[jj] = ia;
            }
          }
        }
        __syncthreads();
      }
    }
    for (int64_t i = tid; i < p.k; i += NT) {
      const bool ok = i < kb;
      if (p.values) p.values[ob + i] = ok ? key_float(sk[i]) : -INFINITY;
      if (p.idx64) p.idx64[ob + i] = ok ? static_cast<int64_t>(si[i]) + skip : -1;
      if (p.idx32) p.idx32[ob + i] = ok ? static_cast<int32_t>(si[i]) + skip : -1;
    }
  } else {
    // ascending index: bitmap, then a popcount scan over its words
    uint32_t* bits = rsm;
    const int nwords = (nv + 31) >> 5;
    for (int i = tid; i < nwords; i += NT) bits[i] = 0u;
    __syncthreads();
#pragma unroll
    for (int it = 0; it < ITEMS; ++it)
      if ((take >> it) & 1u) {
        const int i = it * NT + tid;
        atomicOr(&bits[i >> 5], 1u << (i & 31));
      }
    __syncthreads();
    const int per = (nwords + NT - 1) / NT;
    const int w0 = tid * per, w1 = min(nwords, w0 + per);
    uint32_t cnt = 0u;
    for (int w = w0; w < w1; ++w) cnt += __popc(bits[w]);
    uint32_t pos = block_exclusive_scan<NT>(cnt, scratch, nullptr);
    for (int w = w0; w < w1; ++w) {
      uint32_t m = bits[w];
      while (m) {
        const int bpos = __ffs(m) - 1;
        m &= m - 1u;
        const int i = (w << 5) | bpos;
        if (p.values) p.values[ob + pos] = __ldg(row + i);
        if (p.idx64) p.idx64[ob + pos] = i + skip;
        if (p.idx32) p.idx32[ob + pos] = i + skip;
        ++pos;
      }
    }
    for (int64_t i = kb + tid; i < p.k; i += NT) {
      if (p.values) p.values[ob + i] = -INFINITY;
      if (p.idx64) p.idx64[ob + i] = -1;
      if (p.idx32) p.idx32[ob + i] = -1;
    }
  }
}

// Rows of any length: keys staged in shared memory up to kSmemKeys entries, re-read
// from global memory beyond.  Four 8-bit radix passes.
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
  const int64_t nv_all = p.causal ? visible_keys(p.n, p.first_pos + j, p.kb) : p.n;
  const int64_t skip = lmin(p.skip, nv_all);
  const int64_t nv = nv_all - skip;
  const int64_t ob = seg * p.out_bstride + j * p.out_stride;
  const int64_t kb = lmin(p.k, nv);
  const float* row = p.scores + r * p.row_stride + skip;
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
          // a belongs before b: (key desc, index asc), or index asc for index order
          const bool a_first = p.sorted ? (ka > kb2 || (ka == kb2 && ia < ib)) : ia < ib;
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
    if (p.idx64) p.idx64[ob + i] = ok ? static_cast<int64_t>(si[i]) + skip : -1;
    if (p.idx32) p.idx32[ob + i] = ok ? static_cast<int32_t>(si[i]) + skip : -1;
  }
}

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_indexer_scores(const void* q_idx, int32_t q_dtype, const int64_t* q_strides,
                                      const void* k_idx, int32_t k_dtype, const int64_t* k_strides,
                                      const float* k_scale, int64_t scale_group, int64_t scale_batch_stride,
                                      const void* head_weights, int32_t w_dtype, const int64_t* w_strides,
                                      int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D, int32_t causal,
                                      int64_t offset, int64_t key_block, int64_t t_begin, int64_t t_end, float* scores,
                                      int64_t row_stride, int32_t* status, void* stream) {
  if (!q_idx || !k_idx || !head_weights || !scores || !q_strides || !k_strides || !w_strides)
    return set_error(LINATTN_EINVAL, "indexer_scores: NULL pointer");
  const bool qok = q_dtype == LINATTN_F32 || q_dtype == LINATTN_F16 || q_dtype == LINATTN_BF16;
  if (!qok || !(w_dtype == LINATTN_F32 || w_dtype == LINATTN_F16 || w_dtype == LINATTN_BF16))
    return set_error(LINATTN_EUNSUPPORTED, "indexer_scores: q / weights dtype");
  if (k_dtype == LINATTN_FP8E4M3 && (!k_scale || scale_group < 1))
    return set_error(LINATTN_EINVAL, "indexer_scores: fp8 keys need k_scale and scale_group");
  if (H < 1 || D < 1 || H * D > 512) return set_error(LINATTN_EUNSUPPORTED, "indexer_scores: H * D must be <= 512");
  if (causal < 0 || causal > 2) return set_error(LINATTN_EINVAL, "indexer_scores: causal must be 0, 1 or 2");
  if (key_block < 1) return set_error(LINATTN_EINVAL, "indexer_scores: key_block must be >= 1");
  if (t_begin < 0 || t_end > Tq || t_begin > t_end || row_stride < Tk)
    return set_error(LINATTN_EINVAL, "indexer_scores: bad query range or row stride");
  if (B == 0 || t_end == t_begin || Tk == 0) return LINATTN_OK;
  IndexerParams p;
  p.q = q_idx; p.q_dtype = q_dtype; p.k = k_idx; p.k_scale = k_scale; p.group = scale_group > 0 ? scale_group : 1;
  p.w = head_weights; p.w_dtype = w_dtype; p.B = B; p.Tq = t_end; p.Tk = Tk; p.H = H; p.D = D;
  for (int i = 0; i < 4; ++i) { p.qs[i] = q_strides[i]; p.ks[i] = k_strides[i]; }
  for (int i = 0; i < 3; ++i) p.ws[i] = w_strides[i];
  p.ss = scale_batch_stride; p.causal = causal; p.offset = offset; p.kb = key_block; p.t_begin = t_begin;
  p.scores = scores;
  p.row_stride = row_stride;
  {
    cudaError_t me = cudaSuccess;
    if (indexer_scores_mma(q_idx, q_dtype, q_strides, k_idx, k_dtype, k_strides, k_scale, scale_group,
                           scale_batch_stride, head_weights, w_dtype, w_strides, B, Tq, Tk, H, D, causal, offset,
                           key_block,
                           t_begin, t_end, scores, row_stride, status, static_cast<cudaStream_t>(stream), &me)) {
      if (me != cudaSuccess) {
        char msg[256];
        snprintf(msg, sizeof(msg), "indexer_scores: %s", cudaGetErrorString(me));
        return set_error(LINATTN_ECUDA, msg);
      }
      return LINATTN_OK;
    }
  }
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

// Short rows (n <= 32 * ITEMS <= 2048) in index order: one warp per row, eight rows
// per CTA.  Lane l holds entries i = it * 32 + l (coalesced loads) as order-preserving
// keys; the k-th largest key is found by a binary search over the key range with warp
// counts (eight independent partial sums per lane, and an early exit once exactly k
// keys reach the probe); the keys above it and the lowest-index copies of it are then
// written in ascending index order by ballots over the entry blocks.  Same selection
// and output as row_topk_reg_kernel's index-order path.
template <int ITEMS>
__global__ void __launch_bounds__(256) row_topk_warp_kernel(const RowTopkParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= p.rows) return;  // warp-uniform
  const int64_t seg = r / p.period, j = r % p.period;
  const int nv_all = static_cast<int>(p.causal ? visible_keys(p.n, p.first_pos + j, p.kb) : p.n);
  const int skip = static_cast<int>(lmin(p.skip, nv_all));
  const int nv = nv_all - skip;  // candidates: entries skip .. nv_all - 1, indexed from 0 here
  const int64_t ob = seg * p.out_bstride + j * p.out_stride;
  const int kb = static_cast<int>(lmin(p.k, nv));
  const float* row = p.scores + r * p.row_stride + skip;
  uint32_t key[ITEMS];
  uint32_t kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const int i = it * 32 + lane;
    key[it] = i < nv ? float_key(__ldg(row + i)) : 0u;  // candidate keys are > 0 (even -inf's)
    if (i < nv) {
      kmin = min(kmin, key[it]);
      kmax = max(kmax, key[it]);
    }
  }
  auto count_ge = [&](uint32_t t) -> uint32_t {
    uint32_t cc[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) cc[it & 7] += key[it] >= t ? 1u : 0u;
    return __reduce_add_sync(0xffffffffu, ((cc[0] + cc[1]) + (cc[2] + cc[3])) + ((cc[4] + cc[5]) + (cc[6] + cc[7])));
  };
  uint32_t lo = __reduce_min_sync(0xffffffffu, kmin), hi = __reduce_max_sync(0xffffffffu, kmax);
  // largest t with count(key >= t) >= kb (the kb-th largest key), or any t that exactly
  // kb keys reach (then the keys >= t are the selection, ties included)
  while (lo < hi && kb > 0) {
    const uint32_t mid = lo + ((hi - lo + 1u) >> 1);
    const uint32_t c = count_ge(mid);
    if (c == static_cast<uint32_t>(kb)) {
      lo = mid;
      break;
    }
    if (c > static_cast<uint32_t>(kb)) lo = mid;
    else hi = mid - 1u;
  }
  const uint32_t kstar = lo;
  uint32_t n_gt = 0u;
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) n_gt += key[it] > kstar ? 1u : 0u;
  // copies of kstar to take, lowest index first
  const uint32_t remaining = kb > 0 ? static_cast<uint32_t>(kb) - __reduce_add_sync(0xffffffffu, n_gt) : 0u;
  const unsigned lt = (1u << lane) - 1u;
  uint32_t n_sel = 0u, eq_taken = 0u;
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    if (kb == 0) break;
    const int i = it * 32 + lane;
    const bool gt = key[it] > kstar;
    const bool eq = i < nv && key[it] == kstar;
    const unsigned eq_mask = __ballot_sync(0xffffffffu, eq);
    const bool take = gt || (eq && eq_taken + __popc(eq_mask & lt) < remaining);
    const unsigned take_mask = __ballot_sync(0xffffffffu, take);
    if (take) {
      const int64_t pos = ob + n_sel + __popc(take_mask & lt);
      if (p.values) p.values[pos] = key_float(key[it]);
      if (p.idx64) p.idx64[pos] = i + skip;
      if (p.idx32) p.idx32[pos] = i + skip;
    }
    n_sel += __popc(take_mask);
    eq_taken += __popc(eq_mask);
  }
  for (int64_t i = kb + lane; i < p.k; i += 32) {
    if (p.values) p.values[ob + i] = -INFINITY;
    if (p.idx64) p.idx64[ob + i] = -1;
    if (p.idx32) p.idx32[ob + i] = -1;
  }
}

extern "C" int linattn_row_topk(const float* scores, int64_t rows, int64_t n, int64_t row_stride, int64_t k,
                                int32_t causal, int64_t first_pos, int64_t key_block, int64_t period, int64_t skip,
                                int32_t sorted, float* values,
                                int64_t* idx_i64, int32_t* idx_i32, int64_t out_stride, int64_t out_batch_stride,
                                void* stream) {
  if (!scores) return set_error(LINATTN_EINVAL, "row_topk: scores is NULL");
  if (n < 1 || n >= (int64_t(1) << 31)) return set_error(LINATTN_EUNSUPPORTED, "row_topk: row length must be in [1, 2^31)");
  if (k < 1 || k > 4096) return set_error(LINATTN_EUNSUPPORTED, "row_topk: k must be in [1, 4096]");
  if (row_stride < n || out_stride < k || period < 1 || key_block < 1)
    return set_error(LINATTN_EINVAL, "row_topk: bad strides or key_block");
  if (rows == 0) return LINATTN_OK;
  if (rows > 0x7fffffff) return set_error(LINATTN_EUNSUPPORTED, "row_topk: too many rows");
  int64_t kp = 1;
  while (kp < k) kp <<= 1;
  RowTopkParams p;
  p.scores = scores; p.rows = rows; p.n = n; p.row_stride = row_stride; p.k = k; p.kpow2 = kp; p.causal = causal;
  p.first_pos = first_pos; p.kb = key_block; p.period = period; p.values = values; p.idx64 = idx_i64; p.idx32 = idx_i32;
  p.out_stride = out_stride; p.out_bstride = out_batch_stride; p.sorted = sorted ? 1 : 0; p.skip = skip < 0 ? 0 : skip;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(rows);
  cudaError_t e = cudaSuccess;
  if (!sorted && n <= 2048) {
    const unsigned wgrid = static_cast<unsigned>((rows + 7) / 8);
    if (n <= 512) row_topk_warp_kernel<16><<<wgrid, 256, 0, st>>>(p);
    else if (n <= 1024) row_topk_warp_kernel<32><<<wgrid, 256, 0, st>>>(p);
    else row_topk_warp_kernel<64><<<wgrid, 256, 0, st>>>(p);
    e = cudaGetLastError();
  } else if (n <= 32768) {
    const size_t smem = sorted ? static_cast<size_t>(2 * kp) * sizeof(uint32_t)
                               : static_cast<size_t>((n + 31) / 32) * sizeof(uint32_t);
    auto go = [&](auto kernel, int nt) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e == cudaSuccess) kernel<<<grid, nt, smem, st>>>(p);
      if (e == cudaSuccess) e = cudaGetLastError();
    };
    if (n <= 4096) go(row_topk_reg_kernel<512, 8>, 512);
    else if (n <= 8192) go(row_topk_reg_kernel<512, 16>, 512);
    else if (n <= 16384) go(row_topk_reg_kernel<1024, 16>, 1024);
    else go(row_topk_reg_kernel<1024, 32>, 1024);
  } else {
    const size_t smem = static_cast<size_t>(2 * kp) * sizeof(uint32_t);
    e = cudaFuncSetAttribute(row_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess) {
      row_topk_kernel<<<grid, 512, smem, st>>>(p);
      e = cudaGetLastError();
    }
  }
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "row_topk: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
