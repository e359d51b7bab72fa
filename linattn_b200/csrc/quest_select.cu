// Quest page scoring and top-k page selection with the GQA union.
//
// quest_scores_kernel: s[b,h,t,p] = sum_d max(q_d*min_d, q_d*max_d) in fp32.  Each
//   product of two 16-bit (or fp32) values is computed with one fma against the
//   bound picked by the sign of q_d, which equals max(q*min, q*max).  Bandwidth-bound:
//   every metadata row is one 16-byte load per lane, D/8 lanes per page; the partial
//   sums of the GQ query heads that share the metadata are reduced across the lanes
//   with a transposing butterfly (log2(D/8) shuffle rounds, halving the values
//   carried per round), so the metadata is read once for all heads of a group.
// page_topk_kernel: per (batch, head group, query) CTA, radix select (4 passes of 8
//   bits over order-preserving keys) of the k largest scores; ties at the k-th value
//   resolved by lowest page index; output sorted by (score desc, index asc); then the
//   union bitmap over the group's heads is compacted to an ascending page list.
#include "launchers.cuh"

namespace linattn {

// Reduce v[G] over aligned groups of LPR lanes.  On return, lane l (cl = l % LPR)
// holds sums for NV = max(1, G/LPR) heads: heads cl*NV + i when G >= LPR, else head
// cl / (LPR/G) (replicated over LPR/G lanes).
template <int G, int LPR>
__device__ __forceinline__ void transpose_reduce(float (&v)[G], int lane) {
  int n = G;
#pragma unroll
  for (int off = LPR / 2; off >= 1; off >>= 1) {
    if (n > 1) {
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < G / 2; ++i) {
        if (i < n / 2) {
          const float send = upper ? v[i] : v[i + n / 2];
          const float keep = upper ? v[i + n / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      n >>= 1;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
}

template <int G, int LPR>
struct ReduceLayout {
  static constexpr int NV = G >= LPR ? G / LPR : 1;
  static constexpr int REP = G >= LPR ? 1 : LPR / G;
  __device__ static int head(int cl, int i) { return G >= LPR ? cl * NV + i : cl / REP; }
  __device__ static bool writer(int cl) { return G >= LPR ? true : (cl % REP) == 0; }
};

struct ScoreParams {
  const void* q;
  int q_dtype;
  int64_t B, Hq, Tq;
  int64_t qs[4];
  linattn_meta_t meta;
  int64_t P, n_pages, offset;
  int sink_pages;
  const int32_t* n_pages_b;
  float* scores;
  int32_t* status;
  int pages_per_cta;
};

template <typename TM, int D, int GQ>
__global__ void __launch_bounds__(256) quest_scores_kernel(const ScoreParams p) {
  constexpr int LPR = D / 8;
  constexpr int PPW = 32 / LPR;
  using RL = ReduceLayout<GQ, LPR>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / LPR, cl = lane % LPR;
  const int64_t Hm = p.meta.n_heads;
  const int64_t hm = blockIdx.y % Hm, b = blockIdx.y / Hm;
  const int64_t Gq = p.Hq / Hm;
  const int64_t p_begin = static_cast<int64_t>(blockIdx.x) * p.pages_per_cta;
  const int64_t p_end = min(p_begin + p.pages_per_cta, p.n_pages);
  int64_t nb = p.n_pages_b ? static_cast<int64_t>(p.n_pages_b[b]) : p.n_pages;
  nb = min(nb, p.n_pages);
  const TM* mins = static_cast<const TM*>(p.meta.mins);
  const TM* maxs = static_cast<const TM*>(p.meta.maxs);
  const int64_t n_hc = (Gq + GQ - 1) / GQ;
  for (int64_t combo = 0; combo < p.Tq * n_hc; ++combo) {
    const int64_t t = combo / n_hc, hc = combo % n_hc;
    float qv[GQ][8];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
      const int64_t hg = hc * GQ + g;
      const int64_t h = hm * Gq + hg;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        qv[g][c] = hg < Gq ? load_any(p.q, b * p.qs[0] + h * p.qs[1] + t * p.qs[2] + (cl * 8 + c) * p.qs[3],
                                      p.q_dtype)
                           : 0.f;
    }
    const int64_t qpos = p.offset + t;
    const int64_t own = min(qpos / p.P, nb - 1);
    for (int64_t p0 = p_begin + warp * PPW; p0 < p_end; p0 += 8 * PPW) {
      const int64_t pg = p0 + sub;
      float acc[GQ];
#pragma unroll
      for (int g = 0; g < GQ; ++g) acc[g] = 0.f;
      bool live = pg < p_end && pg < nb && pg * p.P <= qpos;
      if (live) {
        int64_t phys = pg;
        if (p.meta.page_table) {
          phys = p.meta.page_table[b * p.meta.page_table_stride + pg];
          if (phys < 0 || phys >= p.meta.num_phys_pages) {
            report(p.status, LINATTN_DEV_BAD_ID);
            live = false;
          }
        }
        if (live) {
          const int64_t off = b * p.meta.stride_b + phys * p.meta.stride_page + hm * p.meta.stride_head + cl * 8;
          float mn[8], mx[8];
          load8(mins + off, mn);
          load8(maxs + off, mx);
#pragma unroll
          for (int g = 0; g < GQ; ++g)
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[g] = fmaf(qv[g][c], qv[g][c] >= 0.f ? mx[c] : mn[c], acc[g]);
        }
      }
      transpose_reduce<GQ, LPR>(acc, lane);
      if (pg < p_end && RL::writer(cl)) {
        const bool visible = pg < nb && pg * p.P <= qpos;
#pragma unroll
        for (int i = 0; i < RL::NV; ++i) {
          const int hg = static_cast<int>(hc * GQ) + RL::head(cl, i);
          if (hg >= Gq) continue;
          float s = live ? acc[i] : -INFINITY;
          if (!visible) s = -INFINITY;
          if (visible && (pg == own || pg < p.sink_pages)) s = INFINITY;
          const int64_t h = hm * Gq + hg;
          p.scores[((b * p.Hq + h) * p.Tq + t) * p.n_pages + pg] = s;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// top-k + union
// ---------------------------------------------------------------------------------

__global__ void __launch_bounds__(256) page_topk_kernel(const TopkParams p) {
  extern __shared__ uint32_t smem[];
  const int64_t n = p.n;
  const int64_t W = (n + 31) / 32;
  uint32_t* keys = smem;
  uint32_t* bitmap = keys + n;
  uint32_t* sel_idx = bitmap + W;
  uint32_t* sel_key = sel_idx + p.topk;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t scratch[9];
  __shared__ uint32_t sh_digit, sh_remaining, sh_count, sh_tokens;
  const int tid = threadIdx.x;
  const int64_t n_groups = p.Hq / p.group;
  const int64_t unit = blockIdx.x;
  const int64_t t = unit % p.Tq;
  const int64_t hg = (unit / p.Tq) % n_groups;
  const int64_t b = unit / (p.Tq * n_groups);
  int64_t nb = p.n_pages_b ? static_cast<int64_t>(p.n_pages_b[b]) : n;
  nb = lmax(0, min(nb, n));
  const int64_t kb = nb > 0 ? lmax(1, min(p.topk, nb)) : 0;
  const uint32_t neg_inf_key = float_key(-INFINITY);
  for (int64_t w = tid; w < W; w += 256) bitmap[w] = 0u;

  for (int64_t g = 0; g < p.group; ++g) {
    const int64_t h = hg * p.group + g;
    const int64_t row = (b * p.Hq + h) * p.Tq + t;
    const float* srow = p.scores + row * n;
    for (int64_t i = tid; i < nb; i += 256) keys[i] = float_key(srow[i]);
    __syncthreads();
    // ---- radix select: kstar = k-th largest key, need_eq = copies of kstar to take
    uint32_t prefix = 0u, mask = 0u, remaining = static_cast<uint32_t>(kb);
    if (kb > 0) {
      for (int shift = 24; shift >= 0; shift -= 8) {
        hist[tid] = 0u;
        __syncthreads();
        for (int64_t i = tid; i < nb; i += 256) {
          const uint32_t key = keys[i];
          if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        const uint32_t c = hist[255 - tid];
        const uint32_t above = block_exclusive_scan<256>(c, scratch, nullptr);
        if (above < remaining && above + c >= remaining) {
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
    // ---- gather: all keys > kstar, and the lowest-index need_eq keys == kstar
    if (tid == 0) sh_count = 0u;
    const int64_t chunk = (nb + 255) / 256;
    const int64_t i0 = lmin(nb, tid * chunk), i1 = lmin(nb, i0 + chunk);
    uint32_t n_eq = 0u;
    for (int64_t i = i0; i < i1; ++i) n_eq += keys[i] == kstar ? 1u : 0u;
    uint32_t eq_seen = block_exclusive_scan<256>(n_eq, scratch, nullptr);
    if (kb > 0) {
      for (int64_t i = i0; i < i1; ++i) {
        const uint32_t key = keys[i];
        bool take = key > kstar;
        if (key == kstar) {
          take = eq_seen < need_eq;
          ++eq_seen;
        }
        if (take) {
          const uint32_t pos = atomicAdd(&sh_count, 1u);
          if (pos < static_cast<uint32_t>(kb)) {
            sel_idx[pos] = static_cast<uint32_t>(i);
            sel_key[pos] = key;
          }
        }
      }
    }
    __syncthreads();
    // ---- rank sort (score desc, index asc) and write
    for (int64_t i = tid; i < kb; i += 256) {
      const uint32_t ki = sel_key[i], ii = sel_idx[i];
      int64_t rank = 0;
      for (int64_t j = 0; j < kb; ++j) {
        const uint32_t kj = sel_key[j], ij = sel_idx[j];
        rank += (kj > ki || (kj == ki && ij < ii)) ? 1 : 0;
      }
      if (p.ids64) p.ids64[row * p.topk + rank] = ii;
      if (p.ids32) p.ids32[row * p.topk + rank] = static_cast<int32_t>(ii);
      if (p.union_ids && ki > neg_inf_key) atomicOr(&bitmap[ii >> 5], 1u << (ii & 31u));
    }
    for (int64_t r = kb + tid; r < p.topk; r += 256) {
      if (p.ids64) p.ids64[row * p.topk + r] = -1;
      if (p.ids32) p.ids32[row * p.topk + r] = -1;
    }
    __syncthreads();
  }
  if (p.union_ids == nullptr) return;
  // ---- compact the union bitmap into an ascending page list
  const int64_t wpt = (W + 255) / 256;
  const int64_t w0 = lmin(W, tid * wpt), w1 = lmin(W, w0 + wpt);
  uint32_t cnt = 0u;
  for (int64_t w = w0; w < w1; ++w) cnt += __popc(bitmap[w]);
  if (tid == 0) sh_tokens = 0u;
  uint32_t total = 0u;
  uint32_t pos = block_exclusive_scan<256>(cnt, scratch, &total);
  const int64_t len = p.seq_lens ? static_cast<int64_t>(p.seq_lens[b]) : p.seq_len;
  const int64_t limit = min(len, p.offset + t + 1);
  const int64_t uoff = ((b * n_groups + hg) * p.Tq + t) * p.max_union;
  uint32_t tokens = 0u;
  for (int64_t w = w0; w < w1; ++w) {
    uint32_t bits = bitmap[w];
    while (bits) {
      const int bit = __ffs(bits) - 1;
      bits &= bits - 1u;
      const int64_t pg = w * 32 + bit;
      if (pos < p.max_union) p.union_ids[uoff + pos] = static_cast<int32_t>(pg);
      ++pos;
      const int64_t nv = lmin(p.P, lmax(0, limit - pg * p.P));
      tokens += static_cast<uint32_t>(nv);
    }
  }
  for (int64_t j = total + tid; j < p.max_union; j += 256) p.union_ids[uoff + j] = -1;
  if (p.union_tokens) atomicAdd(&sh_tokens, tokens);
  __syncthreads();
  if (tid == 0) {
    const int64_t u = (b * n_groups + hg) * p.Tq + t;
    if (total > p.max_union) report(p.status, LINATTN_DEV_OVERFLOW);
    p.union_count[u] = static_cast<int32_t>(lmin(total, p.max_union));
    if (p.union_tokens) p.union_tokens[u] = static_cast<int32_t>(sh_tokens);
  }
}

// ---------------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------------
template <typename TM, int D>
static cudaError_t launch_scores_d(const ScoreParams& p, int64_t Gq, dim3 grid, cudaStream_t stream) {
  if (Gq >= 8) quest_scores_kernel<TM, D, 8><<<grid, 256, 0, stream>>>(p);
  else if (Gq >= 4) quest_scores_kernel<TM, D, 4><<<grid, 256, 0, stream>>>(p);
  else if (Gq >= 2) quest_scores_kernel<TM, D, 2><<<grid, 256, 0, stream>>>(p);
  else quest_scores_kernel<TM, D, 1><<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

template <typename TM>
static cudaError_t launch_scores_t(const ScoreParams& p, int64_t D, int64_t Gq, dim3 grid, cudaStream_t stream) {
  switch (D) {
    case 8: return launch_scores_d<TM, 8>(p, Gq, grid, stream);
    case 16: return launch_scores_d<TM, 16>(p, Gq, grid, stream);
    case 32: return launch_scores_d<TM, 32>(p, Gq, grid, stream);
    case 64: return launch_scores_d<TM, 64>(p, Gq, grid, stream);
    case 128: return launch_scores_d<TM, 128>(p, Gq, grid, stream);
    case 256: return launch_scores_d<TM, 256>(p, Gq, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_quest_scores(const void* q, int q_dtype, int64_t B, int64_t Hq, int64_t Tq, int64_t D,
                                const int64_t* qs, const linattn_meta_t& meta, int64_t P, int64_t n_pages,
                                int64_t offset, int sink_pages, const int32_t* n_pages_b, float* scores,
                                int32_t* status, cudaStream_t stream) {
  ScoreParams p;
  p.q = q; p.q_dtype = q_dtype; p.B = B; p.Hq = Hq; p.Tq = Tq;
  for (int i = 0; i < 4; ++i) p.qs[i] = qs[i];
  p.meta = meta; p.P = P; p.n_pages = n_pages; p.offset = offset; p.sink_pages = sink_pages;
  p.n_pages_b = n_pages_b; p.scores = scores; p.status = status;
  p.pages_per_cta = 64;
  const int64_t chunks = (n_pages + p.pages_per_cta - 1) / p.pages_per_cta;
  const int64_t Gq = Hq / meta.n_heads;
  if (chunks == 0 || B * meta.n_heads == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(B * meta.n_heads));
  switch (meta.dtype) {
    case LINATTN_F32: return launch_scores_t<float>(p, D, Gq, grid, stream);
    case LINATTN_F16: return launch_scores_t<__half>(p, D, Gq, grid, stream);
    case LINATTN_BF16: return launch_scores_t<__nv_bfloat16>(p, D, Gq, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

size_t page_topk_smem_bytes(int64_t n, int64_t topk) {
  return static_cast<size_t>(n + (n + 31) / 32 + 2 * topk) * sizeof(uint32_t);
}

cudaError_t launch_page_topk(const TopkParams& p, cudaStream_t stream) {
  const size_t smem = page_topk_smem_bytes(p.n, p.topk);
  static bool configured = false;  // per process; the attribute is per function
  if (!configured || smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(page_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem < 48 * 1024 ? 48 * 1024 : smem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int64_t units = p.B * (p.Hq / p.group) * p.Tq;
  if (units == 0) return cudaSuccess;
  page_topk_kernel<<<static_cast<unsigned>(units), 256, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace linattn
