// Sequence-sharded (and chunked) Quest decode: the global top-k of the candidates of
// all shards / chunks and the GQA union of the selected pages one shard owns.
//
// Each of R shards proposes, per (sequence, query head), its local top-k pages with
// their scores (global page ids); after an all-gather every shard holds all R * K
// candidates (rank-major).  One CTA per (sequence, kv head) ranks each head's
// candidates by a 64-bit key (order-preserving score, then the bitwise complement of
// the page id, so equal scores go to the lowest page: the single-cache top-k's
// tie-break); each block of K arrives sorted by that key (the candidates kernel
// writes them so) and the blocks hold disjoint pages, so a k-way merge of the block
// heads yields the global order.  The first k go
// to `sel`, and those in this shard's range [page_lo_b, page_hi_b) to a bitmap that
// compacts to the ascending local page list the attention reads.  With the union
// left out (union_ids NULL) the kernel is a shard's pre-merge of its own chunks: its
// top-k ids and scores, in key order, form the one block of K the shard exchanges.
// No counterpart in the reference (it
// never shards the KV sequence); the selection equals page_select_torch's top-k
// (src/linattn/kernels/triton/quest_pages.py:57-78) over the union of the shards' pages
// whenever each shard's k candidates include its share of the global top-k, which
// holds because a page in the global top-k is in its own shard's top-k.
#include <cstdio>

#include "launchers.cuh"

namespace linattn {

namespace {

struct ShardMergeParams {
  const float* scores;   // (R, B, Hq, K)
  const int32_t* ids;    // (R, B, Hq, K) global page ids, -1 = none
  int64_t R, B, Hq, K, rs, topk, G;  // rs: elements between shards' blocks
  const int32_t* page_lo;  // (B) first global page of this shard
  const int32_t* page_hi;  // (B) one past its last
  int64_t max_local;       // local pages (bitmap size)
  int32_t* sel;            // (B, Hq, topk) global ids, (score desc, id asc), -1 padded; or NULL
  float* sel_scores;       // (B, Hq, topk) their scores (-inf past the last), or NULL
  int32_t* union_ids;      // (B, Hkv, max_union) local ids ascending, -1 padded; NULL: no union
  int32_t* union_count;    // (B, Hkv)
  int64_t max_union;
  const int32_t* seq_lens;  // (B) tokens of each sequence (for union_tokens)
  int64_t P;
  int32_t* union_tokens;    // (B, Hkv) tokens of the union pages, or NULL
};

__device__ __forceinline__ unsigned long long cand_key(const ShardMergeParams& p, int64_t off) {
  // both loads issued together (the score is read even for an empty slot)
  const int32_t id = __ldcg(p.ids + off);
  const float sc = __ldcg(p.scores + off);
  return id >= 0 ? (static_cast<unsigned long long>(float_key(sc)) << 32) |
                       static_cast<unsigned long long>(~static_cast<uint32_t>(id))
                 : 0ull;  // empty slots rank last
}

// Merge-path tree over the R sorted blocks of one head (topk <= 256), one warp: level
// by level, blocks j and j + s (s = 1, 2, 4, ...) merge into the top min(topk, La + Lb)
// keys at block j's place.  Output o of a merge is found on its own: i = the number of
// A keys among the first o outputs is the first mid in [max(0, o - Lb), min(o, La)]
// with A[mid] < B[o - 1 - mid] (A wins ties, which only empty slots have: keys are
// unique), and output o = max(A[i], B[o - i]).  A lane computes outputs lane, lane +
// 32, ... into registers; they overwrite the blocks after the whole merge has read
// them.  Returns the merged length; block 0 then holds the keys in order.
__device__ __forceinline__ int tree_merge_blocks(unsigned long long* kw, int R, int K, int topk, int lane) {
  const int L0 = K < topk ? K : topk;
  // at level s, block j (a multiple of 2s) holds the merge of original blocks j ..
  // min(R, j + s) - 1, truncated to topk
  for (int s = 1; s < R; s <<= 1) {
    for (int j = 0; j + s < R; j += 2 * s) {
      const int na = s, nb = (R - j - s) < s ? (R - j - s) : s;
      const int La = na * L0 < topk ? na * L0 : topk, Lb = nb * L0 < topk ? nb * L0 : topk;
      const int Lo = La + Lb < topk ? La + Lb : topk;
      const unsigned long long* A = kw + j * K;
      const unsigned long long* B = kw + (j + s) * K;
      unsigned long long out[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int o = lane + 32 * c;
        out[c] = 0ull;
        if (o < Lo) {
          int lo = o - Lb > 0 ? o - Lb : 0, hi = o < La ? o : La;
          while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (A[mid] >= B[o - 1 - mid]) lo = mid + 1;
            else hi = mid;
          }
          const unsigned long long a = lo < La ? A[lo] : 0ull, b = o - lo < Lb ? B[o - lo] : 0ull;
          out[c] = a >= b ? a : b;
        }
      }
      __syncwarp();
      unsigned long long* dst = kw + j * K;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        if (lane + 32 * c < Lo) dst[lane + 32 * c] = out[c];
      __syncwarp();
    }
  }
  return R * L0 < topk ? R * L0 : topk;
}

// The keys of `hpw` heads at a time are staged in shared memory by all threads
// (eight loads in flight per thread: the staging is latency-bound otherwise); then one
// warp per head merges the R sorted blocks: up to 4 blocks by the merge-path tree, more
// (R <= 64, two per lane) step by step: each step the warp takes the largest block head
// (two 32-bit warp max-reductions over the unique 64-bit keys, the heads and the keys
// after them held in registers) and that block advances, so the top-k come out in order
// after k steps.
template <bool TREE>
__global__ void __launch_bounds__(256) shard_merge_kernel(const ShardMergeParams p, int hpw) {
  extern __shared__ unsigned long long msm[];
  const int64_t n = p.R * p.K;
  unsigned long long* keys = msm;                                   // [hpw][R * K]
  uint32_t* bits = reinterpret_cast<uint32_t*>(keys + hpw * n);     // [(max_local + 31) / 32]
  __shared__ uint32_t scratch[256 / 32 + 1];
  __shared__ uint32_t sh_tokens;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) sh_tokens = 0u;
  const int64_t bk = blockIdx.x;  // (b, kv head)
  const int64_t Hkv = p.Hq / p.G;
  const int64_t kvh = bk % Hkv, b = bk / Hkv;
  const int64_t lo = p.page_lo[b], hi = p.page_hi[b];
  const int64_t nwords = (p.max_local + 31) / 32;
  if (p.union_ids)
    for (int64_t i = tid; i < nwords; i += 256) bits[i] = 0u;
  const int K = static_cast<int>(p.K);
  for (int64_t g0 = 0; g0 < p.G; g0 += hpw) {
    const int ng = static_cast<int>(lmin(hpw, p.G - g0));
    __syncthreads();
    // ---- stage: eight candidates in flight per thread; 32-bit index arithmetic
    const int total = ng * static_cast<int>(n);
    const int n32 = static_cast<int>(n);
    const bool pow2 = (K & (K - 1)) == 0;
    const int k_shift = __ffs(K) - 1;
    for (int i0 = tid; i0 < total; i0 += 8 * 256) {
      unsigned long long kx[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * 256;
        kx[u] = 0ull;
        if (i < total) {
          const int g = i / n32, j = i - g * n32;
          const int r = pow2 ? j >> k_shift : j / K, e = j - r * K;
          kx[u] = cand_key(p, r * p.rs + (b * p.Hq + kvh * p.G + g0 + g) * p.K + e);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (i0 + u * 256 < total) keys[i0 + u * 256] = kx[u];
    }
    __syncthreads();
    if (warp >= ng) continue;
    // ---- warp `warp` merges head g0 + warp.  A lane holds the heads of its blocks
    // (lane, lane + 32) and the key after each in registers: a step is the two
    // reductions and the winner's advance, whose next load is off the step's chain.
    const int64_t h = kvh * p.G + g0 + warp;
    const unsigned long long* kw = keys + warp * n;
    const int R32 = static_cast<int>(p.R);
    const bool has0 = lane < R32, has1 = lane + 32 < R32;
    const unsigned long long* b0 = kw + (has0 ? lane * K : 0);
    const unsigned long long* b1 = kw + (has1 ? (lane + 32) * K : 0);
    int p0 = 0, p1 = 0;
    unsigned long long h0 = has0 ? b0[0] : 0ull, h1 = has1 ? b1[0] : 0ull;
    unsigned long long n0 = has0 && K > 1 ? b0[1] : 0ull, n1 = has1 && K > 1 ? b1[1] : 0ull;
    const int topk = static_cast<int>(p.topk);
    int32_t* sel_row = p.sel ? p.sel + (b * p.Hq + h) * p.topk : nullptr;
    float* sc_row = p.sel_scores ? p.sel_scores + (b * p.Hq + h) * p.topk : nullptr;
    int i = 0;
    // TREE (up to 4 blocks, topk <= 256): block 0 ends up holding the top keys in order
    if constexpr (TREE) {
      unsigned long long* kwm = keys + warp * n;
      const int m = tree_merge_blocks(kwm, R32, K, topk, lane);
      int valid = 0;  // keys before the first empty slot
      for (int o = lane; o < m; o += 32) {
        const unsigned long long key = kwm[o];
        valid += key != 0ull;
        if (key == 0ull) continue;
        const int32_t id = static_cast<int32_t>(~static_cast<uint32_t>(key));
        if (sel_row) sel_row[o] = id;
        if (sc_row) sc_row[o] = key_float(static_cast<uint32_t>(key >> 32));
        if (p.union_ids && id >= lo && id < hi && id - lo < p.max_local)
          atomicOr(&bits[(id - lo) >> 5], 1u << ((id - lo) & 31));
      }
      i = __reduce_add_sync(0xffffffffu, static_cast<uint32_t>(valid));
    }
    for (; i < topk && !TREE; ++i) {
      const unsigned long long mine = h0 > h1 ? h0 : h1;
      const uint32_t khi = static_cast<uint32_t>(mine >> 32), klo = static_cast<uint32_t>(mine);
      const uint32_t hmax = __reduce_max_sync(0xffffffffu, khi);
      const uint32_t lmax = __reduce_max_sync(0xffffffffu, khi == hmax ? klo : 0u);
      if (hmax == 0u && lmax == 0u) break;  // every block exhausted (warp-uniform)
      if (khi == hmax && klo == lmax) {     // the unique winner
        const int32_t id = static_cast<int32_t>(~lmax);
        if (sel_row) sel_row[i] = id;
        if (sc_row) sc_row[i] = key_float(hmax);
        if (p.union_ids && id >= lo && id < hi && id - lo < p.max_local)
          atomicOr(&bits[(id - lo) >> 5], 1u << ((id - lo) & 31));
        if (h0 > h1) {
          h0 = n0;
          ++p0;
          n0 = p0 + 1 < K ? b0[p0 + 1] : 0ull;
        } else {
          h1 = n1;
          ++p1;
          n1 = p1 + 1 < K ? b1[p1 + 1] : 0ull;
        }
      }
    }
    for (int64_t r = i + lane; r < p.topk; r += 32) {
      if (p.sel) p.sel[(b * p.Hq + h) * p.topk + r] = -1;
      if (p.sel_scores) p.sel_scores[(b * p.Hq + h) * p.topk + r] = -INFINITY;
    }
  }
  __syncthreads();
  if (p.union_ids == nullptr) return;  // top-k only (a shard's pre-merge of its own chunks)
  // ascending local union: popcount scan over the bitmap words
  const int64_t per = (nwords + 255) / 256;
  const int64_t w0 = lmin(nwords, tid * per), w1 = lmin(nwords, w0 + per);
  uint32_t cnt = 0u;
  for (int64_t w = w0; w < w1; ++w) cnt += __popc(bits[w]);
  uint32_t total = 0u;
  uint32_t pos = block_exclusive_scan<256>(cnt, scratch, &total);
  int32_t* out = p.union_ids + bk * p.max_union;
  const int64_t len = p.seq_lens ? static_cast<int64_t>(p.seq_lens[b]) : 0;
  uint32_t tokens = 0u;
  for (int64_t w = w0; w < w1; ++w) {
    uint32_t m = bits[w];
    while (m) {
      const int bit = __ffs(m) - 1;
      m &= m - 1u;
      if (pos < p.max_union) out[pos] = static_cast<int32_t>(w * 32 + bit);
      ++pos;
      tokens += static_cast<uint32_t>(lmin(p.P, lmax(0, len - (lo + w * 32 + bit) * p.P)));
    }
  }
  for (int64_t i = static_cast<int64_t>(total) + tid; i < p.max_union; i += 256) out[i] = -1;
  if (p.union_tokens) atomicAdd(&sh_tokens, tokens);
  __syncthreads();
  if (tid == 0) {
    p.union_count[bk] = static_cast<int32_t>(total < p.max_union ? total : p.max_union);
    if (p.union_tokens) p.union_tokens[bk] = static_cast<int32_t>(sh_tokens);
  }
}

}  // namespace

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_shard_merge(const float* scores, const int32_t* ids, int64_t R, int64_t B, int64_t Hq,
                                   int64_t K, int64_t rank_stride, int64_t topk, int64_t n_kv_heads, const int32_t* page_lo,
                                   const int32_t* page_hi, int64_t max_local, int32_t* sel, float* sel_scores,
                                   int32_t* union_ids,
                                   int32_t* union_count, int64_t max_union, const int32_t* seq_lens,
                                   int64_t page_size, int32_t* union_tokens, void* stream) {
  if (!scores || !ids || !page_lo || !page_hi || (union_ids && !union_count) || (!union_ids && !sel))
    return set_error(LINATTN_EINVAL, "shard_merge: NULL pointer");
  if (R < 1 || K < 1 || topk < 1 || n_kv_heads < 1 || Hq % n_kv_heads || max_local < 1 ||
      (union_ids && max_union < 1))
    return set_error(LINATTN_EINVAL, "shard_merge: bad sizes");
  if (rank_stride != 0 && rank_stride < B * Hq * K) return set_error(LINATTN_EINVAL, "shard_merge: rank_stride");
  if (R * K > 4096 || R > 64 || max_local > (int64_t(1) << 20))
    return set_error(LINATTN_EUNSUPPORTED, "shard_merge: at most 64 blocks, 4096 candidates and 2^20 local pages");
  if (B * n_kv_heads == 0) return LINATTN_OK;
  ShardMergeParams p;
  p.scores = scores; p.ids = ids; p.R = R; p.B = B; p.Hq = Hq; p.K = K;
  p.rs = rank_stride ? rank_stride : B * Hq * K; p.topk = topk; p.G = Hq / n_kv_heads;
  p.page_lo = page_lo; p.page_hi = page_hi; p.max_local = max_local; p.sel = sel; p.sel_scores = sel_scores;
  p.union_ids = union_ids; p.union_count = union_count; p.max_union = max_union;
  if (union_tokens && (!seq_lens || page_size < 1))
    return set_error(LINATTN_EINVAL, "shard_merge: union_tokens needs seq_lens and page_size");
  p.seq_lens = seq_lens; p.P = page_size; p.union_tokens = union_tokens;
  const size_t bits_bytes = union_ids ? static_cast<size_t>((max_local + 31) / 32) * 4 : 0;
  const size_t head_bytes = static_cast<size_t>(R * K) * 8;
  // as many heads per pass as 160 KiB hold (at most 8: the per-head counters)
  const int hpw = static_cast<int>(lmax(1, lmin(lmin(8, p.G), static_cast<int64_t>((160 * 1024) / head_bytes))));
  const size_t smem = hpw * head_bytes + bits_bytes;
  if (smem > 200 * 1024) return set_error(LINATTN_EUNSUPPORTED, "shard_merge: shared memory");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // few blocks: the merge-path tree (log2 R levels of parallel outputs); more blocks:
  // the step-by-step k-way merge (the tree's work grows as R x topk: config 5's 8 ranks
  // x 64 keys take the k-way merge 35 us, the tree as long; 16 chunks 54 us against 65)
  const bool tree = topk <= 256 && R <= 4;
  auto kern = tree ? shard_merge_kernel<true> : shard_merge_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) {
    kern<<<static_cast<unsigned>(B * n_kv_heads), 256, smem, st>>>(p, hpw);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "shard_merge: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}

