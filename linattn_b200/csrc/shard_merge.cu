// Sequence-sharded (and chunked) Quest decode: the global top-k of the candidates of
// all shards / chunks and the GQA union of the selected pages one shard owns.
//
// Each of R shards proposes, per (sequence, query head), its local top-k pages with
// their scores (global page ids); after an all-gather every shard holds all R * K
// candidates (rank-major).  One CTA per (sequence, kv head) ranks each head's
// candidates by a 64-bit key (order-preserving score, then the bitwise complement of
// the page id, so equal scores go to the lowest page: the single-cache top-k's
// tie-break), bitonic-sorted in shared memory, takes the first k, and marks the pages
// of this shard's range [page_lo_b, page_hi_b) in a bitmap; the bitmap compacts to the
// ascending local page list the attention reads.  No counterpart in the reference (it
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
  int64_t R, B, Hq, K, rs, topk, G, np2;  // rs: elements between shards' blocks
  const int32_t* page_lo;  // (B) first global page of this shard
  const int32_t* page_hi;  // (B) one past its last
  int64_t max_local;       // local pages (bitmap size)
  int32_t* sel;            // (B, Hq, topk) global ids, (score desc, id asc), -1 padded; or NULL
  int32_t* union_ids;      // (B, Hkv, max_union) local ids ascending, -1 padded
  int32_t* union_count;    // (B, Hkv)
  int64_t max_union;
  const int32_t* seq_lens;  // (B) tokens of each sequence (for union_tokens)
  int64_t P;
  int32_t* union_tokens;    // (B, Hkv) tokens of the union pages, or NULL
};

__global__ void __launch_bounds__(256) shard_merge_kernel(const ShardMergeParams p) {
  extern __shared__ unsigned long long msm[];
  unsigned long long* keys = msm;                                    // [np2]
  uint32_t* bits = reinterpret_cast<uint32_t*>(keys + p.np2);        // [(max_local + 31) / 32]
  __shared__ uint32_t scratch[256 / 32 + 1];
  __shared__ uint32_t sh_tokens;
  const int tid = threadIdx.x;
  if (tid == 0) sh_tokens = 0u;
  const int64_t bk = blockIdx.x;  // (b, kv head)
  const int64_t Hkv = p.Hq / p.G;
  const int64_t kvh = bk % Hkv, b = bk / Hkv;
  const int64_t lo = p.page_lo[b], hi = p.page_hi[b];
  const int64_t nwords = (p.max_local + 31) / 32;
  for (int64_t i = tid; i < nwords; i += 256) bits[i] = 0u;
  const int64_t n = p.R * p.K;
  for (int64_t g = 0; g < p.G; ++g) {
    const int64_t h = kvh * p.G + g;
    __syncthreads();
    for (int64_t i = tid; i < p.np2; i += 256) {
      unsigned long long key = 0ull;  // padding and empty slots sort last
      if (i < n) {
        const int64_t r = i / p.K, e = i % p.K;
        const int64_t off = r * p.rs + (b * p.Hq + h) * p.K + e;
        const int32_t id = p.ids[off];
        if (id >= 0)
          key = (static_cast<unsigned long long>(float_key(p.scores[off])) << 32) |
                static_cast<unsigned long long>(~static_cast<uint32_t>(id));
      }
      keys[i] = key;
    }
    __syncthreads();
    // bitonic sort, descending
    for (int64_t size = 2; size <= p.np2; size <<= 1) {
      for (int64_t stride = size >> 1; stride > 0; stride >>= 1) {
        for (int64_t i = tid; i < p.np2; i += 256) {
          const int64_t j = i ^ stride;
          if (j > i) {
            const bool desc = (i & size) == 0;
            const unsigned long long a = keys[i], c = keys[j];
            if ((a > c) != desc && a != c) {
              keys[i] = c;
              keys[j] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    for (int64_t i = tid; i < p.topk; i += 256) {
      const unsigned long long key = i < n ? keys[i] : 0ull;
      const int32_t id = key ? static_cast<int32_t>(~static_cast<uint32_t>(key & 0xffffffffull)) : -1;
      if (p.sel) p.sel[(b * p.Hq + h) * p.topk + i] = id;
      if (id >= lo && id < hi && id - lo < p.max_local) atomicOr(&bits[(id - lo) >> 5], 1u << ((id - lo) & 31));
    }
  }
  __syncthreads();
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
                                   const int32_t* page_hi, int64_t max_local, int32_t* sel, int32_t* union_ids,
                                   int32_t* union_count, int64_t max_union, const int32_t* seq_lens,
                                   int64_t page_size, int32_t* union_tokens, void* stream) {
  if (!scores || !ids || !page_lo || !page_hi || !union_ids || !union_count)
    return set_error(LINATTN_EINVAL, "shard_merge: NULL pointer");
  if (R < 1 || K < 1 || topk < 1 || n_kv_heads < 1 || Hq % n_kv_heads || max_local < 1 || max_union < 1)
    return set_error(LINATTN_EINVAL, "shard_merge: bad sizes");
  if (rank_stride != 0 && rank_stride < B * Hq * K) return set_error(LINATTN_EINVAL, "shard_merge: rank_stride");
  int64_t np2 = 1;
  while (np2 < R * K) np2 <<= 1;
  if (np2 > 4096 || max_local > (int64_t(1) << 20))
    return set_error(LINATTN_EUNSUPPORTED, "shard_merge: at most 4096 candidates and 2^20 local pages");
  if (B * n_kv_heads == 0) return LINATTN_OK;
  ShardMergeParams p;
  p.scores = scores; p.ids = ids; p.R = R; p.B = B; p.Hq = Hq; p.K = K;
  p.rs = rank_stride ? rank_stride : B * Hq * K; p.topk = topk; p.G = Hq / n_kv_heads;
  p.np2 = np2; p.page_lo = page_lo; p.page_hi = page_hi; p.max_local = max_local; p.sel = sel;
  p.union_ids = union_ids; p.union_count = union_count; p.max_union = max_union;
  if (union_tokens && (!seq_lens || page_size < 1))
    return set_error(LINATTN_EINVAL, "shard_merge: union_tokens needs seq_lens and page_size");
  p.seq_lens = seq_lens; p.P = page_size; p.union_tokens = union_tokens;
  const size_t smem = static_cast<size_t>(np2) * 8 + static_cast<size_t>((max_local + 31) / 32) * 4;
  if (smem > 200 * 1024) return set_error(LINATTN_EUNSUPPORTED, "shard_merge: shared memory");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaFuncSetAttribute(shard_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e == cudaSuccess) {
    shard_merge_kernel<<<static_cast<unsigned>(B * n_kv_heads), 256, smem, st>>>(p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "shard_merge: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}

