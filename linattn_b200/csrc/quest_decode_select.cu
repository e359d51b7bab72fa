// Fused Quest selection for decode: page scores -> top-k per query head -> GQA union,
// one CTA per (sequence, kv head), no intermediate buffer in HBM.
//
// Metadata layout: [B, H_kv, max_pages, 2, D] (logical page order per sequence and
// kv head, min row then max row), so one (sequence, kv head) is a single contiguous
// stream of n_pages * 2 * D elements.  Thread 0 streams it through an NSTG-deep ring
// of CH-page chunks with 1-D TMA bulk copies (no tensor map, no multicast); all warps
// score each chunk for the G query heads of the group (q in registers, D/8 lanes per
// page, transposing butterfly over the head partials) into shared memory.  Then warp
// g runs a radix select (4 x 8-bit passes over order-preserving keys, warp-private
// histogram) for head g, takes ties at the k-th value by lowest page index, sorts its
// k pages by (score desc, index asc), writes them and sets the group's union bitmap;
// the CTA compacts the bitmap into an ascending page list.
//
// Decode semantics: the query sits at position seq_len_b - 1, so every page below
// n_pages_b is visible, the own page is n_pages_b - 1, and it and the first
// `sink_pages` pages are forced to +inf (quest_pages.py:67-75 at T_q == 1).
//
// Candidates form (linattn_quest_decode_candidates): the page axis is cut into chunks
// of `chunk` pages, one CTA per (sequence, kv head, chunk); each CTA writes every
// head's top-k of its chunk as (score, page + page_base[b]) candidates sorted by
// (score desc, page asc), and the global top-k + GQA union is taken by the shard
// merge kernel over all chunks (and, in the sequence-sharded decode, all ranks).  A
// page of the global top-k is in its chunk's top-k, so the result is the same
// selection; long sequences get many CTAs and short per-CTA selections.
//
// Histogram passes aggregate equal bins across the warp (match.any) before the shared
// memory atomic, so keys that share a digit (most keys share the top byte) cost one
// atomic per warp instead of 32 serialised ones.
#include <cstdio>

#include "launchers.cuh"

namespace linattn {

namespace {

constexpr int CH = 32;    // pages per ring stage

template <int G, int LPR>
__device__ __forceinline__ void group_reduce(float (&v)[G], int lane) {
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

struct DecodeSelectParams {
  const void* q;
  int q_dtype;
  int64_t B, Hq, Hkv;
  int64_t qs[4];
  const void* meta;
  int64_t max_pages;
  const int32_t* n_pages_b;
  const int32_t* seq_lens;
  int64_t P;
  int topk;
  int sink_pages;
  int force_last;  // the own (last visible) page is forced in
  int32_t* ids;      // (B, Hq, topk)
  float* scores;     // optional (B, Hq, max_pages)
  int32_t* union_ids;
  int32_t* union_count;
  int64_t max_union;
  int32_t* union_tokens;
  int32_t* status;
  int64_t chunk;              // pages per CTA (blockIdx.y = chunk index)
  float* cand_scores;         // candidates form: (n_chunks, B, Hq, topk), chunk stride cand_stride
  int32_t* cand_ids;
  int64_t cand_stride;
  const int32_t* page_base;   // per sequence, added to candidate page ids (NULL = 0)
};

}  // namespace

// ---------------------------------------------------------------------------------
// per-head selection and output (shared by both scoring paths)
// ---------------------------------------------------------------------------------
// Warp g (< G) selects for query head kvh*G + g over the chunk's scores sc[g][0, nb):
// the k-th largest order-preserving key (a binary search over the key range with
// warp-wide counts of register-held keys for nb <= 2048; else a radix select, 4 x
// 8-bit passes over a warp-private histogram with match.any-aggregated atomics),
// every key above it plus the lowest-index copies of it, ranked by (score desc,
// index asc).  Writes the ids (and marks the union bitmap) or, in the candidates
// form, (score, page) candidates.
// Ranks the kb taken entries (sel_idx / sel_key) by (score desc, index asc) and
// writes the ids (marking the union bitmap) or the candidates.
// The entries of two lists (A: na entries, B: nb_ entries; B may be empty) ranked
// together by (score desc, index asc); the first kb by rank are written as ids (and
// marked in the union bitmap) or, in the candidates form, as (score, page) candidates.
__device__ __forceinline__ void write_selection2(const DecodeSelectParams& p, const float* srow,
                                                 const uint32_t* idx_a, const uint32_t* key_a, int64_t na,
                                                 const uint32_t* idx_b, const uint32_t* key_b, int64_t nb_,
                                                 int64_t kb, uint32_t* bitmap, int64_t pg0, int64_t b, int64_t h,
                                                 int lane) {
  const uint32_t neg_inf_key = float_key(-INFINITY);
  const int64_t n = na + nb_;
  const bool cand = p.cand_scores != nullptr;
  const int64_t off = cand ? static_cast<int64_t>(blockIdx.y) * p.cand_stride + (b * p.Hq + h) * p.topk
                           : (b * p.Hq + h) * p.topk;
  const int64_t id0 = pg0 + (p.page_base ? static_cast<int64_t>(p.page_base[b]) : 0);
  for (int64_t i = lane; i < n; i += 32) {
    const uint32_t ki = i < na ? key_a[i] : key_b[i - na], ii = i < na ? idx_a[i] : idx_b[i - na];
    // unrolled so that eight independent shared loads are in flight per step
    int rank = 0;
    const int na32 = static_cast<int>(na), nb32 = static_cast<int>(nb_);
#pragma unroll 8
    for (int j = 0; j < na32; ++j) {
      const uint32_t kj = key_a[j], ij = idx_a[j];
      rank += (kj > ki || (kj == ki && ij < ii)) ? 1 : 0;
    }
#pragma unroll 8
    for (int j = 0; j < nb32; ++j) {
      const uint32_t kj = key_b[j], ij = idx_b[j];
      rank += (kj > ki || (kj == ki && ij < ii)) ? 1 : 0;
    }
    if (rank >= kb) continue;
    if (cand) {
      p.cand_scores[off + rank] = srow[ii];
      p.cand_ids[off + rank] = static_cast<int32_t>(id0 + ii);
    } else {
      p.ids[off + rank] = static_cast<int32_t>(ii);
      if (ki > neg_inf_key) atomicOr(&bitmap[ii >> 5], 1u << (ii & 31u));
    }
  }
  for (int64_t r = kb + lane; r < p.topk; r += 32) {
    if (cand) {
      p.cand_scores[off + r] = -INFINITY;
      p.cand_ids[off + r] = -1;
    } else {
      p.ids[off + r] = -1;
    }
  }
}

__device__ __forceinline__ void write_selection(const DecodeSelectParams& p, const float* srow,
                                                const uint32_t* sel_idx, const uint32_t* sel_key, int64_t kb,
                                                uint32_t* bitmap, int64_t pg0, int64_t b, int64_t h, int lane) {
  write_selection2(p, srow, sel_idx, sel_key, kb, nullptr, nullptr, 0, kb, bitmap, pg0, b, h, lane);
}

// Register form for nb <= 32 * ITEMS: lane holds keys i = j * 32 + lane; the k-th
// largest key is found by a binary search over the key range with warp-wide counts
// (no shared-memory histogram, no atomics), then the same gather and ranking.
// With idx_off >= 0 the selection is only gathered (its indices shifted by idx_off,
// in this warp's slot of `sel`) for a merge with another warp's; otherwise written.
template <int ITEMS>
__device__ __forceinline__ void select_head_reg(const DecodeSelectParams& p, const float* srow, uint32_t* sel,
                                                uint32_t* bitmap, int64_t nb, int64_t pg0, int64_t b, int64_t h,
                                                int warp, int lane, int64_t idx_off = -1) {
  const int64_t kb = nb > 0 ? lmax(1, lmin(p.topk, nb)) : 0;
  uint32_t* sel_idx = sel + warp * 2 * p.topk;
  uint32_t* sel_key = sel_idx + p.topk;
  const uint32_t shift = idx_off > 0 ? static_cast<uint32_t>(idx_off) : 0u;
  uint32_t key[ITEMS];
  uint32_t kmax = 0u, kmin = 0xffffffffu;
#pragma unroll
  for (int j = 0; j < ITEMS; ++j) {
    const int64_t i = j * 32 + lane;
    key[j] = i < nb ? float_key(srow[i]) : 0u;  // real keys are > 0 (float_key(-inf) > 0)
    if (i < nb) {
      kmax = key[j] > kmax ? key[j] : kmax;
      kmin = key[j] < kmin ? key[j] : kmin;
    }
  }
  uint32_t lo = __reduce_min_sync(0xffffffffu, kmin), hi = __reduce_max_sync(0xffffffffu, kmax);
  // count(key >= t) over the warp, with 8 independent partial sums (short add chains)
  auto count_ge = [&](uint32_t t) -> uint32_t {
    uint32_t cc[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) cc[j & 7] += key[j] >= t ? 1u : 0u;
    return __reduce_add_sync(0xffffffffu, ((cc[0] + cc[1]) + (cc[2] + cc[3])) + ((cc[4] + cc[5]) + (cc[6] + cc[7])));
  };
  // largest t with count(key >= t) >= kb (the kb-th largest key), or any t with
  // count(key >= t) == kb exactly (then the keys >= t are the selection, ties included)
  bool exact = false;
  while (lo < hi && kb > 0) {
    const uint32_t mid = lo + ((hi - lo + 1u) >> 1);
    const uint32_t c = count_ge(mid);
    if (c == static_cast<uint32_t>(kb)) {
      lo = mid;
      exact = true;
      break;
    }
    if (c > static_cast<uint32_t>(kb)) lo = mid;
    else hi = mid - 1u;
  }
  const uint32_t kstar = lo;
  uint32_t n_ge = 0u, n_eq = 0u;
#pragma unroll
  for (int j = 0; j < ITEMS; ++j) {
    n_ge += key[j] >= kstar ? 1u : 0u;
    n_eq += key[j] == kstar ? 1u : 0u;
  }
  const uint32_t tot_ge = __reduce_add_sync(0xffffffffu, n_ge);
  if (kb > 0 && (exact || tot_ge == static_cast<uint32_t>(kb))) {
    // every key >= kstar is selected: place each lane's keys after an exclusive scan of
    // the lanes' counts (the order inside sel does not matter, the ranking sorts)
    uint32_t pos = n_ge;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, pos, o);
      if (lane >= o) pos += y;
    }
    pos -= n_ge;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      if (key[j] >= kstar && j * 32 + lane < nb) {
        sel_idx[pos] = static_cast<uint32_t>(j * 32 + lane) + shift;
        sel_key[pos] = key[j];
        ++pos;
      }
    }
  } else {
    // ties at the k-th key: every key > kstar and the first `remaining` keys == kstar
    // (index order)
    const uint32_t remaining = static_cast<uint32_t>(kb) - (tot_ge - __reduce_add_sync(0xffffffffu, n_eq));
    uint32_t n_sel = 0u, eq_taken = 0u;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      const int64_t i = j * 32 + lane;
      const bool gt = kb > 0 && key[j] > kstar;
      const bool eq = kb > 0 && i < nb && key[j] == kstar;
      const unsigned eq_mask = __ballot_sync(0xffffffffu, eq);
      const uint32_t eq_rank = eq_taken + __popc(eq_mask & ((1u << lane) - 1u));
      const bool take = gt || (eq && eq_rank < remaining);
      const unsigned take_mask = __ballot_sync(0xffffffffu, take);
      if (take) {
        const uint32_t pos = n_sel + __popc(take_mask & ((1u << lane) - 1u));
        sel_idx[pos] = static_cast<uint32_t>(i) + shift;
        sel_key[pos] = key[j];
      }
      n_sel += __popc(take_mask);
      eq_taken += __popc(eq_mask);
    }
  }
  __syncwarp();
  if (idx_off < 0) write_selection(p, srow, sel_idx, sel_key, kb, bitmap, pg0, b, h, lane);
}

// Split form (G <= 4, so every head has two of the eight consumer warps): warp g and
// warp g + G each select the top kb of one half of head g's scores, and after a CTA
// barrier warp g ranks the two halves' picks together (a pick of the head's top kb is
// in its half's top kb, ties included, since its half holds no more keys that beat it).
// Every thread of the CTA calls this (the split form has a CTA-wide barrier).
__device__ __forceinline__ void write_one(const DecodeSelectParams& p, const float* srow, int rank, uint32_t ki,
                                          uint32_t ii, uint32_t neg_inf_key, int64_t off, int64_t id0,
                                          uint32_t* bitmap) {
  if (p.cand_scores) {
    p.cand_scores[off + rank] = srow[ii];
    p.cand_ids[off + rank] = static_cast<int32_t>(id0 + ii);
  } else {
    p.ids[off + rank] = static_cast<int32_t>(ii);
    if (ki > neg_inf_key) atomicOr(&bitmap[ii >> 5], 1u << (ii & 31u));
  }
}

// (score desc, index asc) as one descending 64-bit key: score key high, ~index low
__device__ __forceinline__ unsigned long long pick_key(uint32_t key, uint32_t idx) {
  return (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(~idx);
}

// A warp sorts its n <= 64 picks (sel_idx / sel_key) by (score desc, index asc) in
// place: a bitonic network over 64 positions, two per lane (lane and lane + 32).
__device__ __forceinline__ void sort_picks_desc(uint32_t* sel_idx, uint32_t* sel_key, int n, int lane) {
  unsigned long long v[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int e = lane + 32 * r;
    v[r] = e < n ? pick_key(sel_key[e], sel_idx[e]) : 0ull;  // empty slots sort last
  }
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 32) {  // k == 64: positions lane and lane + 32, the lower keeps the larger
        const unsigned long long mx = v[0] > v[1] ? v[0] : v[1], mn = v[0] > v[1] ? v[1] : v[0];
        v[0] = mx;
        v[1] = mn;
      } else {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int pos = lane + 32 * r;
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, v[r], j);
          // descending overall: in a block sorted downwards the lower position keeps
          // the larger key, in one sorted upwards the smaller
          const bool keep_max = ((pos & j) == 0) == ((pos & k) == 0);
          const unsigned long long mx = v[r] > other ? v[r] : other, mn = v[r] > other ? other : v[r];
          v[r] = keep_max ? mx : mn;
        }
      }
    }
  }
  __syncwarp();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int e = lane + 32 * r;
    if (e < n) {
      sel_key[e] = static_cast<uint32_t>(v[r] >> 32);
      sel_idx[e] = ~static_cast<uint32_t>(v[r]);
    }
  }
  __syncwarp();
}

// Ranks of two lists each sorted by (score desc, index asc): an entry's rank is its
// position in its own list plus the number of entries of the other list above it (a
// binary search); the first kb by rank are written.
__device__ __forceinline__ void write_sorted_pair(const DecodeSelectParams& p, const float* srow,
                                                  const uint32_t* idx_a, const uint32_t* key_a, int na,
                                                  const uint32_t* idx_b, const uint32_t* key_b, int nb_, int64_t kb,
                                                  uint32_t* bitmap, int64_t pg0, int64_t b, int64_t h, int lane) {
  const uint32_t neg_inf_key = float_key(-INFINITY);
  const bool cand = p.cand_scores != nullptr;
  const int64_t off = cand ? static_cast<int64_t>(blockIdx.y) * p.cand_stride + (b * p.Hq + h) * p.topk
                           : (b * p.Hq + h) * p.topk;
  const int64_t id0 = pg0 + (p.page_base ? static_cast<int64_t>(p.page_base[b]) : 0);
  for (int e = lane; e < na + nb_; e += 32) {
    const bool in_a = e < na;
    const int i = in_a ? e : e - na;
    const uint32_t ki = in_a ? key_a[i] : key_b[i], ii = in_a ? idx_a[i] : idx_b[i];
    const unsigned long long me = pick_key(ki, ii);
    const uint32_t* ok = in_a ? key_b : key_a;
    const uint32_t* oi = in_a ? idx_b : idx_a;
    int lo = 0, hi = in_a ? nb_ : na;  // first position of the other list below `me`
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (pick_key(ok[mid], oi[mid]) > me) lo = mid + 1;
      else hi = mid;
    }
    const int rank = i + lo;
    if (rank < kb) write_one(p, srow, rank, ki, ii, neg_inf_key, off, id0, bitmap);
  }
  for (int64_t r = kb + lane; r < p.topk; r += 32) {
    if (cand) {
      p.cand_scores[off + r] = -INFINITY;
      p.cand_ids[off + r] = -1;
    } else {
      p.ids[off + r] = -1;
    }
  }
}

template <int G, int ITEMS>
__device__ __forceinline__ void select_heads_split(const DecodeSelectParams& p, const float* sc, uint32_t* bitmap,
                                                   uint32_t* sel, int64_t nb, int64_t pg0, int64_t b, int64_t kvh,
                                                   int warp, int lane) {
  const int64_t kb = lmax(1, lmin(p.topk, nb));
  const int g = warp % G, half = warp / G;
  const int64_t n0 = (nb + 1) / 2;
  const float* srow = sc + g * p.chunk;
  const int64_t h = kvh * G + g;
  const bool sorted = kb <= 64;  // picks per half fit the 64-position sort
  if (warp < 2 * G) {
    if (p.scores && half == 0) {
      float* dst = p.scores + (b * p.Hq + h) * p.max_pages + pg0;
      const int64_t span = lmin(p.chunk, p.max_pages - pg0);
      for (int64_t i = lane; i < span; i += 32) dst[i] = i < nb ? srow[i] : -INFINITY;
    }
    const int64_t off = half ? n0 : 0, n = half ? nb - n0 : n0;
    select_head_reg<ITEMS>(p, srow + off, sel, bitmap, n, pg0, b, h, warp, lane, off);
    if (sorted) {
      uint32_t* si = sel + warp * 2 * p.topk;
      sort_picks_desc(si, si + p.topk, static_cast<int>(lmin(kb, n)), lane);
    }
  }
  __syncthreads();
  if (warp < G) {
    const uint32_t* a = sel + g * 2 * p.topk;
    const uint32_t* c = sel + (g + G) * 2 * p.topk;
    if (sorted)
      write_sorted_pair(p, srow, a, a + p.topk, static_cast<int>(lmin(kb, n0)), c, c + p.topk,
                        static_cast<int>(lmin(kb, nb - n0)), kb, bitmap, pg0, b, h, lane);
    else
      write_selection2(p, srow, a, a + p.topk, lmin(kb, n0), c, c + p.topk, lmin(kb, nb - n0), kb, bitmap, pg0, b,
                       h, lane);
  }
}

template <int G>
__device__ __forceinline__ void select_heads(const DecodeSelectParams& p, const float* sc, uint32_t* hist,
                                             uint32_t* bitmap, uint32_t* sel, int64_t nb, int64_t pg0, int64_t b,
                                             int64_t kvh, int warp, int lane) {
  if constexpr (G <= 4) {
    // CTA-uniform choice (nb is the CTA's page count)
    if (nb > 512 && nb <= 1024) return select_heads_split<G, 16>(p, sc, bitmap, sel, nb, pg0, b, kvh, warp, lane);
    if (nb > 1024 && nb <= 2048) return select_heads_split<G, 32>(p, sc, bitmap, sel, nb, pg0, b, kvh, warp, lane);
  }
  if (warp >= G) return;
  const int64_t kb = nb > 0 ? lmax(1, lmin(p.topk, nb)) : 0;
  const int g = warp;
  const int64_t h = kvh * G + g;
  const float* srow = sc + g * p.chunk;
  uint32_t* hw = hist + warp * 256;
  uint32_t* sel_idx = sel + warp * 2 * p.topk;
  uint32_t* sel_key = sel_idx + p.topk;
  if (p.scores) {
    float* dst = p.scores + (b * p.Hq + h) * p.max_pages + pg0;
    const int64_t span = lmin(p.chunk, p.max_pages - pg0);
    for (int64_t i = lane; i < span; i += 32) dst[i] = i < nb ? srow[i] : -INFINITY;
  }
  if (nb <= 256) return select_head_reg<8>(p, srow, sel, bitmap, nb, pg0, b, h, warp, lane);
  if (nb <= 512) return select_head_reg<16>(p, srow, sel, bitmap, nb, pg0, b, h, warp, lane);
  if (nb <= 1024) return select_head_reg<32>(p, srow, sel, bitmap, nb, pg0, b, h, warp, lane);
  if (nb <= 2048) return select_head_reg<64>(p, srow, sel, bitmap, nb, pg0, b, h, warp, lane);
  // longer chunks: radix select over shared memory
  uint32_t prefix = 0u, mask = 0u, remaining = static_cast<uint32_t>(kb);
  for (int shift = 24; shift >= 0 && kb > 0; shift -= 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) hw[lane * 8 + j] = 0u;
    __syncwarp();
    for (int64_t i0 = 0; i0 < nb; i0 += 32) {  // warp-uniform trip count
      const int64_t i = i0 + lane;
      const uint32_t key = i < nb ? float_key(srow[i]) : 0u;
      const bool act = i < nb && (key & mask) == prefix;
      const uint32_t bin = (key >> shift) & 255u;
      const unsigned am = __ballot_sync(0xffffffffu, act);
      if (act) {
        const unsigned peers = __match_any_sync(am, bin);
        if ((peers & ((1u << lane) - 1u)) == 0u) atomicAdd(&hw[bin], static_cast<uint32_t>(__popc(peers)));
      }
    }
    __syncwarp();
    // lane owns the 8 bins 255 - (lane*8 + j): counts in descending bin order
    uint32_t cnt[8], local = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      cnt[j] = hw[255 - (lane * 8 + j)];
      local += cnt[j];
    }
    uint32_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    uint32_t above = incl - local;  // keys in higher bins than this lane's
    int found = -1;
    uint32_t rem_new = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (found < 0 && above < remaining && above + cnt[j] >= remaining) {
        found = 255 - (lane * 8 + j);
        rem_new = remaining - above;
      }
      above += cnt[j];
    }
    const unsigned who = __ballot_sync(0xffffffffu, found >= 0);
    const int src = __ffs(who) - 1;
    const uint32_t digit = static_cast<uint32_t>(__shfl_sync(0xffffffffu, found, src));
    remaining = __shfl_sync(0xffffffffu, rem_new, src);
    prefix |= digit << shift;
    mask |= 0xffu << shift;
    __syncwarp();
  }
  // gather: every key > kstar, and the first `remaining` keys == kstar (index order)
  const uint32_t kstar = prefix;
  uint32_t n_sel = 0u, eq_taken = 0u;
  for (int64_t i0 = 0; i0 < nb && kb > 0; i0 += 32) {
    const int64_t i = i0 + lane;
    const uint32_t key = i < nb ? float_key(srow[i]) : 0u;
    const bool gt = i < nb && key > kstar;
    const bool eq = i < nb && key == kstar;
    const unsigned eq_mask = __ballot_sync(0xffffffffu, eq);
    const uint32_t eq_rank = eq_taken + __popc(eq_mask & ((1u << lane) - 1u));
    const bool take = gt || (eq && eq_rank < remaining);
    const unsigned take_mask = __ballot_sync(0xffffffffu, take);
    if (take) {
      const uint32_t pos = n_sel + __popc(take_mask & ((1u << lane) - 1u));
      sel_idx[pos] = static_cast<uint32_t>(i);
      sel_key[pos] = key;
    }
    n_sel += __popc(take_mask);
    eq_taken += __popc(eq_mask);
  }
  __syncwarp();
  write_selection(p, srow, sel_idx, sel_key, kb, bitmap, pg0, b, h, lane);
}

// The union bitmap of a (sequence, kv head) compacted to an ascending page list, with
// its count and token count.  All NT threads of the CTA take part.
template <int NT>
__device__ __forceinline__ void compact_union(const DecodeSelectParams& p, const uint32_t* bitmap, int64_t W,
                                              int64_t b, int64_t kvh, uint32_t* scan_tmp, uint32_t* sh_tokens) {
  const int tid = threadIdx.x;
  const int64_t wpt = (W + NT - 1) / NT;
  const int64_t w0 = lmin(W, tid * wpt), w1 = lmin(W, w0 + wpt);
  uint32_t cnt = 0u;
  for (int64_t w = w0; w < w1; ++w) cnt += __popc(bitmap[w]);
  uint32_t total = 0u;
  uint32_t pos = block_exclusive_scan<NT>(cnt, scan_tmp, &total);
  const int64_t len = p.seq_lens[b];
  const int64_t uoff = (b * p.Hkv + kvh) * p.max_union;
  uint32_t tokens = 0u;
  for (int64_t w = w0; w < w1; ++w) {
    uint32_t bits = bitmap[w];
    while (bits) {
      const int bit = __ffs(bits) - 1;
      bits &= bits - 1u;
      const int64_t pg = w * 32 + bit;
      if (pos < p.max_union) p.union_ids[uoff + pos] = static_cast<int32_t>(pg);
      ++pos;
      tokens += static_cast<uint32_t>(lmin(p.P, lmax(0, len - pg * p.P)));
    }
  }
  for (int64_t j = total + tid; j < p.max_union; j += NT) p.union_ids[uoff + j] = -1;
  atomicAdd(sh_tokens, tokens);
  __syncthreads();
  if (tid == 0) {
    if (total > p.max_union) report(p.status, LINATTN_DEV_OVERFLOW);
    p.union_count[b * p.Hkv + kvh] = static_cast<int32_t>(lmin(total, p.max_union));
    if (p.union_tokens) p.union_tokens[b * p.Hkv + kvh] = static_cast<int32_t>(*sh_tokens);
  }
}

// ---------------------------------------------------------------------------------
// CUDA-core scoring (fp32 q, or q and metadata of different 16-bit types)
// ---------------------------------------------------------------------------------
template <typename TM, int D, int G, int NSTG>
__global__ void __launch_bounds__(256, 1) quest_decode_select_kernel(const DecodeSelectParams p) {
  constexpr int LPR = D / 8;               // lanes per page
  constexpr int PPW = 32 / LPR;            // pages per warp step
  constexpr int PAGE_ELEMS = 2 * D;
  constexpr int CHUNK_BYTES = CH * PAGE_ELEMS * static_cast<int>(sizeof(TM));
  constexpr int NV = G >= LPR ? G / LPR : 1;
  constexpr int REP = G >= LPR ? 1 : LPR / G;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;                                                   // NSTG chunks
  float* sc = reinterpret_cast<float*>(smem + NSTG * CHUNK_BYTES);        // [G][chunk]
  uint32_t* hist = reinterpret_cast<uint32_t*>(sc + G * p.chunk);         // [8 warps][256]
  uint32_t* bitmap = hist + 8 * 256;                                      // [ceil(chunk/32)]
  uint32_t* sel = bitmap + (p.chunk + 31) / 32;                           // [8 warps][2][topk]
  __shared__ __align__(8) uint64_t bar[NSTG];
  __shared__ uint32_t scan_tmp[9];
  __shared__ uint32_t sh_tokens;

  // the attention launch that follows (a programmatic dependent) may start its set-up
  // now; its reads of what this grid writes wait for this grid's end
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t kvh = blockIdx.x % p.Hkv, b = blockIdx.x / p.Hkv;
  const int64_t nb_all = lmin(p.n_pages_b[b], p.max_pages);  // the sequence's pages
  const int64_t pg0 = static_cast<int64_t>(blockIdx.y) * p.chunk;  // this CTA's first page
  const int64_t nb = lmax(0, lmin(nb_all - pg0, p.chunk));      // and its page count
  const int64_t W = (p.chunk + 31) / 32;
  for (int64_t w = tid; w < W; w += 256) bitmap[w] = 0u;
  if (tid == 0) {
    for (int s = 0; s < NSTG; ++s) mbar_init(&bar[s], 1);
    mbar_fence_init();
    sh_tokens = 0u;
  }
  __syncthreads();

  const TM* base = static_cast<const TM*>(p.meta) + ((b * p.Hkv + kvh) * p.max_pages + pg0) * PAGE_ELEMS;
  const int64_t n_chunks = (nb + CH - 1) / CH;
  auto issue = [&](int64_t c) {
    const int s = static_cast<int>(c % NSTG);
    const uint32_t pages = static_cast<uint32_t>(lmin(CH, nb - c * CH));
    const uint32_t bytes = pages * PAGE_ELEMS * static_cast<uint32_t>(sizeof(TM));
    mbar_arrive_expect_tx(&bar[s], bytes);
    bulk_g2s(ring + s * CHUNK_BYTES, base + c * CH * PAGE_ELEMS, bytes, &bar[s]);
  };
  if (tid == 0)
    for (int64_t c = 0; c < n_chunks && c < NSTG; ++c) issue(c);

  // q of the G heads: lane covers channels [cl*8, cl*8+8)
  const int sub = lane / LPR, cl = lane % LPR;
  float qv[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < 8; ++c)
      qv[g][c] = load_any(p.q, b * p.qs[0] + (kvh * G + g) * p.qs[1] + (cl * 8 + c) * p.qs[3], p.q_dtype);

  bool abort = false;
  for (int64_t c = 0; c < n_chunks; ++c) {
    const int s = static_cast<int>(c % NSTG);
    if (!mbar_wait_bounded(&bar[s], static_cast<uint32_t>((c / NSTG) & 1))) {
      report(p.status, LINATTN_DEV_TIMEOUT);
      abort = true;
    }
    if (__syncthreads_or(abort)) {
      abort = true;
      break;
    }
    const TM* chunk = reinterpret_cast<const TM*>(ring + s * CHUNK_BYTES);
    const int64_t pages = lmin(CH, nb - c * CH);
    for (int pp = warp * PPW; pp < CH; pp += 8 * PPW) {
      const int pg = pp + sub;
      float acc[G];
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = 0.f;
      if (pg < pages) {
        float mn[8], mx[8];
        load8(chunk + pg * PAGE_ELEMS + cl * 8, mn);
        load8(chunk + pg * PAGE_ELEMS + D + cl * 8, mx);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[g] = fmaf(qv[g][e], qv[g][e] >= 0.f ? mx[e] : mn[e], acc[g]);
      }
      group_reduce<G, LPR>(acc, lane);
      if (pg < pages && (cl % REP) == 0) {
        const int64_t page = c * CH + pg;
        const int64_t gpage = pg0 + page;
        const bool forced = (p.force_last && gpage == nb_all - 1) || gpage < p.sink_pages;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int g = G >= LPR ? cl * NV + i : cl / REP;
          sc[g * p.chunk + page] = forced ? INFINITY : acc[i];
        }
      }
    }
    __syncthreads();  // chunk s consumed
    if (tid == 0 && c + NSTG < n_chunks) issue(c + NSTG);
  }
  if (abort) {
    if (tid == 0)  // bounded wait for copies still in flight
      for (int64_t c = 0; c < n_chunks && c < NSTG; ++c)
        (void)mbar_wait_bounded(&bar[c % NSTG], static_cast<uint32_t>((c / NSTG) & 1));
    __syncthreads();
    return;
  }
  select_heads<G>(p, sc, hist, bitmap, sel, nb, pg0, b, kvh, warp, lane);
  if (p.cand_scores) return;  // the union is taken after the merge of all chunks
  __syncthreads();
  compact_union<256>(p, bitmap, W, b, kvh, scan_tmp, &sh_tokens);
}

// ---------------------------------------------------------------------------------
// Tensor-core scoring (q and metadata of the same 16-bit type)
// ---------------------------------------------------------------------------------
// max(q_d*min_d, q_d*max_d) = min(q_d,0)*min_d + max(q_d,0)*max_d exactly (one of the
// two products is zero), so the scores of a stage of pages are one GEMM: the stage's
// metadata rows [min row | max row] (pages x 2D, as stored) times [min(q,0) ; max(q,0)]
// (2D x heads).  mma.sync m16n8k16 with the pages as M (16 per warp tile), the G <= 8
// heads of the group as N, fp32 accumulation of exact 16-bit products.
//
// A producer warp streams the chunk's rows with 2-D TMA boxes (64 channels x MP pages,
// 128-byte swizzle, no multicast) through an NS-stage ring (full / empty mbarriers);
// stages alternate between two groups of four consumer warps, each warp taking one
// 16-page tile of its stages (ldmatrix from the swizzled tile, 2D/16 MMAs).
constexpr int MP = 64;  // pages per stage of the tensor-core path

__device__ __forceinline__ void qs_ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void qs_tma_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <typename TM>
__device__ __forceinline__ void qs_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void qs_mma<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                      uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void qs_mma<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t qs_pack(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(lo)) | (static_cast<uint32_t>(__bfloat16_as_ushort(hi)) << 16);
}
__device__ __forceinline__ uint32_t qs_pack(__half lo, __half hi) {
  return static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}
// the negative / positive part of a 16-bit value, exactly (sign test on the bits)
template <typename TM>
__device__ __forceinline__ TM qs_part(TM x, bool positive) {
  const uint16_t bits = sizeof(TM) == 2 ? *reinterpret_cast<const uint16_t*>(&x) : 0;
  const bool neg = (bits & 0x8000u) != 0;
  uint16_t out = (neg != positive) ? bits : static_cast<uint16_t>(0);
  return *reinterpret_cast<const TM*>(&out);
}

template <typename TM, int D, int G, int NS>
__global__ void __launch_bounds__(288, 2) quest_select_mma_kernel(const DecodeSelectParams p,
                                                                  const __grid_constant__ CUtensorMap tm) {
  constexpr int NQ = 2 * D / 64;             // 128-byte column blocks per page row
  constexpr int BOX_BYTES = MP * 128;
  constexpr int STAGE_BYTES = NQ * BOX_BYTES;
  constexpr int KSTEPS = 2 * D / 16;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* ring = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);  // 1024-aligned for the swizzle
  float* sc = reinterpret_cast<float*>(ring + NS * STAGE_BYTES);           // [G][chunk]
  uint32_t* hist = reinterpret_cast<uint32_t*>(sc + G * p.chunk);          // [8 warps][256]
  uint32_t* bitmap = hist + 8 * 256;                                       // [ceil(chunk/32)]
  uint32_t* sel = bitmap + (p.chunk + 31) / 32;                            // [8 warps][2][topk]
  __shared__ __align__(8) uint64_t full_bar[NS];
  __shared__ __align__(8) uint64_t empty_bar[NS];
  __shared__ uint32_t scan_tmp[10];
  __shared__ uint32_t sh_tokens;

  // the attention launch that follows (a programmatic dependent) may start its set-up
  // now; its reads of what this grid writes wait for this grid's end
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t kvh = blockIdx.x % p.Hkv, b = blockIdx.x / p.Hkv;
  const int64_t nb_all = lmin(p.n_pages_b[b], p.max_pages);
  const int64_t pg0 = static_cast<int64_t>(blockIdx.y) * p.chunk;
  const int64_t nb = lmax(0, lmin(nb_all - pg0, p.chunk));
  const int64_t W = (p.chunk + 31) / 32;
  for (int64_t w = tid; w < W; w += 288) bitmap[w] = 0u;
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 4);  // the four consumer warps of the slot's group
    }
    mbar_fence_init();
    sh_tokens = 0u;
  }
  __syncthreads();

  const int64_t n_st = (nb + MP - 1) / MP;
  bool abort = false;
  int64_t issued = 0;
  if (warp == 8) {
    // ---- producer
    if (lane == 0) {
      const int row0 = static_cast<int>((b * p.Hkv + kvh) * p.max_pages + pg0);
      for (int64_t c = 0; c < n_st; ++c) {
        const int s = static_cast<int>(c % NS);
        if (c >= NS && !mbar_wait_bounded(&empty_bar[s], static_cast<uint32_t>(((c / NS) - 1) & 1))) {
          report(p.status, LINATTN_DEV_TIMEOUT);
          abort = true;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
        uint8_t* dst = ring + s * STAGE_BYTES;
#pragma unroll
        for (int qq = 0; qq < NQ; ++qq)
          qs_tma_2d(dst + qq * BOX_BYTES, &tm, qq * 64, row0 + static_cast<int>(c * MP), &full_bar[s]);
        ++issued;
      }
    }
  } else {
    // ---- consumers: B fragments of [min(q,0) ; max(q,0)] for head n = lane / 4
    const int gid = lane >> 2, tig = lane & 3;
    uint32_t qb[KSTEPS][2];
    {
      const TM* qrow = static_cast<const TM*>(p.q) + b * p.qs[0] + (kvh * G + (gid < G ? gid : 0)) * p.qs[1];
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int k = ks * 16 + r * 8 + 2 * tig;  // k and k + 1
          const bool positive = k >= D;              // the max half of the row
          const int ch = positive ? k - D : k;
          TM lo = qrow[ch * p.qs[3]], hi = qrow[(ch + 1) * p.qs[3]];
          lo = qs_part(lo, positive);
          hi = qs_part(hi, positive);
          qb[ks][r] = gid < G ? qs_pack(lo, hi) : 0u;
        }
      }
    }
    const int grp = warp >> 2, mt = warp & 3;
    const int mi = lane >> 3, ri = lane & 7;
    const uint32_t ring_s = smem_u32(ring);
    for (int64_t c = grp; c < n_st; c += 2) {
      const int s = static_cast<int>(c % NS);
      // warp-uniform outcome: every lane goes on to the warp-collective MMAs, or none
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full_bar[s], static_cast<uint32_t>((c / NS) & 1)))) {
        if (lane == 0) report(p.status, LINATTN_DEV_TIMEOUT);
        abort = true;
        break;
      }
      const int64_t pages = lmin(MP, nb - c * MP);
      if (mt * 16 < pages) {
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};  // two chains: min / max halves
        const uint32_t st = ring_s + static_cast<uint32_t>(s) * STAGE_BYTES;
        const int row = mt * 16 + (mi & 1) * 8 + ri;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) {
          const int chunk16 = ks * 2 + (mi >> 1);  // 16-byte chunk of the page row
          const uint32_t addr = st + static_cast<uint32_t>((chunk16 >> 3) * BOX_BYTES + row * 128 +
                                                           (((chunk16 & 7) ^ (row & 7)) << 4));
          uint32_t a[4];
          qs_ldsm_x4(addr, a);
          qs_mma<TM>(ks < KSTEPS / 2 ? d0 : d1, a, qb[ks][0], qb[ks][1]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int pr = mt * 16 + gid + (i >> 1) * 8;  // page within the stage
          const int hh = 2 * tig + (i & 1);             // head within the group
          const int64_t page = c * MP + pr;
          if (hh < G && pr < pages) {
            const int64_t gpage = pg0 + page;
            const bool forced = (p.force_last && gpage == nb_all - 1) || gpage < p.sink_pages;
            sc[hh * p.chunk + page] = forced ? INFINITY : d0[i] + d1[i];
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_1(&empty_bar[s]);
    }
  }
  if (__syncthreads_or(abort)) {
    if (warp == 8 && lane == 0)  // bounded wait for the copies still in flight
      for (int64_t c = lmax(0, issued - NS); c < issued; ++c)
        (void)mbar_wait_bounded(&full_bar[c % NS], static_cast<uint32_t>((c / NS) & 1));
    __syncthreads();
    return;
  }
  select_heads<G>(p, sc, hist, bitmap, sel, nb, pg0, b, kvh, warp, lane);
  if (p.cand_scores) return;
  __syncthreads();
  compact_union<288>(p, bitmap, W, b, kvh, scan_tmp, &sh_tokens);
}

// Shared memory of the two scoring paths.  Ring stages: the CUDA-core path uses 8
// (single-CTA form, one CTA per SM streams the whole sequence) or 4 (candidates form);
// the tensor-core path 4 or 2 stages of MP pages, the latter so that two CTAs share
// an SM.
size_t select_rest_smem(int64_t chunk, int64_t G, int64_t topk) {
  return static_cast<size_t>(G) * chunk * 4 + 8 * 256 * 4 + static_cast<size_t>((chunk + 31) / 32) * 4 +
         static_cast<size_t>(8) * 2 * topk * 4;
}
size_t quest_decode_select_smem(int64_t chunk, int64_t G, int64_t topk, int64_t D, bool mma, bool cand) {
  if (mma) return 1024 + static_cast<size_t>(cand ? 2 : 4) * 2 * D * MP * 2 + select_rest_smem(chunk, G, topk);
  return static_cast<size_t>(cand ? 4 : 8) * CH * 2 * D * 2 + select_rest_smem(chunk, G, topk);
}

template <bool MMA, bool CAND, typename TM, int D, int G>
static cudaError_t launch_one(const DecodeSelectParams& p, const CUtensorMap& tm, unsigned n_chunks, size_t smem,
                              cudaStream_t stream) {
  static int configured[64] = {};
  const int dev = device_index();
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const dim3 grid(static_cast<unsigned>(p.B * p.Hkv), n_chunks);
  if constexpr (MMA) {
    constexpr int NS = CAND ? 2 : 4;
    if (configured[dev] < static_cast<int>(smem)) {
      cudaError_t e = cudaFuncSetAttribute(quest_select_mma_kernel<TM, D, G, NS>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      configured[dev] = static_cast<int>(smem);
    }
    quest_select_mma_kernel<TM, D, G, NS><<<grid, 288, smem, stream>>>(p, tm);
  } else {
    constexpr int NS = CAND ? 4 : 8;
    if (configured[dev] < static_cast<int>(smem)) {
      cudaError_t e = cudaFuncSetAttribute(quest_decode_select_kernel<TM, D, G, NS>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      configured[dev] = static_cast<int>(smem);
    }
    quest_decode_select_kernel<TM, D, G, NS><<<grid, 256, smem, stream>>>(p);
  }
  return cudaGetLastError();
}

template <bool MMA, bool CAND, typename TM, int D>
static cudaError_t launch_g(const DecodeSelectParams& p, const CUtensorMap& tm, int G, unsigned n_chunks,
                            size_t smem, cudaStream_t stream) {
  switch (G) {
    case 1: return launch_one<MMA, CAND, TM, D, 1>(p, tm, n_chunks, smem, stream);
    case 2: return launch_one<MMA, CAND, TM, D, 2>(p, tm, n_chunks, smem, stream);
    case 4: return launch_one<MMA, CAND, TM, D, 4>(p, tm, n_chunks, smem, stream);
    case 8: return launch_one<MMA, CAND, TM, D, 8>(p, tm, n_chunks, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <bool MMA, bool CAND, typename TM>
static cudaError_t launch_d(const DecodeSelectParams& p, const CUtensorMap& tm, int D, int G, unsigned n_chunks,
                            size_t smem, cudaStream_t stream) {
  switch (D) {
    case 64: return launch_g<MMA, CAND, TM, 64>(p, tm, G, n_chunks, smem, stream);
    case 128: return launch_g<MMA, CAND, TM, 128>(p, tm, G, n_chunks, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <bool MMA, typename TM>
static cudaError_t launch_c(const DecodeSelectParams& p, const CUtensorMap& tm, int D, int G, unsigned n_chunks,
                            size_t smem, cudaStream_t stream) {
  return p.cand_scores ? launch_d<MMA, true, TM>(p, tm, D, G, n_chunks, smem, stream)
                       : launch_d<MMA, false, TM>(p, tm, D, G, n_chunks, smem, stream);
}

}  // namespace linattn

using namespace linattn;

namespace {

int check_select_args(const void* q, int32_t q_dtype, int64_t Hq, int64_t D, const int64_t* q_strides,
                      const void* meta, int32_t meta_dtype, int64_t n_kv_heads, int64_t max_pages,
                      const int32_t* n_pages_b, int64_t topk, const char* who) {
  char msg[160];
  auto fail = [&](int code, const char* what) {
    snprintf(msg, sizeof(msg), "%s: %s", who, what);
    return set_error(code, msg);
  };
  if (!q || !q_strides || !meta || !n_pages_b) return fail(LINATTN_EINVAL, "NULL pointer");
  if (q_dtype != LINATTN_F32 && q_dtype != LINATTN_F16 && q_dtype != LINATTN_BF16)
    return fail(LINATTN_EUNSUPPORTED, "q dtype");
  if (meta_dtype != LINATTN_F16 && meta_dtype != LINATTN_BF16)
    return fail(LINATTN_EUNSUPPORTED, "metadata must be f16 or bf16");
  if (D != 64 && D != 128) return fail(LINATTN_EUNSUPPORTED, "head_dim must be 64 or 128");
  if (n_kv_heads <= 0 || Hq % n_kv_heads) return fail(LINATTN_EINVAL, "H_kv must divide H_q");
  const int64_t G = Hq / n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return fail(LINATTN_EUNSUPPORTED, "group size must be 1, 2, 4 or 8");
  if (topk < 1 || topk > 1024 || max_pages < 1) return fail(LINATTN_EINVAL, "bad topk / max_pages");
  if (reinterpret_cast<uintptr_t>(meta) % 16) return fail(LINATTN_EINVAL, "meta alignment");
  return LINATTN_OK;
}

int launch_select_on(const DecodeSelectParams& p, int32_t q_dtype, int32_t meta_dtype, int64_t D,
                     unsigned n_chunks, const char* who, void* stream) {
  const int64_t G = p.Hq / p.Hkv;
  const bool cand = p.cand_scores != nullptr;
  // tensor cores when q and the metadata share a 16-bit type (the products stay exact)
  const bool mma = q_dtype == meta_dtype && p.B * p.Hkv * p.max_pages < (int64_t(1) << 31) &&
                   reinterpret_cast<uintptr_t>(p.meta) % 16 == 0;
  const size_t smem = quest_decode_select_smem(p.chunk, G, p.topk, D, mma, cand);
  char msg[256];
  if (smem > 220 * 1024) {
    snprintf(msg, sizeof(msg), "%s: too many pages per CTA for the fused kernel", who);
    return set_error(LINATTN_EUNSUPPORTED, msg);
  }
  if (p.B * p.Hkv == 0 || n_chunks == 0) return LINATTN_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tm;
  cudaError_t e;
  if (mma) {
    const CUtensorMapDataType cu = meta_dtype == LINATTN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (!tensor_map_2d(&tm, p.meta, cu, 2 * D, p.B * p.Hkv * p.max_pages, 2 * D * 2, 64, MP)) {
      snprintf(msg, sizeof(msg), "%s: tensor map encoding failed", who);
      return set_error(LINATTN_ECUDA, msg);
    }
    e = meta_dtype == LINATTN_BF16
            ? launch_c<true, __nv_bfloat16>(p, tm, static_cast<int>(D), static_cast<int>(G), n_chunks, smem, st)
            : launch_c<true, __half>(p, tm, static_cast<int>(D), static_cast<int>(G), n_chunks, smem, st);
  } else {
    e = meta_dtype == LINATTN_BF16
            ? launch_c<false, __nv_bfloat16>(p, tm, static_cast<int>(D), static_cast<int>(G), n_chunks, smem, st)
            : launch_c<false, __half>(p, tm, static_cast<int>(D), static_cast<int>(G), n_chunks, smem, st);
  }
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "%s: %s", who, cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}

}  // namespace

extern "C" int linattn_quest_decode_select(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t D,
                                           const int64_t* q_strides, const void* meta, int32_t meta_dtype,
                                           int64_t n_kv_heads, int64_t max_pages, const int32_t* n_pages_b,
                                           const int32_t* seq_lens, int64_t page_size, int64_t topk,
                                           int32_t sink_pages, int32_t force_last, int32_t* ids, float* scores,
                                           int32_t* union_ids,
                                           int32_t* union_count, int64_t max_union, int32_t* union_tokens,
                                           int32_t* status, void* stream) {
  int rc = check_select_args(q, q_dtype, Hq, D, q_strides, meta, meta_dtype, n_kv_heads, max_pages, n_pages_b, topk,
                             "quest_decode_select");
  if (rc) return rc;
  if (!seq_lens || !ids || !union_ids || !union_count)
    return set_error(LINATTN_EINVAL, "quest_decode_select: NULL pointer");
  if (page_size < 1 || max_union < 1) return set_error(LINATTN_EINVAL, "quest_decode_select: bad page_size / max_union");
  DecodeSelectParams p{};
  p.q = q; p.q_dtype = q_dtype; p.B = B; p.Hq = Hq; p.Hkv = n_kv_heads;
  for (int i = 0; i < 4; ++i) p.qs[i] = q_strides[i];
  p.meta = meta; p.max_pages = max_pages; p.n_pages_b = n_pages_b; p.seq_lens = seq_lens; p.P = page_size;
  p.topk = static_cast<int>(topk); p.sink_pages = sink_pages; p.force_last = force_last ? 1 : 0;
  p.ids = ids; p.scores = scores;
  p.union_ids = union_ids; p.union_count = union_count; p.max_union = max_union; p.union_tokens = union_tokens;
  p.status = status;
  p.chunk = max_pages;
  return launch_select_on(p, q_dtype, meta_dtype, D, 1u, "quest_decode_select", stream);
}

extern "C" int linattn_quest_decode_candidates(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t D,
                                               const int64_t* q_strides, const void* meta, int32_t meta_dtype,
                                               int64_t n_kv_heads, int64_t max_pages, const int32_t* n_pages_b,
                                               int64_t topk, int32_t sink_pages, int32_t force_last,
                                               int64_t chunk_pages, const int32_t* page_base, float* cand_scores,
                                               int32_t* cand_ids, int64_t cand_stride, float* scores,
                                               int32_t* status, void* stream) {
  int rc = check_select_args(q, q_dtype, Hq, D, q_strides, meta, meta_dtype, n_kv_heads, max_pages, n_pages_b, topk,
                             "quest_decode_candidates");
  if (rc) return rc;
  if (!cand_scores || !cand_ids) return set_error(LINATTN_EINVAL, "quest_decode_candidates: NULL pointer");
  if (chunk_pages < 1) return set_error(LINATTN_EINVAL, "quest_decode_candidates: chunk_pages must be >= 1");
  const int64_t n_chunks = (max_pages + chunk_pages - 1) / chunk_pages;
  if (cand_stride < B * Hq * topk) return set_error(LINATTN_EINVAL, "quest_decode_candidates: cand_stride");
  if (n_chunks > 65535) return set_error(LINATTN_EUNSUPPORTED, "quest_decode_candidates: too many chunks");
  DecodeSelectParams p{};
  p.q = q; p.q_dtype = q_dtype; p.B = B; p.Hq = Hq; p.Hkv = n_kv_heads;
  for (int i = 0; i < 4; ++i) p.qs[i] = q_strides[i];
  p.meta = meta; p.max_pages = max_pages; p.n_pages_b = n_pages_b; p.P = 1;
  p.topk = static_cast<int>(topk); p.sink_pages = sink_pages; p.force_last = force_last ? 1 : 0;
  p.scores = scores; p.status = status;
  p.chunk = lmin(chunk_pages, max_pages);
  p.cand_scores = cand_scores; p.cand_ids = cand_ids; p.cand_stride = cand_stride; p.page_base = page_base;
  return launch_select_on(p, q_dtype, meta_dtype, D, static_cast<unsigned>(n_chunks), "quest_decode_candidates",
                          stream);
}
