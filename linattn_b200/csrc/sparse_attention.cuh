// Sparse (paged, block-list) attention for decode-shaped work.
//
// One CTA = one (batch, list head, query) unit x one split of its page list x one
// chunk of up to G query heads.  All G heads share every K/V row that is read, so
// a page is fetched from HBM once per GQA group.
//
// Data path: each page's valid rows are contiguous (P rows x D elements), so warp 0
// moves them with 1-D TMA bulk copies (cp.async.bulk, no tensor map, no multicast)
// into a STAGES-deep ring of shared-memory tiles of TR rows, completing on one
// mbarrier per stage.  Consumers wait with a bounded try_wait (a give-up sets
// LINATTN_DEV_TIMEOUT; no wait is unbounded).
//
// Math (fp32, CUDA cores): QK with D/8 lanes per row and a transposing butterfly
// over the G head partials; online softmax in the log2 domain (scale*log2(e) is
// folded into q); PV with each thread owning a channel pair for all G heads and a
// row subset.  fp8 e4m3 rows are dequantised in registers; the per-(page, head)
// scales fold into the scores (K) and into the probabilities (V).
#pragma once

#include "common.cuh"

namespace linattn {

struct AttnParams {
  const void* q;
  int q_dtype;
  int out_dtype;  // of `out` (q's dtype, or f32 for partials that are merged later)
  int64_t B, Hq, Tq;
  int64_t qs[4];
  linattn_kv_t kv;
  linattn_lists_t lists;
  int causal;
  int64_t offset;
  float scale_log2;  // softmax scale * log2(e)
  void* out;
  int64_t os[4];
  float* lse_out;
  int n_splits;
  int n_head_chunks;
  int heads_per_list;  // G_total
  float* ws_o;         // [S, B*Hq*Tq, D] when n_splits > 1
  float* ws_lse;       // [S, B*Hq*Tq]
  int32_t* status;
};

template <int G, int LPR>
__device__ __forceinline__ void attn_transpose_reduce(float (&v)[G], int lane) {
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

template <typename T, int D, int G>
struct AttnShape {
  static constexpr int EB = sizeof(T);
  static constexpr int TR0 = 16384 / (D * EB);
  static constexpr int TR = TR0 < 64 ? TR0 : 64;  // tile rows
  static constexpr int TILE_BYTES = TR * D * EB;  // one of K or V
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int STAGES = STAGE_BYTES <= 16384 ? 4 : 3;
  static constexpr int LPR = D / 8 < 32 ? D / 8 : 32;  // QK lanes per row
  static constexpr int CPL = D / LPR;                 // QK channels per lane (8, or 8*k for D > 256)
  static constexpr int RPW = 32 / LPR;                // rows per warp step
  static constexpr int PAIRS = D / 2;
  static constexpr int NRG = 256 / PAIRS;  // PV row groups
  static constexpr int MAXSLOT = TR;       // page slots per tile (page_size 1)
  static constexpr size_t RING_BYTES = static_cast<size_t>(STAGES) * STAGE_BYTES;
  static constexpr size_t RED_BYTES = static_cast<size_t>(NRG) * G * D * 4;
  static constexpr size_t SMEM_BYTES = (RING_BYTES > RED_BYTES ? RING_BYTES : RED_BYTES);
  static_assert(D % 8 == 0 && D <= 256, "head_dim");
  static_assert(PAIRS <= 256, "head_dim");
};

template <typename T, int D, int G>
__global__ void __launch_bounds__(256, 2) sparse_attention_kernel(const AttnParams p) {
  using S = AttnShape<T, D, G>;
  constexpr int TR = S::TR, STAGES = S::STAGES, LPR = S::LPR, RPW = S::RPW;
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ int32_t st_nv[STAGES][S::MAXSLOT];
  __shared__ int64_t st_off[STAGES][S::MAXSLOT];
  __shared__ float st_ks[STAGES][S::MAXSLOT];
  __shared__ float st_vs[STAGES][S::MAXSLOT];
  __shared__ unsigned long long st_rows[STAGES];  // row-valid bit mask of the tile
  __shared__ float s_s[G][TR];
  __shared__ __align__(16) float p_s[TR][G];
  __shared__ float alpha_s[G];
  __shared__ float m_fin[G], l_fin[G];
  __shared__ int sh_abort;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // ---- unit decode
  const int64_t S_ = p.n_splits;
  int64_t bid = blockIdx.x;
  const int split = static_cast<int>(bid % S_);
  bid /= S_;
  const int hc = static_cast<int>(bid % p.n_head_chunks);
  const int64_t unit = bid / p.n_head_chunks;
  const int64_t t = unit % p.Tq;
  const int64_t lh = (unit / p.Tq) % p.lists.n_heads;
  const int64_t b = unit / (p.Tq * p.lists.n_heads);
  const int64_t h0 = lh * p.heads_per_list + static_cast<int64_t>(hc) * G;
  const int n_heads_here = static_cast<int>(lmin(G, p.heads_per_list - static_cast<int64_t>(hc) * G));
  const int64_t kvh = h0 / (p.Hq / p.kv.n_kv_heads);

  const int64_t P = p.kv.page_size;
  const int64_t len_b = p.kv.seq_lens ? static_cast<int64_t>(p.kv.seq_lens[b]) : p.kv.seq_len;
  const int64_t limit = p.causal ? min(len_b, p.offset + t + 1) : len_b;

  // ---- this split's slice of the list
  const int64_t lbase = b * p.lists.stride_b + lh * p.lists.stride_h + t * p.lists.stride_t;
  int64_t list_len = p.lists.max_len;
  if (p.lists.counts)
    list_len = lmin(list_len, p.lists.counts[b * p.lists.cstride_b + lh * p.lists.cstride_h +
                                                     t * p.lists.cstride_t]);
  const int64_t per = (list_len + S_ - 1) / S_;
  const int64_t j0 = lmin(list_len, split * per);
  const int64_t j1 = lmin(list_len, j0 + per);
  const bool small_pages = P <= TR;
  const int64_t PR = small_pages ? P : TR;              // rows per slot
  const int64_t PPT = small_pages ? TR / P : 1;          // slots per tile
  const int64_t segs = small_pages ? 1 : P / TR;         // tiles per page (P > TR)
  const int64_t n_tiles = small_pages ? (j1 - j0 + PPT - 1) / PPT : (j1 - j0) * segs;

  const T* kbase = static_cast<const T*>(p.kv.k) + b * p.kv.stride_b + kvh * p.kv.stride_head;
  const T* vbase = static_cast<const T*>(p.kv.v) + b * p.kv.stride_b + kvh * p.kv.stride_head;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full_bar[s], 1);
    mbar_fence_init();
    sh_abort = 0;
  }
  __syncthreads();

  // ---- producer: warp 0 fills stage `s` with tile `tile`.  Pass 1: one lane per
  // page slot resolves list id -> physical page -> valid row count; the warp sums the
  // bytes and lane 0 arms the stage barrier.  Pass 2: each lane issues its slot's K
  // and V bulk copies.
  auto issue = [&](int64_t tile, int s) {
    uint8_t* kdst = ring + static_cast<size_t>(s) * S::STAGE_BYTES;
    uint8_t* vdst = kdst + S::TILE_BYTES;
    uint32_t bytes = 0;
    unsigned long long rows = 0ull;
    for (int64_t slot0 = 0; slot0 < PPT; slot0 += 32) {
      const int64_t slot = slot0 + lane;
      int64_t nv = 0, eoff = 0;
      float ks = 1.f, vs = 1.f;
      if (slot < PPT) {
        const int64_t j = small_pages ? j0 + tile * PPT + slot : j0 + tile / segs;
        const int64_t seg = small_pages ? 0 : tile % segs;
        if (j < j1) {
          const int64_t id = p.lists.ids_dtype == LINATTN_I64
                                 ? static_cast<const int64_t*>(p.lists.ids)[lbase + j]
                                 : static_cast<int64_t>(static_cast<const int32_t*>(p.lists.ids)[lbase + j]);
          if (id >= 0) {
            nv = lmax(0, lmin(PR, limit - (id * P + seg * TR)));
            int64_t phys = id;
            if (nv > 0 && p.kv.page_table) {
              phys = id < p.kv.page_table_stride ? p.kv.page_table[b * p.kv.page_table_stride + id] : -1;
              if (phys < 0 || phys >= p.kv.num_phys_pages) {
                report(p.status, LINATTN_DEV_BAD_ID);
                nv = 0;
              }
            }
            if (nv > 0) {
              eoff = phys * p.kv.stride_page + seg * TR * D;
              if (p.kv.k_scale) {
                ks = p.kv.k_scale[phys * p.kv.scale_stride_page + kvh * p.kv.scale_stride_head];
                vs = p.kv.v_scale[phys * p.kv.scale_stride_page + kvh * p.kv.scale_stride_head];
              }
            }
          }
        }
        st_nv[s][slot] = static_cast<int32_t>(nv);
        st_off[s][slot] = eoff;
        st_ks[s][slot] = ks;
        st_vs[s][slot] = vs;
      }
      uint32_t my_bytes = static_cast<uint32_t>(2 * nv * D * S::EB);
      unsigned long long my_rows = 0ull;
      if (nv > 0) my_rows = (nv >= 64 ? ~0ull : ((1ull << nv) - 1ull)) << (slot * PR);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        my_bytes += __shfl_xor_sync(0xffffffffu, my_bytes, o);
        my_rows |= __shfl_xor_sync(0xffffffffu, my_rows, o);
      }
      bytes += my_bytes;
      rows |= my_rows;
    }
    __syncwarp();
    if (lane == 0) {
      st_rows[s] = rows;
      mbar_arrive_expect_tx(&full_bar[s], bytes);
    }
    __syncwarp();
    for (int64_t slot0 = 0; slot0 < PPT; slot0 += 32) {
      const int64_t slot = slot0 + lane;
      if (slot >= PPT) continue;
      const int64_t nv = st_nv[s][slot];
      if (nv <= 0) continue;
      const int64_t eoff = st_off[s][slot];
      const uint32_t nbytes = static_cast<uint32_t>(nv * D * S::EB);
      bulk_g2s(kdst + slot * PR * D * S::EB, kbase + eoff, nbytes, &full_bar[s]);
      bulk_g2s(vdst + slot * PR * D * S::EB, vbase + eoff, nbytes, &full_bar[s]);
    }
  };

  if (warp == 0) {
    for (int64_t tile = 0; tile < n_tiles && tile < STAGES; ++tile) issue(tile, static_cast<int>(tile));
  }

  // ---- q in registers, pre-scaled; lane cl covers channels [cl*CPL, cl*CPL + CPL)
  const int sub = lane / LPR, cl = lane % LPR;
  float qv[G][S::CPL];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < S::CPL; ++c)
      qv[g][c] = g < n_heads_here
                     ? load_any(p.q, b * p.qs[0] + (h0 + g) * p.qs[1] + t * p.qs[2] + (cl * S::CPL + c) * p.qs[3],
                                p.q_dtype) *
                           p.scale_log2
                     : 0.f;
  // PV ownership
  const int cp = tid % S::PAIRS, rg = tid / S::PAIRS;
  float acc[G][2];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // softmax state of head `warp` (warps < G)

  int64_t consumed = 0;
  for (int64_t tile = 0; tile < n_tiles; ++tile) {
    const int s = static_cast<int>(tile % STAGES);
    const uint32_t par = static_cast<uint32_t>((tile / STAGES) & 1);
    if (!mbar_wait_bounded(&full_bar[s], par)) {
      report(p.status, LINATTN_DEV_TIMEOUT);
      sh_abort = 1;
    }
    __syncthreads();
    if (sh_abort) break;
    consumed = tile + 1;
    const T* Ks = reinterpret_cast<const T*>(ring + static_cast<size_t>(s) * S::STAGE_BYTES);
    const T* Vs = reinterpret_cast<const T*>(ring + static_cast<size_t>(s) * S::STAGE_BYTES + S::TILE_BYTES);
    const unsigned long long rows = st_rows[s];
    // ---- QK
    for (int rb = warp * RPW; rb < TR; rb += 8 * RPW) {
      const int r = rb + sub;
      const bool valid = r < TR && ((rows >> r) & 1ull);
      float dots[G];
#pragma unroll
      for (int g = 0; g < G; ++g) dots[g] = 0.f;
      if (valid) {
#pragma unroll
        for (int c8 = 0; c8 < S::CPL; c8 += 8) {
          float kf[8];
          load8(Ks + r * D + cl * S::CPL + c8, kf);
#pragma unroll
          for (int g = 0; g < G; ++g)
#pragma unroll
            for (int c = 0; c < 8; ++c) dots[g] = fmaf(qv[g][c8 + c], kf[c], dots[g]);
        }
      }
      attn_transpose_reduce<G, LPR>(dots, lane);
      constexpr int NV = G >= LPR ? G / LPR : 1;
      constexpr int REP = G >= LPR ? 1 : LPR / G;
      if (r < TR && (cl % REP) == 0) {
        const float ks = valid ? st_ks[s][r / PR] : 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int g = G >= LPR ? cl * NV + i : cl / REP;
          s_s[g][r] = valid ? dots[i] * ks : -INFINITY;
        }
      }
    }
    __syncthreads();
    // ---- online softmax, warp g owns head g
    if (warp < G) {
      const int g = warp;
      float x0 = lane < TR ? s_s[g][lane] : -INFINITY;
      float x1 = lane + 32 < TR ? s_s[g][lane + 32] : -INFINITY;
      float mt = fmaxf(x0, x1);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
      const float m_new = fmaxf(m_run, mt);
      float alpha = 1.f, p0 = 0.f, p1 = 0.f;
      if (m_new != -INFINITY) {
        alpha = exp2f(m_run - m_new);
        p0 = exp2f(x0 - m_new);
        p1 = exp2f(x1 - m_new);
      }
      float ps = p0 + p1;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l_run = l_run * alpha + ps;
      m_run = m_new;
      const unsigned long long rows = st_rows[s];
      if (lane < TR) p_s[lane][g] = ((rows >> lane) & 1ull) ? p0 * st_vs[s][lane / PR] : 0.f;
      if (lane + 32 < TR) p_s[lane + 32][g] = ((rows >> (lane + 32)) & 1ull) ? p1 * st_vs[s][(lane + 32) / PR] : 0.f;
      if (lane == 0) alpha_s[g] = alpha;
    }
    __syncthreads();
    // ---- PV
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float a = alpha_s[g];
      acc[g][0] *= a;
      acc[g][1] *= a;
    }
    for (int r = rg; r < TR; r += S::NRG) {
      if (!((rows >> r) & 1ull)) continue;
      const float2 v2 = load2(Vs + r * D + cp * 2);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pr = p_s[r][g];
        acc[g][0] = fmaf(pr, v2.x, acc[g][0]);
        acc[g][1] = fmaf(pr, v2.y, acc[g][1]);
      }
    }
    __syncthreads();  // stage s fully consumed
    if (warp == 0 && tile + STAGES < n_tiles) issue(tile + STAGES, s);
  }

  // ---- unwind after a give-up: wait (bounded) for copies still in flight
  if (sh_abort) {
    if (tid == 0) {
      for (int64_t tile = consumed; tile < n_tiles && tile < consumed + STAGES; ++tile) {
        const int s = static_cast<int>(tile % STAGES);
        (void)mbar_wait_bounded(&full_bar[s], static_cast<uint32_t>((tile / STAGES) & 1));
      }
    }
    __syncthreads();
  }

  // ---- reduce the PV row groups and write
  if (warp < G && lane == 0) {
    m_fin[warp] = m_run;
    l_fin[warp] = l_run;
  }
  float* red = reinterpret_cast<float*>(ring);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    red[(rg * G + g) * D + cp * 2] = acc[g][0];
    red[(rg * G + g) * D + cp * 2 + 1] = acc[g][1];
  }
  __syncthreads();
  const int64_t rows_total = p.B * p.Hq * p.Tq;
  for (int idx = tid; idx < G * D; idx += 256) {
    const int g = idx / D, c = idx % D;
    if (g >= n_heads_here) continue;
    float sum = 0.f;
#pragma unroll 4
    for (int r = 0; r < S::NRG; ++r) sum += red[(r * G + g) * D + c];
    const float l = l_fin[g];
    const float o = l > 0.f ? sum / l : 0.f;
    const int64_t h = h0 + g;
    const int64_t row = (b * p.Hq + h) * p.Tq + t;
    const float lse = l > 0.f ? (m_fin[g] + log2f(l)) * 0.69314718055994531f : -INFINITY;
    if (p.n_splits == 1) {
      store_any(p.out, b * p.os[0] + h * p.os[1] + t * p.os[2] + c * p.os[3], p.out_dtype, o);
      if (p.lse_out && c == 0) p.lse_out[row] = lse;
    } else {
      p.ws_o[(static_cast<int64_t>(split) * rows_total + row) * D + c] = o;
      if (c == 0) p.ws_lse[static_cast<int64_t>(split) * rows_total + row] = lse;
    }
  }
}

}  // namespace linattn
