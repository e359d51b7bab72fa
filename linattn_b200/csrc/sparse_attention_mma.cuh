// Sparse (paged, block-list) attention on the tensor cores, for 16-bit and fp8 KV.
//
// Work: the (batch, list head, query, head chunk) units of linattn_sparse_attention,
// each cut into `n_splits` equal slices of its page list ("items").  A persistent
// grid (one CTA of NW warps per SM) hands items out through an atomic counter, so
// ragged lists (GQA unions of different sizes) leave no tail.
//
// Every warp is self-contained (no inter-warp signalling after set-up):
// * it grabs items and resolves each item's list entries once (list id -> page
//   table -> physical page -> row of the [rows, D] view of the pool) into one of two
//   shared-memory table slots, one item ahead and while its ring is full, so the
//   global-load latency overlaps the copies in flight;
// * it keeps its STG-stage ring of TRW-row tiles full from the tables: per tile,
//   one lane per row decides whether the row is read (position < the causal or
//   sequence limit), lane 0 arms the stage's mbarrier with the byte count, and the
//   first lane of each page segment issues TMA tiled loads through tensor maps over
//   the K and V pools (64-column x box_rows boxes, 128-byte swizzle, no multicast);
// * it computes with the heads as the narrow dimension: S^T = K Q^T and
//   O^T += V^T P^T with mma.sync m16n8k16, tokens / channels as the 16-row M side and
//   up to 8 query heads of the GQA group as N = 8.  K and V^T fragments come from
//   ldmatrix (plain / .trans) on the swizzled tiles (the swizzle XORs each 16-byte
//   chunk index with the row mod 8, so every phase hits eight bank groups); P^T moves
//   from the accumulator layout to the B-operand layout with movmatrix.trans.  The
//   online softmax runs per head (column) in the log2 domain; P is split into two
//   16-bit parts (hi + lo) so its rounding stays near fp32 precision, and the running
//   sum uses the unrounded fp32 P.
// fp8 (e4m3, one scale per (page, kv head)) KV, D = 128, pages of >= 32 rows: tiles of
// 32 one-byte rows (one 128-byte box row each, same 4 KiB per K or V tile), so a tile
// never spans two pages and its two scales are per-tile constants.  Fragments come
// straight from the swizzled tile (no ldmatrix):
// * S^T = K Q^T runs on the e4m3 tensor-core mma (m16n8k32) with the K codes as they
//   are: the channels are permuted identically in q and K so that a lane's A fragments
//   are two 16-byte loads per row.  q (times a per-head power of two putting its
//   largest |q| in [2^7, 2^8)) is split into NQT e4m3 terms q1 + q2/16 (+ q3/256),
//   each an mma of its own: two terms hold a bf16 q exactly, three an f16 q (every
//   element down to 2^-13 of the largest).  The K scale folds into the score scale.
// * O^T += V^T P^T runs in f16: V^T fragments pair two tokens per channel with byte
//   permutes and convert them exactly (cvt e4m3x2 -> f16x2); the output channels are
//   permuted instead (undone in the epilogue).  P is a single f16 part carrying the
//   ratio of the page's V scale to the one o is kept in (o is rebased when that ratio
//   leaves [2^-4, 2^4]).
// Every wait is bounded (a give-up reports LINATTN_DEV_TIMEOUT and unwinds after
// waiting, bounded, for the copies in flight).
#pragma once

#include <cuda.h>

#include <type_traits>

#include "sparse_attention.cuh"

namespace linattn {

template <typename T> struct MmaOp;
template <> struct MmaOp<__nv_bfloat16> {
  __device__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ static uint32_t pack(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
  __device__ static float2 unpack(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  }
};
template <> struct MmaOp<__half> {
  __device__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ static uint32_t pack(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
  __device__ static float2 unpack(uint32_t v) { return __half22float2(*reinterpret_cast<const __half2*>(&v)); }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Geometry for head_dim D and EB-byte KV elements: every K or V tile is 4 KiB
// (D=128: 16 rows of bf16/f16 or 32 rows of fp8; D=64 16-bit: 32 rows).
template <int D, int EB = 2>
struct MmaShape {
  static constexpr int ROWB = D * EB;             // bytes per K/V row
  static constexpr int TRW = 4096 / ROWB;         // tile rows
  static constexpr int NHALF = ROWB / 128;        // 128-byte column blocks
  static constexpr int HALF_BYTES = TRW * 128;    // one column block of a tile
  static constexpr int TILE_BYTES = NHALF * HALF_BYTES;  // one of K or V (4 KiB)
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int STG = 3;                   // stages per warp
  static constexpr int NW = 8;                    // warps per CTA
  static constexpr int ITEM_MAX = 128;            // list entries per item (host guarantees)
  static constexpr int ENT_BYTES = EB == 1 ? 16 : 8;  // table entry: int2, or int4 with the fp8 scales
  static constexpr size_t RING_BYTES = static_cast<size_t>(NW) * STG * STAGE_BYTES;
  static constexpr size_t TABLE_BYTES = static_cast<size_t>(NW) * 2 * ITEM_MAX * ENT_BYTES;
  static constexpr size_t SMEM_BYTES = 1024 + RING_BYTES + TABLE_BYTES;  // + alignment slack
  static constexpr int MT = TRW / 16;             // token 16-blocks per tile
  static constexpr int KS = D / 16;               // channel 16-blocks
  static_assert(NHALF >= 1 && TRW <= 32, "tile geometry");
};

// An item as resolved by its warp (one of two slots per warp).
struct MmaItem {
  int32_t b, t, h0, n_heads, split, n, n_tiles, limit;
};

// A filled ring stage as the consumer sees it (two 16-byte words).
struct __align__(16) MmaStage {
  uint32_t rows;   // valid-row mask of the tile
  uint32_t holes;  // rows a box wrote that the tile does not use
  int32_t b, t;
  uint32_t h0nh;   // first head | n_heads << 24 | first tile << 30 | last tile << 31
  int32_t split;
  float ks, vs;    // fp8: the tile's page scales (a tile never spans two pages)
};

// Swizzled byte offset of 16-byte chunk `chunk` (0 .. ROWB/16-1) of tile row `row`.
template <int D, int EB = 2>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>((chunk >> 3) * MmaShape<D, EB>::HALF_BYTES + row * 128 +
                               (((chunk & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

// The two e4m3 codes in the low 16 bits of v (low byte first) -> f16x2 (low half
// first), exactly: every e4m3 value is an f16.
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v & 0xffffu), __NV_E4M3);
  return static_cast<uint32_t>(h.x) | (static_cast<uint32_t>(h.y) << 16);
}

// d += a * b over k = 32 e4m3 codes per row (fp32 accumulation).
__device__ __forceinline__ void mma_e4m3(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t word_of(const uint4& u, int i) {
  return i == 0 ? u.x : i == 1 ? u.y : i == 2 ? u.z : u.w;
}

// T: the KV element type (bf16 / f16, or fp8e4m3 for the fp8 mode described at the
// top of the file); D: head_dim; NQT: fp8 mode, e4m3 terms of q (2 for a bf16 q, 3 for
// an f16 q).
template <typename T, int D, int NQT = 1>
__global__ void __launch_bounds__(32 * MmaShape<D, sizeof(T)>::NW, 1)
    sparse_attention_mma_kernel(const AttnParams p, const __grid_constant__ CUtensorMap tmk,
                                const __grid_constant__ CUtensorMap tmv, int box_rows, int* __restrict__ counter,
                                int64_t n_items) {
  constexpr bool F8 = sizeof(T) == 1;
  static_assert(!F8 || D == 128, "fp8 tiles hold one 128-byte row per token");
  static_assert(!F8 || NQT == 2 || NQT == 3, "fp8 mode splits q into 2 or 3 terms");
  using S = MmaShape<D, sizeof(T)>;
  using M = MmaOp<std::conditional_t<F8, __half, T>>;
  using Ent = std::conditional_t<F8, int4, int2>;  // {row position, pool row[, k scale, v scale]}
  constexpr int TRW = S::TRW, STG = S::STG;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // 128-byte swizzled TMA destinations want 1024-byte alignment
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  __shared__ __align__(8) uint64_t full_bar[S::NW][STG];
  __shared__ MmaStage st[S::NW][STG];
  __shared__ MmaItem items[S::NW][2];

  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint8_t* ring = smem + static_cast<size_t>(w) * STG * S::STAGE_BYTES;
  Ent* tables = reinterpret_cast<Ent*>(smem + S::RING_BYTES) + w * 2 * S::ITEM_MAX;
  if (lane == 0) {
    for (int s = 0; s < STG; ++s) mbar_init(&full_bar[w][s], 1);
    mbar_fence_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmv)) : "memory");
  }
  // rows never copied must hold finite values
  for (int i = lane; i < STG * S::STAGE_BYTES / 16; i += 32)
    reinterpret_cast<uint4*>(ring)[i] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  // launched as a programmatic dependent: everything above is set-up; the lists, the
  // counter and q may come from the previous kernel, so wait for it (a no-op when
  // nothing is in flight before this launch).  The split merge behind this launch may
  // start its own set-up now.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int64_t S_ = p.n_splits;
  const int64_t P = p.kv.page_size;
  const int64_t heads_per_kv = p.Hq / p.kv.n_kv_heads;
  const int64_t rows_total = p.B * p.Hq * p.Tq;
  const bool small_pages = P <= TRW;
  const int64_t PPT = small_pages ? TRW / P : 1;
  const int64_t segs = small_pages ? 1 : (P + TRW - 1) / TRW;
  // per-tile row -> (entry, row in page) in 32-bit arithmetic; shifts when P and the
  // segment count are powers of two (the common case), division otherwise
  const int P32 = static_cast<int>(P), PPT32 = static_cast<int>(PPT), segs32 = static_cast<int>(segs);
  const bool pow2 = (P32 & (P32 - 1)) == 0 && (segs32 & (segs32 - 1)) == 0;
  const int p_shift = __ffs(P32) - 1, seg_shift = __ffs(segs32) - 1;

  // ---- item resolution: grab items until one has tiles (writing empty ones)
  int res_count = 0;           // items resolved into slots so far
  bool exhausted = false;      // the counter ran past n_items
  auto resolve = [&]() {
    const int k = res_count & 1;
    while (true) {
      int v = 0;
      if (lane == 0) v = atomicAdd(counter, 1);
      const int64_t item = static_cast<int64_t>(__shfl_sync(0xffffffffu, v, 0));
      if (item >= n_items) {
        exhausted = true;
        return;
      }
      int64_t x = item;
      const int split = static_cast<int>(x % S_);
      x /= S_;
      const int hc = static_cast<int>(x % p.n_head_chunks);
      const int64_t unit = x / p.n_head_chunks;
      const int64_t t = unit % p.Tq;
      const int64_t lh = (unit / p.Tq) % p.lists.n_heads;
      const int64_t b = unit / (p.Tq * p.lists.n_heads);
      const int64_t h0 = lh * p.heads_per_list + hc * 8;
      const int nh = static_cast<int>(lmin(8, p.heads_per_list - hc * 8));
      const int64_t lbase = b * p.lists.stride_b + lh * p.lists.stride_h + t * p.lists.stride_t;
      int64_t len = p.lists.max_len;
      if (p.lists.counts)
        len = lmin(len, p.lists.counts[b * p.lists.cstride_b + lh * p.lists.cstride_h + t * p.lists.cstride_t]);
      const int64_t per = (len + S_ - 1) / S_;
      const int64_t j0 = lmin(len, split * per);
      const int64_t n = lmin(lmin(len, j0 + per) - j0, S::ITEM_MAX);
      const int64_t ntiles = small_pages ? (n + PPT - 1) / PPT : n * segs;
      if (ntiles == 0) {
        // empty item: (o, lse) = (0, -inf)
        for (int g = 0; g < nh; ++g) {
          const int64_t h = h0 + g;
          const int64_t row = (b * p.Hq + h) * p.Tq + t;
          if (p.n_splits == 1) {
            for (int cc = lane; cc < D; cc += 32)
              store_any(p.out, b * p.os[0] + h * p.os[1] + t * p.os[2] + cc * p.os[3], p.out_dtype, 0.f);
            if (p.lse_out && lane == 0) p.lse_out[row] = -INFINITY;
          } else if (lane == 0) {
            p.ws_lse[static_cast<int64_t>(split) * rows_total + row] = -INFINITY;
          }
        }
        continue;
      }
      const int64_t len_b = p.kv.seq_lens ? static_cast<int64_t>(p.kv.seq_lens[b]) : p.kv.seq_len;
      const int64_t kvh = h0 / heads_per_kv;
      Ent* table = tables + k * S::ITEM_MAX;
      for (int64_t e = lane; e < n; e += 32) {
        const int64_t id = p.lists.ids_dtype == LINATTN_I64
                               ? static_cast<const int64_t*>(p.lists.ids)[lbase + j0 + e]
                               : static_cast<int64_t>(static_cast<const int32_t*>(p.lists.ids)[lbase + j0 + e]);
        int rowpos = -1, y0 = 0;
        float ksc = 0.f, vsc = 0.f;
        if (id >= 0 && id * P < len_b) {
          int64_t ph = id;
          if (p.kv.page_table) {
            ph = id < p.kv.page_table_stride ? p.kv.page_table[b * p.kv.page_table_stride + id] : -1;
            if (ph < 0 || ph >= p.kv.num_phys_pages) {
              report(p.status, LINATTN_DEV_BAD_ID);
              ph = -1;
            }
          }
          if (ph >= 0) {
            rowpos = static_cast<int>(id * P);
            // first row of this (page, kv head) in the [rows, D] view of the pool
            y0 = static_cast<int>((b * p.kv.stride_b + ph * p.kv.stride_page + kvh * p.kv.stride_head) / D);
            if constexpr (F8) {
              const int64_t si = ph * p.kv.scale_stride_page + kvh * p.kv.scale_stride_head;
              ksc = p.kv.k_scale[si];
              vsc = p.kv.v_scale[si];
            }
          }
        }
        if constexpr (F8)
          table[e] = make_int4(rowpos, y0, __float_as_int(ksc), __float_as_int(vsc));
        else
          table[e] = make_int2(rowpos, y0);
      }
      if (lane == 0) {
        MmaItem& d = items[w][k];
        d.b = static_cast<int32_t>(b);
        d.t = static_cast<int32_t>(t);
        d.h0 = static_cast<int32_t>(h0);
        d.n_heads = nh;
        d.split = split;
        d.n = static_cast<int32_t>(n);
        d.n_tiles = static_cast<int32_t>(ntiles);
        d.limit = static_cast<int32_t>(p.causal ? lmin(len_b, p.offset + t + 1) : len_b);
      }
      __syncwarp();
      ++res_count;
      return;
    }
  };

  // ---- production: item pi of the resolved sequence, tile ptile of it, into ring
  // stage ps.  The item's fields live in registers from its first tile on.  Returns
  // false when the next tile needs an item that is not resolved yet (or none is left).
  int pi = 0, ptile = 0, ps = 0, in_flight = 0;
  int p_ntiles = -1, p_n = 0, p_limit = 0, p_b = 0, p_t = 0, p_split = 0;
  uint32_t p_h0nh = 0u;
  auto issue = [&]() -> bool {
    while (true) {
      if (pi >= res_count) return false;
      if (p_ntiles < 0) {
        const MmaItem& it = items[w][pi & 1];
        p_ntiles = it.n_tiles;
        p_n = it.n;
        p_limit = it.limit;
        p_b = it.b;
        p_t = it.t;
        p_split = it.split;
        p_h0nh = static_cast<uint32_t>(it.h0) | (static_cast<uint32_t>(it.n_heads) << 24);
      }
      if (ptile < p_ntiles) break;
      ++pi;  // the slot of item pi-1 is free again
      ptile = 0;
      p_ntiles = -1;
    }
    const Ent* table = tables + (pi & 1) * S::ITEM_MAX;
    const int s = ps;
    uint8_t* kdst = ring + static_cast<size_t>(s) * S::STAGE_BYTES;
    uint8_t* vdst = kdst + S::TILE_BYTES;
    const int k = ptile;
    const int r = lane;
    int e, rp, slot;
    if (small_pages) {
      slot = pow2 ? (r >> p_shift) : r / P32;
      rp = pow2 ? (r & (P32 - 1)) : r - slot * P32;
      e = k * PPT32 + slot;
    } else {
      slot = 0;
      e = pow2 ? (k >> seg_shift) : k / segs32;
      rp = (k - e * segs32) * TRW + r;
    }
    bool valid = false;
    int y = 0;
    float tks = 0.f, tvs = 0.f;  // fp8: row 0's page scales are the tile's (pages >= TRW rows)
    if (r < TRW && slot < PPT32 && e < p_n && rp < P32) {
      const Ent ent = table[e];
      valid = ent.x >= 0 && ent.x + rp < p_limit;
      y = ent.y + rp;
      if constexpr (F8) {
        tks = __int_as_float(ent.z);
        tvs = __int_as_float(ent.w);
      }
    }
    const uint32_t mask = __ballot_sync(0xffffffffu, valid);
    const uint32_t box_mask = box_rows >= 32 ? 0xffffffffu : ((1u << box_rows) - 1u);
    int n_boxes = 0;
    uint32_t loaded = 0u;
    for (int r0b = 0; r0b < TRW; r0b += box_rows)
      if ((mask >> r0b) & box_mask) {
        ++n_boxes;
        loaded |= box_mask << r0b;
      }
    if (lane == 0) {
      MmaStage m;
      m.rows = mask;
      m.holes = loaded & ~mask;
      m.b = p_b;
      m.t = p_t;
      m.h0nh = p_h0nh | (k == 0 ? 1u << 30 : 0u) | (k + 1 == p_ntiles ? 1u << 31 : 0u);
      m.split = p_split;
      m.ks = tks;
      m.vs = tvs;
      st[w][s] = m;
      mbar_arrive_expect_tx(&full_bar[w][s], static_cast<uint32_t>(n_boxes) * S::NHALF * box_rows * 128u * 2u);
    }
    __syncwarp();
    if (r < TRW && (r & (box_rows - 1)) == 0 && ((mask >> r) & box_mask)) {
#pragma unroll
      for (int h = 0; h < S::NHALF; ++h) {
        tma_load_2d(kdst + h * S::HALF_BYTES + r * 128, &tmk, h * (128 * D / S::ROWB), y, &full_bar[w][s]);
        tma_load_2d(vdst + h * S::HALF_BYTES + r * 128, &tmv, h * (128 * D / S::ROWB), y, &full_bar[w][s]);
      }
    }
    ++ptile;
    ps = ps + 1 == STG ? 0 : ps + 1;
    ++in_flight;
    return true;
  };

  // ---- consumer state
  const int mi = lane >> 3, ri = lane & 7;
  const int hA = (lane & 3) * 2;   // this thread's two heads (accumulator columns)
  const int tk = lane >> 2;        // its token / channel row within a 16-row block
  const int lq = lane & 3;         // its quad position (k pairs 2lq, 2lq+1, 2lq+8, 2lq+9)
  // q B fragments: 16-bit KV, per channel block; fp8, term t / k-step j at [4t + j]
  uint32_t qb[F8 ? 4 * NQT : S::KS][2];
  float o[S::KS][4];               // O^T: channel blocks x (row tk, tk+8) x heads (hA, hA+1)
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  int32_t cb = 0, ct = 0, ch0 = 0, cnh = 0, csplit = 0;
  const float sl2 = p.scale_log2;
  // fp8: the q power-of-two factors undone on heads hA, hA+1, and the V scale that o is
  // currently expressed in (o_true = o * cvs; 0 until a page with a nonzero V scale)
  float qfA = 1.f, qfB = 1.f, cvs = 1.f;
  const uint32_t ring_s = smem_u32(ring);

  int cs = 0;          // ring stage consumed next
  uint32_t cph = 0u;   // its fill phase parity
  bool abort = false;
  while (true) {
    // keep one item resolved ahead of production (the loads overlap the copies in
    // flight), then top the ring up; both have exactly one call site
    if (!exhausted && res_count <= pi + 1) resolve();
    while (in_flight < STG && issue()) {
    }
    if (in_flight == 0) {
      if (exhausted && pi >= res_count) break;
      continue;
    }
    const int s = cs;
    // the stage record was written when the tile was issued: an item's q loads and
    // set-up go out before the wait for its first tile, so their latency overlaps it
    const MmaStage sd = st[w][s];
    const bool first = (sd.h0nh >> 30) & 1u, last = sd.h0nh >> 31;
    if (first) {
      cb = sd.b;
      ct = sd.t;
      ch0 = static_cast<int32_t>(sd.h0nh & 0xffffffu);
      cnh = static_cast<int32_t>((sd.h0nh >> 24) & 0x3fu);
      csplit = sd.split;
      const int64_t qoff = static_cast<int64_t>(cb) * p.qs[0] + static_cast<int64_t>(ch0 + tk) * p.qs[1] +
                           static_cast<int64_t>(ct) * p.qs[2];
      if constexpr (F8) {
        // Channels are permuted identically in q and K (the sum over them is unchanged):
        // in k-step j, this lane's A / B k-quads (4lq .. 4lq+3) and (16+4lq .. 16+4lq+3)
        // are channels 32lq + 8j + {0..3} and {4..7}, so a lane reads 32 contiguous K
        // bytes per row (chunks 2lq, 2lq+1) and 32 contiguous q channels.
        float v[32];
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = tk < cnh ? load_any(p.q, qoff + static_cast<int64_t>(32 * lq + i) * p.qs[3], p.q_dtype) : 0.f;
          amax = fmaxf(amax, fabsf(v[i]));
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const int ex = amax > 0.f ? static_cast<int>((__float_as_uint(amax) >> 23) & 0xffu) - 127 : 0;
        const int e2 = max(-126, min(126, 7 - ex));  // both 2^e2 and 2^-e2 stay normal floats
        const float up = __uint_as_float(static_cast<uint32_t>(127 + e2) << 23);
        const float down = __uint_as_float(static_cast<uint32_t>(127 - e2) << 23);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= up;
        // term t: e4m3 (round to nearest even) of 16^t times what the earlier terms left
#pragma unroll
        for (int t = 0; t < NQT; ++t) {
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            uint32_t word = 0u;
#pragma unroll
            for (int hp = 0; hp < 2; ++hp) {
              const int i = 4 * r + 2 * hp;
              const uint32_t c2 = __nv_cvt_float2_to_fp8x2(make_float2(v[i], v[i + 1]), __NV_SATFINITE, __NV_E4M3);
              word |= c2 << (16 * hp);
              const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(c2), __NV_E4M3);
              const float2 back = __half22float2(*reinterpret_cast<const __half2*>(&h));
              v[i] = (v[i] - back.x) * 16.f;
              v[i + 1] = (v[i + 1] - back.y) * 16.f;
            }
            qb[4 * t + (r >> 1)][r & 1] = word;
          }
        }
        qfA = __shfl_sync(0xffffffffu, down, hA * 4);
        qfB = __shfl_sync(0xffffffffu, down, hA * 4 + 4);
        cvs = 0.f;
      } else {
        const T* qrow = static_cast<const T*>(p.q) + qoff;
#pragma unroll
        for (int kk = 0; kk < S::KS; ++kk) {
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int col = kk * 16 + hA + (e >> 1) * 8 + (e & 1);  // B fragment: k = channels, n = head tk
            v[e] = tk < cnh ? to_float(qrow[col * p.qs[3]]) : 0.f;
          }
          qb[kk][0] = M::pack(v[0], v[1]);
          qb[kk][1] = M::pack(v[2], v[3]);
        }
      }
#pragma unroll
      for (int n = 0; n < S::KS; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      mA = mB = -INFINITY;
      lA = lB = 0.f;
    }
    if (!mbar_wait_bounded(&full_bar[w][s], cph)) {
      report(p.status, LINATTN_DEV_TIMEOUT);
      abort = true;
      break;
    }
    const uint32_t kst = ring_s + static_cast<uint32_t>(s) * S::STAGE_BYTES;
    const uint32_t vst = kst + S::TILE_BYTES;
    const uint8_t* kptr = ring + static_cast<size_t>(s) * S::STAGE_BYTES;
    const uint8_t* vptr = kptr + S::TILE_BYTES;
    // rows a box brought in but the tile does not use: zero their V so that P = 0
    // meets finite values in P V
    const uint32_t holes = sd.holes;
    if (holes) {
      uint8_t* vrows = ring + static_cast<size_t>(s) * S::STAGE_BYTES + S::TILE_BYTES;
      constexpr int CPR = S::ROWB / 16;  // 16-byte chunks per row
      for (int i = lane; i < TRW * CPR; i += 32) {
        const int row = i / CPR, chunk = i % CPR;
        if ((holes >> row) & 1u)
          *reinterpret_cast<uint4*>(vrows + swz<D, sizeof(T)>(row, chunk)) = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }
    // ---- S^T = K Q^T: tokens (16 per block) x heads (8)
    float sc[S::MT][4], sc2[S::MT][4];  // two accumulation chains (even / odd channel blocks)
#pragma unroll
    for (int mt = 0; mt < S::MT; ++mt) {
      sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.f;
      sc2[mt][0] = sc2[mt][1] = sc2[mt][2] = sc2[mt][3] = 0.f;
    }
    if constexpr (F8) {
#pragma unroll
      for (int mt = 0; mt < S::MT; ++mt) {
        // rows tk and tk+8 of the block, chunks 2lq and 2lq+1 (lanes of a quarter warp
        // hit 8 distinct chunks under the swizzle)
        uint4 k0[2], k1[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          k0[h] = *reinterpret_cast<const uint4*>(kptr + swz<D, 1>(mt * 16 + tk, 2 * lq + h));
          k1[h] = *reinterpret_cast<const uint4*>(kptr + swz<D, 1>(mt * 16 + tk + 8, 2 * lq + h));
        }
        float acc[NQT][4];
#pragma unroll
        for (int t = 0; t < NQT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int h = j >> 1, wd = 2 * (j & 1);
          const uint32_t a0 = word_of(k0[h], wd), a1 = word_of(k1[h], wd);
          const uint32_t a2 = word_of(k0[h], wd + 1), a3 = word_of(k1[h], wd + 1);
#pragma unroll
          for (int t = 0; t < NQT; ++t) mma_e4m3(acc[t], a0, a1, a2, a3, qb[4 * t + j][0], qb[4 * t + j][1]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float x = fmaf(acc[1][i], 0.0625f, acc[0][i]);
          if constexpr (NQT == 3) x = fmaf(acc[2][i], 0.00390625f, x);
          sc[mt][i] = x;
        }
      }
    } else {
#pragma unroll
      for (int kk = 0; kk < S::KS; ++kk) {
#pragma unroll
        for (int mt = 0; mt < S::MT; ++mt) {
          uint32_t a[4];
          ldsm_x4(kst + swz<D>(mt * 16 + (mi & 1) * 8 + ri, kk * 2 + (mi >> 1)), a[0], a[1], a[2], a[3]);
          M::mma((kk & 1) ? sc2[mt] : sc[mt], a, qb[kk][0], qb[kk][1]);
        }
      }
    }
#pragma unroll
    for (int mt = 0; mt < S::MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[mt][i] += sc2[mt][i];
    // ---- online softmax per head (column); unread rows -> -inf.  The running maxima
    // mA / mB are lazy: they move only when a score exceeds them by more than 8 (log2
    // domain; one warp vote per tile), so P <= 2^8, and o is rescaled only then.  The
    // row sums lA / lB are per-lane partials (this lane's rows), summed over the lanes
    // of a head column once, at the end of the item.  fp8: P also carries vs / cvs
    // (exp2 offset lr) and the row sums take it back out (ir).
    const float fA = F8 ? sl2 * sd.ks * qfA : sl2, fB = F8 ? sl2 * sd.ks * qfB : sl2;
    bool over = false;
#pragma unroll
    for (int mt = 0; mt < S::MT; ++mt) {
      const bool v0 = (sd.rows >> (mt * 16 + tk)) & 1u;
      const bool v1 = (sd.rows >> (mt * 16 + tk + 8)) & 1u;
      sc[mt][0] = v0 ? sc[mt][0] * fA : -INFINITY;
      sc[mt][1] = v0 ? sc[mt][1] * fB : -INFINITY;
      sc[mt][2] = v1 ? sc[mt][2] * fA : -INFINITY;
      sc[mt][3] = v1 ? sc[mt][3] * fB : -INFINITY;
      over |= fmaxf(sc[mt][0], sc[mt][2]) > mA + 8.f || fmaxf(sc[mt][1], sc[mt][3]) > mB + 8.f;
    }
    float lr = 0.f, ir = 1.f;
    bool pv = true, rebase = false;
    if constexpr (F8) {
      if (sd.vs == 0.f) {
        pv = false;  // the page's V is 0: it adds nothing to o
      } else if (cvs == 0.f) {
        cvs = sd.vs;  // first page with a V scale: o is still 0
      } else if (sd.vs != cvs) {
        lr = log2f(sd.vs / cvs);
        if (fabsf(lr) > 4.f) {
          rebase = true;
          lr = 0.f;
        } else {
          ir = cvs / sd.vs;
        }
      }
    }
    if (rebase || __any_sync(0xffffffffu, over)) {
      float tA = -INFINITY, tB = -INFINITY;
#pragma unroll
      for (int mt = 0; mt < S::MT; ++mt) {
        tA = fmaxf(tA, fmaxf(sc[mt][0], sc[mt][2]));
        tB = fmaxf(tB, fmaxf(sc[mt][1], sc[mt][3]));
      }
#pragma unroll
      for (int off = 4; off <= 16; off <<= 1) {
        tA = fmaxf(tA, __shfl_xor_sync(0xffffffffu, tA, off));
        tB = fmaxf(tB, __shfl_xor_sync(0xffffffffu, tB, off));
      }
      const float nA = fmaxf(mA, tA), nB = fmaxf(mB, tB);
      const float aA = nA == -INFINITY ? 1.f : exp2f(mA - nA);
      const float aB = nB == -INFINITY ? 1.f : exp2f(mB - nB);
      lA *= aA;
      lB *= aB;
      mA = nA;
      mB = nB;
      float oA = aA, oB = aB;
      if (rebase) {
        const float r = cvs / sd.vs;
        oA *= r;
        oB *= r;
        cvs = sd.vs;
      }
#pragma unroll
      for (int n = 0; n < S::KS; ++n) {
        o[n][0] *= oA;
        o[n][1] *= oB;
        o[n][2] *= oA;
        o[n][3] *= oB;
      }
    }
    const float oA_ = mA - lr, oB_ = mB - lr;  // exp2 offsets
    float sA = 0.f, sB = 0.f;
#pragma unroll
    for (int mt = 0; mt < S::MT; ++mt) {
      sc[mt][0] = mA == -INFINITY ? 0.f : exp2f(sc[mt][0] - oA_);
      sc[mt][2] = mA == -INFINITY ? 0.f : exp2f(sc[mt][2] - oA_);
      sc[mt][1] = mB == -INFINITY ? 0.f : exp2f(sc[mt][1] - oB_);
      sc[mt][3] = mB == -INFINITY ? 0.f : exp2f(sc[mt][3] - oB_);
      sA += sc[mt][0] + sc[mt][2];
      sB += sc[mt][1] + sc[mt][3];
    }
    lA = fmaf(sA, ir, lA);
    lB = fmaf(sB, ir, lB);
    if constexpr (F8) {
      // ---- O^T += V^T P^T with one f16 P.  Output rows are permuted: in channel block
      // dm, accumulator rows tk / tk+8 are channels 16tk + 2dm / 16tk + 2dm + 1, so a
      // lane reads one 16-byte chunk (channels 16tk .. 16tk+15) of each of its four
      // token rows (2lq, 2lq+1, 2lq+8, 2lq+9) and pairs tokens per channel with byte
      // permutes.
      if (pv) {
#pragma unroll
        for (int mt = 0; mt < S::MT; ++mt) {
          const uint32_t bh0 = movmatrix_t(M::pack(sc[mt][0], sc[mt][1]));
          const uint32_t bh1 = movmatrix_t(M::pack(sc[mt][2], sc[mt][3]));
          uint4 vw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            vw[i] = *reinterpret_cast<const uint4*>(vptr + swz<D, 1>(mt * 16 + 2 * lq + (i & 1) + (i >> 1) * 8, tk));
#pragma unroll
          for (int dm = 0; dm < S::KS; ++dm) {
            const uint32_t sel = (dm & 1) ? 0x7362u : 0x5140u;
            const uint32_t p01 = __byte_perm(word_of(vw[0], dm >> 1), word_of(vw[1], dm >> 1), sel);
            const uint32_t p89 = __byte_perm(word_of(vw[2], dm >> 1), word_of(vw[3], dm >> 1), sel);
            const uint32_t a[4] = {e4m3x2_f16x2(p01), e4m3x2_f16x2(p01 >> 16), e4m3x2_f16x2(p89),
                                   e4m3x2_f16x2(p89 >> 16)};
            M::mma(o[dm], a, bh0, bh1);
          }
        }
      }
    } else {
      // ---- O^T += V^T P^T  (P = hi + lo in the 16-bit type)
#pragma unroll
      for (int mt = 0; mt < S::MT; ++mt) {
        const uint32_t h0 = M::pack(sc[mt][0], sc[mt][1]);  // tokens tk,   heads hA, hA+1
        const uint32_t h1 = M::pack(sc[mt][2], sc[mt][3]);  // tokens tk+8
        const float2 r0 = M::unpack(h0), r1 = M::unpack(h1);
        const uint32_t l0 = M::pack(sc[mt][0] - r0.x, sc[mt][1] - r0.y);
        const uint32_t l1 = M::pack(sc[mt][2] - r1.x, sc[mt][3] - r1.y);
        const uint32_t bh0 = movmatrix_t(h0), bh1 = movmatrix_t(h1);
        const uint32_t bl0 = movmatrix_t(l0), bl1 = movmatrix_t(l1);
#pragma unroll
        for (int dm = 0; dm < S::KS; ++dm) {
          uint32_t a[4];
          ldsm_x4_t(vst + swz<D>(mt * 16 + (mi >> 1) * 8 + ri, dm * 2 + (mi & 1)), a[0], a[1], a[2], a[3]);
          M::mma(o[dm], a, bh0, bh1);
          M::mma(o[dm], a, bl0, bl1);
        }
      }
    }
    __syncwarp();
    if (holes) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before the next TMA fill
    --in_flight;
    cs = cs + 1 == STG ? 0 : cs + 1;
    if (cs == 0) cph ^= 1u;
    // ---- item finished: write (o, lse) for its heads
    if (last) {
#pragma unroll
      for (int off = 4; off <= 16; off <<= 1) {
        lA += __shfl_xor_sync(0xffffffffu, lA, off);
        lB += __shfl_xor_sync(0xffffffffu, lB, off);
      }
      const float iA = lA > 0.f ? cvs / lA : 0.f, iB = lB > 0.f ? cvs / lB : 0.f;
      const float lseA = lA > 0.f ? (mA + log2f(lA)) * 0.69314718055994531f : -INFINITY;
      const float lseB = lB > 0.f ? (mB + log2f(lB)) * 0.69314718055994531f : -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int g = hA + j;
        if (g >= cnh) continue;
        const int64_t h = ch0 + g;
        const int64_t row = (static_cast<int64_t>(cb) * p.Hq + h) * p.Tq + ct;
        const float inv = j ? iB : iA;
        // (channel, value) pairs of this lane for head g: 16-bit KV rows dm*16+tk and
        // dm*16+tk+8; fp8 channels 16tk .. 16tk+15 in order
        float* wo = nullptr;
        if (p.n_splits == 1) {
          const int64_t ob = static_cast<int64_t>(cb) * p.os[0] + h * p.os[1] + static_cast<int64_t>(ct) * p.os[2];
          if (F8 && p.out_dtype == LINATTN_F32 && p.os[3] == 1) wo = static_cast<float*>(p.out) + ob;
          if (!wo) {
#pragma unroll
            for (int dm = 0; dm < S::KS; ++dm) {
              const int c0 = F8 ? 16 * tk + 2 * dm : dm * 16 + tk, c1 = F8 ? c0 + 1 : c0 + 8;
              store_any(p.out, ob + c0 * p.os[3], p.out_dtype, o[dm][j] * inv);
              store_any(p.out, ob + c1 * p.os[3], p.out_dtype, o[dm][2 + j] * inv);
            }
          }
          if (p.lse_out && tk == 0) p.lse_out[row] = j ? lseB : lseA;
        } else {
          wo = p.ws_o + (static_cast<int64_t>(csplit) * rows_total + row) * D;
          if (tk == 0) p.ws_lse[static_cast<int64_t>(csplit) * rows_total + row] = j ? lseB : lseA;
        }
        if (wo) {
          if constexpr (F8) {
            float* w16 = wo + 16 * tk;
            if ((reinterpret_cast<uintptr_t>(w16) & 15u) == 0) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                reinterpret_cast<float4*>(w16)[i] = make_float4(o[2 * i][j] * inv, o[2 * i][2 + j] * inv,
                                                                o[2 * i + 1][j] * inv, o[2 * i + 1][2 + j] * inv);
            } else {
#pragma unroll
              for (int dm = 0; dm < S::KS; ++dm) {
                w16[2 * dm] = o[dm][j] * inv;
                w16[2 * dm + 1] = o[dm][2 + j] * inv;
              }
            }
          } else {
#pragma unroll
            for (int dm = 0; dm < S::KS; ++dm) {
              wo[dm * 16 + tk] = o[dm][j] * inv;
              wo[dm * 16 + tk + 8] = o[dm][2 + j] * inv;
            }
          }
        }
      }
    }
  }
  if (abort) {
    for (; in_flight > 0; --in_flight) {
      (void)mbar_wait_bounded(&full_bar[w][cs], cph);
      cs = cs + 1 == STG ? 0 : cs + 1;
      if (cs == 0) cph ^= 1u;
    }
  }
}

}  // namespace linattn
