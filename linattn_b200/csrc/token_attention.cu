// Token-sparse attention (DSA / CSA): every query attends to the union of
//   * the tokens of its own list (top-k indexer selection, any order, -1 padded;
//     an entry stands for `block` consecutive tokens: 1 for DSA, the compression
//     ratio for CSA's pooled groups),
//   * the first `sink` tokens, and
//   * the `window` tokens ending at its position,
// restricted to positions < T_k (and <= offset + t when causal).  This is the masked
// attention of BlockSelectionAttention.attend (src/linattn/variants/selection.py:86-116)
// with the DSA selection of DSAAttention.select (:738-763): selection OR sink OR window,
// then causal; the union counts each token once.
//
// One warp per item = (batch, query, chunk of up to 8 query heads that share a kv
// head and a list); items are ordered chunk-major so that the warps in flight read
// one kv head's K / V (L2-resident) at a time.  Per 16-row tile (D = 128; 32 rows for
// D = 64) the warp resolves the tile's tokens (list ids copied three tiles ahead into a
// per-warp ring, then
// the sink and window ranges as virtual entries; list ids inside those ranges are
// dropped) and gathers the K and V rows with zero-filling 16-byte cp.async into a
// 128-byte-swizzled 3-stage ring, each stage completing on an mbarrier through
// cp.async.mbarrier.arrive.noinc (32 arrivals per phase).  The math is the
// transposed formulation of the paged decode kernel: S^T = K Q^T and O^T += V^T P^T
// with mma.sync m16n8k16, heads as the N = 8 side, online softmax per head in the
// log2 domain (hardware ex2; the running maximum lazy, as in the paged kernel: it moves
// only past a margin of 8, one warp vote per tile; row sums per lane until the end),
// P split into 16-bit hi + lo parts, or one f16 part when V
// is given as an f16 copy (a bf16 V scaled by a power of two per (b, kv head), undone
// on the output).
#include <cstdio>

#include "launchers.cuh"
#include "sparse_attention_mma.cuh"

namespace linattn {

struct TokenAttnParams {
  const void* q;
  int q_dtype;
  int64_t qs[4];
  const void* k;
  const void* v;
  int64_t kv_sb, kv_sh, kv_st;  // K / V element strides: batch, kv head, token (rows contiguous)
  int64_t B, Hq, Tq, Tk;
  linattn_lists_t lists;
  int64_t sink, window, block;
  int causal;
  int64_t offset;
  float scale_log2;
  void* out;
  int64_t os[4];
  float* lse_out;
  int32_t* reads_out;  // (B, H_q, T_q) tokens read per query, or NULL
  int diag_fallback;   // a query with nothing to read reads token min(offset + t, T_k - 1)
  const float* v_unscale;  // non-NULL: V is an f16 copy scaled per (b, kv head); o is multiplied back
  int32_t* status;
  int64_t heads_per_kv, heads_per_list, chunk_heads, n_items;
};

namespace {

constexpr int TNW = 8;   // warps per CTA
constexpr int TSTG = 3;  // ring stages per warp (8 warps x 3 x 8 KiB = 192 KiB)
constexpr int TIDR = TSTG + 1;  // list-id ring slots per warp (tiles)

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;  // 0: write 16 zero bytes, read nothing
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_small(uint32_t dst, const void* src, int bytes, bool valid) {
  const int sz = valid ? bytes : 0;
  if (bytes == 8)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

}  // namespace

__device__ __forceinline__ float tok_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// VF16: V arrives as an f16 copy (exact for a bf16 V scaled by a power of two per
// (b, kv head)), so P V takes one f16 P part instead of 16-bit hi + lo parts.
template <typename T, int D, bool VF16>
__global__ void __launch_bounds__(32 * TNW, 1) token_attention_kernel(const TokenAttnParams p) {
  using S = MmaShape<D>;
  using M = MmaOp<T>;
  constexpr int TRW = S::TRW;
  constexpr int CPR = D / 8;                 // 16-byte chunks per row = lanes per row in a copy
  constexpr int RPI = 32 / CPR;              // rows per copy instruction (2 for D = 128, 4 for D = 64)
  constexpr int NCI = TRW / RPI;             // copy instructions per tile, for each of K and V
  extern __shared__ __align__(128) uint8_t tsmem_raw[];
  uint8_t* smem = tsmem_raw + ((1024 - (smem_u32(tsmem_raw) & 1023)) & 1023);
  __shared__ __align__(8) uint64_t full_bar[TNW][TSTG];
  __shared__ uint32_t stage_rows[TNW][TSTG];
  __shared__ __align__(8) int64_t id_ring[TNW][TIDR][MmaShape<D>::TRW];  // raw list ids (int32 in the low word)

  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * TNW + w;
  if (item >= p.n_items) return;
  uint8_t* ring = smem + static_cast<size_t>(w) * TSTG * S::STAGE_BYTES;
  if (lane == 0) {
    for (int s = 0; s < TSTG; ++s) mbar_init(&full_bar[w][s], 32);
    mbar_fence_init();
  }
  __syncwarp();

  // ---- item: chunk-major order (chunk, b, t)
  const int64_t t = item % p.Tq;
  const int64_t b = (item / p.Tq) % p.B;
  const int64_t chunk = item / (p.Tq * p.B);
  const int64_t h0 = chunk * p.chunk_heads;
  const int nh = static_cast<int>(lmin(p.chunk_heads, p.Hq - h0));
  const int64_t kvh = h0 / p.heads_per_kv;
  const int64_t lh = h0 / p.heads_per_list;
  const int64_t lbase = b * p.lists.stride_b + lh * p.lists.stride_h + t * p.lists.stride_t;
  int64_t n_list = p.lists.max_len;
  if (p.lists.counts)
    n_list = lmin(n_list, p.lists.counts[b * p.lists.cstride_b + lh * p.lists.cstride_h + t * p.lists.cstride_t]);
  const int64_t pos = p.offset + t;
  const int64_t limit = p.causal ? lmin(p.Tk, pos + 1) : p.Tk;
  const int64_t n_sink = lmax(0, lmin(p.sink, limit));
  const int64_t w_end = p.window > 0 ? lmin(limit, pos + 1) : 0;
  const int64_t w_lo = p.window > 0 ? lmax(n_sink, pos - p.window + 1) : 0;
  const int64_t n_win = lmax(0, w_end - w_lo);
  const int64_t n_lt = n_list * p.block;  // list tokens
  const int64_t ne = n_lt + n_sink + n_win;
  const int64_t n_tiles = (ne + TRW - 1) / TRW;

  const T* kbase = static_cast<const T*>(p.k) + b * p.kv_sb + kvh * p.kv_sh;
  const T* vbase = static_cast<const T*>(p.v) + b * p.kv_sb + kvh * p.kv_sh;
  const int row = lane % TRW, part = lane / TRW;  // this lane's tile row and chunk range
  // token of virtual token e (-1: not read): list tokens, then the sink and window
  // ranges; list tokens inside those ranges are dropped (the union counts them once)
  auto token_of = [&](int64_t e, int64_t id) -> int64_t {
    if (e < n_lt) {
      const int64_t tok = p.block == 1 ? id : id * p.block + (e - (e / p.block) * p.block);
      const bool ok = id >= 0 && tok < limit && tok >= n_sink && !(tok >= w_lo && tok < w_end);
      return ok ? tok : -1;
    }
    if (e < n_lt + n_sink) return e - n_lt;
    if (e < ne) return w_lo + (e - n_lt - n_sink);
    return -1;
  };
  const bool ids64 = p.lists.ids_dtype == LINATTN_I64;
  const int id_bytes = ids64 ? 8 : 4;
  const char* id_src = static_cast<const char*>(p.lists.ids) + lbase * id_bytes;
  // list ids of tile k's rows (lane r < TRW: row r) -> id-ring slot k % TIDR.  With
  // `async`, a cp.async completing with the stage copies of the issuing tile.
  auto fetch_ids = [&](int64_t k, bool async) {
    if (lane >= TRW) return;
    const int64_t e = k * TRW + lane;
    const bool ok = e < n_lt;
    const int64_t j = !ok ? 0 : (p.block == 1 ? e : e / p.block);
    int64_t* slot = &id_ring[w][k % TIDR][lane];
    if (async) {
      cp_async_small(smem_u32(slot), id_src + j * id_bytes, id_bytes, ok);
    } else {
      *slot = !ok ? 0 : (ids64 ? reinterpret_cast<const int64_t*>(id_src)[j]
                               : static_cast<int64_t>(reinterpret_cast<const int32_t*>(id_src)[j]));
    }
  };
  for (int64_t k = 0; k < TSTG; ++k) fetch_ids(k, false);
  __syncwarp();

  int64_t produced = 0;
  auto issue = [&]() {
    const int s = static_cast<int>(produced % TSTG);
    // this lane's row token (lanes < TRW); the tile's ids arrived TSTG tiles ago
    int32_t tok = -1;
    if (lane < TRW) {
      const int64_t e = produced * TRW + lane;
      int64_t id = -1;
      if (e < n_lt) {
        const int64_t raw = id_ring[w][produced % TIDR][lane];
        id = ids64 ? raw : static_cast<int64_t>(static_cast<int32_t>(raw & 0xffffffffll));
      }
      int64_t t64 = token_of(e, id);
      if (produced == n_tiles)  // the fallback tile: the diagonal token alone
        t64 = (lane == 0 && pos >= 0 && p.Tk > 0) ? lmin(pos, p.Tk - 1) : -1;
      tok = static_cast<int32_t>(t64);
    }
    __syncwarp();
    // ids of tile produced + TSTG, into the slot freed by tile produced - 1
    fetch_ids(produced + TSTG, true);
    const uint32_t kdst = smem_u32(ring + static_cast<size_t>(s) * S::STAGE_BYTES);
    const uint32_t vdst = kdst + S::TILE_BYTES;
    // whole rows per instruction: lanes c of row (i RPI + lane / CPR) copy chunk c
    const int c = lane % CPR;
#pragma unroll
    for (int i = 0; i < NCI; ++i) {
      const int r = i * RPI + lane / CPR;
      const int32_t tr = __shfl_sync(0xffffffffu, tok, r);
      const int64_t ro = static_cast<int64_t>(tr < 0 ? 0 : tr) * p.kv_st + c * 8;
      cp_async16(kdst + swz<D>(r, c), kbase + ro, tr >= 0);
      cp_async16(vdst + swz<D>(r, c), vbase + ro, tr >= 0);
    }
    const uint32_t mask = __ballot_sync(0xffffffffu, lane < TRW && tok >= 0);
    if (lane == 0) stage_rows[w][s] = mask;
    cp_async_arrive(&full_bar[w][s]);
    ++produced;
  };

  // ---- query fragments (B operand: channels x heads)
  const int mi = lane >> 3, ri = lane & 7;
  const int hA = (lane & 3) * 2;
  const int tk = lane >> 2;
  uint32_t qb[S::KS][2];
  {
    const T* qrow = static_cast<const T*>(p.q) + b * p.qs[0] + (h0 + tk) * p.qs[1] + t * p.qs[2];
#pragma unroll
    for (int kk = 0; kk < S::KS; ++kk) {
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = kk * 16 + hA + (e >> 1) * 8 + (e & 1);
        v[e] = tk < nh ? to_float(qrow[col * p.qs[3]]) : 0.f;
      }
      qb[kk][0] = M::pack(v[0], v[1]);
      qb[kk][1] = M::pack(v[2], v[3]);
    }
  }
  float o[S::KS][4];
#pragma unroll
  for (int n = 0; n < S::KS; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  const float sl2 = p.scale_log2;
  const uint32_t ring_s = smem_u32(ring);

  bool abort = false;
  // tiles to run; one more (the diagonal token) if nothing else was read
  int64_t consumed = 0, total = (n_tiles == 0 && p.diag_fallback) ? 1 : n_tiles;
  uint32_t n_read = 0;
  while (consumed < total) {
    while (produced < total && produced - consumed < TSTG) issue();
    const int s = static_cast<int>(consumed % TSTG);
    if (!mbar_wait_bounded(&full_bar[w][s], static_cast<uint32_t>((consumed / TSTG) & 1))) {
      report(p.status, LINATTN_DEV_TIMEOUT);
      abort = true;
      break;
    }
    const uint32_t rows = stage_rows[w][s];
    n_read += __popc(rows);
    const uint32_t kst = ring_s + static_cast<uint32_t>(s) * S::STAGE_BYTES;
    const uint32_t vst = kst + S::TILE_BYTES;
    float sc[S::MT][4], sc2[S::MT][4];
#pragma unroll
    for (int mt = 0; mt < S::MT; ++mt) {
      sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.f;
      sc2[mt][0] = sc2[mt][1] = sc2[mt][2] = sc2[mt][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < S::KS; ++kk) {
#pragma unroll
      for (int mt = 0; mt < S::MT; ++mt) {
        uint32_t a[4];
        ldsm_x4(kst + swz<D>(mt * 16 + (mi & 1) * 8 + ri, kk * 2 + (mi >> 1)), a[0], a[1], a[2], a[3]);
        M::mma((kk & 1) ? sc2[mt] : sc[mt], a, qb[kk][0], qb[kk][1]);
      }
    }
#pragma unroll
    for (int mt = 0; mt < S::MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[mt][i] += sc2[mt][i];
    // online softmax per head (column), the running maxima lazy: they move only when a
    // score exceeds them by more than 8 (log2 units; one warp vote per tile), so P <=
    // 2^8 and o is rescaled only then; the row sums are per-lane partials, summed over
    // a head column's lanes once, after the last tile
    bool over = false;
#pragma unroll
    for (int mt = 0; mt < S::MT; ++mt) {
      const bool v0 = (rows >> (mt * 16 + tk)) & 1u;
      const bool v1 = (rows >> (mt * 16 + tk + 8)) & 1u;
      sc[mt][0] = v0 ? sc[mt][0] * sl2 : -INFINITY;
      sc[mt][1] = v0 ? sc[mt][1] * sl2 : -INFINITY;
      sc[mt][2] = v1 ? sc[mt][2] * sl2 : -INFINITY;
      sc[mt][3] = v1 ? sc[mt][3] * sl2 : -INFINITY;
      over |= fmaxf(sc[mt][0], sc[mt][2]) > mA + 8.f || fmaxf(sc[mt][1], sc[mt][3]) > mB + 8.f;
    }
    if (__any_sync(0xffffffffu, over)) {
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
      const float aA = nA == -INFINITY ? 1.f : tok_ex2(mA - nA);
      const float aB = nB == -INFINITY ? 1.f : tok_ex2(mB - nB);
      lA *= aA;
      lB *= aB;
      mA = nA;
      mB = nB;
#pragma unroll
      for (int n = 0; n < S::KS; ++n) {
        o[n][0] *= aA;
        o[n][1] *= aB;
        o[n][2] *= aA;
        o[n][3] *= aB;
      }
    }
#pragma unroll
    for (int mt = 0; mt < S::MT; ++mt) {
      sc[mt][0] = mA == -INFINITY ? 0.f : tok_ex2(sc[mt][0] - mA);
      sc[mt][2] = mA == -INFINITY ? 0.f : tok_ex2(sc[mt][2] - mA);
      sc[mt][1] = mB == -INFINITY ? 0.f : tok_ex2(sc[mt][1] - mB);
      sc[mt][3] = mB == -INFINITY ? 0.f : tok_ex2(sc[mt][3] - mB);
      lA += sc[mt][0] + sc[mt][2];
      lB += sc[mt][1] + sc[mt][3];
    }
#pragma unroll
    for (int mt = 0; mt < S::MT; ++mt) {
      if constexpr (VF16) {
        using MH = MmaOp<__half>;
        const uint32_t bh0 = movmatrix_t(MH::pack(sc[mt][0], sc[mt][1]));
        const uint32_t bh1 = movmatrix_t(MH::pack(sc[mt][2], sc[mt][3]));
#pragma unroll
        for (int dm = 0; dm < S::KS; ++dm) {
          uint32_t a[4];
          ldsm_x4_t(vst + swz<D>(mt * 16 + (mi >> 1) * 8 + ri, dm * 2 + (mi & 1)), a[0], a[1], a[2], a[3]);
          MH::mma(o[dm], a, bh0, bh1);
        }
        continue;
      }
      const uint32_t h0p = M::pack(sc[mt][0], sc[mt][1]);
      const uint32_t h1p = M::pack(sc[mt][2], sc[mt][3]);
      const float2 r0 = M::unpack(h0p), r1 = M::unpack(h1p);
      const uint32_t l0 = M::pack(sc[mt][0] - r0.x, sc[mt][1] - r0.y);
      const uint32_t l1 = M::pack(sc[mt][2] - r1.x, sc[mt][3] - r1.y);
      const uint32_t bh0 = movmatrix_t(h0p), bh1 = movmatrix_t(h1p);
      const uint32_t bl0 = movmatrix_t(l0), bl1 = movmatrix_t(l1);
#pragma unroll
      for (int dm = 0; dm < S::KS; ++dm) {
        uint32_t a[4];
        ldsm_x4_t(vst + swz<D>(mt * 16 + (mi >> 1) * 8 + ri, dm * 2 + (mi & 1)), a[0], a[1], a[2], a[3]);
        M::mma(o[dm], a, bh0, bh1);
        M::mma(o[dm], a, bl0, bl1);
      }
    }
    __syncwarp();  // every lane is done with the stage before it is refilled
    ++consumed;
    if (consumed == n_tiles && total == n_tiles && n_read == 0 && p.diag_fallback) total = n_tiles + 1;
  }
  if (abort) {
    for (int64_t c2 = consumed; c2 < produced; ++c2)
      (void)mbar_wait_bounded(&full_bar[w][c2 % TSTG], static_cast<uint32_t>((c2 / TSTG) & 1), 200000000ull);
    return;
  }
  // ---- (o, lse) of the item's heads
#pragma unroll
  for (int off = 4; off <= 16; off <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, off);
    lB += __shfl_xor_sync(0xffffffffu, lB, off);
  }
  const float vs = VF16 ? p.v_unscale[b * (p.Hq / p.heads_per_kv) + kvh] : 1.f;
  const float iA = lA > 0.f ? vs / lA : 0.f, iB = lB > 0.f ? vs / lB : 0.f;
  const float lseA = lA > 0.f ? (mA + log2f(lA)) * 0.69314718055994531f : -INFINITY;
  const float lseB = lB > 0.f ? (mB + log2f(lB)) * 0.69314718055994531f : -INFINITY;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int g = hA + j;
    if (g >= nh) continue;
    const int64_t h = h0 + g;
    const float inv = j ? iB : iA;
    const int64_t ob = b * p.os[0] + h * p.os[1] + t * p.os[2];
#pragma unroll
    for (int dm = 0; dm < S::KS; ++dm) {
      store_any(p.out, ob + (dm * 16 + tk) * p.os[3], p.q_dtype, o[dm][j] * inv);
      store_any(p.out, ob + (dm * 16 + tk + 8) * p.os[3], p.q_dtype, o[dm][2 + j] * inv);
    }
    if (p.lse_out && tk == 0) p.lse_out[(b * p.Hq + h) * p.Tq + t] = j ? lseB : lseA;
    if (p.reads_out && tk == 0) p.reads_out[(b * p.Hq + h) * p.Tq + t] = static_cast<int32_t>(n_read);
  }
}

namespace {

template <typename T, int D>
cudaError_t launch_tok(const TokenAttnParams& p, cudaStream_t st) {
  constexpr size_t smem = 1024 + static_cast<size_t>(TNW) * TSTG * MmaShape<D>::STAGE_BYTES;
  auto kern = p.v_unscale ? token_attention_kernel<T, D, true> : token_attention_kernel<T, D, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>((p.n_items + TNW - 1) / TNW);
  kern<<<grid, 32 * TNW, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_token_attention(const TokenAttnParams& p, int dtype, int D, cudaStream_t st) {
  if (p.v_unscale && dtype != LINATTN_BF16) return cudaErrorInvalidValue;
  if (dtype == LINATTN_BF16) {
    if (D == 128) return launch_tok<__nv_bfloat16, 128>(p, st);
    if (D == 64) return launch_tok<__nv_bfloat16, 64>(p, st);
  } else if (dtype == LINATTN_F16) {
    if (D == 128) return launch_tok<__half, 128>(p, st);
    if (D == 64) return launch_tok<__half, 64>(p, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_token_attention(const void* q, int32_t dtype, int64_t B, int64_t Hq, int64_t Tq,
                                       const int64_t* q_strides, const void* k, const void* v,
                                       const float* v_unscale, int64_t Hkv,
                                       int64_t Tk, int64_t D, const int64_t* kv_strides,
                                       const linattn_lists_t* lists, int64_t block, int64_t sink, int64_t window,
                                       int32_t causal,
                                       int64_t offset, float scale, int32_t diag_fallback, void* out,
                                       const int64_t* out_strides, float* lse_out, int32_t* reads_out,
                                       int32_t* status, void* stream) {
  if (!q || !k || !v || !out || !lists || !q_strides || !kv_strides || !out_strides)
    return set_error(LINATTN_EINVAL, "token_attention: NULL pointer");
  if (dtype != LINATTN_BF16 && dtype != LINATTN_F16)
    return set_error(LINATTN_EUNSUPPORTED, "token_attention: q / K / V must be bf16 or f16 (one type)");
  if (v_unscale && dtype != LINATTN_BF16)
    return set_error(LINATTN_EINVAL, "token_attention: an f16 V copy (v_unscale) goes with bf16 q / K");
  if (D != 64 && D != 128) return set_error(LINATTN_EUNSUPPORTED, "token_attention: head_dim must be 64 or 128");
  if (Hkv < 1 || Hq % Hkv) return set_error(LINATTN_EINVAL, "token_attention: H_q must be a multiple of H_kv");
  if (lists->n_heads < 1 || Hq % lists->n_heads)
    return set_error(LINATTN_EINVAL, "token_attention: H_q must be a multiple of the list heads");
  if (lists->ids_dtype != LINATTN_I32 && lists->ids_dtype != LINATTN_I64)
    return set_error(LINATTN_EINVAL, "token_attention: ids must be int32 or int64");
  if (kv_strides[2] < D || reinterpret_cast<uintptr_t>(k) % 16 || reinterpret_cast<uintptr_t>(v) % 16 ||
      (kv_strides[0] * 2) % 16 || (kv_strides[1] * 2) % 16 || (kv_strides[2] * 2) % 16)
    return set_error(LINATTN_EINVAL, "token_attention: K/V rows must be contiguous and 16-byte aligned");
  if (sink < 0 || window < 0 || block < 1)
    return set_error(LINATTN_EINVAL, "token_attention: sink, window must be >= 0 and block >= 1");
  const int64_t hpk = Hq / Hkv, hpl = Hq / lists->n_heads;
  if (hpk % hpl && hpl % hpk)
    return set_error(LINATTN_EUNSUPPORTED, "token_attention: heads per kv head and per list must divide one another");
  if (B == 0 || Hq == 0 || Tq == 0) return LINATTN_OK;
  TokenAttnParams p;
  p.q = q; p.q_dtype = dtype;
  for (int i = 0; i < 4; ++i) { p.qs[i] = q_strides[i]; p.os[i] = out_strides[i]; }
  p.k = k; p.v = v; p.kv_sb = kv_strides[0]; p.kv_sh = kv_strides[1]; p.kv_st = kv_strides[2];
  p.B = B; p.Hq = Hq; p.Tq = Tq; p.Tk = Tk; p.lists = *lists;
  p.sink = sink; p.window = window; p.block = block; p.causal = causal; p.offset = offset;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out; p.lse_out = lse_out; p.reads_out = reads_out; p.diag_fallback = diag_fallback ? 1 : 0;
  p.v_unscale = v_unscale;
  p.status = status;
  p.heads_per_kv = hpk; p.heads_per_list = hpl;
  // a chunk: consecutive heads sharing a kv head and a list, at most 8 (a divisor of both)
  const int64_t m = lmin(hpk, hpl);
  int64_t c = lmin(8, m);
  while (m % c) --c;
  p.chunk_heads = c;
  const int64_t n_chunks = Hq / p.chunk_heads;
  p.n_items = n_chunks * B * Tq;
  const cudaError_t e = launch_token_attention(p, dtype, static_cast<int>(D), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "token_attention: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
