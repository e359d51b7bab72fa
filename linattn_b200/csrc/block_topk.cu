// Block scores + causal top-k + forced-block merge in one kernel: the block selectors
// of MInference (pooled q-block . pooled k-block, selection.py:339-353), MoBA (token q .
// pooled k-block, selection.py:635-649) and NSA's selection branch (token q . pooled
// k-block, native_sparse.py:78-92), and the block-sparse prefill's sink + window + top-k
// lists.
//
// Row r of (b, h) holds a query vector a_r (D channels); candidate c of (b, h / G) holds
// b_c.  score(r, c) = scale * sum_d a_r[d] * b_c[d], accumulated in fp32 in channel
// order d = 0 .. D-1 (one FMA chain per score, so a score does not depend on the tile it
// was computed in).  Row r reads candidates c in [skip, min(lim_r, NC - 1)],
// lim_r = floor((first_pos + r) / key_block); the top k by (score desc, index asc) are
// kept and then merged with the forced blocks [0, sink) and [own - window + 1, own]
// (own = floor((merge_pos + r) / own_div), and own itself with force_own), giving an
// ascending -1 padded list and its count.  The score matrix never leaves the chip.
//
// Layout: a CTA of 256 threads owns a tile of 128 rows (G' heads of one kv head x
// 128 / G' rows, so the heads of a GQA group share each candidate tile) and walks
// candidate tiles of 128.  Rows of D + 4 floats in shared memory: A, staged once, and
// two candidate buffers filled by 16-byte cp.async copies, the next tile in flight
// while the current one is scored.  Each thread computes an 8 x 8 block of scores
// (rows ty*8 + i, candidates tx + 16 j; 256 FMA per 16 loads of 16 bytes), the block
// goes to shared memory over the consumed candidate buffer, and two threads per row
// scan it (one per 64 candidates), each keeping its best k (k <= 32) sorted in
// registers: a score enters only when strictly greater than the current k-th, so
// among equal scores the lower index (seen first) stays.  The two halves' lists are
// merged by (score desc, index asc) at the end.
#include <cstdio>

#include "launchers.cuh"

namespace linattn {

namespace {

constexpr int BT_ROWS = 128;    // rows per CTA tile
constexpr int BT_CANDS = 128;   // candidates per tile
constexpr int BT_THREADS = 256;
constexpr int BT_SPAD = BT_CANDS + 1;  // score tile row pitch (floats): conflict-free row scans
constexpr int BT_MAXD = 128;

// Row pitch (floats) of the A and candidate tiles: D + 4 keeps rows 16-byte aligned
// and puts the rows a quarter-warp reads (consecutive candidates) in distinct bank
// groups when D % 32 == 0.
__host__ __device__ constexpr int bt_pitch(int d) { return ((d + 3) / 4) * 4 + 4; }
// floats of one candidate buffer: a candidate tile, or the score tile written over it
__host__ __device__ constexpr int bt_buf(int d) {
  return bt_pitch(d) * BT_CANDS > BT_ROWS * BT_SPAD ? bt_pitch(d) * BT_CANDS : BT_ROWS * BT_SPAD;
}

__device__ __forceinline__ void cp_async16(float* smem_dst, const void* gmem_src) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

struct BlockTopkParams {
  const void* a;
  int a_dtype;
  int a_vec;      // unit channel stride, 16-byte aligned rows (fp32: D % 4 == 0; 16-bit: D % 8 == 0)
  int64_t as[4];  // (B, Hq, R, D) element strides
  const void* bm;
  int b_dtype;
  int b_vec;      // the same for the candidates
  int64_t bs[4];  // (B, Hkv, NC, D)
  int64_t B, Hq, Hkv, R, NC, D;
  int G, Gt, rt;  // group size, heads per tile, rows per head per tile
  int64_t r_chunks;
  float scale;
  int k;
  int64_t first_pos, key_block, skip;
  int64_t merge_pos, own_div, sink, window;
  int force_own;
  int32_t* out;
  int64_t n_max;
  int32_t* counts;
  int32_t* topk_out;   // optional (B, Hq, R, k), score order
  float* scores_out;   // optional (B, Hq, R, NC)
};

__device__ __forceinline__ int64_t floor_div(int64_t a, int64_t b) {
  const int64_t q = a / b;
  return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}

__device__ __forceinline__ float load_elem(const void* base, int64_t idx, int dtype) {
  switch (dtype) {
    case LINATTN_F32: return static_cast<const float*>(base)[idx];
    case LINATTN_F16: return __half2float(static_cast<const __half*>(base)[idx]);
    default: return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(base)[idx]) << 16);
  }
}

// Stage `n_rows` rows of D channels (row i at element offset row_off(i)) into rows of
// `pt` floats at dst, zero-filling channels >= D and rows >= n_valid.  fp32 vector rows
// go by cp.async (the caller commits and waits); 16-bit vector rows by 16-byte loads,
// eight in flight per thread; anything else element by element, eight in flight.
template <typename RowOff>
__device__ __forceinline__ void stage_rows(float* dst, int pt, int n_rows, int n_valid, int D, const void* src,
                                           int dtype, int vec, int64_t cstride, RowOff row_off) {
  const int tid = threadIdx.x;
  if (vec && dtype == LINATTN_F32) {
    const int n4 = pt / 4;
    for (int e = tid; e < n_rows * n4; e += BT_THREADS) {
      const int i = e / n4, d = (e - i * n4) * 4;
      float* to = dst + i * pt + d;
      if (i < n_valid && d < D) cp_async16(to, static_cast<const float*>(src) + row_off(i) + d);
      else *reinterpret_cast<float4*>(to) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  } else if (vec) {
    const int n8 = pt / 8;  // D % 8 == 0, so pt = D + 4: the last 4 floats are zeroed below
    const int total = n_rows * n8;
    for (int e0 = tid; e0 < total; e0 += 8 * BT_THREADS) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * BT_THREADS;
        const int i = e / n8, d = (e - i * n8) * 8;
        v[u] = (e < total && i < n_valid)
                   ? *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(src) + row_off(i) + d)
                   : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * BT_THREADS;
        if (e >= total) break;
        const int i = e / n8, d = (e - i * n8) * 8;
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        float f[8];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          if (dtype == LINATTN_F16) {
            const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[x]));
            f[2 * x] = t.x;
            f[2 * x + 1] = t.y;
          } else {
            f[2 * x] = __uint_as_float(w[x] << 16);
            f[2 * x + 1] = __uint_as_float(w[x] & 0xffff0000u);
          }
        }
        float* to = dst + i * pt + d;
        *reinterpret_cast<float4*>(to) = make_float4(f[0], f[1], f[2], f[3]);
        *reinterpret_cast<float4*>(to + 4) = make_float4(f[4], f[5], f[6], f[7]);
      }
    }
    for (int i = tid; i < n_rows; i += BT_THREADS)
      *reinterpret_cast<float4*>(dst + i * pt + n8 * 8) = make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
    const int total = n_rows * pt;
    for (int e0 = tid; e0 < total; e0 += 8 * BT_THREADS) {
      float f[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * BT_THREADS;
        const int i = e / pt, d = e - i * pt;
        f[u] = (e < total && i < n_valid && d < D) ? load_elem(src, row_off(i) + d * cstride, dtype) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * BT_THREADS;
        if (e < total) dst[e] = f[u];
      }
    }
  }
}

// DT: the head size at compile time (64, 128), or 0 for any D <= 128 read from p.D
template <int DT, int KMAX>
__global__ void __launch_bounds__(BT_THREADS, 1) block_topk_kernel(const BlockTopkParams p) {
  const int D = DT > 0 ? DT : static_cast<int>(p.D);
  const int PT = bt_pitch(D);
  const int BUF = bt_buf(D);
  extern __shared__ __align__(16) float smem[];
  float* As = smem;                      // [BT_ROWS][PT]
  float* Bbuf = smem + BT_ROWS * PT;     // two buffers of BUF floats
  const int tid = threadIdx.x;

  // tile -> (b, kv head, head sub-group, row chunk); the last row chunks (most
  // candidates under the causal rule) are scheduled first
  int64_t t = blockIdx.x;
  const int64_t rc = p.r_chunks - 1 - t % p.r_chunks;
  t /= p.r_chunks;
  const int n_sub = p.G / p.Gt;
  const int sub = static_cast<int>(t % n_sub);
  t /= n_sub;
  const int64_t kvh = t % p.Hkv;
  const int64_t b = t / p.Hkv;
  const int64_t r0 = rc * p.rt;
  const int64_t h0 = kvh * p.G + static_cast<int64_t>(sub) * p.Gt;

  const int64_t r_last = (r0 + p.rt < p.R ? r0 + p.rt : p.R) - 1;
  int64_t c_hi = floor_div(p.first_pos + r_last, p.key_block);  // lim is non-decreasing in r
  if (c_hi > p.NC - 1) c_hi = p.NC - 1;
  const int64_t c_lo = p.skip;
  const int64_t c_first = (c_lo / BT_CANDS) * BT_CANDS;
  const int n_tiles = c_hi >= c_lo ? static_cast<int>((c_hi - c_first) / BT_CANDS + 1) : 0;

  // ---- stage A (rows past R zero) and the first candidate tile
  const int64_t a_base = b * p.as[0];
  stage_rows(As, PT, BT_ROWS, BT_ROWS, D, p.a, p.a_dtype, p.a_vec, p.as[3], [&](int i) -> int64_t {
    const int64_t r = r0 + i % p.rt;
    return r < p.R ? a_base + (h0 + i / p.rt) * p.as[1] + r * p.as[2] : a_base;  // rows past R read row 0
  });
  const int64_t b_base = b * p.bs[0] + kvh * p.bs[1];
  auto stage_cands = [&](int tile) {
    const int64_t c0 = c_first + static_cast<int64_t>(tile) * BT_CANDS;
    const int n_c = static_cast<int>(c_hi - c0 + 1 < BT_CANDS ? c_hi - c0 + 1 : BT_CANDS);
    stage_rows(Bbuf + (tile & 1) * BUF, PT, BT_CANDS, n_c, D, p.bm, p.b_dtype, p.b_vec, p.bs[3],
               [&](int j) -> int64_t { return b_base + (c0 + j) * p.bs[2]; });
  };
  if (n_tiles > 0) stage_cands(0);
  cp_async_commit();

  // ---- this thread's row scan: row my_i, candidates [64 * half, 64 * half + 64) of a tile
  const int my_i = tid & (BT_ROWS - 1), half = tid >> 7;
  const int64_t my_r = r0 + my_i % p.rt;
  const int64_t my_h = h0 + my_i / p.rt;
  const bool my_ok = my_r < p.R;
  int64_t my_lim = my_ok ? floor_div(p.first_pos + my_r, p.key_block) : -1;
  if (my_lim > p.NC - 1) my_lim = p.NC - 1;
  float tv[KMAX];
  int32_t ti[KMAX];
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    tv[j] = -INFINITY;
    ti[j] = -1;
  }
  float* sout_row = (p.scores_out && my_ok) ? p.scores_out + ((b * p.Hq + my_h) * p.R + my_r) * p.NC : nullptr;

  // thread's 8 x 8 score block: rows ty*8 + i, candidates tx + 16*j
  const int ty = tid / 16, tx = tid % 16;
  for (int tile = 0; tile < n_tiles; ++tile) {
    const int64_t c0 = c_first + static_cast<int64_t>(tile) * BT_CANDS;
    float* Bs = Bbuf + (tile & 1) * BUF;
    // the next tile's copies go out now and land while this one is scored and scanned;
    // its buffer was last read by the previous tile's scan, which the barrier at the end
    // of the previous iteration closed
    if (tile + 1 < n_tiles) stage_cands(tile + 1);
    cp_async_commit();
    cp_async_wait_prev();
    __syncthreads();  // tile `tile` (and A) visible to every thread
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    // each score is one FMA chain over d = 0, 1, 2, ... (the zero padding adds +0)
#pragma unroll 1
    for (int d = 0; d < D; d += 4) {
      float4 av[8], bv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) av[i] = *reinterpret_cast<const float4*>(As + (ty * 8 + i) * PT + d);
#pragma unroll
      for (int j = 0; j < 8; ++j) bv[j] = *reinterpret_cast<const float4*>(Bs + (tx + 16 * j) * PT + d);
      // channel by channel over all 64 scores: 64 independent FMAs between two that
      // depend on each other
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i].x, bv[j].x, acc[i][j]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i].y, bv[j].y, acc[i][j]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i].z, bv[j].z, acc[i][j]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i].w, bv[j].w, acc[i][j]);
    }
    __syncthreads();  // every thread is done with this candidate buffer
    float* S = Bs;     // [BT_ROWS][BT_SPAD]
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) S[(ty * 8 + i) * BT_SPAD + tx + 16 * j] = acc[i][j] * p.scale;
    __syncthreads();
    // ---- scan this thread's half of row my_i: [max(c0 + 64 half, skip), min(c0 + 64 half + 63, lim)]
    if (my_ok) {
      const int64_t g_lo = c0 + 64 * half, g_hi = g_lo + 63;
      const int64_t lo64 = g_lo > c_lo ? g_lo : c_lo;
      const int64_t hi64 = g_hi < my_lim ? g_hi : my_lim;
      const int lo = static_cast<int>(lo64 - c0), hi = static_cast<int>(hi64 - c0);
      const float* srow = S + my_i * BT_SPAD;
      if (sout_row)
        for (int c = lo; c <= hi; ++c) sout_row[c0 + c] = srow[c];
      // pass 1, branch-free: the candidates above the current k-th best, as a bit mask;
      // pass 2 inserts just those (the k-th best only rises, so each is checked again)
      const float thr = tv[KMAX - 1];
      const int base = 64 * half;
      unsigned long long above = 0ull;
#pragma unroll 16
      for (int c = 0; c < 64; ++c) {
        const bool in = c + base >= lo && c + base <= hi;
        above |= static_cast<unsigned long long>(in && srow[base + c] > thr) << c;
      }
      while (above) {
        const int c = base + __ffsll(static_cast<long long>(above)) - 1;
        above &= above - 1ull;
        const float sc = srow[c];
        if (sc > tv[KMAX - 1]) {
          tv[KMAX - 1] = sc;
          ti[KMAX - 1] = static_cast<int32_t>(c0 + c);
#pragma unroll
          for (int j = KMAX - 1; j > 0; --j) {
            if (tv[j] > tv[j - 1]) {
              const float fv = tv[j]; tv[j] = tv[j - 1]; tv[j - 1] = fv;
              const int32_t fi = ti[j]; ti[j] = ti[j - 1]; ti[j - 1] = fi;
            }
          }
        }
      }
    }
    __syncthreads();  // the scan is done with this buffer before the next refill of it
  }
  cp_async_wait_all();
  __syncthreads();
  // ---- merge the two halves' lists (both sorted by score desc, index asc); half 1
  // hands its list over through shared memory (the A tile is no longer needed)
  float* xv = As;                                                 // [BT_ROWS][KMAX]
  int32_t* xi = reinterpret_cast<int32_t*>(As + BT_ROWS * KMAX);  // [BT_ROWS][KMAX]
  if (half == 1) {
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      xv[my_i * KMAX + j] = tv[j];
      xi[my_i * KMAX + j] = ti[j];
    }
  }
  __syncthreads();
  if (half == 1 || !my_ok) return;
  const int kk = p.k;
  // half 0's list is in registers (tv, ti); walk it by shifting: the head is always at
  // index 0, so no dynamic register indexing is needed
  int32_t top[KMAX];
  int c = 0;
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    const float vb = c < KMAX ? xv[my_i * KMAX + c] : -INFINITY;
    const int32_t ib = c < KMAX ? xi[my_i * KMAX + c] : -1;
    const float va = tv[0];
    const int32_t ia = ti[0];
    const bool take_a = ia >= 0 && (ib < 0 || va > vb || (va == vb && ia < ib));
    top[j] = take_a ? ia : ib;
    if (take_a) {
#pragma unroll
      for (int x = 0; x + 1 < KMAX; ++x) {
        tv[x] = tv[x + 1];
        ti[x] = ti[x + 1];
      }
      tv[KMAX - 1] = -INFINITY;
      ti[KMAX - 1] = -1;
    } else if (ib >= 0) {
      ++c;
    }
  }

  // ---- the row's top k (score order), then the ascending merge with the forced blocks
  const int64_t row = (b * p.Hq + my_h) * p.R + my_r;
  if (p.topk_out) {
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
      if (j < kk) p.topk_out[row * kk + j] = top[j];
  }
  // keep the first k, ascending by index (invalid entries sort last)
  int32_t sid[KMAX];
#pragma unroll
  for (int j = 0; j < KMAX; ++j) sid[j] = (j < kk && top[j] >= 0) ? top[j] : 0x7fffffff;
#pragma unroll
  for (int x = 1; x < KMAX; ++x)
#pragma unroll
    for (int y = x; y > 0; --y)
      if (sid[y] < sid[y - 1]) {
        const int32_t f = sid[y]; sid[y] = sid[y - 1]; sid[y - 1] = f;
      }
  const int64_t pos = p.merge_pos + my_r;
  int64_t own = pos < 0 ? -1 : pos / p.own_div;
  if (own > p.NC - 1) own = p.NC - 1;
  const int64_t s_end = p.sink < own + 1 ? p.sink : own + 1;
  int64_t w_lo = p.window > 0 ? (s_end > own - p.window + 1 ? s_end : own - p.window + 1) : own + 1;
  if (p.force_own && w_lo > own) w_lo = s_end > own ? s_end : own;
  int32_t* o = p.out + row * p.n_max;
  int64_t n = 0, last = -1;
  for (int64_t f = 0; f < s_end && n < p.n_max; ++f) {
    o[n++] = static_cast<int32_t>(f);
    last = f;
  }
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    const int64_t v = sid[j];
    if (v != 0x7fffffff && v > last && v <= own && v < w_lo && n < p.n_max) {
      o[n++] = static_cast<int32_t>(v);
      last = v;
    }
  }
  for (int64_t f = (w_lo > last + 1 ? w_lo : last + 1); f <= own && n < p.n_max; ++f) o[n++] = static_cast<int32_t>(f);
  const int64_t n_done = n;
  for (int64_t i = n_done; i < p.n_max; ++i) o[i] = -1;
  if (p.counts) p.counts[row] = static_cast<int32_t>(n_done);
}

template <int DT, int KMAX>
cudaError_t launch_block_topk(const BlockTopkParams& p, unsigned grid, cudaStream_t st) {
  const int d = DT > 0 ? DT : static_cast<int>(p.D);
  const size_t smem = (static_cast<size_t>(BT_ROWS) * bt_pitch(d) + 2 * static_cast<size_t>(bt_buf(d))) * 4;
  cudaError_t e = cudaFuncSetAttribute(block_topk_kernel<DT, KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  block_topk_kernel<DT, KMAX><<<grid, BT_THREADS, smem, st>>>(p);
  return cudaGetLastError();
}

bool rows_vec(int dtype, const void* base, const int64_t* s, int64_t D) {
  const int per16 = dtype == LINATTN_F32 ? 4 : 8;  // elements in 16 bytes
  return s[3] == 1 && D % per16 == 0 && (reinterpret_cast<uintptr_t>(base) & 15) == 0 && s[0] % per16 == 0 &&
         s[1] % per16 == 0 && s[2] % per16 == 0;
}

}  // namespace

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_block_score_topk(const void* a, int32_t a_dtype, const int64_t* a_strides, const void* bm,
                                        int32_t b_dtype, const int64_t* b_strides, int64_t B, int64_t Hq,
                                        int64_t Hkv, int64_t R, int64_t NC, int64_t D, float scale, int64_t k,
                                        int64_t first_pos, int64_t key_block, int64_t skip, int64_t merge_pos,
                                        int64_t own_div, int64_t sink, int64_t window, int32_t force_own,
                                        int32_t* out, int64_t n_max, int32_t* counts, int32_t* topk_out,
                                        float* scores_out, void* stream) {
  if (!a || !bm || !a_strides || !b_strides || !out) return set_error(LINATTN_EINVAL, "block_score_topk: NULL pointer");
  for (int32_t dt : {a_dtype, b_dtype})
    if (dt != LINATTN_F32 && dt != LINATTN_F16 && dt != LINATTN_BF16)
      return set_error(LINATTN_EUNSUPPORTED, "block_score_topk: a and b must be f32, f16 or bf16");
  if (D < 1 || D > BT_MAXD) return set_error(LINATTN_EUNSUPPORTED, "block_score_topk: D must be 1 .. 128");
  if (Hkv < 1 || Hq % Hkv != 0) return set_error(LINATTN_EINVAL, "block_score_topk: H_q must be a multiple of H_kv");
  if (k < 1 || k > 32) return set_error(LINATTN_EUNSUPPORTED, "block_score_topk: k must be 1 .. 32");
  if (key_block < 1 || own_div < 1 || NC < 1 || n_max < 1 || skip < 0)
    return set_error(LINATTN_EINVAL, "block_score_topk: bad sizes");
  if (n_max < k + (sink > 0 ? sink : 0) + (window > 1 ? window : 1))
    return set_error(LINATTN_EINVAL, "block_score_topk: n_max must be >= k + sink + max(window, 1)");
  if (B == 0 || Hq == 0 || R == 0) return LINATTN_OK;
  BlockTopkParams p;
  p.a = a; p.a_dtype = a_dtype; p.bm = bm; p.b_dtype = b_dtype;
  for (int i = 0; i < 4; ++i) {
    p.as[i] = a_strides[i];
    p.bs[i] = b_strides[i];
  }
  p.a_vec = rows_vec(a_dtype, a, a_strides, D);
  p.b_vec = rows_vec(b_dtype, bm, b_strides, D);
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.R = R; p.NC = NC; p.D = D;
  p.G = static_cast<int>(Hq / Hkv);
  int gt = 1;
  while (gt * 2 <= 8 && p.G % (gt * 2) == 0) gt *= 2;
  p.Gt = gt;
  p.rt = BT_ROWS / gt;
  p.r_chunks = (R + p.rt - 1) / p.rt;
  p.scale = scale; p.k = static_cast<int>(k);
  p.first_pos = first_pos; p.key_block = key_block; p.skip = skip;
  p.merge_pos = merge_pos; p.own_div = own_div; p.sink = sink < 0 ? 0 : sink; p.window = window < 0 ? 0 : window;
  p.force_own = force_own ? 1 : 0;
  p.out = out; p.n_max = n_max; p.counts = counts; p.topk_out = topk_out; p.scores_out = scores_out;
  const int64_t tiles = B * Hkv * (p.G / gt) * p.r_chunks;
  if (tiles > 0x7fffffff) return set_error(LINATTN_EUNSUPPORTED, "block_score_topk: too many row tiles");
  const unsigned grid = static_cast<unsigned>(tiles);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  const int kmax = k <= 16 ? 16 : 32;
  if (D == 128)
    e = kmax == 16 ? launch_block_topk<128, 16>(p, grid, st) : launch_block_topk<128, 32>(p, grid, st);
  else if (D == 64)
    e = kmax == 16 ? launch_block_topk<64, 16>(p, grid, st) : launch_block_topk<64, 32>(p, grid, st);
  else
    e = kmax == 16 ? launch_block_topk<0, 16>(p, grid, st) : launch_block_topk<0, 32>(p, grid, st);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "block_score_topk: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
