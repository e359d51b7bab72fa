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
// ascending -1 padded list and its count.
//
// Layout: a CTA of 128 threads scores a tile of 64 rows (G' heads of one kv head x
// 64 / G' rows, so the heads of a GQA group share each candidate tile) against
// candidate tiles of 128.  A (channel-major) and the candidate tile (channel-major,
// staged from L2) live in shared memory; each thread computes an 8 x 8 block of scores
// with 64 FMA per pair of 16-byte loads.  The tile's scores then go to shared memory
// (over the candidate tile, which is no longer needed) and thread i < 64 scans row i,
// keeping its top k (k <= 32) sorted in registers: a score enters only when strictly
// greater than the current k-th, so among equal scores the lower index (seen first)
// stays.  Two CTAs fit an SM, so one computes while the other scans and loads.
#include <cstdio>

#include "launchers.cuh"

namespace linattn {

namespace {

constexpr int BT_ROWS = 64;     // rows per CTA tile
constexpr int BT_CANDS = 128;   // candidates per tile
constexpr int BT_THREADS = 128;
constexpr int BT_SPAD = BT_CANDS + 1;  // score tile row pitch (floats): conflict-free row scans
constexpr int BT_APAD = BT_ROWS + 4;   // A pitch (floats): 16-byte rows, 4-way staging conflicts at most

struct BlockTopkParams {
  const void* a;
  int a_dtype;
  int64_t as[4];  // (B, Hq, R, D) element strides
  const void* bm;
  int b_dtype;
  int b_vec;      // fp32 candidates, unit channel stride, 16-byte aligned rows
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

template <int D, int KMAX>
__global__ void __launch_bounds__(BT_THREADS, 2) block_topk_kernel(const BlockTopkParams p) {
  extern __shared__ __align__(16) float smem[];
  float* As = smem;                        // [D][BT_APAD]
  float* Bs = smem + D * BT_APAD;          // [D][BT_CANDS], then the score tile [BT_ROWS][BT_SPAD]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

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

  // ---- stage A channel-major: a warp per row, lanes over channels (coalesced reads)
  for (int i = warp; i < BT_ROWS; i += BT_THREADS / 32) {
    const int64_t r = r0 + i % p.rt;
    const int64_t h = h0 + i / p.rt;
    const bool ok = r < p.R;
    const int64_t base = b * p.as[0] + h * p.as[1] + r * p.as[2];
    for (int d = lane; d < D; d += 32) As[d * BT_APAD + i] = ok ? load_elem(p.a, base + d * p.as[3], p.a_dtype) : 0.f;
  }
  const int64_t r_last = (r0 + p.rt < p.R ? r0 + p.rt : p.R) - 1;
  int64_t c_hi = floor_div(p.first_pos + r_last, p.key_block);  // lim is non-decreasing in r
  if (c_hi > p.NC - 1) c_hi = p.NC - 1;
  const int64_t c_lo = p.skip;

  // ---- the row this thread scans (thread i < 64 owns tile row i)
  const bool scanner = tid < BT_ROWS;
  const int my_i = tid;
  const int64_t my_r = r0 + my_i % p.rt;
  const int64_t my_h = h0 + my_i / p.rt;
  const bool my_ok = scanner && my_r < p.R;
  int64_t my_lim = my_ok ? floor_div(p.first_pos + my_r, p.key_block) : -1;
  if (my_lim > p.NC - 1) my_lim = p.NC - 1;
  float tv[KMAX];
  int32_t ti[KMAX];
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    tv[j] = -INFINITY;
    ti[j] = -1;
  }
  const int kk = p.k;

  // thread's 8 x 8 score block: rows ty*8 .. +7, candidates tx*4 .. +3 and 64 + tx*4 .. +3
  const int ty = tid / 16, tx = tid % 16;
  for (int64_t c0 = (c_lo / BT_CANDS) * BT_CANDS; c0 <= c_hi; c0 += BT_CANDS) {
    __syncthreads();  // A staged / the previous score tile scanned
    // ---- stage the candidate tile, channel-major: thread j loads candidate c0 + j
    {
      const int j = tid;  // BT_THREADS == BT_CANDS
      const int64_t c = c0 + j;
      const bool ok = c <= c_hi && c < p.NC;
      const int64_t base = b * p.bs[0] + kvh * p.bs[1] + c * p.bs[2];
      if (p.b_vec) {
        const float* src = static_cast<const float*>(p.bm) + base;
#pragma unroll 4
        for (int d = 0; d < D; d += 4) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (ok) v = *reinterpret_cast<const float4*>(src + d);
          Bs[(d + 0) * BT_CANDS + j] = v.x;
          Bs[(d + 1) * BT_CANDS + j] = v.y;
          Bs[(d + 2) * BT_CANDS + j] = v.z;
          Bs[(d + 3) * BT_CANDS + j] = v.w;
        }
      } else {
        for (int d = 0; d < D; ++d)
          Bs[d * BT_CANDS + j] = ok ? load_elem(p.bm, base + d * p.bs[3], p.b_dtype) : 0.f;
      }
    }
    __syncthreads();
    // ---- 8 x 8 scores per thread
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; ++d) {
      const float4 a0 = *reinterpret_cast<const float4*>(As + d * BT_APAD + ty * 8);
      const float4 a1 = *reinterpret_cast<const float4*>(As + d * BT_APAD + ty * 8 + 4);
      const float4 b0 = *reinterpret_cast<const float4*>(Bs + d * BT_CANDS + tx * 4);
      const float4 b1 = *reinterpret_cast<const float4*>(Bs + d * BT_CANDS + 64 + tx * 4);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();  // every thread is done with the candidate tile
    float* S = Bs;     // [BT_ROWS][BT_SPAD]
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int cj = j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4);
        S[(ty * 8 + i) * BT_SPAD + cj] = acc[i][j] * p.scale;
      }
    __syncthreads();
    // ---- scan: row my_i over candidates [max(c0, skip), min(c0 + 127, lim)]
    if (my_ok) {
      const int64_t lo = c0 > c_lo ? c0 : c_lo;
      const int64_t hi = (c0 + BT_CANDS - 1 < my_lim) ? c0 + BT_CANDS - 1 : my_lim;
      const float* srow = S + my_i * BT_SPAD;
      float* sout = p.scores_out ? p.scores_out + ((b * p.Hq + my_h) * p.R + my_r) * p.NC : nullptr;
      for (int64_t c = lo; c <= hi; ++c) {
        const float s = srow[c - c0];
        if (sout) sout[c] = s;
        // the row keeps its best KMAX >= k (the first k of them are its top k)
        if (s > tv[KMAX - 1]) {
          tv[KMAX - 1] = s;
          ti[KMAX - 1] = static_cast<int32_t>(c);
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
  }
  if (!my_ok) return;

  // ---- the row's top k (score order), then the ascending merge with the forced blocks
  const int64_t row = (b * p.Hq + my_h) * p.R + my_r;
  if (p.topk_out) {
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
      if (j < kk) p.topk_out[row * kk + j] = ti[j];
  }
  // keep the first k, ascending by index (invalid entries -1 sort last)
  int32_t sid[KMAX];
#pragma unroll
  for (int j = 0; j < KMAX; ++j) sid[j] = (j < kk && ti[j] >= 0) ? ti[j] : 0x7fffffff;
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

template <int D, int KMAX>
cudaError_t launch_block_topk(const BlockTopkParams& p, unsigned grid, cudaStream_t st) {
  const size_t a_bytes = size_t(D) * BT_APAD * 4;
  size_t b_bytes = size_t(D) * BT_CANDS * 4;
  const size_t s_bytes = size_t(BT_ROWS) * BT_SPAD * 4;
  if (s_bytes > b_bytes) b_bytes = s_bytes;
  const size_t smem = a_bytes + b_bytes;
  cudaError_t e = cudaFuncSetAttribute(block_topk_kernel<D, KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  block_topk_kernel<D, KMAX><<<grid, BT_THREADS, smem, st>>>(p);
  return cudaGetLastError();
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
  if (D != 64 && D != 128) return set_error(LINATTN_EUNSUPPORTED, "block_score_topk: D must be 64 or 128");
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
  p.b_vec = b_dtype == LINATTN_F32 && b_strides[3] == 1 && (reinterpret_cast<uintptr_t>(bm) & 15) == 0 &&
            b_strides[0] % 4 == 0 && b_strides[1] % 4 == 0 && b_strides[2] % 4 == 0;
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
  else
    e = kmax == 16 ? launch_block_topk<64, 16>(p, grid, st) : launch_block_topk<64, 32>(p, grid, st);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "block_score_topk: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
