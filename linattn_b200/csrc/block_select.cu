// Block selection helpers for block-sparse prefill (MInference block-sparse, MoBA,
// sink + window + top-k).
//
// block_mean_kernel: mean of each block of `block` rows along the token axis, the
//   tail block padded by repeating the last row (block_reduce, src/linattn/core.py:103-120),
//   fp32 out.  One CTA per (b, h, block); threads over channels, so every row read is
//   coalesced.
// merge_lists_kernel: per row, the ascending union of a top-k list (-1 padded, any
//   order) with the forced blocks: [0, sink), [own - window + 1, own] and own
//   (MInference's own block, selection.py:350-351; MoBA's own block, :645-646), clipped to
//   [0, own]; duplicates removed.  One thread per row (lists are short).
#include <cstdio>

#include "launchers.cuh"

namespace linattn {

namespace {

struct BlockMeanParams {
  const void* x;
  int dtype;
  int64_t B, H, T, D, s[4];
  int64_t block, nb;
  float* out;  // (B, H, nb, D) contiguous
};

__global__ void block_mean_kernel(const BlockMeanParams p) {
  const int64_t unit = blockIdx.x;  // (b, h, blk)
  const int64_t blk = unit % p.nb;
  const int64_t bh = unit / p.nb;
  const int64_t h = bh % p.H, b = bh / p.H;
  const int64_t t0 = blk * p.block;
  const float inv = 1.f / static_cast<float>(p.block);
  for (int64_t c = threadIdx.x; c < p.D; c += blockDim.x) {
    float acc = 0.f;
    const int64_t base = b * p.s[0] + h * p.s[1] + c * p.s[3];
    for (int64_t i = 0; i < p.block; ++i) {
      const int64_t t = lmin(t0 + i, p.T - 1);  // the tail repeats the last row
      acc += load_any(p.x, base + t * p.s[2], p.dtype);
    }
    p.out[unit * p.D + c] = acc * inv;
  }
}

// 16-bit rows with unit channel stride and 16-byte aligned rows: each thread sums 8
// channels of one block with 16-byte loads, eight rows in flight, in the same row
// order as block_mean_kernel (bit-identical means); D / 8 threads per block.
template <bool BF16>
__global__ void __launch_bounds__(128) block_mean_vec_kernel(const BlockMeanParams p, int64_t units) {
  const int tpu = static_cast<int>(p.D / 8);  // threads per (b, h, block); divides 128
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * (128 / tpu) + threadIdx.x / tpu;
  if (unit >= units) return;
  const int c0 = (threadIdx.x % tpu) * 8;
  const int64_t blk = unit % p.nb, bh = unit / p.nb;
  const int64_t h = bh % p.H, b = bh / p.H;
  const int64_t t0 = blk * p.block;
  const uint16_t* base = static_cast<const uint16_t*>(p.x) + b * p.s[0] + h * p.s[1] + c0;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int64_t i0 = 0; i0 < p.block; i0 += 8) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t t = lmin(t0 + lmin(i0 + u, p.block - 1), p.T - 1);  // the tail repeats the last row
      v[u] = *reinterpret_cast<const uint4*>(base + t * p.s[2]);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (i0 + u >= p.block) break;
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float lo, hi;
        if constexpr (BF16) {
          lo = __uint_as_float(w[q] << 16);
          hi = __uint_as_float(w[q] & 0xffff0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[q]));
          lo = f.x;
          hi = f.y;
        }
        acc[2 * q] += lo;
        acc[2 * q + 1] += hi;
      }
    }
  }
  const float inv = 1.f / static_cast<float>(p.block);
  float* o = p.out + unit * p.D + c0;
  reinterpret_cast<float4*>(o)[0] = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
  reinterpret_cast<float4*>(o)[1] = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
}

struct MergeParams {
  const int32_t* topk;
  int64_t rows, k;
  int64_t period, first_pos, own_div, n_blocks;
  int64_t sink, window;
  int force_own;
  int32_t* out;
  int64_t n_max;
  int32_t* counts;
};

__global__ void merge_lists_kernel(const MergeParams p) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= p.rows) return;
  const int64_t pos = p.first_pos + r % p.period;
  const int64_t own = pos < 0 ? -1 : lmin(pos / p.own_div, p.n_blocks - 1);
  const int32_t* tk = p.topk + r * p.k;
  int32_t* o = p.out + r * p.n_max;
  // forced ranges, ascending and disjoint: [0, s_end) and [w_lo, own]
  const int64_t s_end = lmin(p.sink, own + 1);
  int64_t w_lo = p.window > 0 ? lmax(s_end, own - p.window + 1) : own + 1;
  if (p.force_own && w_lo > own) w_lo = lmax(s_end, own);
  int64_t n = 0, last = -1;
  auto emit = [&](int64_t v) {
    if (v > last && n < p.n_max) {
      o[n++] = static_cast<int32_t>(v);
      last = v;
    }
  };
  // top-k ids are ascending when produced in index order; sort defensively (k small)
  int64_t prev = -1;
  for (int64_t f = 0; f < s_end; ++f) emit(f);
  while (true) {
    int64_t best = -1;
    for (int64_t i = 0; i < p.k; ++i) {
      const int64_t v = tk[i];
      if (v > prev && v <= own && (best < 0 || v < best)) best = v;
    }
    if (best < 0) break;
    prev = best;
    if (best >= w_lo) break;  // the forced tail covers the rest
    emit(best);
  }
  for (int64_t f = w_lo; f <= own; ++f) emit(f);
  for (int64_t i = n; i < p.n_max; ++i) o[i] = -1;
  if (p.counts) p.counts[r] = static_cast<int32_t>(n);
}

}  // namespace

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_block_mean(const void* x, int32_t dtype, int64_t B, int64_t H, int64_t T, int64_t D,
                                  const int64_t* strides, int64_t block, float* out, void* stream) {
  if (!x || !out || !strides) return set_error(LINATTN_EINVAL, "block_mean: NULL pointer");
  if (dtype != LINATTN_F32 && dtype != LINATTN_F16 && dtype != LINATTN_BF16)
    return set_error(LINATTN_EUNSUPPORTED, "block_mean: dtype must be f32, f16 or bf16");
  if (block < 1) return set_error(LINATTN_EINVAL, "block_mean: block must be >= 1");
  if (B == 0 || H == 0 || T == 0 || D == 0) return LINATTN_OK;
  BlockMeanParams p;
  p.x = x; p.dtype = dtype; p.B = B; p.H = H; p.T = T; p.D = D;
  for (int i = 0; i < 4; ++i) p.s[i] = strides[i];
  p.block = block; p.nb = (T + block - 1) / block; p.out = out;
  const int64_t units = B * H * p.nb;
  if (units > 0x7fffffff) return set_error(LINATTN_EUNSUPPORTED, "block_mean: too many blocks");
  const bool vec = dtype != LINATTN_F32 && D % 8 == 0 && 128 % (D / 8) == 0 && p.s[3] == 1 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0 && p.s[0] % 8 == 0 && p.s[1] % 8 == 0 &&
                   p.s[2] % 8 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (vec) {
    const int64_t per_cta = 128 / (D / 8);
    const unsigned grid = static_cast<unsigned>((units + per_cta - 1) / per_cta);
    if (dtype == LINATTN_BF16)
      block_mean_vec_kernel<true><<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(p, units);
    else
      block_mean_vec_kernel<false><<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(p, units);
  } else {
    block_mean_kernel<<<static_cast<unsigned>(units), D >= 128 ? 128 : 64, 0, static_cast<cudaStream_t>(stream)>>>(p);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "block_mean: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}

extern "C" int linattn_merge_block_lists(const int32_t* topk, int64_t rows, int64_t k, int64_t period,
                                         int64_t first_pos, int64_t own_div, int64_t n_blocks, int64_t sink,
                                         int64_t window, int32_t force_own, int32_t* out, int64_t n_max,
                                         int32_t* counts, void* stream) {
  if (!out || (k > 0 && !topk)) return set_error(LINATTN_EINVAL, "merge_block_lists: NULL pointer");
  if (period < 1 || own_div < 1 || n_blocks < 1 || n_max < 1 || k < 0)
    return set_error(LINATTN_EINVAL, "merge_block_lists: bad sizes");
  if (rows == 0) return LINATTN_OK;
  MergeParams p;
  p.topk = topk; p.rows = rows; p.k = k; p.period = period; p.first_pos = first_pos; p.own_div = own_div;
  p.n_blocks = n_blocks; p.sink = sink < 0 ? 0 : sink; p.window = window < 0 ? 0 : window;
  p.force_own = force_own ? 1 : 0; p.out = out; p.n_max = n_max; p.counts = counts;
  const unsigned grid = static_cast<unsigned>((rows + 127) / 128);
  merge_lists_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "merge_block_lists: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
