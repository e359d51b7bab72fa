// Split-KV (o, lse) merge: o = sum_s exp(lse_s - L) o_s / sum_s exp(lse_s - L),
// L = max_s lse_s, lse = L + log(sum_s exp(lse_s - L)).  One warp per output row,
// lanes over channels; used after the in-GPU KV split and after the NCCL all-gather
// of per-GPU partials in the sequence-sharded decode.  Part s of o starts at
// o_parts + s * o_part_stride and its lse at lse_parts + s * lse_part_stride (dense
// (S, rows, D) / (S, rows) by default), so one gathered buffer holding every rank's
// [o | lse] block is read in place.
#include "common.cuh"

namespace linattn {

// One CTA per output row, one thread per channel: every thread reads all parts'
// lse (broadcast loads), so the max, the weights and the o loads (coalesced across
// threads, independent across parts) need no dependent round trips.
__global__ void __launch_bounds__(256) lse_combine_kernel(const float* __restrict__ o_parts,
                                                          const float* __restrict__ lse_parts, int64_t S,
                                                          int64_t rows, int64_t D, int64_t o_ps, int64_t l_ps,
                                                          void* out, int out_dtype,
                                                          int64_t H, int64_t Tq, int64_t os0, int64_t os1,
                                                          int64_t os2, int64_t os3, float* lse_out) {
  const int64_t row = blockIdx.x;
  const int c = threadIdx.x;
  float L = -INFINITY;
  for (int64_t s = 0; s < S; ++s) L = fmaxf(L, lse_parts[s * l_ps + row]);
  float acc = 0.f, W = 0.f;
  if (L != -INFINITY) {
#pragma unroll 8
    for (int64_t s = 0; s < S; ++s) {
      const float ls = lse_parts[s * l_ps + row];
      if (ls == -INFINITY) continue;  // empty part: its o is not read (it may be unwritten)
      const float w = __expf(ls - L);
      W += w;
      if (c < D) acc = fmaf(w, o_parts[s * o_ps + row * D + c], acc);
    }
  }
  if (c < D) {
    const int64_t t = row % Tq, h = (row / Tq) % H, b = row / (Tq * H);
    store_any(out, b * os0 + h * os1 + t * os2 + c * os3, out_dtype, W > 0.f ? acc / W : 0.f);
  }
  if (lse_out && c == 0) lse_out[row] = W > 0.f ? L + logf(W) : -INFINITY;
}

cudaError_t launch_lse_combine(const float* o_parts, const float* lse_parts, int64_t S, int64_t rows, int64_t D,
                               void* out, int out_dtype, int64_t H, int64_t Tq, const int64_t* os, float* lse_out,
                               cudaStream_t stream, int64_t o_part_stride, int64_t lse_part_stride) {
  if (rows == 0) return cudaSuccess;
  const int threads = static_cast<int>(lmax(32, (D + 31) / 32 * 32));
  const int64_t o_ps = o_part_stride > 0 ? o_part_stride : rows * D;
  const int64_t l_ps = lse_part_stride > 0 ? lse_part_stride : rows;
  lse_combine_kernel<<<static_cast<unsigned>(rows), threads, 0, stream>>>(o_parts, lse_parts, S, rows, D, o_ps,
                                                                           l_ps, out, out_dtype, H, Tq, os[0],
                                                                           os[1], os[2], os[3], lse_out);
  return cudaGetLastError();
}

}  // namespace linattn
