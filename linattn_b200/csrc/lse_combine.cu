// Split-KV (o, lse) merge: o = sum_s exp(lse_s - L) o_s / sum_s exp(lse_s - L),
// L = max_s lse_s, lse = L + log(sum_s exp(lse_s - L)).  One warp per output row,
// lanes over channels; used after the in-GPU KV split and after the NCCL all-gather
// of per-GPU partials in the sequence-sharded decode.
#include "common.cuh"

namespace linattn {

__global__ void __launch_bounds__(256) lse_combine_kernel(const float* __restrict__ o_parts,
                                                          const float* __restrict__ lse_parts, int64_t S,
                                                          int64_t rows, int64_t D, void* out, int out_dtype,
                                                          int64_t H, int64_t Tq, int64_t os0, int64_t os1,
                                                          int64_t os2, int64_t os3, float* lse_out) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float L = -INFINITY;
  for (int64_t s = 0; s < S; ++s) L = fmaxf(L, lse_parts[s * rows + row]);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  float W = 0.f;
  if (L != -INFINITY) {
    for (int64_t s = 0; s < S; ++s) {
      const float ls = lse_parts[s * rows + row];
      if (ls == -INFINITY) continue;  // empty part: its o is not read (it may be unwritten)
      const float w = __expf(ls - L);
      W += w;
      const float* op = o_parts + (s * rows + row) * D;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t c = lane + 32 * i;
        if (c < D) acc[i] = fmaf(w, op[c], acc[i]);
      }
    }
  }
  const int64_t t = row % Tq, h = (row / Tq) % H, b = row / (Tq * H);
  const float inv = W > 0.f ? 1.f / W : 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t c = lane + 32 * i;
    if (c < D) store_any(out, b * os0 + h * os1 + t * os2 + c * os3, out_dtype, acc[i] * inv);
  }
  if (lse_out && lane == 0) lse_out[row] = W > 0.f ? L + logf(W) : -INFINITY;
}

cudaError_t launch_lse_combine(const float* o_parts, const float* lse_parts, int64_t S, int64_t rows, int64_t D,
                               void* out, int out_dtype, int64_t H, int64_t Tq, const int64_t* os, float* lse_out,
                               cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>((rows * 32 + 255) / 256);
  lse_combine_kernel<<<grid, 256, 0, stream>>>(o_parts, lse_parts, S, rows, D, out, out_dtype, H, Tq, os[0], os[1],
                                               os[2], os[3], lse_out);
  return cudaGetLastError();
}

}  // namespace linattn
