// Split-KV (o, lse) merge: o = sum_s exp(lse_s - L) o_s / sum_s exp(lse_s - L),
// L = max_s lse_s, lse = L + log(sum_s exp(lse_s - L)).  One warp per output row,
// lanes over channels; used after the in-GPU KV split and after the NCCL all-gather
// of per-GPU partials in the sequence-sharded decode.  Part s of o starts at
// o_parts + s * o_part_stride and its lse at lse_parts + s * lse_part_stride (dense
// (S, rows, D) / (S, rows) by default), so one gathered buffer holding every rank's
// [o | lse] block is read in place.
#include "common.cuh"

namespace linattn {

// One CTA per output row, one thread per channel.  Every warp fetches the parts' lse
// 32 at a time (lane s holds part s of the group, one round trip for all of them),
// reduces the max and broadcasts each part's weight by shuffle, so the o loads
// (coalesced across threads, independent across parts) follow in a second round trip.
__global__ void __launch_bounds__(256) lse_combine_kernel(const float* __restrict__ o_parts,
                                                          const float* __restrict__ lse_parts, int64_t S,
                                                          int64_t rows, int64_t D, int64_t o_ps, int64_t l_ps,
                                                          void* out, int out_dtype,
                                                          int64_t H, int64_t Tq, int64_t os0, int64_t os1,
                                                          int64_t os2, int64_t os3, float* lse_out) {
  // a programmatic dependent of the attention launch: the parts are its output
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t row = blockIdx.x;
  const int c = threadIdx.x, lane = c & 31;
  float L = -INFINITY;
  for (int64_t s0 = 0; s0 < S; s0 += 32)
    L = fmaxf(L, s0 + lane < S ? lse_parts[(s0 + lane) * l_ps + row] : -INFINITY);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) L = fmaxf(L, __shfl_xor_sync(0xffffffffu, L, off));
  float acc = 0.f, W = 0.f;
  if (L != -INFINITY) {
    for (int64_t s0 = 0; s0 < S; s0 += 32) {
      const float ls = s0 + lane < S ? lse_parts[(s0 + lane) * l_ps + row] : -INFINITY;
      const float wl = ls == -INFINITY ? 0.f : __expf(ls - L);
      const int n = static_cast<int>(lmin(32, S - s0));
      const float* op = o_parts + s0 * o_ps + row * D + c;
#pragma unroll 8
      for (int j = 0; j < n; ++j) {
        const float w = __shfl_sync(0xffffffffu, wl, j);
        W += w;
        // an empty part (lse = -inf) is not read: its o may be unwritten
        if (w != 0.f && c < D) acc = fmaf(w, op[j * o_ps], acc);
      }
    }
  }
  if (c < D) {
    const int64_t t = row % Tq, h = (row / Tq) % H, b = row / (Tq * H);
    store_any(out, b * os0 + h * os1 + t * os2 + c * os3, out_dtype, W > 0.f ? acc / W : 0.f);
  }
  if (lse_out && c == 0) lse_out[row] = W > 0.f ? L + logf(W) : -INFINITY;
}

// Clears the tensor-core attention's work counter (the workspace header) in place of a
// memset node, as a kernel that can itself start early behind the previous
// kernel (programmatic dependent launch) and lets the attention launch behind it: it
// clears, allows its dependents, then waits for its own prerequisite so that it ends
// only after the previous kernel (whose results the attention reads) has ended.
__global__ void __launch_bounds__(256) attn_counters_clear_kernel(int4* __restrict__ words, int n16) {
  for (int i = threadIdx.x; i < n16; i += blockDim.x) words[i] = make_int4(0, 0, 0, 0);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

cudaError_t launch_attn_counters_clear(void* words, int64_t bytes, cudaStream_t stream) {
  if (bytes <= 0 || bytes % 16 || bytes > (int64_t{1} << 30)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_counters_clear_kernel, static_cast<int4*>(words), static_cast<int>(bytes / 16));
}

cudaError_t launch_lse_combine(const float* o_parts, const float* lse_parts, int64_t S, int64_t rows, int64_t D,
                               void* out, int out_dtype, int64_t H, int64_t Tq, const int64_t* os, float* lse_out,
                               cudaStream_t stream, int64_t o_part_stride, int64_t lse_part_stride) {
  if (rows == 0) return cudaSuccess;
  const int threads = static_cast<int>(lmax(32, (D + 31) / 32 * 32));
  const int64_t o_ps = o_part_stride > 0 ? o_part_stride : rows * D;
  const int64_t l_ps = lse_part_stride > 0 ? lse_part_stride : rows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows));
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, lse_combine_kernel, o_parts, lse_parts, S, rows, D, o_ps, l_ps, out, out_dtype, H,
                            Tq, os[0], os[1], os[2], os[3], lse_out);
}

}  // namespace linattn
