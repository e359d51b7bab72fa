// linattn_read_bandwidth: the read roof of a buffer, for the roofline of kernels whose
// reads hit L2 (the DSA token attention's gathered rows) rather than HBM.  A persistent
// grid (two CTAs per SM) reads the buffer `reps` times with 16-byte loads, eight in
// flight per thread, and folds what it read into one word per CTA so the loads stay
// live.  A buffer that fits the 126 MB L2 measures L2 reads; a larger one, HBM reads.
// Measurement utility only: no counterpart in the reference.
#include <cstdio>

#include "launchers.cuh"

namespace linattn {

namespace {

__global__ void __launch_bounds__(512) read_probe_kernel(const uint4* __restrict__ buf, int64_t n16, int reps,
                                                         uint32_t* __restrict__ sink) {
  uint32_t acc = 0u;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int r = 0; r < reps; ++r) {
    int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + 7 * stride < n16; i += 8 * stride) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldcg(buf + i + u * stride);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
    }
    for (; i < n16; i += stride) {
      const uint4 v = __ldcg(buf + i);
      acc ^= v.x ^ v.y ^ v.z ^ v.w;
    }
  }
  // one word per CTA: the xor of its threads' folds
  for (int off = 16; off >= 1; off >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, off);
  if ((threadIdx.x & 31) == 0) atomicXor(sink + blockIdx.x, acc);
}

}  // namespace

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_read_bandwidth(const void* buf, int64_t bytes, int32_t reps, uint32_t* sink,
                                      int64_t sink_words, void* stream) {
  if (!buf || !sink) return set_error(LINATTN_EINVAL, "read_bandwidth: NULL pointer");
  if (bytes < 16 || bytes % 16 || (reinterpret_cast<uintptr_t>(buf) & 15) || reps < 1)
    return set_error(LINATTN_EINVAL, "read_bandwidth: bytes must be a positive multiple of 16 at a 16-byte address");
  const int64_t grid = lmin(2 * static_cast<int64_t>(sm_count()), sink_words);
  if (grid < 1) return set_error(LINATTN_EINVAL, "read_bandwidth: sink_words must be >= 1");
  read_probe_kernel<<<static_cast<unsigned>(grid), 512, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(buf), bytes / 16, reps, sink);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "read_bandwidth: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
