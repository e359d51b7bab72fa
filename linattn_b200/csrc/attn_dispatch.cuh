// Instantiation helper: one translation unit per KV element type includes this
// with ATTN_T set, so the template instances compile in parallel.
#pragma once
#include "launchers.cuh"
#include "sparse_attention_mma.cuh"

namespace linattn {

template <typename T, int D, int G>
static cudaError_t launch_one(const AttnParams& p, unsigned grid, cudaStream_t stream) {
  using S = AttnShape<T, D, G>;
  static bool configured[64] = {};
  const int dev = device_index();
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(sparse_attention_kernel<T, D, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(S::SMEM_BYTES));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  sparse_attention_kernel<T, D, G><<<grid, 256, S::SMEM_BYTES, stream>>>(p);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_g(const AttnParams& p, int G, unsigned grid, cudaStream_t stream) {
  switch (G) {
    case 1: return launch_one<T, D, 1>(p, grid, stream);
    case 2: return launch_one<T, D, 2>(p, grid, stream);
    case 4: return launch_one<T, D, 4>(p, grid, stream);
    case 8: return launch_one<T, D, 8>(p, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_dg(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream) {
  switch (D) {
    case 8: if constexpr (sizeof(T) >= 2) return launch_g<T, 8>(p, G, grid, stream); else return cudaErrorInvalidValue;
    case 16: return launch_g<T, 16>(p, G, grid, stream);
    case 32: return launch_g<T, 32>(p, G, grid, stream);
    case 64: return launch_g<T, 64>(p, G, grid, stream);
    case 128: return launch_g<T, 128>(p, G, grid, stream);
    case 256: return launch_g<T, 256>(p, G, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

int sm_count();

template <typename T, int D, int NQT = 1>
static cudaError_t launch_mma_d(const AttnParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int box_rows,
                                int* counter, int64_t n_items, cudaStream_t stream) {
  using S = MmaShape<D, sizeof(T)>;
  static bool configured[64] = {};
  const int dev = device_index();
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(sparse_attention_mma_kernel<T, D, NQT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(S::SMEM_BYTES));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int64_t want = (n_items + S::NW - 1) / S::NW;
  const int grid = static_cast<int>(lmax(1, lmin(sm_count(), want)));
  // programmatic dependent launch: the CTAs may start (set-up only) while the
  // previous kernel in the stream finishes; griddepcontrol.wait orders every read
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(32 * S::NW);
  cfg.dynamicSmemBytes = S::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sparse_attention_mma_kernel<T, D, NQT>, p, tmk, tmv, box_rows, counter, n_items);
}

template <typename T>
static cudaError_t launch_mma(const AttnParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int box_rows, int D,
                              int* counter, int64_t n_items, cudaStream_t stream) {
  if constexpr (sizeof(T) == 1) {
    // q as e4m3 terms: two hold a bf16 q exactly, an f16 q takes three
    if (D != 128) return cudaErrorInvalidValue;
    if (p.q_dtype == LINATTN_BF16) return launch_mma_d<T, 128, 2>(p, tmk, tmv, box_rows, counter, n_items, stream);
    if (p.q_dtype == LINATTN_F16) return launch_mma_d<T, 128, 3>(p, tmk, tmv, box_rows, counter, n_items, stream);
    return cudaErrorInvalidValue;
  } else {
    switch (D) {
      case 64: return launch_mma_d<T, 64>(p, tmk, tmv, box_rows, counter, n_items, stream);
      case 128: return launch_mma_d<T, 128>(p, tmk, tmv, box_rows, counter, n_items, stream);
      default: return cudaErrorInvalidValue;
    }
  }
}

template <typename T>
constexpr int tile_rows(int D) {
  return (16384 / (D * static_cast<int>(sizeof(T)))) < 64 ? (16384 / (D * static_cast<int>(sizeof(T)))) : 64;
}

}  // namespace linattn
