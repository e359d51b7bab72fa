// Shared device helpers for the sm_100a kernels of linattn_b200.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "linattn_b200.h"

namespace linattn {

// ---------------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------------
struct fp8e4m3 {
  uint8_t x;
};

template <typename T> struct ElemBytes { static constexpr int value = sizeof(T); };

// Convert 8 consecutive elements at `p` (16-byte aligned for 16-bit types, 8-byte for
// fp8, 32-byte for fp32) to float.
__device__ __forceinline__ void load8(const float* p, float (&f)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
__device__ __forceinline__ void load8(const __half* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ float2 fp8x2_to_float2(uint16_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
__device__ __forceinline__ void load8(const fp8e4m3* p, float (&f)[8]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const uint32_t w[2] = {u.x, u.y};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float2 lo = fp8x2_to_float2(static_cast<uint16_t>(w[i] & 0xffffu));
    const float2 hi = fp8x2_to_float2(static_cast<uint16_t>(w[i] >> 16));
    f[4 * i] = lo.x; f[4 * i + 1] = lo.y; f[4 * i + 2] = hi.x; f[4 * i + 3] = hi.y;
  }
}

// Two consecutive elements -> float2.
__device__ __forceinline__ float2 load2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 load2(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
__device__ __forceinline__ float2 load2(const __nv_bfloat16* p) {
  const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ float2 load2(const fp8e4m3* p) {
  return fp8x2_to_float2(*reinterpret_cast<const uint16_t*>(p));
}

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

// Load one element of a runtime-typed tensor as float (q vectors, weights).
__device__ __forceinline__ float load_any(const void* base, int64_t idx, int dtype) {
  switch (dtype) {
    case LINATTN_F32: return static_cast<const float*>(base)[idx];
    case LINATTN_F16: return __half2float(static_cast<const __half*>(base)[idx]);
    case LINATTN_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
    default: return 0.f;
  }
}
__device__ __forceinline__ void store_any(void* base, int64_t idx, int dtype, float v) {
  switch (dtype) {
    case LINATTN_F32: static_cast<float*>(base)[idx] = v; break;
    case LINATTN_F16: static_cast<__half*>(base)[idx] = __float2half_rn(v); break;
    case LINATTN_BF16: static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v); break;
    default: break;
  }
}

__host__ __device__ __forceinline__ int64_t lmin(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t lmax(int64_t a, int64_t b) { return a > b ? a : b; }

// ---------------------------------------------------------------------------------
// order-preserving float keys (larger float -> larger key; -0 folded onto +0)
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t float_key(float f) {
  const uint32_t b = __float_as_uint(f + 0.0f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}

// ---------------------------------------------------------------------------------
// device status
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void report(int32_t* status, int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// ---------------------------------------------------------------------------------
// mbarrier + 1-D bulk copy (TMA, no tensor map, no multicast)
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for the phase with `parity` to complete, giving up after ~`limit_ns` (or
// 2^28 polls, whichever is first).  Returns false on give-up; the caller reports
// LINATTN_DEV_TIMEOUT and unwinds.  No wait in this library is unbounded.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < (1u << 28); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && global_ns() - t0 > limit_ns) return false;
  }
  return false;
}
// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte
// aligned) completing on `bar` (complete_tx).  The CTA is its own cluster.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------------
// block-wide exclusive scan of one uint32 per thread (blockDim.x == 256)
// ---------------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* scratch /*[NT/32 + 1]*/,
                                                         uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < NT / 32 ? scratch[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < NT / 32) scratch[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const uint32_t warp_base = warp > 0 ? scratch[warp - 1] : 0u;
  if (total) *total = scratch[NT / 32 - 1];
  const uint32_t excl = warp_base + x - v;
  __syncthreads();  // scratch reusable after return
  return excl;
}

}  // namespace linattn
