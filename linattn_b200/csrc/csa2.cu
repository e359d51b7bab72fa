// CSA2 compressed KV: mean-pool groups of `ratio` tokens, then store them through the
// group-wise FP4 (E2M1) or FP8 (e4m3) codec and hand the dequantised values back in the
// input dtype (CSA2Attention.compressed_kv, src/linattn/variants/csa2.py:77-85, with
// block_reduce, src/linattn/core.py:103-120, and the codec of
// src/linattn/kv/quant.py:76-109).  One CTA per pooled row (b, h, group), one thread per
// channel, one warp per 32-channel quantisation group.  The arithmetic follows the
// reference step by step so that codes agree bit for bit: the mean is rounded to the
// input dtype first (the reference pools in that dtype; a no-op for f32), scale = max(absmax, 1e-8) / 6
// (or / 448) by true division, x / scale by true division, FP4 takes the nearest grid
// magnitude with ties to the smaller one (argmin's first index), FP8 rounds to nearest
// even; the dequantised value (magnitude x scale in fp32) is rounded to the dtype.
#include <cstdio>

#include "launchers.cuh"

namespace linattn {

namespace {

struct PoolQuantParams {
  const void* x;
  int dtype;
  int64_t B, H, T, D, s[4];
  int64_t ratio, G;
  int bits;
  void* out;  // (B, H, G, D) contiguous, dtype
};

__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == LINATTN_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == LINATTN_F16) return __half2float(__float2half_rn(v));
  return v;
}

__global__ void __launch_bounds__(256) csa2_pool_quant_kernel(const PoolQuantParams p) {
  const int64_t unit = blockIdx.x;  // (b, h, g)
  const int64_t g = unit % p.G, bh = unit / p.G;
  const int64_t h = bh % p.H, b = bh / p.H;
  const int c = threadIdx.x;
  const bool live = c < p.D;
  float x = 0.f;
  if (live) {
    // the tail group repeats the last row
    float acc = 0.f;
    const int64_t base = b * p.s[0] + h * p.s[1] + c * p.s[3];
    for (int64_t i = 0; i < p.ratio; ++i) {
      const int64_t t = lmin(g * p.ratio + i, p.T - 1);
      acc += load_any(p.x, base + t * p.s[2], p.dtype);
    }
    x = round_to(acc / static_cast<float>(p.ratio), p.dtype);
  }
  float y = x;
  if (p.bits == 4 || p.bits == 8) {
    float amax = live ? fabsf(x) : 0.f;  // channels past D pad the group with zeros
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = fmaxf(amax, 1e-8f) / (p.bits == 4 ? 6.f : 448.f);
    const float n = x / scale;
    if (p.bits == 4) {
      const float grid[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
      const float a = fabsf(n);
      float mag = grid[0];
      float bd = fabsf(a - grid[0]);
#pragma unroll
      for (int i = 1; i < 8; ++i) {
        const float d = fabsf(a - grid[i]);
        if (d < bd) {  // strict: ties keep the smaller magnitude
          bd = d;
          mag = grid[i];
        }
      }
      y = (n < 0.f ? -mag : mag) * scale;
    } else {
      const __nv_fp8_storage_t code = __nv_cvt_float_to_fp8(n, __NV_SATFINITE, __NV_E4M3);
      const __half_raw hr = __nv_cvt_fp8_to_halfraw(code, __NV_E4M3);
      y = __half2float(*reinterpret_cast<const __half*>(&hr)) * scale;
    }
    y = round_to(y, p.dtype);
  }
  if (live) {
    const int64_t o = unit * p.D + c;
    if (p.dtype == LINATTN_BF16) static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(y);
    else if (p.dtype == LINATTN_F16) static_cast<__half*>(p.out)[o] = __float2half_rn(y);
    else static_cast<float*>(p.out)[o] = y;
  }
}

}  // namespace

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_csa2_pool_quant(const void* x, int32_t dtype, int64_t B, int64_t H, int64_t T, int64_t D,
                                       const int64_t* strides, int64_t ratio, int32_t bits, int32_t group,
                                       void* out, void* stream) {
  if (!x || !out || !strides) return set_error(LINATTN_EINVAL, "csa2_pool_quant: NULL pointer");
  if (dtype != LINATTN_BF16 && dtype != LINATTN_F16 && dtype != LINATTN_F32)
    return set_error(LINATTN_EUNSUPPORTED, "csa2_pool_quant: dtype must be bf16, f16 or f32");
  if (bits != 4 && bits != 8 && bits != 16) return set_error(LINATTN_EINVAL, "csa2_pool_quant: bits must be 4, 8 or 16");
  if (bits != 16 && group != 32)
    return set_error(LINATTN_EUNSUPPORTED, "csa2_pool_quant: quantisation groups of 32 channels only");
  if (ratio < 1 || D < 1 || D > 256 || B < 0 || H < 0 || T < 0)
    return set_error(LINATTN_EINVAL, "csa2_pool_quant: bad sizes (ratio >= 1, 1 <= D <= 256)");
  if (B == 0 || H == 0 || T == 0) return LINATTN_OK;
  PoolQuantParams p;
  p.x = x; p.dtype = dtype; p.B = B; p.H = H; p.T = T; p.D = D;
  for (int i = 0; i < 4; ++i) p.s[i] = strides[i];
  p.ratio = ratio; p.G = (T + ratio - 1) / ratio; p.bits = bits; p.out = out;
  const int64_t units = B * H * p.G;
  if (units > 0x7fffffff) return set_error(LINATTN_EUNSUPPORTED, "csa2_pool_quant: too many groups");
  const unsigned threads = static_cast<unsigned>((D + 31) / 32 * 32);
  csa2_pool_quant_kernel<<<static_cast<unsigned>(units), threads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "csa2_pool_quant: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
