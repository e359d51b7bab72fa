// CSA2 compressed KV: mean-pool groups of `ratio` tokens, then store them through the
// group-wise FP4 (E2M1) or FP8 (e4m3) codec and hand the dequantised values back in the
// input dtype (CSA2Attention.compressed_kv, src/linattn/variants/csa2.py:77-85, with
// block_reduce, src/linattn/core.py:103-120, and the codec of
// src/linattn/kv/quant.py:76-109).  Scalar form: one CTA per pooled row (b, h, group), one
// thread per channel, one warp per 32-channel quantisation group; vector form below.  The arithmetic follows the
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

// x / scale stored as FP4 (nearest E2M1 magnitude, the smaller one on ties, sign kept)
// or FP8 e4m3 (round to nearest even, saturating), returned dequantised in fp32.
__device__ __forceinline__ float codec_roundtrip(float x, float scale, int bits) {
  const float n = x / scale;
  if (bits == 4) {
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
    return (n < 0.f ? -mag : mag) * scale;
  }
  const __nv_fp8_storage_t code = __nv_cvt_float_to_fp8(n, __NV_SATFINITE, __NV_E4M3);
  const __half_raw hr = __nv_cvt_fp8_to_halfraw(code, __NV_E4M3);
  return __half2float(*reinterpret_cast<const __half*>(&hr)) * scale;
}

__device__ __forceinline__ void store8(float* p, const float (&f)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&t);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void store8(__half* p, const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 t = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&t);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Vector form (D a multiple of 32, 16-byte aligned rows): a thread owns 8 consecutive
// channels (one 16-byte load per row for 16-bit types), D / 8 threads a pooled row and
// 256 / (D / 8) pooled rows a CTA; four rows of loads in flight per thread; a 32-channel
// quantisation group is four adjacent lanes (absmax by two shuffles).  Same arithmetic,
// same summation order as the scalar form.
template <typename T>
__global__ void __launch_bounds__(256) csa2_pool_quant_vec_kernel(const PoolQuantParams p, int64_t units) {
  const int tpu = static_cast<int>(p.D / 8);
  const int per_cta = 256 / tpu;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * per_cta + threadIdx.x / tpu;
  // threads past the CTA's last whole row (256 % tpu of them) and past the last unit
  // idle; no early exit: every lane takes part in the shuffles
  const bool live = static_cast<int>(threadIdx.x) < per_cta * tpu && unit < units;
  const int c0 = (threadIdx.x % tpu) * 8;
  const int64_t uu = live ? unit : 0;
  const int64_t g = uu % p.G, bh = uu / p.G;
  const int64_t h = bh % p.H, b = bh / p.H;
  const T* base = static_cast<const T*>(p.x) + b * p.s[0] + h * p.s[1] + c0;
  float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (live) {
    for (int64_t i0 = 0; i0 < p.ratio; i0 += 4) {
      float v[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        // the tail group repeats the last row; slots past the ratio re-read its last row
        const int64_t t = lmin(g * p.ratio + lmin(i0 + u, p.ratio - 1), p.T - 1);
        load8(base + t * p.s[2], v[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (i0 + u >= p.ratio) break;
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] += v[u][j];
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = round_to(x[j] / static_cast<float>(p.ratio), p.dtype);
  if (p.bits == 4 || p.bits == 8) {
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(x[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float scale = fmaxf(amax, 1e-8f) / (p.bits == 4 ? 6.f : 448.f);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = round_to(codec_roundtrip(x[j], scale, p.bits), p.dtype);
  }
  if (live) store8(static_cast<T*>(p.out) + unit * p.D + c0, x);
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
    y = round_to(codec_roundtrip(x, scale, p.bits), p.dtype);
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
  const int esz = dtype == LINATTN_F32 ? 4 : 2;
  const bool vec = D % 32 == 0 && strides[3] == 1 && strides[0] % 8 == 0 && strides[1] % 8 == 0 &&
                   strides[2] % 8 == 0 && reinterpret_cast<uintptr_t>(x) % (8 * esz) == 0 &&
                   reinterpret_cast<uintptr_t>(out) % (8 * esz) == 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (vec) {
    const int64_t per_cta = 256 / (D / 8);
    const unsigned grid = static_cast<unsigned>((units + per_cta - 1) / per_cta);
    if (dtype == LINATTN_BF16) csa2_pool_quant_vec_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p, units);
    else if (dtype == LINATTN_F16) csa2_pool_quant_vec_kernel<__half><<<grid, 256, 0, st>>>(p, units);
    else csa2_pool_quant_vec_kernel<float><<<grid, 256, 0, st>>>(p, units);
  } else {
    const unsigned threads = static_cast<unsigned>((D + 31) / 32 * 32);
    csa2_pool_quant_kernel<<<static_cast<unsigned>(units), threads, 0, st>>>(p);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "csa2_pool_quant: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
