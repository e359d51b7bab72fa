// Lightning-indexer scores on the tensor cores.
//
// I[b,t,s] = scale_s * sum_h w[b,t,h] * ReLU(q[b,t,h,:] . k[b,s,h,:]), fp32 accumulate
// (src/linattn/kernels/triton/fused_indexer.py:52-60).  One CTA = 64 queries x a chunk
// of key tiles (64 keys each); 8 warps = 4 (16 queries) x 2 (32 keys of a tile).
//
// * Key tiles arrive by TMA (2-D map over the [B*T_k, H*D] key rows, 128-byte boxes
//   with 128-byte swizzle) into a 4-stage ring; thread 0 refills a stage after the
//   CTA barrier that ends its use.
// * The product is mma.sync m16n8k16 with fp32 accumulation.  The 16 channels of one
//   k-step are permuted identically in q and k (logical k = {2c, 2c+1, 2c+8, 2c+9} ->
//   physical 4c..4c+3 for lane quad c), so a lane's B fragment is one contiguous
//   4-element read of a key row: 4 bytes for fp8 (two cvt.rn.f16x2.e4m3x2) or 8 bytes
//   for 16-bit keys.  The sum over channels is unchanged by the permutation.
// * fp8 e4m3 keys are multiplied as f16 (exact).  A bf16 query is then scaled per
//   (t, h) by a power of two so that its largest element sits in [2^14, 2^15): every
//   element above 2^-32 of the largest is exact in f16, and the scale is undone
//   exactly in the head weight.  bf16 / f16 keys with a query of the same type run
//   bf16 / f16 products without conversion.
// * Query fragments (all heads) live in registers for the CTA's lifetime; the
//   per-head dot products are ReLU'd and folded into the weighted sum in registers.
#include <cudaTypedefs.h>

#include <cstdio>

#include "launchers.cuh"
#include "sparse_attention_mma.cuh"

namespace linattn {

namespace {

constexpr int XQ = 64;    // queries per CTA
constexpr int XK = 64;    // keys per tile
constexpr int XSTG = 4;   // ring stages
constexpr int XKCT = 32;  // key tiles per CTA

struct IndexerMmaParams {
  const void* q;
  int q_dtype;
  int64_t qs[4];
  const float* k_scale;
  int64_t group, ss;
  const void* w;
  int w_dtype;
  int64_t ws[3];
  int64_t Tq, Tk;  // Tq = t_end
  int causal;      // 0: none, 1: mask and write -inf, 2: mask, skip tiles past every query
  int64_t offset, kb, t_begin;  // key s is visible from t iff s * kb <= offset + t
  float* scores;
  int64_t row_stride;
  int32_t* status;
};

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t v16) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v16), __NV_E4M3);
  return static_cast<uint32_t>(h.x) | (static_cast<uint32_t>(h.y) << 16);
}

template <typename MT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  return MmaOp<__half>::pack(lo, hi);
}
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  return MmaOp<__nv_bfloat16>::pack(lo, hi);
}

}  // namespace

// KEB: key element bytes (1 = fp8 e4m3 -> f16 products, 2 = same type as MT).
template <typename MT, int KEB, int H, int D, bool SCALE_Q>
__global__ void __launch_bounds__(256, 2)
    indexer_mma_kernel(const IndexerMmaParams p, const __grid_constant__ CUtensorMap tmk) {
  constexpr int HD = H * D;
  constexpr int KS = D / 16;                 // k-steps per head
  constexpr int ROW_BYTES = HD * KEB;        // one key row
  constexpr int NBOX = ROW_BYTES / 128;      // 128-byte boxes per row
  constexpr int BOX_BYTES = XK * 128;
  constexpr int STAGE_BYTES = NBOX * BOX_BYTES;
  extern __shared__ __align__(1024) unsigned char xsmem_raw[];
  unsigned char* xsmem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(xsmem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full_bar[XSTG];
  __shared__ float col_scale[XKCT * XK];  // key scales of this CTA's key range (fp8)

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wq = warp & 3, wk = warp >> 2;
  const int g = lane >> 2, c = lane & 3;
  const int64_t b = blockIdx.z;
  const int64_t q0 = p.t_begin + static_cast<int64_t>(blockIdx.y) * XQ;
  const int64_t t_last = lmin(p.Tq, q0 + XQ) - 1;
  const int64_t n_tiles_all = (p.Tk + XK - 1) / XK;
  const int64_t kt0 = static_cast<int64_t>(blockIdx.x) * XKCT;
  const int64_t kt_chunk_end = lmin(n_tiles_all, kt0 + XKCT);
  int64_t kt_end = kt_chunk_end;
  if (p.causal) {
    // tiles with a key visible from the block's last query
    const int64_t pos = p.offset + t_last;
    kt_end = pos < 0 ? kt0 : lmin(kt_end, (pos / p.kb) / XK + 1);
  }
  const int64_t n = lmax(0, kt_end - kt0);
  const int64_t rows_per_b = p.Tq - p.t_begin;

  if (tid == 0) {
    for (int s = 0; s < XSTG; ++s) mbar_init(&full_bar[s], 1);
    mbar_fence_init();
  }
  __syncthreads();
  auto issue = [&](int stage, int64_t kt) {
    mbar_arrive_expect_tx(&full_bar[stage], STAGE_BYTES);
    const int y = static_cast<int>(b * p.Tk + kt * XK);
#pragma unroll
    for (int bx = 0; bx < NBOX; ++bx)
      tma_load_2d(xsmem + stage * STAGE_BYTES + bx * BOX_BYTES, &tmk, bx * (128 / KEB), y, &full_bar[stage]);
  };
  if (tid == 0)
    for (int s = 0; s < XSTG && s < n; ++s) issue(s, kt0 + s);
  if (p.k_scale) {
    // one group index per key; the groups of a 64-key tile are consecutive
    for (int e = tid; e < n * XK; e += 256) {
      const int64_t col = kt0 * XK + e;
      col_scale[e] = col < p.Tk ? p.k_scale[b * p.ss + col / p.group] : 0.f;
    }
  }

  // ---- query fragments and weights (rows r0 = q0 + 16 wq + g, r1 = r0 + 8)
  const int64_t r0 = q0 + wq * 16 + g, r1 = r0 + 8;
  const bool v0 = r0 <= t_last, v1 = r1 <= t_last;
  uint32_t a[H][KS][4];
  float wv[2][H];
#pragma unroll
  for (int h = 0; h < H; ++h) {
    float x[2][KS][4];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int64_t r = rr ? r1 : r0;
      const bool ok = rr ? v1 : v0;
      const int64_t base = b * p.qs[0] + r * p.qs[1] + h * p.qs[2];
#pragma unroll
      for (int j = 0; j < KS; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          x[rr][j][e] = ok ? load_any(p.q, base + (16 * j + 4 * c + e) * p.qs[3], p.q_dtype) : 0.f;
      wv[rr][h] = ok ? load_any(p.w, b * p.ws[0] + r * p.ws[1] + h * p.ws[2], p.w_dtype) : 0.f;
      if (SCALE_Q) {
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < KS; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) m = fmaxf(m, fabsf(x[rr][j][e]));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        // power of two that lifts the largest element into [2^14, 2^15), within 2^+-64
        int ex = 0;
        if (m > 0.f) ex = 14 - (static_cast<int>((__float_as_uint(m) >> 23) & 0xffu) - 127);
        ex = ex < -64 ? -64 : (ex > 64 ? 64 : ex);
        const float up = __uint_as_float(static_cast<uint32_t>(127 + ex) << 23);
        const float down = __uint_as_float(static_cast<uint32_t>(127 - ex) << 23);
#pragma unroll
        for (int j = 0; j < KS; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) x[rr][j][e] *= up;
        wv[rr][h] *= down;
      }
    }
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      a[h][j][0] = pack2<MT>(x[0][j][0], x[0][j][1]);
      a[h][j][1] = pack2<MT>(x[1][j][0], x[1][j][1]);
      a[h][j][2] = pack2<MT>(x[0][j][2], x[0][j][3]);
      a[h][j][3] = pack2<MT>(x[1][j][2], x[1][j][3]);
    }
  }

  int64_t stalled = -1;  // first tile whose copy did not arrive in time
  for (int64_t i = 0; i < n; ++i) {
    const int stage = static_cast<int>(i % XSTG);
    const bool late = !mbar_wait_bounded(&full_bar[stage], static_cast<uint32_t>((i / XSTG) & 1));
    if (__syncthreads_or(late)) {
      stalled = i;
      break;
    }
    const int64_t s0 = (kt0 + i) * XK;
    const uint32_t sbase = smem_u32(xsmem + stage * STAGE_BYTES);
    float tot[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) tot[nt][0] = tot[nt][1] = tot[nt][2] = tot[nt][3] = 0.f;
#pragma unroll
    for (int h = 0; h < H; ++h) {
      float acc[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
      for (int j = 0; j < KS; ++j) {
        const int off = (h * D + 16 * j + 4 * c) * KEB;  // byte offset in the key row
        const int box = off >> 7, chunk = (off & 127) >> 4, within = off & 15;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int row = wk * 32 + nt * 8 + g;
          const uint32_t addr = sbase + box * BOX_BYTES + row * 128 + (((chunk ^ (row & 7)) << 4) | within);
          uint32_t b0, b1;
          if (KEB == 1) {
            const uint32_t v = lds32(addr);
            b0 = e4m3x2_to_f16x2(v & 0xffffu);
            b1 = e4m3x2_to_f16x2(v >> 16);
          } else {
            const uint2 v = lds64(addr);
            b0 = v.x;
            b1 = v.y;
          }
          MmaOp<MT>::mma(acc[nt], a[h][j], b0, b1);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        tot[nt][0] = fmaf(wv[0][h], fmaxf(acc[nt][0], 0.f), tot[nt][0]);
        tot[nt][1] = fmaf(wv[0][h], fmaxf(acc[nt][1], 0.f), tot[nt][1]);
        tot[nt][2] = fmaf(wv[1][h], fmaxf(acc[nt][2], 0.f), tot[nt][2]);
        tot[nt][3] = fmaf(wv[1][h], fmaxf(acc[nt][3], 0.f), tot[nt][3]);
      }
    }
    // every warp is done with this stage: refill it
    __syncthreads();
    if (tid == 0 && i + XSTG < n) issue(stage, kt0 + i + XSTG);
    // ---- epilogue: key scales, causal mask, store
    const bool diag = p.causal && (s0 + XK - 1) * p.kb > p.offset + q0;
    float* out0 = p.scores + (b * rows_per_b + r0 - p.t_begin) * p.row_stride;
    float* out1 = out0 + 8 * p.row_stride;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int64_t col = s0 + wk * 32 + nt * 8 + 2 * c;
      float sc0 = 1.f, sc1 = 1.f;
      if (p.k_scale) {
        const int lc = static_cast<int>(col - kt0 * XK);
        sc0 = col_scale[lc];
        sc1 = col_scale[lc + 1];
      }
      float o[4] = {tot[nt][0] * sc0, tot[nt][1] * sc1, tot[nt][2] * sc0, tot[nt][3] * sc1};
      if (diag) {
        if (col * p.kb > p.offset + r0) o[0] = -INFINITY;
        if ((col + 1) * p.kb > p.offset + r0) o[1] = -INFINITY;
        if (col * p.kb > p.offset + r1) o[2] = -INFINITY;
        if ((col + 1) * p.kb > p.offset + r1) o[3] = -INFINITY;
      }
      if (col + 1 < p.Tk && (p.row_stride & 1) == 0) {
        if (v0) *reinterpret_cast<float2*>(out0 + col) = make_float2(o[0], o[1]);
        if (v1) *reinterpret_cast<float2*>(out1 + col) = make_float2(o[2], o[3]);
      } else {
        if (v0 && col < p.Tk) out0[col] = o[0];
        if (v0 && col + 1 < p.Tk) out0[col + 1] = o[1];
        if (v1 && col < p.Tk) out1[col] = o[2];
        if (v1 && col + 1 < p.Tk) out1[col + 1] = o[3];
      }
    }
  }
  if (stalled >= 0) {
    // report, then give the copies still in flight (tiles stalled .. stalled + XSTG - 1)
    // a bounded time to land before the CTA releases its shared memory
    if (tid == 0) {
      report(p.status, LINATTN_DEV_TIMEOUT);
      for (int64_t j = stalled; j < n && j < stalled + XSTG; ++j)
        mbar_wait_bounded(&full_bar[j % XSTG], static_cast<uint32_t>((j / XSTG) & 1), 200000000ull);
    }
    return;
  }
  // ---- causal, mode 1: tiles of this chunk after every query of the block hold -inf
  if (p.causal == 1 && kt_end < kt_chunk_end) {
    const int64_t c0 = lmax(kt0, kt_end) * XK, c1 = lmin(p.Tk, kt_chunk_end * XK);
    const int64_t w = c1 - c0;
    for (int64_t e = tid; e < XQ * w; e += 256) {
      const int64_t r = q0 + e / w, col = c0 + e % w;
      if (r <= t_last) p.scores[(b * rows_per_b + r - p.t_begin) * p.row_stride + col] = -INFINITY;
    }
  }
}

namespace {

template <typename MT, int KEB, int H, int D, bool SCALE_Q>
cudaError_t launch_t(const IndexerMmaParams& p, const CUtensorMap& tm, dim3 grid, cudaStream_t st) {
  constexpr int STAGE_BYTES = H * D * KEB / 128 * XK * 128;
  constexpr int smem = XSTG * STAGE_BYTES + 1024;
  auto kern = indexer_mma_kernel<MT, KEB, H, D, SCALE_Q>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, 256, smem, st>>>(p, tm);
  return cudaGetLastError();
}

template <typename MT, int KEB, bool SCALE_Q>
cudaError_t launch_hd(int H, int D, const IndexerMmaParams& p, const CUtensorMap& tm, dim3 grid, cudaStream_t st) {
#define LINATTN_IDX_CASE(HH, DD) \
  if (H == HH && D == DD) return launch_t<MT, KEB, HH, DD, SCALE_Q>(p, tm, grid, st);
  LINATTN_IDX_CASE(1, 64)
  LINATTN_IDX_CASE(2, 64)
  LINATTN_IDX_CASE(4, 64)
  LINATTN_IDX_CASE(1, 128)
  LINATTN_IDX_CASE(2, 128)
  LINATTN_IDX_CASE(4, 32)
  LINATTN_IDX_CASE(8, 32)
  LINATTN_IDX_CASE(4, 16)
  LINATTN_IDX_CASE(8, 16)
#undef LINATTN_IDX_CASE
  return cudaErrorInvalidValue;
}

}  // namespace

// The tensor-core path; returns false (nothing launched) when the call is not
// eligible, so the caller runs the CUDA-core kernel instead.
bool indexer_scores_mma(const void* q, int q_dtype, const int64_t* qs, const void* k, int k_dtype, const int64_t* ks,
                        const float* k_scale, int64_t group, int64_t ss, const void* w, int w_dtype, const int64_t* ws,
                        int64_t B, int64_t Tq, int64_t Tk, int64_t H, int64_t D, int causal, int64_t offset,
                        int64_t key_block, int64_t t_begin, int64_t t_end, float* scores, int64_t row_stride, int32_t* status,
                        cudaStream_t st, cudaError_t* err) {
  *err = cudaSuccess;
  if (q_dtype != LINATTN_F16 && q_dtype != LINATTN_BF16) return false;
  const bool fp8 = k_dtype == LINATTN_FP8E4M3;
  if (!fp8 && k_dtype != q_dtype) return false;
  const int keb = fp8 ? 1 : 2;
  const bool shape_ok = (H == 1 && D == 64) || (H == 2 && D == 64) || (H == 4 && D == 64) || (H == 1 && D == 128) ||
                        (H == 2 && D == 128) || (H == 4 && D == 32) || (H == 8 && D == 32) ||
                        (H == 4 && D == 16) || (H == 8 && D == 16);  // CSA2 / DSA plugin indexer shapes
  if (!shape_ok || (H * D * keb) % 128 != 0) return false;
  if (ks[3] != 1 || ks[2] != D || ks[1] != H * D || (B > 1 && ks[0] != Tk * H * D)) return false;
  if (reinterpret_cast<uintptr_t>(k) % 16 != 0 || B * Tk >= (int64_t(1) << 31) - XK) return false;
  if ((t_end - t_begin + XQ - 1) / XQ > 65535 || B > 65535) return false;
  CUtensorMap tm;
  const CUtensorMapDataType cu = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                     : (k_dtype == LINATTN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  if (!tensor_map_2d(&tm, k, cu, H * D, B * Tk, H * D * keb, 128 / keb, XK)) return false;
  IndexerMmaParams p;
  p.q = q; p.q_dtype = q_dtype;
  for (int i = 0; i < 4; ++i) p.qs[i] = qs[i];
  p.k_scale = fp8 ? k_scale : nullptr; p.group = group > 0 ? group : 1; p.ss = ss;
  p.w = w; p.w_dtype = w_dtype;
  for (int i = 0; i < 3; ++i) p.ws[i] = ws[i];
  p.Tq = t_end; p.Tk = Tk; p.causal = causal; p.offset = offset; p.kb = key_block; p.t_begin = t_begin;
  p.scores = scores; p.row_stride = row_stride; p.status = status;
  const int64_t n_tiles = (Tk + XK - 1) / XK;
  dim3 grid(static_cast<unsigned>((n_tiles + XKCT - 1) / XKCT), static_cast<unsigned>((t_end - t_begin + XQ - 1) / XQ),
            static_cast<unsigned>(B));
  const int h = static_cast<int>(H), d = static_cast<int>(D);
  if (fp8)
    *err = q_dtype == LINATTN_BF16 ? launch_hd<__half, 1, true>(h, d, p, tm, grid, st)
                                   : launch_hd<__half, 1, false>(h, d, p, tm, grid, st);
  else if (q_dtype == LINATTN_BF16)
    *err = launch_hd<__nv_bfloat16, 2, false>(h, d, p, tm, grid, st);
  else
    *err = launch_hd<__half, 2, false>(h, d, p, tm, grid, st);
  return true;
}

}  // namespace linattn
