// Block-sparse causal prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Every query row reads the 64-token key blocks of its own ascending block list (one
// list per `rows_per_list` consecutive queries: 64 for per-q-block lists such as
// MInference's block-sparse pattern or sink + window + top-k, 1 for MoBA's per-token
// routing), plus the tokens below `sink`, causally (key <= offset + t) and below T_k.
// (MInferenceAttention._block_sparse / MoBAAttention.select + the masked attention of
// BlockSelectionAttention.attend, src/linattn/variants/selection.py:86-116, 339-353,
// 635-649.)
//
// One CTA = 128 query rows of one (batch, head); it walks the ascending union of its
// rows' lists, 64 keys at a time, and a row ignores (-inf) the blocks not in its list.
// Warp roles (192 threads, one CTA per SM):
//   warp 0     TMEM allocation (256 columns) and the TMA producer: Q (two 128x64 boxes)
//              once, then K and V blocks (two 64x64 boxes each, 128-byte swizzle) into
//              a 3-stage ring;
//   warp 1     one thread issues tcgen05.mma (kind::f16, M = 128, fp32 accumulators in
//              TMEM): S_j = Q K_j^T (N = 64) into one of two S buffers, then
//              O += P_{j-1} V_{j-1} (N = 128, V read MN-major), and commits each to the
//              mbarriers the other roles wait on;
//   warps 2-5  softmax, one thread per row (TMEM lane): tcgen05.ld of its S row, masks,
//              online softmax in the log2 domain, P written into swizzled shared
//              tiles (the A operand of the PV product): for bf16 as hi + lo parts
//              (two products, P to ~2^-17), for f16 one tile with the row sum of the
//              rounded P (O / l an exact weighted mean of V rows).  O is rescaled in TMEM
//              only when a row's running maximum grows by more than 8 (a factor 256),
//              so P stays below 2^8 and the rare rescale waits for the PV in flight.
//              The epilogue reads O from TMEM, divides by the row sum and stores.
// Every mbarrier wait is bounded (LINATTN_DEV_TIMEOUT on give-up); TMEM is released on
// every path.
#include <cudaTypedefs.h>

#include <cstdio>
#include <type_traits>

#include "launchers.cuh"
#include "sparse_attention_mma.cuh"

namespace linattn {

struct PrefillParams {
  int64_t B, Hq, Hkv, Tq, Tk;
  const int32_t* ids;     // (B, Hq, n_list_rows, n_max) ascending block ids, -1 padded
  const int32_t* counts;  // (B, Hq, n_list_rows) or NULL
  int64_t ls_b, ls_h, ls_r, n_max, rows_per_list, cs_b, cs_h, cs_r;
  int64_t sink;           // tokens [0, sink) are read by every row
  int causal;
  int64_t offset;
  float scale_log2;
  void* out;
  int64_t os[4];
  int out_dtype;
  float* lse;             // (B, Hq, Tq) or NULL
  int64_t n_tiles;        // query tiles of 128 per (b, head)
  int64_t n_kb;           // key blocks
  int32_t* status;
};

namespace {

constexpr int PQ = 128;          // query rows per CTA
constexpr int PK = 64;           // keys per block
constexpr int PKST = 3;          // K / V ring stages
constexpr int PLMAX = 64;        // longest list a row may have
constexpr int PMAXKB = 4096;     // key blocks (T_k <= 2^18)
constexpr int BOXB = 64 * 128;   // one 64-row x 128-byte box
constexpr int QBYTES = 2 * PQ * 128;           // Q: two 128 x 64 boxes
constexpr int STAGE = 4 * BOXB;                // K (2 boxes) + V (2 boxes)
constexpr int PBYTES = PQ * 128;               // P: 128 rows x 64 keys (16-bit)
// bf16: P = hi + lo (two tiles per buffer, 2^-17 relative); f16: one tile (2^-11)
constexpr int SMEM_DYN = 1024 + QBYTES + PKST * STAGE + 2 * 2 * PBYTES;

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;  // 128-byte swizzle
  return d;
}
// kind::f16 instruction descriptor: fp32 accumulate, A / B type `ab` (0 f16, 1 bf16)
__host__ __device__ constexpr uint32_t umma_idesc(int ab, int m, int n, int b_mn_major) {
  return (1u << 4) | (static_cast<uint32_t>(ab) << 7) | (static_cast<uint32_t>(ab) << 10) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

#define LINATTN_R8(i) "=r"(v[i]), "=r"(v[i + 1]), "=r"(v[i + 2]), "=r"(v[i + 3]), "=r"(v[i + 4]), "=r"(v[i + 5]), \
                      "=r"(v[i + 6]), "=r"(v[i + 7])
// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : LINATTN_R8(0), LINATTN_R8(8), LINATTN_R8(16), LINATTN_R8(24)
      : "r"(taddr));
}
#undef LINATTN_R8
#define LINATTN_W8(i) "r"(v[i]), "r"(v[i + 1]), "r"(v[i + 2]), "r"(v[i + 3]), "r"(v[i + 4]), "r"(v[i + 5]), \
                      "r"(v[i + 6]), "r"(v[i + 7])
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      LINATTN_W8(0), LINATTN_W8(8), LINATTN_W8(16), LINATTN_W8(24)
      : "memory");
}
#undef LINATTN_W8
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace

template <typename T>
__global__ void __launch_bounds__(192, 1)
    prefill_umma_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tmq,
                        const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  using M = MmaOp<T>;
  constexpr int AB = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC_S = umma_idesc(AB, PQ, PK, 0);
  constexpr uint32_t IDESC_O = umma_idesc(AB, PQ, 128, 1);
  extern __shared__ __align__(128) uint8_t psmem_raw[];
  uint8_t* smem = psmem_raw + ((1024 - (smem_u32(psmem_raw) & 1023)) & 1023);
  uint8_t* sq = smem;                          // Q boxes
  uint8_t* skv = sq + QBYTES;                  // ring: [K box0, K box1, V box0, V box1] per stage
  uint8_t* sp = skv + PKST * STAGE;            // P buffers: [hi, lo] x 2
  constexpr bool SPLIT = AB == 1;              // bf16 P as hi + lo
  __shared__ __align__(8) uint64_t q_full, o_done, kv_full[PKST], kv_empty[PKST], s_full[2], s_free[2],
      p_full[2], p_free[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ uint32_t bitmap[PMAXKB / 32];
  __shared__ uint16_t ulist[PMAXKB];
  __shared__ uint16_t rlist[PQ][PLMAX + 2];  // odd word stride: rows in distinct banks
  __shared__ int n_union, dead;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // ---- tile: (b, head, query tile), longest tiles first
  const int64_t tile = blockIdx.x;
  const int64_t qt = p.n_tiles - 1 - tile % p.n_tiles;
  const int64_t bh = tile / p.n_tiles;
  const int64_t h = bh % p.Hq, b = bh / p.Hq;
  const int64_t kvh = h / (p.Hq / p.Hkv);
  const int64_t t0 = qt * PQ;

  // ---- set-up: barriers, TMEM, the union of the rows' block lists
  const int nwords = static_cast<int>((p.n_kb + 31) / 32);
  for (int i = tid; i < nwords; i += 192) bitmap[i] = 0u;
  if (tid == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&o_done, 1);
    for (int s = 0; s < PKST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], PQ);
      mbar_init(&p_full[s], PQ);
      mbar_init(&p_free[s], 1);
    }
    dead = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(&tmem_base_sh))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  // softmax threads: row r = TMEM lane (32 x (warp % 4) + lane)
  const bool is_sm = warp >= 2;
  const int r = is_sm ? 32 * (warp & 3) + lane : 0;
  const int64_t t = t0 + r;
  const bool row_ok = is_sm && t < p.Tq;
  const int64_t pos = p.offset + t;
  int my_n = 0;
  if (row_ok) {
    const int64_t lr = t / p.rows_per_list;
    const int32_t* ids = p.ids + b * p.ls_b + h * p.ls_h + lr * p.ls_r;
    int64_t cnt = p.n_max;
    if (p.counts) cnt = lmin(cnt, static_cast<int64_t>(p.counts[b * p.cs_b + h * p.cs_h + lr * p.cs_r]));
    const int64_t vis = p.causal ? (pos < 0 ? -1 : pos / PK) : p.n_kb - 1;  // last visible block
    for (int64_t i = 0; i < cnt && my_n < PLMAX; ++i) {
      const int32_t blk = ids[i];
      if (blk < 0 || blk >= p.n_kb || blk > vis) continue;
      if (my_n > 0 && blk <= rlist[r][my_n - 1]) continue;  // ascending lists only
      rlist[r][my_n++] = static_cast<uint16_t>(blk);
      atomicOr(&bitmap[blk >> 5], 1u << (blk & 31));
    }
    if (p.sink > 0) {
      const int64_t sb = lmin((p.sink - 1) / PK, vis);
      for (int64_t blk = 0; blk <= sb; ++blk) atomicOr(&bitmap[blk >> 5], 1u << (blk & 31));
    }
  }
  __syncthreads();
  if (warp == 1) {
    // ascending union: popcount scan over the bitmap words
    int base = 0;
    for (int w0 = 0; w0 < nwords; w0 += 32) {
      const uint32_t word = w0 + lane < nwords ? bitmap[w0 + lane] : 0u;
      const int c = __popc(word);
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int at = base + incl - c;
      uint32_t m = word;
      while (m) {
        const int bit = __ffs(m) - 1;
        m &= m - 1u;
        ulist[at++] = static_cast<uint16_t>(((w0 + lane) << 5) | bit);
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) n_union = base;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int n = n_union;
  const uint32_t tmem = tmem_base_sh;  // columns [0, 64): S0, [64, 128): S1, [128, 256): O

  if (warp == 0) {
    // ================= TMA producer
    if (lane == 0 && n > 0) {
      const int qrow = static_cast<int>((b * p.Hq + h) * p.Tq + t0);
      mbar_arrive_expect_tx(&q_full, QBYTES);
      tma_load_2d(sq, &tmq, 0, qrow, &q_full);
      tma_load_2d(sq + PQ * 128, &tmq, 64, qrow, &q_full);
      const int64_t kv0 = (b * p.Hkv + kvh) * p.Tk;
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j % PKST;
        if (j >= PKST && !mbar_wait_bounded(&kv_empty[st], static_cast<uint32_t>(((j / PKST) - 1) & 1))) {
          report(p.status, LINATTN_DEV_TIMEOUT);
          dead = 1;
          break;
        }
        if (dead) break;
        uint8_t* dst = skv + st * STAGE;
        const int y = static_cast<int>(kv0 + static_cast<int64_t>(ulist[j]) * PK);
        mbar_arrive_expect_tx(&kv_full[st], STAGE);
        tma_load_2d(dst, &tmk, 0, y, &kv_full[st]);
        tma_load_2d(dst + BOXB, &tmk, 64, y, &kv_full[st]);
        tma_load_2d(dst + 2 * BOXB, &tmv, 0, y, &kv_full[st]);
        tma_load_2d(dst + 3 * BOXB, &tmv, 64, y, &kv_full[st]);
        issued = j + 1;
      }
      if (dead) {
        // let the copies in flight land (bounded) before the CTA gives up its smem
        for (int j = issued > PKST ? issued - PKST : 0; j < issued; ++j)
          (void)mbar_wait_bounded(&kv_full[j % PKST], static_cast<uint32_t>((j / PKST) & 1), 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer
    if (lane == 0 && n > 0) {
      bool ok = mbar_wait_bounded(&q_full, 0);
      const uint32_t sq_a = smem_u32(sq), skv_a = smem_u32(skv), sp_a = smem_u32(sp);
      auto pv = [&](int j) -> bool {
        const int pb = j & 1;
        if (!mbar_wait_bounded(&p_full[pb], static_cast<uint32_t>((j >> 1) & 1))) return false;
        tc_fence_after();
        const uint32_t vb = skv_a + (j % PKST) * STAGE + 2 * BOXB;
#pragma unroll
        for (int kk = 0; kk < PK / 16; ++kk) {
          const uint64_t bd = umma_desc(vb + kk * 2048, BOXB, 1024);
          const uint64_t a = umma_desc(sp_a + (2 * pb) * PBYTES + kk * 32, 16, 1024);
          umma_f16(tmem + 128, a, bd, IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
          if (SPLIT) umma_f16(tmem + 128, umma_desc(sp_a + (2 * pb + 1) * PBYTES + kk * 32, 16, 1024), bd, IDESC_O, 1u);
        }
        umma_commit(&o_done);
        umma_commit(&p_free[pb]);
        umma_commit(&kv_empty[j % PKST]);
        return true;
      };
      for (int j = 0; ok && j < n; ++j) {
        const int st = j % PKST, sb = j & 1;
        ok = mbar_wait_bounded(&kv_full[st], static_cast<uint32_t>((j / PKST) & 1));
        if (ok && j >= 2) ok = mbar_wait_bounded(&s_free[sb], static_cast<uint32_t>(((j >> 1) - 1) & 1));
        if (!ok) break;
        tc_fence_after();
        const uint32_t kb = skv_a + st * STAGE;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = umma_desc(sq_a + (kk >> 2) * (PQ * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = umma_desc(kb + (kk >> 2) * BOXB + (kk & 3) * 32, 16, 1024);
          umma_f16(tmem + sb * 64, a, bd, IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        if (j >= 1) ok = pv(j - 1);
      }
      if (ok) ok = pv(n - 1);
      if (!ok) {
        report(p.status, LINATTN_DEV_TIMEOUT);
        dead = 1;
      }
    }
  } else {
    // ================= softmax (one thread per query row)
    // tcgen05.ld / st are warp-collective: every branch around them is warp-uniform
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
    float m_used = -INFINITY, l = 0.f;
    int ptr = 0;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int sb = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[sb], static_cast<uint32_t>((j >> 1) & 1)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[2][32];
      tmem_ld32(lane_addr + sb * 64, sv[0]);
      tmem_ld32(lane_addr + sb * 64 + 32, sv[1]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[sb]);
      // which keys of block ulist[j] this row reads
      const int blk = ulist[j];
      while (ptr < my_n && rlist[r][ptr] < blk) ++ptr;
      const bool member = row_ok && ptr < my_n && rlist[r][ptr] == blk;
      const int64_t key0 = static_cast<int64_t>(blk) * PK;
      int64_t kend = member ? PK : lmin(PK, p.sink - key0);   // keys [key0, key0 + kend) are read
      if (!row_ok) kend = 0;
      kend = lmin(kend, p.Tk - key0);
      if (p.causal) kend = lmin(kend, pos - key0 + 1);
      float x[64];
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        x[c] = c < kend ? __uint_as_float(sv[c >> 5][c & 31]) * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, x[c]);
      }
      // running maximum: moved (and O rescaled) only when it grows by more than 8
      const bool first = mx > -INFINITY && m_used == -INFINITY;
      const bool grow = mx > -INFINITY && m_used != -INFINITY && mx > m_used + 8.f;
      if (__any_sync(0xffffffffu, grow)) {
        const float alpha = grow ? exp2f(m_used - mx) : 1.f;
        // O holds blocks < j once PV(j-1) is done: the completion of use (j-1)/2 of P
        // buffer (j-1)%2 (this thread waited for that buffer's previous use, so the
        // parity names exactly this phase)
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&p_free[(j - 1) & 1],
                                                       static_cast<uint32_t>(((j - 1) >> 1) & 1)))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t ov[32];
          tmem_ld32(lane_addr + 128 + cc * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st32(lane_addr + 128 + cc * 32, ov);
        }
        tmem_wait_st();
        l *= alpha;
      }
      if (first || grow) m_used = mx;
      // P = exp2(x - m_used) into the swizzled P tile (row r, 8 chunks of 8 keys)
      const int pb = j & 1;
      if (j >= 2 &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(&p_free[pb], static_cast<uint32_t>(((j >> 1) - 1) & 1)))) {
        ok = false;
        break;
      }
      uint8_t* prow = sp + (2 * pb) * PBYTES + r * 128;
      float sum = 0.f;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t wv[4], wl[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = m_used == -INFINITY ? 0.f : exp2f(x[ch * 8 + 2 * e] - m_used);
          const float c2 = m_used == -INFINITY ? 0.f : exp2f(x[ch * 8 + 2 * e + 1] - m_used);
          wv[e] = M::pack(a, c2);
          const float2 rp = M::unpack(wv[e]);
          if (SPLIT) {
            wl[e] = M::pack(a - rp.x, c2 - rp.y);  // hi + lo carries P to ~2^-17
            sum += a + c2;
          } else {
            sum += rp.x + rp.y;  // the rounded P the product uses: O / l an exact weighted mean
          }
        }
        const int off = (ch ^ (r & 7)) << 4;
        *reinterpret_cast<uint4*>(prow + off) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        if (SPLIT) *reinterpret_cast<uint4*>(prow + PBYTES + off) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
      }
      l += sum;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&p_full[pb]);
    }
    // ---- epilogue: O / l
    if (ok && n > 0 &&
        !__all_sync(0xffffffffu, mbar_wait_bounded(&p_free[(n - 1) & 1], static_cast<uint32_t>(((n - 1) >> 1) & 1))))
      ok = false;
    if (!ok) {
      report(p.status, LINATTN_DEV_TIMEOUT);
      dead = 1;
    }
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t ob = b * p.os[0] + h * p.os[1] + t * p.os[2];
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t ov[32];
      if (ok && n > 0) {  // warp-uniform
        tmem_ld32(lane_addr + 128 + cc * 32, ov);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] = 0u;
      }
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          store_any(p.out, ob + (cc * 32 + i) * p.os[3], p.out_dtype, __uint_as_float(ov[i]) * inv);
      }
    }
    if (row_ok && p.lse)
      p.lse[(b * p.Hq + h) * p.Tq + t] = l > 0.f ? (m_used + log2f(l)) * 0.69314718055994531f : -INFINITY;
  }
  // ---- tear-down: every tcgen05 op of this CTA is complete (the epilogue waited for
  // the last PV; a dead CTA may still have MMAs in flight: wait for them, bounded)
  tc_fence_before();
  __syncthreads();
  if (dead && tid == 32 && n > 0) {
    umma_commit(&o_done);
    (void)mbar_wait_bounded(&o_done, 0, 200000000ull);
    (void)mbar_wait_bounded(&o_done, 1, 200000000ull);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
}

namespace {

template <typename T>
cudaError_t launch_prefill(const PrefillParams& p, const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                           cudaStream_t st) {
  auto kern = prefill_umma_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_DYN);
  if (e != cudaSuccess) return e;
  const int64_t grid = p.B * p.Hq * p.n_tiles;
  kern<<<static_cast<unsigned>(grid), 192, SMEM_DYN, st>>>(p, q, k, v);
  return cudaGetLastError();
}

}  // namespace

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_block_sparse_prefill(const void* q, int32_t dtype, int64_t B, int64_t Hq, int64_t Tq,
                                            const void* k, const void* v, int64_t Hkv, int64_t Tk, int64_t D,
                                            const int32_t* ids, const int32_t* counts, const int64_t* id_strides,
                                            int64_t n_max, int64_t rows_per_list, const int64_t* count_strides,
                                            int64_t sink, int32_t causal, int64_t offset, float scale, void* out,
                                            const int64_t* out_strides, float* lse_out, int32_t* status,
                                            void* stream) {
  if (!q || !k || !v || !ids || !out || !id_strides || !out_strides)
    return set_error(LINATTN_EINVAL, "block_sparse_prefill: NULL pointer");
  if (dtype != LINATTN_BF16 && dtype != LINATTN_F16)
    return set_error(LINATTN_EUNSUPPORTED, "block_sparse_prefill: q / K / V must be bf16 or f16 (one type)");
  if (D != 128) return set_error(LINATTN_EUNSUPPORTED, "block_sparse_prefill: head_dim must be 128");
  if (Hkv < 1 || Hq % Hkv) return set_error(LINATTN_EINVAL, "block_sparse_prefill: H_q must be a multiple of H_kv");
  if (n_max < 1 || n_max > PLMAX || rows_per_list < 1)
    return set_error(LINATTN_EUNSUPPORTED, "block_sparse_prefill: lists must hold 1 .. 64 blocks");
  const int64_t n_kb = (Tk + PK - 1) / PK;
  if (n_kb > PMAXKB) return set_error(LINATTN_EUNSUPPORTED, "block_sparse_prefill: T_k above 2^18");
  if (counts && !count_strides) return set_error(LINATTN_EINVAL, "block_sparse_prefill: counts need strides");
  if (reinterpret_cast<uintptr_t>(q) % 16 || reinterpret_cast<uintptr_t>(k) % 16 || reinterpret_cast<uintptr_t>(v) % 16)
    return set_error(LINATTN_EINVAL, "block_sparse_prefill: q / K / V must be 16-byte aligned");
  if (B * Hq * Tq >= (int64_t(1) << 31) || B * Hkv * Tk >= (int64_t(1) << 31))
    return set_error(LINATTN_EUNSUPPORTED, "block_sparse_prefill: too many rows for 32-bit TMA coordinates");
  if (B == 0 || Hq == 0 || Tq == 0) return LINATTN_OK;
  // q / K / V: contiguous (B, H, T, 128) rows, viewed as 2-D [rows, 128]
  const CUtensorMapDataType cu = dtype == LINATTN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  if (!tensor_map_2d(&tq, q, cu, 128, B * Hq * Tq, 256, 64, PQ) || !tensor_map_2d(&tk, k, cu, 128, B * Hkv * Tk, 256, 64, PK) ||
      !tensor_map_2d(&tv, v, cu, 128, B * Hkv * Tk, 256, 64, PK))
    return set_error(LINATTN_ECUDA, "block_sparse_prefill: tensor map encoding failed");
  PrefillParams p;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.Tq = Tq; p.Tk = Tk;
  p.ids = ids; p.counts = counts;
  p.ls_b = id_strides[0]; p.ls_h = id_strides[1]; p.ls_r = id_strides[2]; p.n_max = n_max;
  p.rows_per_list = rows_per_list;
  p.cs_b = counts ? count_strides[0] : 0; p.cs_h = counts ? count_strides[1] : 0; p.cs_r = counts ? count_strides[2] : 0;
  p.sink = sink < 0 ? 0 : sink; p.causal = causal; p.offset = offset;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out; p.out_dtype = dtype; p.lse = lse_out; p.status = status;
  for (int i = 0; i < 4; ++i) p.os[i] = out_strides[i];
  p.n_tiles = (Tq + PQ - 1) / PQ;
  p.n_kb = n_kb;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = dtype == LINATTN_BF16 ? launch_prefill<__nv_bfloat16>(p, tq, tk, tv, st)
                                              : launch_prefill<__half>(p, tq, tk, tv, st);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "block_sparse_prefill: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
