// Block-sparse causal prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Every query row reads the 64-token key blocks of its own ascending block list (one
// list per `rows_per_list` consecutive queries: 64 for per-q-block lists such as
// MInference's block-sparse pattern or sink + window + top-k, 1 for MoBA's per-token
// routing), plus the tokens below `sink`, causally (key <= offset + t; with causal = c > 1
// the keys are pooled groups of c tokens and key j is read once its group has started,
// j * c <= offset + t + c - 1, NSA's compression-branch rule), with `window` > 0 only keys
// >= offset + t - window + 1 (a token-exact sliding window), and below T_k.
// (MInferenceAttention._block_sparse / MoBAAttention.select + the masked attention of
// BlockSelectionAttention.attend, src/linattn/variants/selection.py:86-116, 339-353,
// 635-649.)
//
// One CTA = 128 query rows of one (batch, head); it walks the ascending union of its
// rows' lists two blocks (128 keys) per step, and a row ignores (-inf) the blocks not
// in its list.  Warp roles (320 threads, one CTA per SM):
//   warp 0     TMEM allocation (512 columns) and two TMA producer lanes: lane 0 Q (two
//              128 x 64 boxes) once, then per step the K rows of two blocks (four 64 x 64
//              boxes, 128-byte swizzle) into a 3-stage K ring freed as soon as S_j is
//              done; lane 1 the V rows into a 2-stage V ring freed by PV_j; both prefetch
//              the blocks of the next steps into L2;
//   warp 1     one thread issues tcgen05.mma (kind::f16, M = 128, fp32 accumulators in
//              TMEM): S_j = Q K_j^T (N = 128 keys) into one of two S buffers, then
//              O += P_{j-1} V_{j-1} (N = 128 channels) with P read from TMEM (A operand)
//              and V from shared memory (MN-major), and commits to the mbarriers the
//              other roles wait on.  MMAs of one thread execute in issue order, so S_{j+2}
//              may be issued into the buffer whose P the earlier PV_j reads;
//   warps 2-9  softmax, two threads per row (TMEM lane): warps 2-5 take every step's
//              first block (64 keys), warps 6-9 its second; each half keeps its own
//              running (O, m, l), the two O accumulators merged in the epilogue.
//              tcgen05.ld of the scores,
//              masks, online softmax in the log2 domain, then P written back over its
//              scores (tcgen05.st): one f16 part when V is f16 (f16 inputs, or a bf16
//              V copied to f16 beforehand with a per-(b, kv head) power-of-two scale),
//              else bf16 hi + lo parts (two products, P to ~2^-17); a block that no row
//              of a warp reads is skipped (P = 0 without exponentials).  O is rescaled in TMEM only when a row's
//              running maximum grows by more than 8, so P stays below 2^8; the rare
//              rescale waits for the PV in flight.  The epilogue reads O from TMEM,
//              divides by the row sum and stores (full tiles: staged in the Q tile and
//              written by two TMA stores).
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
  int window;             // > 0: a row also skips keys below its position - window + 1
  int64_t offset;
  float scale_log2;
  void* out;
  int64_t os[4];
  int out_dtype;
  float* lse;             // (B, Hq, Tq) or NULL
  const float* v_scale;   // (B, Hkv) factor of an f16 V copy, or NULL
  int64_t n_tiles;        // query tiles of 128 per (b, head)
  int64_t n_kb;           // key blocks
  int tma_out;            // out is contiguous (B, H_q, T_q, 128): full tiles leave through TMA stores
  int32_t* status;
};

namespace {

constexpr int PQ = 128;          // query rows per CTA
constexpr int PK = 64;           // keys per list block
constexpr int PSTEP = 128;       // keys per step (two list blocks)
constexpr int PKS = 3;           // K ring stages (steps): freed when S_j is done
constexpr int PVS = 2;           // V ring stages (steps): freed when PV_j is done
constexpr int PPF = 3;           // steps prefetched into L2 ahead of the ring
constexpr int PLMAX = 64;        // longest list a row may have
constexpr int PMAXKB = 4096;     // key blocks (T_k <= 2^18)
constexpr int BOXB = 64 * 128;   // one 64-row x 128-byte box
constexpr int QBYTES = 2 * PQ * 128;           // Q: two 128 x 64 boxes
constexpr int HALFB = PSTEP * 128;             // 128 key rows x 64 channels
constexpr int TILE = 2 * HALFB;                // K or V of one step (two channel halves)
constexpr int SMEM_DYN = 1024 + QBYTES + (PKS + PVS) * TILE;

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
// A operand from TMEM (K-major: lane = row, two 16-bit values per 32-bit column)
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
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
__device__ __forceinline__ void tma_prefetch_2d(const void* tmap, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(tmap)),
               "r"(x), "r"(y)
               : "memory");
}
// 2^x with the hardware approximation (ex2.approx.ftz: relative error ~2^-22; 2^-inf = 0)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace

template <typename TQ, typename TV>
__global__ void __launch_bounds__(320, 1)
    prefill_umma_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tmq,
                        const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                        const __grid_constant__ CUtensorMap tmo) {
  using M = MmaOp<TV>;   // P, packed in V's type
  using MQ = MmaOp<TQ>;  // the output, in q's type
  constexpr int AB_S = std::is_same<TQ, __nv_bfloat16>::value ? 1 : 0;
  constexpr int AB_O = std::is_same<TV, __nv_bfloat16>::value ? 1 : 0;
  constexpr bool SPLIT = AB_O == 1;  // bf16 P as hi + lo
  constexpr uint32_t IDESC_S = umma_idesc(AB_S, PQ, PSTEP, 0);
  constexpr uint32_t IDESC_O = umma_idesc(AB_O, PQ, 128, 1);
  extern __shared__ __align__(128) uint8_t psmem_raw[];
  uint8_t* smem = psmem_raw + ((1024 - (smem_u32(psmem_raw) & 1023)) & 1023);
  uint8_t* sq = smem;          // Q boxes
  uint8_t* sk = sq + QBYTES;        // K ring: [channel half 0, half 1] of 128 key rows per stage
  uint8_t* sv_ring = sk + PKS * TILE;  // V ring, same layout
  __shared__ __align__(8) uint64_t q_full, o_done, k_full[PKS], k_empty[PKS], v_full[PVS], v_empty[PVS], s_full[2],
      p_full[2], pv_done[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ uint32_t bitmap[PMAXKB / 32];
  __shared__ uint16_t ulist[PMAXKB + 1];
  __shared__ uint16_t rlist[PQ][PLMAX + 2];  // odd word stride: rows in distinct banks
  __shared__ int n_union, dead;
  __shared__ int rlen[PQ];              // list length of each row
  __shared__ float xchg[2][2][PQ];      // epilogue: [m | l][block half][row]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // heads fastest: the CTAs in flight share a query tile, so the heads of a GQA group
  // and neighbouring tiles (overlapping windows) read the same K / V blocks from L2
  const int64_t tile = blockIdx.x;
  const int64_t h = tile % p.Hq;
  const int64_t rest = tile / p.Hq;
  const int64_t qt = p.n_tiles - 1 - rest % p.n_tiles;
  const int64_t b = rest / p.n_tiles;
  const int64_t kvh = h / (p.Hq / p.Hkv);
  const int64_t t0 = qt * PQ;

  // ---- set-up: barriers, TMEM, the union of the rows' block lists
  const int nwords = static_cast<int>((p.n_kb + 31) / 32);
  for (int i = tid; i < nwords; i += 320) bitmap[i] = 0u;
  if (tid == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&o_done, 1);
    for (int s = 0; s < PKS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < PVS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 2 * PQ);
      mbar_init(&pv_done[s], 1);
    }
    dead = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_base_sh))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  // softmax threads: row r = TMEM lane (32 x (warp % 4) + lane), block half hb
  const bool is_sm = warp >= 2;
  const int r = is_sm ? 32 * (warp & 3) + lane : 0;
  const int hb = warp >= 6 ? 1 : 0;
  const int64_t t = t0 + r;
  const bool row_ok = is_sm && t < p.Tq;
  const int64_t pos = p.offset + t;
  int my_n = 0;
  // the union only needs, per list, its last row in this tile (the widest causal view)
  const int64_t t_last_row = lmin(p.Tq, t0 + PQ) - 1;
  const bool owner = row_ok && (t == t_last_row || (t + 1) / p.rows_per_list != t / p.rows_per_list);
  if (row_ok && hb == 0) {
    const int64_t lr = t / p.rows_per_list;
    const int32_t* ids = p.ids + b * p.ls_b + h * p.ls_h + lr * p.ls_r;
    int64_t cnt = p.n_max;
    if (p.counts) cnt = lmin(cnt, static_cast<int64_t>(p.counts[b * p.cs_b + h * p.cs_h + lr * p.cs_r]));
    // last visible block: key j is visible iff j * c <= pos + c - 1 (c = p.causal; c = 1 is
    // j <= pos)
    // (so for c > 1 key 0 is already visible from -c < pos < 0)
    const int64_t vis =
        p.causal ? (pos + p.causal - 1 < 0 ? -1 : ((pos + p.causal - 1) / p.causal) / PK) : p.n_kb - 1;
    for (int64_t i0 = 0; i0 < cnt && my_n < PLMAX; i0 += 8) {
      int32_t blk8[8];  // eight independent loads in flight
#pragma unroll
      for (int e = 0; e < 8; ++e) blk8[e] = i0 + e < cnt ? __ldg(ids + i0 + e) : -1;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int32_t blk = blk8[e];
        if (blk < 0 || blk >= p.n_kb || blk > vis || my_n >= PLMAX) continue;
        if (my_n > 0 && blk <= rlist[r][my_n - 1]) continue;  // ascending lists only
        rlist[r][my_n++] = static_cast<uint16_t>(blk);
        if (owner) atomicOr(&bitmap[blk >> 5], 1u << (blk & 31));
      }
    }
    if (p.sink > 0 && t == t_last_row) {
      const int64_t sb = lmin((p.sink - 1) / PK, vis);
      for (int64_t blk = 0; blk <= sb; ++blk) atomicOr(&bitmap[blk >> 5], 1u << (blk & 31));
    }
  }
  if (is_sm && hb == 0) rlen[r] = my_n;
  __syncthreads();
  if (is_sm) my_n = rlen[r];
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
    if (lane == 0) {
      n_union = base;
      // an odd union: the last step repeats its first block (masked for every row)
      if (base & 1) ulist[base] = ulist[base - 1];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int n = n_union;
  const int n_steps = (n + 1) >> 1;
  // columns [0, 128): S / P 0, [128, 256): S / P 1, [256, 384): O of each step's first
  // block, [384, 512): O of its second block (merged in the epilogue)
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ================= TMA producers: lane 0 Q and K (ahead by PKS steps), lane 1 V
    if (lane < 2 && n > 0) {
      const bool is_k = lane == 0;
      const CUtensorMap* tm = is_k ? &tmk : &tmv;
      uint8_t* ring = is_k ? sk : sv_ring;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      const int nst = is_k ? PKS : PVS;
      if (is_k) {
        const int qrow = static_cast<int>((b * p.Hq + h) * p.Tq + t0);
        mbar_arrive_expect_tx(&q_full, QBYTES);
        tma_load_2d(sq, &tmq, 0, qrow, &q_full);
        tma_load_2d(sq + PQ * 128, &tmq, 64, qrow, &q_full);
      }
      const int64_t kv0 = (b * p.Hkv + kvh) * p.Tk;
      auto row_of = [&](int e) { return static_cast<int>(kv0 + static_cast<int64_t>(ulist[e]) * PK); };
      auto prefetch_step = [&](int j) {  // warm L2 (no shared memory involved)
        tma_prefetch_2d(tm, 0, row_of(2 * j));
        tma_prefetch_2d(tm, 64, row_of(2 * j));
        tma_prefetch_2d(tm, 0, row_of(2 * j + 1));
        tma_prefetch_2d(tm, 64, row_of(2 * j + 1));
      };
      int issued = 0;
      for (int j = 0; j < n_steps; ++j) {
        const int st = j % nst;
        if (j >= nst && !mbar_wait_bounded(&empty[st], static_cast<uint32_t>(((j / nst) - 1) & 1))) {
          report(p.status, LINATTN_DEV_TIMEOUT);
          dead = 1;
          break;
        }
        if (dead) break;
        uint8_t* dst = ring + st * TILE;
        const int ya = row_of(2 * j), yb = row_of(2 * j + 1);
        mbar_arrive_expect_tx(&full[st], TILE);
        // 128 key rows per channel half: block a rows 0-63, block b rows 64-127
        tma_load_2d(dst, tm, 0, ya, &full[st]);
        tma_load_2d(dst + BOXB, tm, 0, yb, &full[st]);
        tma_load_2d(dst + HALFB, tm, 64, ya, &full[st]);
        tma_load_2d(dst + HALFB + BOXB, tm, 64, yb, &full[st]);
        issued = j + 1;
        if (j == 0)
          for (int f = 1; f <= PPF && f < n_steps; ++f) prefetch_step(f);
        if (j + PPF + 1 < n_steps) prefetch_step(j + PPF + 1);
      }
      if (dead) {
        // let the copies in flight land (bounded) before the CTA gives up its smem
        for (int j = issued > nst ? issued - nst : 0; j < issued; ++j)
          (void)mbar_wait_bounded(&full[j % nst], static_cast<uint32_t>((j / nst) & 1), 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer
    if (lane == 0 && n > 0) {
      bool ok = mbar_wait_bounded(&q_full, 0);
      const uint32_t sq_a = smem_u32(sq), sk_a = smem_u32(sk), sv_a = smem_u32(sv_ring);
      auto pv = [&](int j) -> bool {
        const int pb = j & 1;
        if (!mbar_wait_bounded(&p_full[pb], static_cast<uint32_t>((j >> 1) & 1))) return false;
        if (!mbar_wait_bounded(&v_full[j % PVS], static_cast<uint32_t>((j / PVS) & 1))) return false;
        tc_fence_after();
        const uint32_t vb = sv_a + (j % PVS) * TILE;
        const uint32_t pt = tmem + pb * 128;  // P of step j, over its scores
        // block half hb of the step (64 keys, P columns [32 hb, 32 hb + 32)) into O_hb
#pragma unroll
        for (int kk = 0; kk < PSTEP / 16; ++kk) {
          const uint32_t od = tmem + 256 + (kk >> 2) * 128;
          const uint64_t bd = umma_desc(vb + kk * 2048, HALFB, 1024);
          // keys [16 kk, 16 kk + 16): P columns 64 (kk / 4) + 8 (kk % 4), lo 32 further
          const uint32_t pcol = pt + 64 * (kk >> 2) + 8 * (kk & 3);
          umma_f16_ts(od, pcol, bd, IDESC_O, (j > 0 || (kk & 3) > 0) ? 1u : 0u);
          if (SPLIT) umma_f16_ts(od, pcol + 32, bd, IDESC_O, 1u);
        }
        umma_commit(&pv_done[pb]);
        umma_commit(&v_empty[j % PVS]);
        return true;
      };
      for (int j = 0; ok && j < n_steps; ++j) {
        const int st = j % PKS, sb = j & 1;
        ok = mbar_wait_bounded(&k_full[st], static_cast<uint32_t>((j / PKS) & 1));
        if (!ok) break;
        tc_fence_after();
        // S_j into buffer sb: its previous P (step j - 2) is read by PV_{j-2}, issued
        // before this point; MMAs run in issue order
        const uint32_t kb = sk_a + st * TILE;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = umma_desc(sq_a + (kk >> 2) * (PQ * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = umma_desc(kb + (kk >> 2) * HALFB + (kk & 3) * 32, 16, 1024);
          umma_f16(tmem + sb * 128, a, bd, IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[st]);
        if (j >= 1) ok = pv(j - 1);
      }
      if (ok) ok = pv(n_steps - 1);
      if (!ok) {
        report(p.status, LINATTN_DEV_TIMEOUT);
        dead = 1;
      }
    }
  } else {
    // ================= softmax (two threads per query row: block half hb)
    // tcgen05.ld / st are warp-collective: every branch around them is warp-uniform
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
    float m_used = -INFINITY, l = 0.f;
    int ptr = 0;
    bool ok = true;
    const int sink32 = static_cast<int>(lmin(p.sink, int64_t(1) << 30)), tk32 = static_cast<int>(p.Tk);
    const int pos32 = static_cast<int>(lmax(lmin(pos, int64_t(1) << 30), -(int64_t(1) << 30)));
    // keys visible from this row under the causal rule (the first lim32 of them), and
    // with a window the first key it reads
    const int cc = p.causal > 0 ? p.causal : 1;
    const int lim32 = pos32 + cc - 1 < 0 ? 0 : (pos32 + cc - 1) / cc + 1;
    const int wlo32 = p.window > 0 ? pos32 - p.window + 1 : 0;
    for (int j = 0; j < n_steps; ++j) {
      const int sb = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[sb], static_cast<uint32_t>((j >> 1) & 1)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[2][32];
      tmem_ld32(lane_addr + sb * 128 + hb * 64, sv[0]);
      tmem_ld32(lane_addr + sb * 128 + hb * 64 + 32, sv[1]);
      tmem_wait_ld();
      // which keys of this thread's block the row reads
      int ke = 0, ks = 0;
      {
        const int e = 2 * j + hb;
        const int blk = ulist[e];
        bool member = false;
        if (e < n) {
          while (ptr < my_n && rlist[r][ptr] < blk) ++ptr;
          member = row_ok && ptr < my_n && rlist[r][ptr] == blk;
        }
        // 32-bit: T_k <= 2^18 and |offset + t| < 2^31 (checked on the host)
        const int key0 = blk * PK;
        int kend = member ? PK : (e < n ? min(PK, sink32 - key0) : 0);
        if (!row_ok) kend = 0;
        kend = min(kend, tk32 - key0);
        if (p.causal) kend = min(kend, lim32 - key0);
        ke = max(0, kend);
        if (p.window > 0) {
          ks = max(0, wlo32 - key0);  // keys [ks, ke) of the block
          if (ks >= ke) ke = ks = 0;
        }
      }
      // raw scores; masks only where needed (scale > 0: max of raw = max / scale).  A
      // block that no row of the warp reads is skipped: P = 0 without exponentials.
      const bool none_in = __all_sync(0xffffffffu, ke == 0);
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
      if (none_in) {
      } else if (ke >= PK && ks == 0) {
#pragma unroll
        for (int c = 0; c < 64; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(sv[c >> 5][c & 31]));
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float v = c >= ks && c < ke ? __uint_as_float(sv[c >> 5][c & 31]) : -INFINITY;
          sv[c >> 5][c & 31] = __float_as_uint(v);
          mx8[c & 7] = fmaxf(mx8[c & 7], v);
        }
      }
      const float mloc = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // this half's running maximum: moved (and O_hb rescaled) only when it grows by
      // more than 8; the two halves keep their own (O, m, l), merged in the epilogue
      const float mx = mloc * p.scale_log2;
      const bool first = mx > -INFINITY && m_used == -INFINITY;
      const bool grow = mx > -INFINITY && m_used != -INFINITY && mx > m_used + 8.f;
      if (__any_sync(0xffffffffu, grow)) {
        const float alpha = grow ? ex2_approx(m_used - mx) : 1.f;
        // O holds steps < j once PV_{j-1} is done (the completion of use (j-1)/2 of
        // buffer (j-1)%2; its previous use finished before S_{j-1}, which this thread saw)
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&pv_done[(j - 1) & 1],
                                                       static_cast<uint32_t>(((j - 1) >> 1) & 1)))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {  // O_hb of this row
          uint32_t ov[32];
          const uint32_t oa = lane_addr + 256 + hb * 128 + cc * 32;
          tmem_ld32(oa, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st32(oa, ov);
        }
        tmem_wait_st();
        l *= alpha;
      }
      if (first || grow) m_used = mx;
      // P = 2^(s * scale - m); masked scores are -inf (P = 0); a row with nothing read
      // yet has m = -inf: P = 0
      const float sl = p.scale_log2;
      const float neg = m_used == -INFINITY ? -INFINITY : -m_used;
      float sum8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum8[i] = 0.f;
      uint32_t hi[32], lo[32];
      if (none_in) {
#pragma unroll
        for (int e = 0; e < 32; ++e) hi[e] = lo[e] = 0u;
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int c = 2 * e;
          const float a = ex2_approx(fmaf(__uint_as_float(sv[c >> 5][c & 31]), sl, neg));
          const float c2 = ex2_approx(fmaf(__uint_as_float(sv[(c + 1) >> 5][(c + 1) & 31]), sl, neg));
          hi[e] = M::pack(a, c2);
          if (SPLIT) {
            const float2 rp = M::unpack(hi[e]);
            lo[e] = M::pack(a - rp.x, c2 - rp.y);
          } else {
            lo[e] = 0u;
          }
          sum8[e & 7] += a + c2;
        }
      }
      // P of this half over its own 64 score columns (hi at [64 hb, 64 hb + 32), lo 32
      // further): the other half may still be reading its scores
      tmem_st32(lane_addr + sb * 128 + hb * 64, hi);
      if (SPLIT) tmem_st32(lane_addr + sb * 128 + hb * 64 + 32, lo);
      l += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    // ---- epilogue: O / l once the last PV is done (exact phase, as above)
    if (ok && n_steps > 0 &&
        !__all_sync(0xffffffffu, mbar_wait_bounded(&pv_done[(n_steps - 1) & 1],
                                                   static_cast<uint32_t>(((n_steps - 1) >> 1) & 1))))
      ok = false;
    if (!ok) {
      report(p.status, LINATTN_DEV_TIMEOUT);
      dead = 1;
    }
    // merge the halves: O = (O_0 2^(m_0 - M) + O_1 2^(m_1 - M)) / (l_0 2^(m_0 - M) + l_1 2^(m_1 - M)),
    // thread hb producing channels [64 hb, 64 hb + 64) from both accumulators
    xchg[0][hb][r] = m_used;
    xchg[1][hb][r] = l;
    asm volatile("bar.sync 2, 256;" ::: "memory");  // every softmax thread reaches this point
    const float m_o = xchg[0][hb ^ 1][r], l_o = xchg[1][hb ^ 1][r];
    const float m_all = fmaxf(m_used, m_o);
    const float f_me = m_used == -INFINITY ? 0.f : ex2_approx(m_used - m_all);
    const float f_o = m_o == -INFINITY ? 0.f : ex2_approx(m_o - m_all);
    const float f0 = hb == 0 ? f_me : f_o, f1 = hb == 0 ? f_o : f_me;
    l = l * f_me + l_o * f_o;
    m_used = m_all;
    tc_fence_after();
    const float vs = p.v_scale ? p.v_scale[b * p.Hkv + kvh] : 1.f;
    const float inv = l > 0.f ? vs / l : 0.f;
    const int64_t ob = b * p.os[0] + h * p.os[1] + t * p.os[2];
    // full tiles with contiguous output: rows staged (swizzled, as TMA boxes) in the Q
    // tile, which every MMA has finished reading, then two TMA stores
    const bool via_tma = p.tma_out && t0 + PQ <= p.Tq;
#pragma unroll 1
    for (int cc = 0; cc < 2; ++cc) {  // this thread's 64 channels
      uint32_t ov[32];
      if (ok && n_steps > 0) {  // warp-uniform
        uint32_t o1[32];
        tmem_ld32(lane_addr + 256 + hb * 64 + cc * 32, ov);
        tmem_ld32(lane_addr + 384 + hb * 64 + cc * 32, o1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          ov[i] = __float_as_uint(__uint_as_float(ov[i]) * f0 + __uint_as_float(o1[i]) * f1);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] = 0u;
      }
      if (via_tma) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int c = cc * 4 + q4;  // 16-byte chunk (8 channels) within the channel half hb
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = MQ::pack(__uint_as_float(ov[q4 * 8 + 2 * e]) * inv, __uint_as_float(ov[q4 * 8 + 2 * e + 1]) * inv);
          *reinterpret_cast<uint4*>(sq + hb * (PQ * 128) + r * 128 + ((c ^ (r & 7)) << 4)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          store_any(p.out, ob + (hb * 64 + cc * 32 + i) * p.os[3], p.out_dtype, __uint_as_float(ov[i]) * inv);
      }
    }
    if (via_tma) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps
      if (r == 0 && hb == 0) {
        const int y = static_cast<int>((b * p.Hq + h) * p.Tq + t0);
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                         reinterpret_cast<uint64_t>(&tmo)), "r"(0), "r"(y), "r"(smem_u32(sq))
                     : "memory");
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                         reinterpret_cast<uint64_t>(&tmo)), "r"(64), "r"(y), "r"(smem_u32(sq + PQ * 128))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // smem read before the CTA exits
      }
    }
    if (row_ok && hb == 0 && p.lse)
      p.lse[(b * p.Hq + h) * p.Tq + t] = l > 0.f ? (m_used + log2f(l)) * 0.69314718055994531f : -INFINITY;
  }
  // ---- tear-down: every tcgen05 op of this CTA is complete (the epilogue waited for
  // the last PV; a dead CTA may still have MMAs in flight: wait for them, bounded)
  tc_fence_before();
  __syncthreads();
  if (dead && tid == 32 && n > 0) {
    umma_commit(&o_done);
    (void)mbar_wait_bounded(&o_done, 0, 200000000ull);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

// bf16 V -> f16 copy for the single-part P product: per (b, kv head) a power-of-two
// scale s >= 1 with max|V| / s <= 2^15 (s = 1 unless |V| exceeds 2^15, so the copy is
// exact for every value in f16's normal range); the prefill multiplies O by s.
__global__ void v_amax_kernel(const __nv_bfloat16* __restrict__ v, int64_t per_head, uint32_t* __restrict__ amax) {
  const int64_t hd = blockIdx.y;
  const __nv_bfloat16* src = v + hd * per_head;
  float m = 0.f;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < per_head;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x * 8) {
    const uint4 w = *reinterpret_cast<const uint4*>(src + i);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[e]));
      m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(amax + hd, __float_as_uint(m));  // m >= 0: bit order = value order
}

__global__ void v_to_f16_kernel(const __nv_bfloat16* __restrict__ v, int64_t per_head,
                                const uint32_t* __restrict__ amax, __half* __restrict__ out, float* __restrict__ scale) {
  const int64_t hd = blockIdx.y;
  const float a = __uint_as_float(amax[hd]);
  float s = 1.f;
  while (a / s > 32768.f && s < 1e30f) s *= 2.f;  // a NaN maximum keeps s = 1 (it propagates)
  const float inv = 1.f / s;                      // a power of two: exact
  if (blockIdx.x == 0 && threadIdx.x == 0) scale[hd] = s;
  const __nv_bfloat16* src = v + hd * per_head;
  __half* dst = out + hd * per_head;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < per_head;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x * 8) {
    const uint4 w = *reinterpret_cast<const uint4*>(src + i);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[e]));
      const __half2 hh = __floats2half2_rn(f.x * inv, f.y * inv);
      o[e] = *reinterpret_cast<const uint32_t*>(&hh);
    }
    *reinterpret_cast<uint4*>(dst + i) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

namespace {

template <typename TQ, typename TV>
cudaError_t launch_prefill(const PrefillParams& p, const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                           const CUtensorMap& o, cudaStream_t st) {
  auto kern = prefill_umma_kernel<TQ, TV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_DYN);
  if (e != cudaSuccess) return e;
  const int64_t grid = p.B * p.Hq * p.n_tiles;
  kern<<<static_cast<unsigned>(grid), 320, SMEM_DYN, st>>>(p, q, k, v, o);
  return cudaGetLastError();
}

}  // namespace

}  // namespace linattn

using namespace linattn;

extern "C" int linattn_prefill_v_to_f16(const void* v, int64_t heads, int64_t per_head, void* out, float* scale,
                                        uint32_t* amax_scratch, void* stream) {
  if (!v || !out || !scale || !amax_scratch) return set_error(LINATTN_EINVAL, "prefill_v_to_f16: NULL pointer");
  if (per_head % 8 || reinterpret_cast<uintptr_t>(v) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return set_error(LINATTN_EINVAL, "prefill_v_to_f16: 16-byte aligned rows of a multiple of 8 elements");
  if (heads < 1 || heads > 65535) return set_error(LINATTN_EINVAL, "prefill_v_to_f16: 1 .. 65535 heads");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(amax_scratch, 0, static_cast<size_t>(heads) * 4, st);
  const int64_t per_block = 256 * 8;
  const unsigned gx = static_cast<unsigned>(lmin((per_head + per_block - 1) / per_block, 4096));
  if (e == cudaSuccess) {
    v_amax_kernel<<<dim3(gx, static_cast<unsigned>(heads)), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(v),
                                                                          per_head, amax_scratch);
    v_to_f16_kernel<<<dim3(gx, static_cast<unsigned>(heads)), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(v), per_head, amax_scratch, static_cast<__half*>(out), scale);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "prefill_v_to_f16: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}

extern "C" int linattn_block_sparse_prefill(const void* q, int32_t dtype, int64_t B, int64_t Hq, int64_t Tq,
                                            const void* k, const void* v, int64_t Hkv, int64_t Tk, int64_t D,
                                            const int32_t* ids, const int32_t* counts, const int64_t* id_strides,
                                            int64_t n_max, int64_t rows_per_list, const int64_t* count_strides,
                                            int64_t sink, int32_t causal, int64_t window, int64_t offset,
                                            float scale, void* out,
                                            const int64_t* out_strides, float* lse_out, const void* v_f16,
                                            const float* v_scale, int32_t* status, void* stream) {
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
  if (v_f16 && (dtype != LINATTN_BF16 || !v_scale))
    return set_error(LINATTN_EINVAL, "block_sparse_prefill: an f16 V copy goes with bf16 inputs and its scales");
  if (reinterpret_cast<uintptr_t>(q) % 16 || reinterpret_cast<uintptr_t>(k) % 16 || reinterpret_cast<uintptr_t>(v) % 16 ||
      reinterpret_cast<uintptr_t>(v_f16) % 16)
    return set_error(LINATTN_EINVAL, "block_sparse_prefill: q / K / V must be 16-byte aligned");
  if (B * Hq * Tq >= (int64_t(1) << 31) || B * Hkv * Tk >= (int64_t(1) << 31))
    return set_error(LINATTN_EUNSUPPORTED, "block_sparse_prefill: too many rows for 32-bit TMA coordinates");
  if (offset < -(int64_t(1) << 30) || offset + Tq >= (int64_t(1) << 30))
    return set_error(LINATTN_EUNSUPPORTED, "block_sparse_prefill: query positions must lie in (-2^30, 2^30)");
  if (causal < 0 || causal > (1 << 20)) return set_error(LINATTN_EINVAL, "block_sparse_prefill: causal must be 0 .. 2^20");
  if (window < 0 || window > (int64_t(1) << 30) || (window > 0 && sink > 0))
    return set_error(LINATTN_EINVAL, "block_sparse_prefill: window must be 0 .. 2^30 and goes without a sink");
  if (B == 0 || Hq == 0 || Tq == 0) return LINATTN_OK;
  // q / K / V: contiguous (B, H, T, 128) rows, viewed as 2-D [rows, 128]
  const CUtensorMapDataType cu = dtype == LINATTN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  if (!tensor_map_2d(&tq, q, cu, 128, B * Hq * Tq, 256, 64, PQ) || !tensor_map_2d(&tk, k, cu, 128, B * Hkv * Tk, 256, 64, PK) ||
      !tensor_map_2d(&tv, v_f16 ? v_f16 : v, v_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : cu, 128, B * Hkv * Tk, 256,
                     64, PK))
    return set_error(LINATTN_ECUDA, "block_sparse_prefill: tensor map encoding failed");
  PrefillParams p;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.Tq = Tq; p.Tk = Tk;
  p.ids = ids; p.counts = counts;
  p.ls_b = id_strides[0]; p.ls_h = id_strides[1]; p.ls_r = id_strides[2]; p.n_max = n_max;
  p.rows_per_list = rows_per_list;
  p.cs_b = counts ? count_strides[0] : 0; p.cs_h = counts ? count_strides[1] : 0; p.cs_r = counts ? count_strides[2] : 0;
  p.sink = sink < 0 ? 0 : sink; p.causal = causal; p.window = static_cast<int>(window); p.offset = offset;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out; p.out_dtype = dtype; p.lse = lse_out; p.status = status;
  p.v_scale = v_f16 ? v_scale : nullptr;
  for (int i = 0; i < 4; ++i) p.os[i] = out_strides[i];
  p.n_tiles = (Tq + PQ - 1) / PQ;
  p.n_kb = n_kb;
  // output through TMA stores when it is contiguous (B, H_q, T_q, 128) and 16-byte aligned
  CUtensorMap to = tq;
  const bool contiguous_out = out_strides[3] == 1 && out_strides[2] == 128 && out_strides[1] == Tq * 128 &&
                              (B == 1 || out_strides[0] == Hq * Tq * 128) && reinterpret_cast<uintptr_t>(out) % 16 == 0;
  p.tma_out = contiguous_out && tensor_map_2d(&to, out, cu, 128, B * Hq * Tq, 256, 64, PQ) ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == LINATTN_F16) e = launch_prefill<__half, __half>(p, tq, tk, tv, to, st);
  else if (v_f16) e = launch_prefill<__nv_bfloat16, __half>(p, tq, tk, tv, to, st);
  else e = launch_prefill<__nv_bfloat16, __nv_bfloat16>(p, tq, tk, tv, to, st);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "block_sparse_prefill: %s", cudaGetErrorString(e));
    return set_error(LINATTN_ECUDA, msg);
  }
  return LINATTN_OK;
}
