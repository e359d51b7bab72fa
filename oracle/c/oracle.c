/*
 * C restatement of the Quest paged decode step.  TEST INFRASTRUCTURE ONLY: the CPU
 * checker for full-size parity and the timed CPU baseline (bench.py
 * `cpu_baseline` / `--impl reference`).  Never on the product path.
 *
 * For every batch b and query head h (decode: one query at position seq_len_b - 1):
 *   scores[p] = sum_d max(q_d*min_d, q_d*max_d)    src/linattn/kernels/triton/quest_pages.py:51-54
 *   own page (the last) and `sink_pages` leading pages forced to +inf, pages past
 *   the sequence excluded                          quest_pages.py:67-75
 *   top-k (score desc, lowest index on ties)       quest_pages.py:76-77 (tie rule fixed)
 * then per kv head the union of the group's pages  src/linattn/variants/selection.py:232-235
 * and, for every query head, exact softmax attention over the union's rows, with the
 * tiled online softmax of the reference's C kernel
 *                                                  src/linattn/kernels/c/decode_attn.c:72-133
 * Element types: 0 = f32, 1 = f16, 2 = bf16 (KV pool and metadata share it).
 * Thread-safe: disjoint unit ranges may run concurrently (ctypes drops the GIL).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t x) {
  uint32_t u = (uint32_t)x << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else { /* subnormal: normalise */
      exp = 113;
      while (!(man & 0x400u)) {
        man <<= 1;
        --exp;
      }
      man &= 0x3ffu;
      u = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (man << 13);
  } else {
    u = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline void load_row(int dtype, const void* base, int64_t off, int n, float* dst) {
  if (dtype == 0) {
    memcpy(dst, (const float*)base + off, sizeof(float) * (size_t)n);
  } else if (dtype == 1) {
    const uint16_t* p = (const uint16_t*)base + off;
    for (int i = 0; i < n; ++i) dst[i] = f16_to_f32(p[i]);
  } else {
    const uint16_t* p = (const uint16_t*)base + off;
    for (int i = 0; i < n; ++i) dst[i] = bf16_to_f32(p[i]);
  }
}

/* insert (score, idx) into the top-k list kept sorted by (score desc, idx asc);
   candidates arrive in ascending idx, so an equal score never displaces */
static inline void topk_push(float s, int idx, float* ts, int* ti, int* n, int k) {
  if (*n == k && !(s > ts[k - 1])) return;
  int pos = *n < k ? (*n)++ : k - 1;
  while (pos > 0 && s > ts[pos - 1]) {
    ts[pos] = ts[pos - 1];
    ti[pos] = ti[pos - 1];
    --pos;
  }
  ts[pos] = s;
  ti[pos] = idx;
}

/* Page selection of one (batch, kv head) unit: top-k per query head of the group,
   union written ascending to ul[0..*cnt).  Returns 2 when the union overflowed. */
static int quest_select_unit(int dtype, const void* q, const void* meta_min, const void* meta_max,
                             const int32_t* page_table, const int32_t* seq_lens, int Hq, int Hkv, int D, int P,
                             int max_pages, int topk, int sink_pages, int unit, int32_t* ul, int32_t* cnt_out,
                             int max_union) {
  const int group = Hq / Hkv;
  const int b = unit / Hkv, kh = unit % Hkv;
  const int len = seq_lens[b];
  const int nb = (len + P - 1) / P;
  const int kb = topk < nb ? topk : nb;
  float qv[512], mn[512], mx[512];
  float* ts = (float*)malloc(sizeof(float) * (size_t)(kb > 0 ? kb : 1));
  int* ti = (int*)malloc(sizeof(int) * (size_t)(kb > 0 ? kb : 1));
  uint8_t* in_union = (uint8_t*)calloc((size_t)(nb > 0 ? nb : 1), 1);
  for (int g = 0; g < group && nb > 0; ++g) {
    const int h = kh * group + g;
    load_row(dtype, q, ((int64_t)b * Hq + h) * D, D, qv);
    int n = 0;
    for (int p = 0; p < nb; ++p) {
      float s;
      if (p == nb - 1 || p < sink_pages) {
        s = INFINITY;
      } else {
        const int phys = page_table[(int64_t)b * max_pages + p];
        const int64_t mo = ((int64_t)phys * Hkv + kh) * D;
        load_row(dtype, meta_min, mo, D, mn);
        load_row(dtype, meta_max, mo, D, mx);
        s = 0.f;
        for (int d = 0; d < D; ++d) {
          const float a = qv[d] * mn[d], c = qv[d] * mx[d];
          s += a > c ? a : c;
        }
      }
      topk_push(s, p, ts, ti, &n, kb);
    }
    for (int i = 0; i < n; ++i) in_union[ti[i]] = 1;
  }
  int cnt = 0, bad = 0;
  for (int p = 0; p < nb; ++p)
    if (in_union[p]) {
      if (cnt < max_union) ul[cnt] = p;
      ++cnt;
    }
  if (cnt > max_union) {
    bad = 2;
    cnt = max_union;
  }
  *cnt_out = cnt;
  free(ts);
  free(ti);
  free(in_union);
  return bad;
}

/* Selection only, for units [unit_begin, unit_end) of the B*Hkv (batch, kv head) units. */
int oracle_quest_select(int dtype, const void* q, const void* meta_min, const void* meta_max,
                        const int32_t* page_table, const int32_t* seq_lens, int B, int Hq, int Hkv, int D, int P,
                        int max_pages, int topk, int sink_pages, int32_t* union_ids, int32_t* union_cnt,
                        int max_union, int unit_begin, int unit_end) {
  if (Hq % Hkv || D > 512 || topk < 1) return 1;
  if (unit_end > B * Hkv) unit_end = B * Hkv;
  int bad = 0;
  for (int unit = unit_begin; unit < unit_end; ++unit)
    bad |= quest_select_unit(dtype, q, meta_min, meta_max, page_table, seq_lens, Hq, Hkv, D, P, max_pages, topk,
                             sink_pages, unit, union_ids + (int64_t)unit * max_union, union_cnt + unit, max_union);
  return bad;
}

/* Selection + attention for units [unit_begin, unit_end); callers run disjoint
   ranges on several threads. */
int oracle_quest_decode(int dtype, const void* q, const void* k_pool, const void* v_pool, const void* meta_min,
                        const void* meta_max, const int32_t* page_table, const int32_t* seq_lens, int B, int Hq,
                        int Hkv, int D, int P, int max_pages, int topk, int sink_pages, float scale, float* out,
                        int32_t* union_ids, int32_t* union_cnt, int max_union, int unit_begin, int unit_end) {
  const int group = Hq / Hkv;
  if (group * Hkv != Hq || D > 512 || topk < 1) return 1;
  if (unit_end > B * Hkv) unit_end = B * Hkv;
  int bad = 0;
  for (int unit = unit_begin; unit < unit_end; ++unit) {
    const int b = unit / Hkv, kh = unit % Hkv;
    const int len = seq_lens[b];
    int32_t* ul = union_ids + (int64_t)unit * max_union;
    bad |= quest_select_unit(dtype, q, meta_min, meta_max, page_table, seq_lens, Hq, Hkv, D, P, max_pages, topk,
                             sink_pages, unit, ul, union_cnt + unit, max_union);
    const int cnt = union_cnt[unit];
    float qv[512], krow[512], vrow[512], acc[512];
    /* attention of each query head of the group over the union's rows */
    for (int g = 0; g < group; ++g) {
      const int h = kh * group + g;
      load_row(dtype, q, ((int64_t)b * Hq + h) * D, D, qv);
      float m = -INFINITY, l = 0.f;
      for (int d = 0; d < D; ++d) acc[d] = 0.f;
      for (int j = 0; j < cnt; ++j) {
        const int p = ul[j];
        const int phys = page_table[(int64_t)b * max_pages + p];
        int rows = len - p * P;
        if (rows > P) rows = P;
        for (int r = 0; r < rows; ++r) {
          const int64_t off = (((int64_t)phys * Hkv + kh) * P + r) * D;
          load_row(dtype, k_pool, off, D, krow);
          float s = 0.f;
          for (int d = 0; d < D; ++d) s += qv[d] * krow[d];
          s *= scale;
          const float m_new = s > m ? s : m;
          const float alpha = expf(m - m_new), pr = expf(s - m_new);
          l = l * alpha + pr;
          load_row(dtype, v_pool, off, D, vrow);
          for (int d = 0; d < D; ++d) acc[d] = acc[d] * alpha + pr * vrow[d];
          m = m_new;
        }
      }
      float* o = out + ((int64_t)b * Hq + h) * D;
      for (int d = 0; d < D; ++d) o[d] = l > 0.f ? acc[d] / l : 0.f;
    }
  }
  return bad;
}
