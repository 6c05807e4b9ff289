/*
 * alut_oracle.c - CPU restatement of the reference's ALUT search path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA library and the
 * CPU baseline of bench.py; it is never linked into, loaded by, or called from the
 * product path (the table_moe package and libalut.so).
 *
 * Every function follows the reference's torch (non-Triton) path of
 * fanyalun/tablemoe-sc26, which scans all K centroids:
 *   oracle_project   table_moe/cache_engine/search.py:476-498 (_project_queries_into)
 *                    and search.py:12-21 (_normalize_last_dim)
 *   oracle_search    table_moe/cache_engine/search.py:566-602 (_search_decode_offline_from_low_into)
 *                    table_moe/cache_engine/search.py:661-697 (_search_offline_dot_from_low_into)
 *   oracle_gather    table_moe/cache_engine/manager.py:212-213 (gather_values)
 *   oracle_combine   table_moe/models/qwen3_vl_moe/cached_layers.py:455-465 restricted to the
 *                    lookup slots, with table_moe/skip/pruning.py:55-73
 *                    (renormalize_surviving_weights)
 *
 * Rounding: torch computes a 16-bit op in fp32 and rounds the result once to the tensor
 * dtype; `round_mode` (0 = fp32, 1 = bf16, 2 = fp16) reproduces that for the projected
 * query, the norm, the normalised query and the scores. The scores of a row are summed in
 * fp32 in increasing l; torch's bmm may sum in another order, which moves a score by a
 * few ulp - the parity rule exempts slots whose top-2 gap is below 1e-5 relative, and
 * oracle_search reports that gap (computed in double) for every slot.
 *
 * Multithreaded with OpenMP over tokens when built with -fopenmp.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static float round_bf16(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) { /* inf / nan */
    if (u & 0x007fffffu) u |= 0x00400000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest even */
  }
  u &= 0xffff0000u;
  memcpy(&v, &u, 4);
  return v;
}

static float round_f16(float v) { return (float)(_Float16)v; }

static float rnd(float v, int mode) {
  if (mode == 1) return round_bf16(v);
  if (mode == 2) return round_f16(v);
  return v;
}

float oracle_round(float v, int mode) { return rnd(v, mode); }

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* q_low[t] = x[t] @ proj[m_t] + bias[m_t], rounded to the table dtype, then optionally
 * L2-normalised (norm <= eps -> 0). x: [Q,H]; proj: [2][H,L]; bias: [2][L]. */
void oracle_project(int64_t Q, int64_t H, int64_t L, const float* x, const uint8_t* is_vision,
                    const float* proj, const float* bias, int round_mode, int normalize,
                    float eps, float* q_low) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < Q; ++t) {
    const int m = is_vision[t] ? 0 : 1;
    const float* P = proj + (int64_t)m * H * L;
    const float* b = bias + (int64_t)m * L;
    float* out = q_low + t * L;
    for (int64_t l = 0; l < L; ++l) out[l] = 0.f;
    for (int64_t h = 0; h < H; ++h) {
      const float xv = x[t * H + h];
      const float* row = P + h * L;
      for (int64_t l = 0; l < L; ++l) out[l] = fmaf(xv, row[l], out[l]);
    }
    for (int64_t l = 0; l < L; ++l) out[l] = rnd(out[l] + b[l], round_mode);
    if (normalize) {
      float ss = 0.f;
      for (int64_t l = 0; l < L; ++l) ss = fmaf(out[l], out[l], ss);
      const float n = rnd(sqrtf(ss), round_mode);
      const float e = rnd(eps, round_mode);
      const float denom = n > e ? n : e;
      for (int64_t l = 0; l < L; ++l) out[l] = (n <= e) ? 0.f : rnd(out[l] / denom, round_mode);
    }
  }
}

/* For every (t, s) with reuse: scores over all K centroids of table (sel[t,s], m_t),
 * first maximal index, hit rule; misses and non-searched slots give hit 0, idx 0.
 * keys: [E,2,K,L]. best/gap (may be NULL) receive the best score and the relative top-2
 * gap (s1 - s2) / max(|s1|, 1e-30) computed in double from the same operands. */
void oracle_search(int64_t Q, int64_t S, int64_t E, int64_t K, int64_t L, const float* q_low,
                   const float* keys, const int64_t* sel, const uint8_t* is_vision,
                   const uint8_t* reuse, float thr_vision, float thr_text, int cmp_ge,
                   int round_mode, uint8_t* out_hit, int64_t* out_idx, float* out_best,
                   double* out_gap) {
  const float tv = rnd(thr_vision, round_mode), tt = rnd(thr_text, round_mode);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t t = 0; t < Q; ++t) {
    const int m = is_vision[t] ? 0 : 1;
    const float* q = q_low + t * L;
    for (int64_t s = 0; s < S; ++s) {
      const int64_t p = t * S + s;
      out_hit[p] = 0;
      out_idx[p] = 0;
      if (out_best) out_best[p] = -INFINITY;
      if (out_gap) out_gap[p] = INFINITY;
      if (reuse && !reuse[p]) continue;
      const int64_t e = sel[p];
      if (e < 0 || e >= E) continue;
      const float* kt = keys + ((e * 2 + m) * K) * L;
      float best = -INFINITY;
      int64_t bi = -1;
      double d1 = -INFINITY, d2 = -INFINITY;
      for (int64_t k = 0; k < K; ++k) {
        const float* row = kt + k * L;
        float acc = 0.f;
        for (int64_t l = 0; l < L; ++l) acc = fmaf(q[l], row[l], acc);
        acc = rnd(acc, round_mode);
        if (bi < 0 || acc > best) {
          best = acc;
          bi = k;
        }
        if (out_gap) { /* exact top-2 for the parity exemption (checker only) */
          double dacc = 0.0;
          for (int64_t l = 0; l < L; ++l) dacc += (double)q[l] * (double)row[l];
          if (dacc > d1) {
            d2 = d1;
            d1 = dacc;
          } else if (dacc > d2) {
            d2 = dacc;
          }
        }
      }
      const float thr = m == 0 ? tv : tt;
      const int hit = cmp_ge ? (best >= thr) : (best > thr);
      if (hit) {
        out_hit[p] = 1;
        out_idx[p] = bi;
      }
      if (out_best) out_best[p] = best;
      if (out_gap) {
        double den = fabs(d1) > 1e-30 ? fabs(d1) : 1e-30;
        out_gap[p] = K > 1 ? (d1 - d2) / den : INFINITY;
      }
    }
  }
}

/* Exact fp64 score of centroid k for slot (t, s), for checking a differing index. */
double oracle_score(int64_t S, int64_t K, int64_t L, const float* q_low, const float* keys,
                    const int64_t* sel, const uint8_t* is_vision, int64_t t, int64_t s,
                    int64_t k) {
  const int m = is_vision[t] ? 0 : 1;
  const int64_t e = sel[t * S + s];
  const float* row = keys + ((e * 2 + m) * K + k) * L;
  double acc = 0.0;
  for (int64_t l = 0; l < L; ++l) acc += (double)q_low[t * L + l] * (double)row[l];
  return acc;
}

static float load_value(const void* values, int value_bf16, int64_t i) {
  if (value_bf16) {
    uint32_t u = (uint32_t)((const uint16_t*)values)[i] << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
  }
  return ((const float*)values)[i];
}

/* out[i,:] = values[eids[i], mids[i], cids[i], :] as fp32. values: [E,2,K,H]. */
void oracle_gather(int64_t n, int64_t K, int64_t H, const void* values, int value_bf16,
                   const int64_t* eids, const int64_t* mids, const int64_t* cids, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const int64_t base = ((eids[i] * 2 + mids[i]) * K + cids[i]) * H;
    for (int64_t h = 0; h < H; ++h) out[i * H + h] = load_value(values, value_bf16, base + h);
  }
}

/* out[t,:] = (accumulate ? out[t,:] : 0) + sum_{s: hit} w~[t,s] * values[sel, m_t, idx, :]
 * with w~ = renormalised weights (renorm 0: as given; 1: to one; 2: to the row sum) over
 * the survivors compute | hit. fp32 accumulation in slot order. */
void oracle_combine(int64_t Q, int64_t S, int64_t E, int64_t K, int64_t H, const void* values,
                    int value_bf16, const int64_t* sel, const uint8_t* is_vision,
                    const uint8_t* hit, const int64_t* idx, const float* w,
                    const uint8_t* compute, int renorm, int accumulate, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < Q; ++t) {
    const int m = is_vision[t] ? 0 : 1;
    float kept = 0.f, tot = 0.f;
    for (int64_t s = 0; s < S; ++s) {
      const int surv = (compute && compute[t * S + s]) || hit[t * S + s];
      kept += surv ? w[t * S + s] : 0.f;
      tot += w[t * S + s];
    }
    float* o = out + t * H;
    if (!accumulate)
      for (int64_t h = 0; h < H; ++h) o[h] = 0.f;
    for (int64_t s = 0; s < S; ++s) {
      const int64_t p = t * S + s;
      if (!hit[p]) continue;
      const int64_t e = sel[p];
      if (e < 0 || e >= E || idx[p] < 0 || idx[p] >= K) continue;
      float ww = w[p];
      if (renorm == 1) ww = kept > 0.f ? ww / kept : 0.f;
      else if (renorm == 2) ww = kept > 0.f ? (ww / kept) * tot : 0.f;
      const int64_t base = ((e * 2 + m) * K + idx[p]) * H;
      for (int64_t h = 0; h < H; ++h) o[h] = fmaf(ww, load_value(values, value_bf16, base + h), o[h]);
    }
  }
}
