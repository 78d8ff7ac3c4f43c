/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for the eviction path.
 *
 * A plain-C restatement of tonghuikang/cache-eviction's decode-time eviction
 * path (code/cache_eviction/sglang_evict_runtime.py, "runtime:" below, and
 * code/cache_eviction/core.py).  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference arm load it; the product path never
 * does.  Its outputs are pinned against fixtures produced by the reference's
 * own functions (tests/golden/make_golden.py).
 *
 * Layouts match include/ce_api.h (host memory here): pools [units, G, P, D]
 * as raw bf16 bits (uint16), scores [L, G, units] fp32, table/req_to_unit
 * [rows, width] int32, pos [rows, L, G, cap] int32.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
  int32_t n, budget, prefix, recent, cursor, policy;
  uint64_t seed;
} or_row_params; /* same bytes as ce_row_params */

enum { POL_PREFIX_SLIDING = 0, POL_RANDOM = 1, POL_RESERVOIR = 2, POL_HEAD_SUM = 3,
       POL_HEAD_MAX = 4, POL_H2O_GLOBAL = 5 };

static inline float bf16f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* core.reservoir_score (core.py:23-30) and runtime reservoir_scores
 * (runtime:358-373): splitmix64 of (seed, layer, KV head, position); the
 * returned integer divided by 2^53 is the reference's double. */
uint64_t or_reservoir53(uint64_t seed, uint64_t layer, uint64_t head, uint64_t pos) {
  uint64_t x = pos * 0x9E3779B97F4A7C15ull + layer * 0xBF58476D1CE4E5B9ull +
               head * 0x94D049BB133111EBull + seed * 0xD1B54A32D192ED03ull + 0x632BE59BD9B4E019ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  x = x ^ (x >> 31);
  return x >> 11;
}

/* fill (runtime:136-152): CSR of compacted residents then the tail. */
void or_fill(const int32_t* table, int64_t ts, const int32_t* r2u, int64_t rs,
             const int32_t* frontier, const int32_t* count, const int64_t* rows,
             const int64_t* seq_lens, int bs, int page, int32_t* indptr, int64_t* indices,
             int32_t* tokens) {
  int64_t off = 0;
  indptr[0] = 0;
  for (int b = 0; b < bs; ++b) {
    const int64_t row = rows[b];
    const int cnt = count[row], fr = frontier[row];
    const int64_t units = (seq_lens[b] + page - 1) / page;
    const int64_t tail = units - fr > 0 ? units - fr : 0;
    for (int i = 0; i < cnt; ++i) indices[off + i] = table[row * ts + i];
    for (int64_t i = 0; i < tail; ++i) indices[off + cnt + i] = r2u[row * rs + fr + i];
    off += cnt + tail;
    indptr[b + 1] = (int32_t)off;
    if (tokens) tokens[b] = (int32_t)((int64_t)cnt * page + seq_lens[b] - (int64_t)fr * page);
  }
}

/* Decode attention with sinks (runtime _verify_decode math, runtime:266-271)
 * plus the per-KV-head H2O scores of _decode_scores / the reference test
 * formula (code/tests/test_sglang_evict.py:71-78), generalised to pages:
 *   p[h,t] = exp(scale*q_h.k_t - logsumexp_t'(scale*q_h.k_t') (+) sink_h)
 *   mode 1: score[g, unit] += sum_{t in unit} sum_{h in g} p[h,t]
 *   mode 2: score[g, unit] += sum_{t in unit} max_{h in g} p[h,t]
 * zero_new: the unit the newest token starts is overwritten (runtime:211-212).
 * q [bs, H, D] bf16 bits; out [bs, H, D] fp32; lse [bs, H] natural log. */
void or_decode(const uint16_t* q, const uint16_t* kpool, const uint16_t* vpool, int64_t pool_units,
               const int32_t* indptr, const int32_t* indices, const int32_t* tokens,
               const float* sinks, const int32_t* modes, float scale, int bs, int H, int G,
               int D, int P, float* scores, int64_t score_sg, int zero_new, float* out,
               float* lse) {
  const int grp = H / G;
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int b = 0; b < bs; ++b) {
    for (int g = 0; g < G; ++g) {
      const int ntok = tokens[b];
      double* s = (double*)malloc(sizeof(double) * (size_t)(ntok > 0 ? ntok : 1) * grp);
      for (int r = 0; r < grp; ++r) {
        const int h = g * grp + r;
        const uint16_t* qh = q + ((int64_t)b * H + h) * D;
        double m = sinks ? (double)sinks[h] : -INFINITY;
        for (int t = 0; t < ntok; ++t) {
          const int unit = indices[indptr[b] + t / P];
          const uint16_t* kr = kpool + (((int64_t)unit * G + g) * P + t % P) * D;
          double acc = 0.0;
          for (int d = 0; d < D; ++d) acc += (double)bf16f(qh[d]) * (double)bf16f(kr[d]);
          s[(int64_t)r * ntok + t] = acc * (double)scale;
          if (s[(int64_t)r * ntok + t] > m) m = s[(int64_t)r * ntok + t];
        }
        double den = sinks ? exp((double)sinks[h] - m) : 0.0;
        for (int t = 0; t < ntok; ++t) den += exp(s[(int64_t)r * ntok + t] - m);
        const double norm = m + log(den);
        if (lse) lse[(int64_t)b * H + h] = (float)norm;
        double o[256];
        for (int d = 0; d < D; ++d) o[d] = 0.0;
        for (int t = 0; t < ntok; ++t) {
          const double pt = exp(s[(int64_t)r * ntok + t] - norm);
          s[(int64_t)r * ntok + t] = pt;
          const int unit = indices[indptr[b] + t / P];
          const uint16_t* vr = vpool + (((int64_t)unit * G + g) * P + t % P) * D;
          for (int d = 0; d < D; ++d) o[d] += pt * (double)bf16f(vr[d]);
        }
        for (int d = 0; d < D; ++d) out[((int64_t)b * H + h) * D + d] = (float)o[d];
      }
      const int mode = modes ? modes[b] : 0;
      if ((mode == 1 || mode == 2) && scores) {
        const int npages = (ntok + P - 1) / P;
        for (int j = 0; j < npages; ++j) {
          double c = 0.0;
          for (int t = j * P; t < (j + 1) * P && t < ntok; ++t) {
            double agg = 0.0;
            for (int r = 0; r < grp; ++r) {
              const double pt = s[(int64_t)r * ntok + t];
              if (mode == 1) agg += pt;
              else if (pt > agg) agg = pt;
            }
            c += agg;
          }
          const int unit = indices[indptr[b] + j];
          float* sp = scores + (int64_t)g * score_sg + unit;
          const int fresh = zero_new && j == npages - 1 && ((ntok - 1) % P) == 0;
          *sp = fresh ? (float)c : (float)((double)*sp + c);
        }
      }
      free(s);
    }
  }
}

/* ---- choose (runtime:376-397) ------------------------------------------- */
typedef struct {
  double key;
  int32_t pos;
  int32_t col;
} or_item;

/* Descending key, ties to the newer (larger) position: the reference's
 * stable argsort over a newest-first pre-order.  NaN sorts above everything. */
/* Prefill / extend scores: _prefill_scores with _probabilities
 * (runtime:314-340).  Entry b's chunk q[qo_indptr[b] .. qo_indptr[b+1])
 * attends to its list of tokens[b] tokens (units indices[indptr[b] ..], page
 * P); list token t is visible to chunk query i when t <= tokens[b] - nq + i
 * (runtime:334-336).  p = exp(s - logaddexp(logsumexp(s), sink_h)) in
 * double; per token: sum over queries of (sum over the group's heads (mode 1)
 * or max (mode 2)); per unit: sum over its tokens, added to scores[g, unit]
 * (or written, for a unit whose first token is in the chunk when zero_new). */
void or_prefill(const uint16_t* q, int64_t q_st, int64_t q_sh, const uint16_t* kpool,
                const int32_t* qo_indptr, const int32_t* indptr, const int32_t* indices,
                const int32_t* tokens, const float* sinks, const int32_t* modes, float scale,
                int bs, int H, int G, int D, int P, float* scores, int64_t score_sg,
                int zero_new) {
  const int grp = H / G;
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int b = 0; b < bs; ++b) {
    for (int g = 0; g < G; ++g) {
      const int mode = modes ? modes[b] : 0;
      if (mode != 1 && mode != 2) continue;
      const int q0 = qo_indptr[b], nq = qo_indptr[b + 1] - q0, ntok = tokens[b];
      const int prefix = ntok - nq;
      if (nq <= 0 || prefix < 0) continue;
      double* contrib = (double*)calloc((size_t)ntok, sizeof(double));
      double* s = (double*)malloc(sizeof(double) * (size_t)ntok * grp);
      for (int i = 0; i < nq; ++i) {
        const int vis = prefix + i + 1; /* tokens [0, vis) */
        for (int r = 0; r < grp; ++r) {
          const int h = g * grp + r;
          const uint16_t* qh = q + (int64_t)(q0 + i) * q_st + (int64_t)h * q_sh;
          double m = -INFINITY;
          for (int t = 0; t < vis; ++t) {
            const int unit = indices[indptr[b] + t / P];
            const uint16_t* kr = kpool + (((int64_t)unit * G + g) * P + t % P) * D;
            double acc = 0.0;
            for (int d = 0; d < D; ++d) acc += (double)bf16f(qh[d]) * (double)bf16f(kr[d]);
            s[(int64_t)r * ntok + t] = acc * (double)scale;
            if (s[(int64_t)r * ntok + t] > m) m = s[(int64_t)r * ntok + t];
          }
          double mm = m;
          if (sinks && (double)sinks[h] > mm) mm = (double)sinks[h];
          double den = sinks ? exp((double)sinks[h] - mm) : 0.0;
          for (int t = 0; t < vis; ++t) den += exp(s[(int64_t)r * ntok + t] - mm);
          const double norm = mm + log(den);
          for (int t = 0; t < vis; ++t) s[(int64_t)r * ntok + t] = exp(s[(int64_t)r * ntok + t] - norm);
        }
        for (int t = 0; t < vis; ++t) {
          double agg = 0.0;
          for (int r = 0; r < grp; ++r) {
            const double pt = s[(int64_t)r * ntok + t];
            if (mode == 1) agg += pt;
            else if (pt > agg) agg = pt;
          }
          contrib[t] += agg;
        }
      }
      const int npages = (ntok + P - 1) / P;
      for (int j = 0; j < npages; ++j) {
        double c = 0.0;
        for (int t = j * P; t < (j + 1) * P && t < ntok; ++t) c += contrib[t];
        const int unit = indices[indptr[b] + j];
        float* sp = scores + (int64_t)g * score_sg + unit;
        *sp = (zero_new && j * P >= prefix) ? (float)c : (float)((double)*sp + c);
      }
      free(s);
      free(contrib);
    }
  }
}

static int cmp_item(const void* a, const void* b) {
  const or_item* x = (const or_item*)a;
  const or_item* y = (const or_item*)b;
  const int xn = isnan(x->key), yn = isnan(y->key);
  if (xn != yn) return xn ? -1 : 1;
  if (!xn && x->key != y->key) return x->key > y->key ? -1 : 1;
  return (x->pos > y->pos) ? -1 : (x->pos < y->pos ? 1 : 0);
}

static int cmp_pos_col(const void* a, const void* b) {
  const or_item* x = (const or_item*)a;
  const or_item* y = (const or_item*)b;
  return (x->pos < y->pos) ? -1 : (x->pos > y->pos ? 1 : 0);
}

static inline int prot(int pos, const or_row_params* q) {
  return pos < q->prefix || pos >= q->n - q->recent || (q->cursor >= 0 && pos >= q->cursor);
}

/* Replay layer error: _replay_layer_difference (runtime:520-546) with
 * _probabilities (314-324) and _visible (241-247).  Query i of the chunk sits
 * at position start + i and sees keys 0 .. start + i of the shadow k/v
 * ([positions, G, D] bf16 bits).  Per head: a = softmax_full V,
 * b = softmax over the head's visible keys V (visible [G, start + count]
 * bytes, NULL = all), both with the sink in the normaliser
 * (logaddexp(logsumexp, sink), so no visible key and a sink give b = 0);
 * error[i] = ||b - a|| / max(||a||, 1e-12) over all H x D values, in double.
 * out_masked (optional) [count, H, D] receives b. */
void or_replay_error(const uint16_t* q, int64_t q_st, int64_t q_sh, const uint16_t* k,
                     const uint16_t* v, const uint8_t* visible, const float* sinks, float scale,
                     int H, int G, int D, int start, int count, double* error,
                     double* out_masked) {
  const int grp = H / G;
  const int end = start + count;
#pragma omp parallel for schedule(dynamic)
  for (int i = 0; i < count; ++i) {
    const int nk = start + i + 1;
    double* s = (double*)malloc(sizeof(double) * (size_t)nk);
    double* a = (double*)malloc(sizeof(double) * (size_t)D);
    double* b = (double*)malloc(sizeof(double) * (size_t)D);
    double num = 0.0, den = 0.0;
    for (int h = 0; h < H; ++h) {
      const int g = h / grp;
      const uint16_t* qh = q + (int64_t)i * q_st + (int64_t)h * q_sh;
      const uint8_t* vis = visible ? visible + (int64_t)g * end : NULL;
      double m = -INFINITY, mv = -INFINITY;
      for (int t = 0; t < nk; ++t) {
        const uint16_t* kr = k + ((int64_t)t * G + g) * D;
        double acc = 0.0;
        for (int d = 0; d < D; ++d) acc += (double)bf16f(qh[d]) * (double)bf16f(kr[d]);
        s[t] = acc * (double)scale;
        if (s[t] > m) m = s[t];
        if ((!vis || vis[t]) && s[t] > mv) mv = s[t];
      }
      const double sink = sinks ? (double)sinks[h] : -INFINITY;
      if (sink > m) m = sink;
      if (sink > mv) mv = sink;
      double z = sinks ? exp(sink - m) : 0.0, zv = (sinks && mv > -INFINITY) ? exp(sink - mv) : 0.0;
      for (int t = 0; t < nk; ++t) {
        z += exp(s[t] - m);
        if (!vis || vis[t]) zv += exp(s[t] - mv);
      }
      for (int d = 0; d < D; ++d) a[d] = b[d] = 0.0;
      for (int t = 0; t < nk; ++t) {
        const double pa = exp(s[t] - m) / z;
        const double pb = (!vis || vis[t]) ? exp(s[t] - mv) / zv : 0.0;
        const uint16_t* vr = v + ((int64_t)t * G + g) * D;
        for (int d = 0; d < D; ++d) {
          const double x = (double)bf16f(vr[d]);
          a[d] += pa * x;
          b[d] += pb * x;
        }
      }
      for (int d = 0; d < D; ++d) {
        num += (b[d] - a[d]) * (b[d] - a[d]);
        den += a[d] * a[d];
        if (out_masked) out_masked[((int64_t)i * H + h) * D + d] = b[d];
      }
    }
    const double na = sqrt(den);
    error[i] = sqrt(num) / (na > 1e-12 ? na : 1e-12);
    free(s);
    free(a);
    free(b);
  }
}

/* One segment: kept columns (protected + chosen) sorted by ascending pos.
 * key[c] is the reference's double key for unprotected columns.  Returns
 * the number kept, or -1 if the protected count exceeds the budget. */
static int choose_segment(const int32_t* pos, const double* key, int N, const or_row_params* q,
                          int32_t* kept_cols, int* nprot_out) {
  or_item* it = (or_item*)malloc(sizeof(or_item) * (size_t)(N > 0 ? N : 1));
  or_item* kp = (or_item*)malloc(sizeof(or_item) * (size_t)(N > 0 ? N : 1));
  int np = 0, nc = 0, nk = 0;
  for (int c = 0; c < N; ++c) {
    if (prot(pos[c], q)) {
      kp[nk].pos = pos[c];
      kp[nk].col = c;
      ++nk;
      ++np;
    } else {
      it[nc].key = key[c];
      it[nc].pos = pos[c];
      it[nc].col = c;
      ++nc;
    }
  }
  *nprot_out = np;
  if (np > q->budget) {
    free(it);
    free(kp);
    return -1;
  }
  int k = (q->policy == POL_PREFIX_SLIDING) ? 0 : q->budget - np;
  if (k > nc) k = nc;
  qsort(it, (size_t)nc, sizeof(or_item), cmp_item);
  for (int i = 0; i < k; ++i) kp[nk++] = it[i];
  qsort(kp, (size_t)nk, sizeof(or_item), cmp_pos_col);
  for (int i = 0; i < nk; ++i) kept_cols[i] = kp[i].col;
  free(it);
  free(kp);
  return nk;
}

/* ce_choose restated: score [problems, segs, n_cols] as double (NULL for
 * reservoir / prefix_sliding).  h2o_global key = fp32 sum over the layer's
 * heads in ascending head order (score_is_f32) or the double sum. */
void or_choose(const int32_t* pos, const int32_t* ncols, int n_cols, const double* score,
               int score_is_f32, const or_row_params* params, int problems, int layers, int heads,
               int head_offset, int32_t* kept, int kept_stride, int32_t* status,
               int32_t* pcount) {
  const int segs = layers * heads;
  int* np_all = (int*)malloc(sizeof(int) * (size_t)problems * segs);
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int i = 0; i < problems; ++i) {
    for (int s = 0; s < segs; ++s) {
      const or_row_params* q = &params[i];
      const int N = ncols ? ncols[i] : n_cols;
      const int l = s / heads, g = s % heads;
      const int64_t base = ((int64_t)i * segs + s) * n_cols;
      double* key = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
      for (int c = 0; c < N; ++c) {
        if (q->policy == POL_RESERVOIR) {
          key[c] = (double)or_reservoir53(q->seed, (uint64_t)l, (uint64_t)(head_offset + g),
                                          (uint64_t)pos[base + c]) / 9007199254740992.0;
        } else if (q->policy == POL_H2O_GLOBAL) {
          if (score_is_f32) {
            float acc = 0.f;
            for (int gg = 0; gg < heads; ++gg)
              acc += (float)score[((int64_t)i * segs + l * heads + gg) * n_cols + c];
            key[c] = acc;
          } else {
            double acc = 0.0;
            for (int gg = 0; gg < heads; ++gg) acc += score[((int64_t)i * segs + l * heads + gg) * n_cols + c];
            key[c] = acc;
          }
        } else if (q->policy == POL_PREFIX_SLIDING || !score) {
          key[c] = 0.0;
        } else {
          key[c] = score[base + c];
        }
      }
      int np = 0;
      int32_t* out = kept + ((int64_t)i * segs + s) * kept_stride;
      int32_t* tmp = (int32_t*)malloc(sizeof(int32_t) * (size_t)(N > 0 ? N : 1));
      const int nk = choose_segment(pos + base, key, N, q, tmp, &np);
      for (int x = 0; x < nk && x < kept_stride; ++x) out[x] = tmp[x];
      np_all[(int64_t)i * segs + s] = np;
      free(tmp);
      free(key);
    }
  }
  for (int i = 0; i < problems; ++i) {
    const int n0 = np_all[(int64_t)i * segs];
    int st = 0;
    for (int s = 1; s < segs; ++s)
      if (np_all[(int64_t)i * segs + s] != n0) st = 3;
    if (st == 0 && n0 > params[i].budget) st = 2;
    status[i] = st;
    if (pcount) pcount[i] = n0;
  }
  free(np_all);
}

/* ---- _boundary (runtime:415-507) ----------------------------------------- *
 * Mutates the state in place.  k_layers/v_layers: host pointers per layer.
 * uniforms: [num_rows, L, G, max_cols] doubles (random rows) or NULL.
 * result [num_rows, 4] as ce_boundary. */
void or_boundary(int32_t* table, int64_t ts, int32_t* r2u, int64_t rs, int32_t* frontier,
                 int32_t* count, int32_t* pos, int64_t prs, int pos_cap, float* scores,
                 int64_t sls, int64_t shs, int64_t pool_units, uint16_t** k_layers,
                 uint16_t** v_layers, int L, int G, int P, int D, int head_offset,
                 const int64_t* swa, const int32_t* rows, const or_row_params* params,
                 int num_rows, const double* uniforms, int max_cols, int live, int32_t* result,
                 int32_t* freed, int64_t freed_stride) {
  const int LG = L * G;
  const int64_t ublk = (int64_t)P * D; /* bf16 elements of one (unit, head) block */
  for (int i = 0; i < num_rows; ++i) {
    const or_row_params* q = &params[i];
    const int row = rows[i];
    const int cnt = count[row], fr = frontier[row];
    const int N = cnt + (q->n - fr);
    int32_t* res = result + i * 4;
    res[0] = 1;
    res[1] = N;
    res[2] = N;
    res[3] = 0;
    if (N <= q->budget) continue; /* runtime:433-435 */
    int32_t* units = (int32_t*)malloc(sizeof(int32_t) * (size_t)N);
    int32_t* ps = (int32_t*)malloc(sizeof(int32_t) * (size_t)LG * N);
    for (int c = 0; c < N; ++c)
      units[c] = c < cnt ? table[row * ts + c] : r2u[row * rs + fr + (c - cnt)]; /* 428 */
    for (int lg = 0; lg < LG; ++lg)
      for (int c = 0; c < N; ++c)
        ps[(int64_t)lg * N + c] = c < cnt ? pos[row * prs + (int64_t)lg * pos_cap + c] : fr + (c - cnt);
    /* keys (_scores, runtime:400-412) */
    double* key = (double*)malloc(sizeof(double) * (size_t)LG * N);
    for (int lg = 0; lg < LG; ++lg) {
      const int l = lg / G, g = lg % G;
      for (int c = 0; c < N; ++c) {
        double k = 0.0;
        switch (q->policy) {
          case POL_RANDOM:
            k = uniforms ? uniforms[((int64_t)i * LG + lg) * max_cols + c] : 0.0;
            break;
          case POL_RESERVOIR:
            k = (double)or_reservoir53(q->seed, (uint64_t)l, (uint64_t)(head_offset + g),
                                       (uint64_t)ps[(int64_t)lg * N + c]) / 9007199254740992.0;
            break;
          case POL_HEAD_SUM:
          case POL_HEAD_MAX:
            k = scores[l * sls + g * shs + units[c]];
            break;
          case POL_H2O_GLOBAL: {
            float acc = 0.f;
            for (int gg = 0; gg < G; ++gg) acc += scores[l * sls + gg * shs + units[c]];
            k = acc;
            break;
          }
          default:
            k = 0.0;
        }
        key[(int64_t)lg * N + c] = k;
      }
    }
    /* choose per (layer, head) */
    int32_t* kept = (int32_t*)malloc(sizeof(int32_t) * (size_t)LG * N);
    int* nk = (int*)malloc(sizeof(int) * LG);
    int* np = (int*)malloc(sizeof(int) * LG);
    for (int lg = 0; lg < LG; ++lg)
      nk[lg] = choose_segment(ps + (int64_t)lg * N, key + (int64_t)lg * N, N, q,
                              kept + (int64_t)lg * N, &np[lg]);
    int mismatch = 0;
    for (int lg = 1; lg < LG; ++lg)
      if (np[lg] != np[0]) mismatch = 1;
    if (mismatch || np[0] > q->budget) {
      res[0] = mismatch ? 3 : 2; /* runtime:388-391 */
      if (!mismatch) res[2] = np[0];
      free(units); free(ps); free(key); free(kept); free(nk); free(np);
      continue;
    }
    const int nprot = np[0];
    const int W = (q->policy == POL_PREFIX_SLIDING) ? 0 : q->budget - nprot;
    /* protected columns of head (0,0) sorted by position (runtime:442-443) */
    int32_t* pcols = (int32_t*)malloc(sizeof(int32_t) * (size_t)(nprot > 0 ? nprot : 1));
    {
      int x = 0;
      for (int k = 0; k < nk[0]; ++k) {
        const int c = kept[k];
        if (prot(ps[c], q)) pcols[x++] = c;
      }
    }
    /* middle survivors per head sorted by position (runtime:444-446) */
    int32_t* mid = (int32_t*)malloc(sizeof(int32_t) * (size_t)LG * (W > 0 ? W : 1));
    for (int lg = 0; lg < LG; ++lg) {
      int x = 0;
      for (int k = 0; k < nk[lg]; ++k) {
        const int c = kept[(int64_t)lg * N + k];
        if (!prot(ps[(int64_t)lg * N + c], q) && x < W) mid[(int64_t)lg * W + x++] = c;
      }
    }
    /* candidates = columns not protected for (0,0), column order (447-451) */
    char* isp = (char*)calloc((size_t)N, 1);
    for (int k = 0; k < nprot; ++k) isp[pcols[k]] = 1;
    int32_t* cand = (int32_t*)malloc(sizeof(int32_t) * (size_t)N);
    int ncand = 0;
    for (int c = 0; c < N; ++c)
      if (!isp[c]) cand[ncand++] = units[c];
    /* relocation: gather every head's sources of a layer, then scatter (452-463) */
    uint16_t* tk = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)G * (W > 0 ? W : 1) * ublk);
    uint16_t* tv = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)G * (W > 0 ? W : 1) * ublk);
    float* tsc = (float*)malloc(sizeof(float) * (size_t)G * (W > 0 ? W : 1));
    for (int l = 0; l < L; ++l) {
      for (int g = 0; g < G; ++g)
        for (int j = 0; j < W; ++j) {
          const int src = units[mid[((int64_t)l * G + g) * W + j]];
          memcpy(tk + ((int64_t)g * W + j) * ublk, k_layers[l] + ((int64_t)src * G + g) * ublk, 2 * ublk);
          memcpy(tv + ((int64_t)g * W + j) * ublk, v_layers[l] + ((int64_t)src * G + g) * ublk, 2 * ublk);
          tsc[(int64_t)g * W + j] = scores[l * sls + g * shs + src];
        }
      for (int g = 0; g < G; ++g)
        for (int j = 0; j < W; ++j) {
          const int dst = cand[j];
          memcpy(k_layers[l] + ((int64_t)dst * G + g) * ublk, tk + ((int64_t)g * W + j) * ublk, 2 * ublk);
          memcpy(v_layers[l] + ((int64_t)dst * G + g) * ublk, tv + ((int64_t)g * W + j) * ublk, 2 * ublk);
          scores[l * sls + g * shs + dst] = tsc[(int64_t)g * W + j];
        }
    }
    /* table, pos, count, frontier (468-473) */
    const int after = nprot + W;
    int32_t* ntab = (int32_t*)malloc(sizeof(int32_t) * (size_t)(after > 0 ? after : 1));
    for (int k = 0; k < nprot; ++k) ntab[k] = units[pcols[k]];
    for (int j = 0; j < W; ++j) ntab[nprot + j] = cand[j];
    for (int lg = 0; lg < LG; ++lg) {
      int32_t* dst = pos + row * prs + (int64_t)lg * pos_cap;
      int32_t* tmp = (int32_t*)malloc(sizeof(int32_t) * (size_t)(after > 0 ? after : 1));
      for (int k = 0; k < nprot; ++k) tmp[k] = ps[(int64_t)lg * N + pcols[k]];
      for (int j = 0; j < W; ++j) tmp[nprot + j] = ps[(int64_t)lg * N + mid[(int64_t)lg * W + j]];
      memcpy(dst, tmp, sizeof(int32_t) * (size_t)after);
      free(tmp);
    }
    memcpy(table + row * ts, ntab, sizeof(int32_t) * (size_t)after);
    count[row] = after;
    frontier[row] = q->n;
    res[0] = 0;
    res[2] = after;
    if (live) {
      const int nleft = ncand - W;
      int bad = 0;
      if (swa)
        for (int k = W; k < ncand; ++k)
          if (swa[cand[k]] != 0) bad = 1; /* 477-479 */
      if (bad) {
        res[0] = 5;
      } else {
        for (int k = W; k < ncand; ++k) {
          freed[i * freed_stride + (k - W)] = cand[k];
          for (int l = 0; l < L; ++l)
            for (int g = 0; g < G; ++g) scores[l * sls + g * shs + cand[k]] = 0.f; /* 481 */
        }
        res[3] = nleft;
        /* pack the row (483-491) */
        int true_u = q->n - q->recent;
        const int cur = q->cursor >= 0 ? q->cursor : q->n;
        if (cur < true_u) true_u = cur;
        int npk = 0;
        int32_t* packed = (int32_t*)malloc(sizeof(int32_t) * (size_t)(after > 0 ? after : 1));
        for (int k = 0; k < after; ++k) {
          int real = 0;
          for (int x = (true_u > 0 ? true_u : 0); x < q->n; ++x)
            if (r2u[row * rs + x] == ntab[k]) { real = 1; break; }
          if (!real) packed[npk++] = ntab[k];
        }
        if (npk > true_u) {
          res[0] = 4;
        } else {
          for (int x = 0; x < true_u; ++x) r2u[row * rs + x] = 0;
          for (int x = 0; x < npk; ++x) r2u[row * rs + x] = packed[x];
        }
        free(packed);
      }
    }
    free(units); free(ps); free(key); free(kept); free(nk); free(np); free(pcols); free(mid);
    free(isp); free(cand); free(tk); free(tv); free(tsc); free(ntab);
  }
}

int or_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void or_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
