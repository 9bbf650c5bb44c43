/*
 * CPU oracle — TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg may load this library, and only as the
 * checker; the product path never calls it.
 *
 * Plain-C restatement of the reference's block selection, written to the
 * exact arithmetic contract the CUDA kernels implement (sequential fp32 sums,
 * one fma chain per score, ranking by (score desc, block id asc)), so that
 * selected indices can be compared bit for bit.
 *
 *   oracle_pool    — block mean/min/max:  reference src/qwen_blocksparse.py:111-116
 *                    (grp>1 mean over the query group first, :113) and
 *                    src/ssa_model.py:113-117 (mean / max pooling of selector features)
 *   oracle_select  — scores + causal top-k:
 *                    layout SSA    src/ssa_model.py:151-162 (own block first, then the
 *                                  top-k content blocks, own excluded, future masked)
 *                    layout FINISH src/qwen_blocksparse.py:87-99 (_finish: causal mask,
 *                                  topk, non-finite -> own, + own + sink, sorted)
 *                    layout RAW    the causal top-k picks in rank order, -1 when fewer
 *                                  (stage 1 of SelectTwoStage, :285-286)
 *                    scores        DOT   q.k of mean-pooled blocks
 *                                  MAXDOT2 src/ssa_model.py:118-119
 *                                  QUEST src/qwen_blocksparse.py:117-120
 *   oracle_select_lsh — LSH candidate selection, the inference branch of LSHBucketSSA
 *                    src/ssa_model.py:438-470: per-round buckets (argmax of the
 *                    projections, :438-439, or the sign bits of n_planes hyperplanes),
 *                    the first `cap` key blocks of each bucket by index (:441-450),
 *                    candidates = the query block's buckets over all rounds,
 *                    deduplicated, own / future excluded (:451-462; block 0 is also
 *                    dropped after an empty slot of an earlier round, because the
 *                    reference dedups ids clamped at 0, :452-457), re-scored by
 *                    scale * cosine, top-k, own block first (:470-476).
 *   oracle_select_scores — _finish top-k of a given score matrix (SelectOracle /
 *                    SelectRandom, src/qwen_blocksparse.py:124-152, :87-99)
 *   oracle_select_qmax — per-token Quest bound maxed over the query block's tokens,
 *                    over all causal blocks (SelectMaxQMax :221-247) or a per-row
 *                    candidate list (SelectTwoStage :270-299)
 *   oracle_csr     — key-block transpose of the active (qblk, slot) entries under the
 *                    masks of src/triton_kernel.py:57-61 (SLOT) or
 *                    src/qwen_blocksparse.py:67-72 (TOKEN).
 *
 * Build: oracle/build.sh (gcc -O2 -ffp-contract=off -fopenmp -fPIC -shared).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* x: (B,H,L,D) with element strides sb, sh, sl (unit D stride), fp32 values. */
void oracle_pool(const float *x, int64_t sb, int64_t sh, int64_t sl, int B, int H, int L, int D,
                 int bs, int grp, float *mean, float *vmin, float *vmax) {
  const int nblk = (L + bs - 1) / bs;
  const int Hout = H / grp;
  for (int b = 0; b < B; ++b)
    for (int ho = 0; ho < Hout; ++ho)
      for (int blk = 0; blk < nblk; ++blk)
        for (int d = 0; d < D; ++d) {
          float sum = 0.f, mn = INFINITY, mx = -INFINITY;
          for (int r = 0; r < bs; ++r) {
            const int64_t gr = (int64_t)blk * bs + r;
            float v = 0.f;
            if (gr < L) {
              if (grp == 1) {
                v = x[b * sb + ho * sh + gr * sl + d];
              } else {
                float t = 0.f;
                for (int g = 0; g < grp; ++g) t = t + x[b * sb + (int64_t)(ho * grp + g) * sh + gr * sl + d];
                v = t / (float)grp;
              }
            }
            sum = sum + v;
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
          }
          const int64_t o = (((int64_t)b * Hout + ho) * nblk + blk) * D + d;
          if (mean) mean[o] = sum / (float)bs;
          if (vmin) vmin[o] = mn;
          if (vmax) vmax[o] = mx;
        }
}

static float score_of(int kind, const float *a, const float *b1, const float *b2, int dim) {
  float s = 0.f, s2 = 0.f;
  for (int d = 0; d < dim; ++d) {
    const float av = a[d];
    if (kind == 2)
      s = fmaf(av, av >= 0.f ? b1[d] : b2[d], s);
    else
      s = fmaf(av, b1[d], s);
    if (kind == 1) s2 = fmaf(av, b2[d], s2);
  }
  return kind == 1 ? fmaxf(s, s2) : s;
}

static int better(float s1, int i1, float s2, int i2) { return s1 > s2 || (s1 == s2 && i1 < i2); }

int oracle_select_width(int layout, int nblk, int topk, int sink) {
  int t;
  if (layout == 0) {
    t = topk < nblk - 1 ? topk : nblk - 1;
    return 1 + (t > 0 ? t : 0);
  }
  t = topk < nblk ? topk : nblk;
  if (layout == 2) return t > 0 ? t : 0; /* RAW: the picks only */
  return (t > 0 ? t : 0) + 1 + (sink ? 1 : 0);
}

static float logsigmoidf_(float x) { return x < 0.f ? x - log1pf(expf(x)) : -log1pf(expf(-x)); }

static int cmp_int(const void *p, const void *q) {
  const int a = *(const int *)p, b = *(const int *)q;
  return (a > b) - (a < b);
}

/* One selection row: query block i of group g.  ls/li/tmp: scratch of T, T, W+1. */
static void select_row(const float *a, const float *b1, const float *b2, int g, int i, int nblk,
                       int dim, int kind, int layout, int causal, int topk, int sink,
                       int32_t *sel, float *score_out, float *gate_out, float *ls, int *li,
                       int *tmp) {
  const int W = oracle_select_width(layout, nblk, topk, sink);
  const int T = layout == 0 ? W - 1 : (layout == 2 ? W : W - 1 - (sink ? 1 : 0));
  const float *A = a + (int64_t)g * nblk * dim;
  const float *B1 = b1 + (int64_t)g * nblk * dim;
  const float *B2 = b2 ? b2 + (int64_t)g * nblk * dim : NULL;
  int n = 0; /* list length */
  for (int j = 0; j < nblk && T > 0; ++j) {
    int ok;
    if (layout == 0)
      ok = j != i && (!causal || j < i);
    else
      ok = j <= i;
    if (!ok) continue;
    const float s = score_of(kind, A + (int64_t)i * dim, B1 + (int64_t)j * dim,
                             B2 ? B2 + (int64_t)j * dim : NULL, dim);
    if (!(s > -INFINITY)) continue; /* -inf / NaN never rank */
    if (n == T && !better(s, j, ls[T - 1], li[T - 1])) continue;
    int pos = n < T ? n : T - 1;
    while (pos > 0 && better(s, j, ls[pos - 1], li[pos - 1])) {
      ls[pos] = ls[pos - 1];
      li[pos] = li[pos - 1];
      --pos;
    }
    ls[pos] = s;
    li[pos] = j;
    if (n < T) ++n;
  }
  int32_t *out = sel + ((int64_t)g * nblk + i) * W;
  if (layout == 0) {
    const float own = score_of(kind, A + (int64_t)i * dim, B1 + (int64_t)i * dim,
                               B2 ? B2 + (int64_t)i * dim : NULL, dim);
    const int64_t ob = ((int64_t)g * nblk + i) * W;
    out[0] = i;
    if (score_out) score_out[ob] = own;
    if (gate_out) gate_out[ob] = logsigmoidf_(own);
    for (int l = 0; l < T; ++l) {
      const int valid = l < n;
      out[1 + l] = valid ? li[l] : i;
      const float sc = valid ? ls[l] : own;
      if (score_out) score_out[ob + 1 + l] = sc;
      if (gate_out) gate_out[ob + 1 + l] = logsigmoidf_(sc);
    }
  } else if (layout == 2) {
    for (int l = 0; l < T; ++l) out[l] = l < n ? li[l] : -1;
  } else {
    for (int l = 0; l < T; ++l) tmp[l] = l < n ? li[l] : i;
    tmp[T] = i;
    if (sink) tmp[T + 1] = 0;
    qsort(tmp, W, sizeof(int), cmp_int);
    for (int l = 0; l < W; ++l) out[l] = tmp[l];
  }
}

/* a, b1, b2: (G, nblk, dim) fp32.  sel: (G, nblk, W).  score/gate optional (SSA).
 * rows: optional list of nrows query blocks (each computed for every group; the
 * other rows of sel are left untouched); NULL = every row.  Rows are independent
 * and run in parallel (OpenMP) with identical arithmetic per row. */
void oracle_select_rows(const float *a, const float *b1, const float *b2, int G, int nblk, int dim,
                        int kind, int layout, int causal, int topk, int sink, const int32_t *rows,
                        int nrows, int32_t *sel, float *score_out, float *gate_out) {
  const int W = oracle_select_width(layout, nblk, topk, sink);
  const int T = layout == 0 ? W - 1 : (layout == 2 ? W : W - 1 - (sink ? 1 : 0));
  const int R = rows ? nrows : nblk;
  const int64_t total = (int64_t)G * R;
#pragma omp parallel
  {
    float *ls = (float *)malloc(sizeof(float) * (T > 0 ? T : 1));
    int *li = (int *)malloc(sizeof(int) * (T > 0 ? T : 1));
    int *tmp = (int *)malloc(sizeof(int) * (W + 1));
#pragma omp for schedule(dynamic, 16)
    for (int64_t t = 0; t < total; ++t) {
      const int g = (int)(t / R);
      const int r = (int)(t % R);
      const int i = rows ? rows[r] : r;
      select_row(a, b1, b2, g, i, nblk, dim, kind, layout, causal, topk, sink, sel, score_out,
                 gate_out, ls, li, tmp);
    }
    free(ls);
    free(li);
    free(tmp);
  }
}

void oracle_select(const float *a, const float *b1, const float *b2, int G, int nblk, int dim,
                   int kind, int layout, int causal, int topk, int sink, int32_t *sel,
                   float *score_out, float *gate_out) {
  oracle_select_rows(a, b1, b2, G, nblk, dim, kind, layout, causal, topk, sink, NULL, 0, sel,
                     score_out, gate_out);
}

static int slot_active(const int32_t *row, int slot, int qblk, int nblk, int mask_mode, int causal) {
  const int kb = row[slot];
  if (kb < 0 || kb >= nblk) return 0;
  if (mask_mode == 0) {
    if (!causal || slot == 0) return 1;
    return kb < qblk;
  }
  for (int j = 0; j < slot; ++j)
    if (row[j] == kb) return 0;
  if (causal && kb > qblk) return 0;
  return 1;
}

/* sel addressed sel[b*sb + h*sh + q*sn + slot].  row_ptr: B*Hs*nblk + 1, col: entries. */
void oracle_csr(const int32_t *sel, int64_t sb, int64_t sh, int64_t sn, int B, int Hs, int nblk,
                int kk, int mask_mode, int causal, int32_t *row_ptr, int32_t *col) {
  const int64_t nbins = (int64_t)B * Hs * nblk;
  memset(row_ptr, 0, sizeof(int32_t) * (nbins + 1));
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < Hs; ++h)
      for (int q = 0; q < nblk; ++q) {
        const int32_t *row = sel + b * sb + h * sh + (int64_t)q * sn;
        for (int s = 0; s < kk; ++s)
          if (slot_active(row, s, q, nblk, mask_mode, causal))
            row_ptr[((int64_t)b * Hs + h) * nblk + row[s] + 1]++;
      }
  for (int64_t i = 0; i < nbins; ++i) row_ptr[i + 1] += row_ptr[i];
  int32_t *fill = (int32_t *)malloc(sizeof(int32_t) * (nbins > 0 ? nbins : 1));
  memcpy(fill, row_ptr, sizeof(int32_t) * nbins);
  /* visiting entries in ascending e = q*kk + slot keeps each bin sorted */
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < Hs; ++h)
      for (int q = 0; q < nblk; ++q) {
        const int32_t *row = sel + b * sb + h * sh + (int64_t)q * sn;
        for (int s = 0; s < kk; ++s)
          if (slot_active(row, s, q, nblk, mask_mode, causal)) {
            const int64_t bin = ((int64_t)b * Hs + h) * nblk + row[s];
            col[fill[bin]++] = q * kk + s;
          }
      }
  free(fill);
}

/* LSH selection (see header).  a, b: (G, nblk, dim) raw summaries; planes:
 * (dim, rounds, nplanes).  sel/score/gate: (G, nblk, W), W = oracle_lsh_width. */
int oracle_lsh_width(int nblk, int topk, int rounds, int cap) {
  int T = topk < (nblk - 1 > 1 ? nblk - 1 : 1) ? topk : (nblk - 1 > 1 ? nblk - 1 : 1);
  int P = rounds * cap;
  return 1 + (T < P ? T : P);
}

static void lsh_normalise(const float *x, float *y, int dim) {
  float ss = 0.f;
  for (int d = 0; d < dim; ++d) ss = fmaf(x[d], x[d], ss);
  float nrm = sqrtf(ss);
  if (nrm < 1e-12f) nrm = 1e-12f;
  for (int d = 0; d < dim; ++d) y[d] = x[d] / nrm;
}

static int lsh_code(const float *y, const float *planes, int dim, int rounds, int nplanes, int r,
                    int sign_hash) {
  int best = 0, bits = 0;
  float bv = 0.f;
  for (int c = 0; c < nplanes; ++c) {
    float v = 0.f;
    for (int d = 0; d < dim; ++d) v = fmaf(y[d], planes[(int64_t)d * rounds * nplanes + r * nplanes + c], v);
    if (c == 0 || v > bv) {
      best = c;
      bv = v;
    }
    if (v > 0.f) bits |= 1 << c;
  }
  return sign_hash ? bits : best;
}

void oracle_select_lsh(const float *a, const float *b, const float *planes, int G, int nblk, int dim,
                       int sign_hash, int rounds, int nplanes, int cap, int causal, int topk,
                       float scale, int32_t *sel, float *score, float *gate) {
  const int NB = sign_hash ? (1 << nplanes) : nplanes;
  const int W = oracle_lsh_width(nblk, topk, rounds, cap);
  const int rk = W - 1, P = rounds * cap;
  float *yq = malloc(sizeof(float) * (size_t)nblk * dim);
  float *yk = malloc(sizeof(float) * (size_t)nblk * dim);
  int *qc = malloc(sizeof(int) * (size_t)nblk * rounds), *kc = malloc(sizeof(int) * (size_t)nblk * rounds);
  int *list = malloc(sizeof(int) * (size_t)rounds * NB * cap), *cnt = malloc(sizeof(int) * (size_t)rounds * NB);
  int *cid = malloc(sizeof(int) * P);
  float *csc = malloc(sizeof(float) * P);
  for (int g = 0; g < G; ++g) {
    const float *ag = a + (int64_t)g * nblk * dim, *bg = b + (int64_t)g * nblk * dim;
    for (int i = 0; i < nblk; ++i) {
      lsh_normalise(ag + (int64_t)i * dim, yq + (int64_t)i * dim, dim);
      lsh_normalise(bg + (int64_t)i * dim, yk + (int64_t)i * dim, dim);
      for (int r = 0; r < rounds; ++r) {
        qc[i * rounds + r] = lsh_code(yq + (int64_t)i * dim, planes, dim, rounds, nplanes, r, sign_hash);
        kc[i * rounds + r] = lsh_code(yk + (int64_t)i * dim, planes, dim, rounds, nplanes, r, sign_hash);
      }
    }
    /* first `cap` key blocks of every (round, bucket), in block order */
    memset(cnt, 0, sizeof(int) * (size_t)rounds * NB);
    for (int r = 0; r < rounds; ++r)
      for (int j = 0; j < nblk; ++j) {
        int c = kc[j * rounds + r], *n = &cnt[r * NB + c];
        if (*n < cap) list[(r * NB + c) * cap + *n] = j;
        ++*n;
      }
    for (int i = 0; i < nblk; ++i) {
      const float *y = yq + (int64_t)i * dim;
      int np = 0, empty_before = 0;
      for (int r = 0; r < rounds; ++r) {
        int c = qc[i * rounds + r], n = cnt[r * NB + c] < cap ? cnt[r * NB + c] : cap;
        for (int p = 0; p < n; ++p) {
          int j = list[(r * NB + c) * cap + p], dup = 0;
          if (j == i || (causal && j > i)) continue;
          /* the reference dedups on ids clamped at 0, so an empty slot of an
           * earlier round (id -1 -> 0) removes block 0 (src/ssa_model.py:452-457) */
          if (j == 0 && empty_before) continue;
          for (int e = 0; e < np && !dup; ++e) dup = cid[e] == j;
          if (dup) continue;
          float s = 0.f;
          for (int d = 0; d < dim; ++d) s = fmaf(y[d], yk[(int64_t)j * dim + d], s);
          cid[np] = j;
          csc[np] = s * scale;
          ++np;
        }
        if (n < cap) empty_before = 1;
      }
      float own = 0.f;
      for (int d = 0; d < dim; ++d) own = fmaf(y[d], yk[(int64_t)i * dim + d], own);
      own *= scale;
      int64_t ob = ((int64_t)g * nblk + i) * W;
      sel[ob] = i;
      if (score) score[ob] = own;
      if (gate) gate[ob] = logsigmoidf_(own);
      for (int t = 0; t < rk; ++t) {
        int bi = -1;
        for (int e = 0; e < np; ++e)
          if (cid[e] >= 0 && (bi < 0 || better(csc[e], cid[e], csc[bi], cid[bi]))) bi = e;
        int pick = bi >= 0 ? cid[bi] : i;
        float ps = bi >= 0 ? csc[bi] : 0.f;
        if (bi >= 0) cid[bi] = -1;
        sel[ob + 1 + t] = pick;
        if (score) score[ob + 1 + t] = ps;
        if (gate) gate[ob + 1 + t] = logsigmoidf_(ps);
      }
    }
  }
  free(yq); free(yk); free(qc); free(kc); free(list); free(cnt); free(cid); free(csc);
}

/* _finish over per-row candidate scores: top T=min(topk,nblk) of (sc[m], id[m])
 * for m < n with finite scores and id <= i, missing -> i, + i (+ sink 0), ascending. */
static void finish_from(const float *sc, const int *id, int n, int i, int nblk, int topk, int sink,
                        int32_t *dst) {
  int T = topk < nblk ? topk : nblk, W = T + 1 + (sink ? 1 : 0);
  int *out = malloc(sizeof(int) * (W > 1 ? W : 1));
  char *used = calloc(n > 0 ? n : 1, 1);
  for (int t = 0; t < T; ++t) {
    int b = -1;
    for (int m = 0; m < n; ++m) {
      if (used[m] || id[m] < 0 || id[m] > i || !(sc[m] > -INFINITY)) continue;
      if (b < 0 || better(sc[m], id[m], sc[b], id[b])) b = m;
    }
    if (b >= 0) used[b] = 1;
    out[t] = b >= 0 ? id[b] : i;
  }
  out[T] = i;
  if (sink) out[T + 1] = 0;
  qsort(out, W, sizeof(int), cmp_int);
  for (int w = 0; w < W; ++w) dst[w] = out[w];
  free(out);
  free(used);
}

int oracle_scores_width(int nblk, int topk, int sink) {
  return (topk < nblk ? topk : nblk) + 1 + (sink ? 1 : 0);
}

/* score: (G, nblk, nblk) contiguous; sel: (G, nblk, W) */
void oracle_select_scores(const float *score, int G, int nblk, int topk, int sink, int32_t *sel) {
  const int W = oracle_scores_width(nblk, topk, sink);
  int *id = malloc(sizeof(int) * nblk);
  float *sc = malloc(sizeof(float) * nblk);
  for (int g = 0; g < G; ++g)
    for (int i = 0; i < nblk; ++i) {
      const float *row = score + ((int64_t)g * nblk + i) * nblk;
      for (int j = 0; j < nblk; ++j) {
        id[j] = j;
        sc[j] = row[j] != row[j] ? -INFINITY : row[j];
      }
      finish_from(sc, id, nblk, i, nblk, topk, sink, sel + ((int64_t)g * nblk + i) * W);
    }
  free(id);
  free(sc);
}

/* qtok: (G, nblk, bs, dim); kmax/kmin: (G, nblk, dim); cand: NULL or (G, nblk, M). */
void oracle_select_qmax(const float *qtok, const float *kmax, const float *kmin, const int32_t *cand,
                        int G, int nblk, int bs, int dim, int M, int topk, int sink, int32_t *sel) {
  const int W = oracle_scores_width(nblk, topk, sink);
  const int NC = cand ? M : nblk;
  int *id = malloc(sizeof(int) * NC);
  float *sc = malloc(sizeof(float) * NC);
  for (int g = 0; g < G; ++g)
    for (int i = 0; i < nblk; ++i) {
      const float *qb = qtok + ((int64_t)g * nblk + i) * bs * dim;
      for (int m = 0; m < NC; ++m) {
        int j = cand ? cand[((int64_t)g * nblk + i) * M + m] : m;
        if (j > i || j >= nblk) j = -1;
        id[m] = j;
        sc[m] = -INFINITY;
        if (j < 0) continue;
        const float *kx = kmax + ((int64_t)g * nblk + j) * dim, *kn = kmin + ((int64_t)g * nblk + j) * dim;
        for (int t = 0; t < bs; ++t) {
          float s = 0.f;
          for (int d = 0; d < dim; ++d) {
            const float q = qb[(int64_t)t * dim + d];
            s = fmaf(q, q >= 0.f ? kx[d] : kn[d], s);
          }
          if (s > sc[m]) sc[m] = s;
        }
      }
      finish_from(sc, id, NC, i, nblk, topk, sink, sel + ((int64_t)g * nblk + i) * W);
    }
  free(id);
  free(sc);
}
