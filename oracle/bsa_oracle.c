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
 *                    scores        DOT   q.k of mean-pooled blocks
 *                                  MAXDOT2 src/ssa_model.py:118-119
 *                                  QUEST src/qwen_blocksparse.py:117-120
 *   oracle_csr     — key-block transpose of the active (qblk, slot) entries under the
 *                    masks of src/triton_kernel.py:57-61 (SLOT) or
 *                    src/qwen_blocksparse.py:67-72 (TOKEN).
 *
 * Build: oracle/build.sh (gcc -O2 -ffp-contract=off -fPIC -shared).
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
  return (t > 0 ? t : 0) + 1 + (sink ? 1 : 0);
}

static float logsigmoidf_(float x) { return x < 0.f ? x - log1pf(expf(x)) : -log1pf(expf(-x)); }

static int cmp_int(const void *p, const void *q) {
  const int a = *(const int *)p, b = *(const int *)q;
  return (a > b) - (a < b);
}

/* a, b1, b2: (G, nblk, dim) fp32.  sel: (G, nblk, W).  score/gate optional (SSA). */
void oracle_select(const float *a, const float *b1, const float *b2, int G, int nblk, int dim,
                   int kind, int layout, int causal, int topk, int sink, int32_t *sel,
                   float *score_out, float *gate_out) {
  const int W = oracle_select_width(layout, nblk, topk, sink);
  const int T = layout == 0 ? W - 1 : W - 1 - (sink ? 1 : 0);
  float *ls = (float *)malloc(sizeof(float) * (T > 0 ? T : 1));
  int *li = (int *)malloc(sizeof(int) * (T > 0 ? T : 1));
  int *tmp = (int *)malloc(sizeof(int) * (W + 1));
  for (int g = 0; g < G; ++g) {
    const float *A = a + (int64_t)g * nblk * dim;
    const float *B1 = b1 + (int64_t)g * nblk * dim;
    const float *B2 = b2 ? b2 + (int64_t)g * nblk * dim : NULL;
    for (int i = 0; i < nblk; ++i) {
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
      } else {
        for (int l = 0; l < T; ++l) tmp[l] = l < n ? li[l] : i;
        tmp[T] = i;
        if (sink) tmp[T + 1] = 0;
        qsort(tmp, W, sizeof(int), cmp_int);
        for (int l = 0; l < W; ++l) out[l] = tmp[l];
      }
    }
  }
  free(ls);
  free(li);
  free(tmp);
}

/* 1 when slot `slot` of `row` is attended under the mask rules, else 0. */
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
