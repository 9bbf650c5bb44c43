// LSH candidate selection: hash pooled block summaries into buckets per round,
// keep the first `cap` key blocks of every bucket (by block index), and pick
// each query block's top-k among the key blocks sharing one of its buckets,
// re-scored by the exact cosine of the summaries.  O(nblk * rounds * (planes +
// cap)); no nblk x nblk matrix.  Follows LSHBucketSSA's inference branch
// (reference src/ssa_model.py:438-470) with two hash rules:
//   ARGMAX: bucket = argmax_c <y, R[:, r, c]>            (src/ssa_model.py:438-439)
//   SIGN:   bucket = sum_c [<y, R[:, r, c]> > 0] << c    (sign of n_planes hyperplanes)
//
// Kernels (all tiny next to the attention read):
//   lsh_hash_kernel    one thread per (summary row): L2-normalise (y = x / max(|x|, 1e-12)),
//                      store y, and the bucket of every round.
//   lsh_bucket_kernel  one warp per (group, round): walks the key blocks in index
//                      order 32 at a time; __match_any_sync gives each block its rank
//                      among earlier blocks of the same bucket, so the first `cap` blocks
//                      of each bucket land in the list in index order (the reference's
//                      cumsum-of-one-hot rank, src/ssa_model.py:444-449).
//   lsh_select_kernel  one warp per (group, query block): up to rounds*cap candidates
//                      (lane-strided), exact scaled cosine, then `rk` rounds of a warp
//                      arg-max by (score desc, block asc); the winner's duplicates are
//                      retired with it, which is the reference's cross-round dedup
//                      (including its drop of block 0 after an earlier empty slot).
// Every dot product is one fp32 fma chain over d = 0..dim-1 from 0, so the
// result is bitwise reproducible and matches the C restatement in the oracle.
#include <algorithm>

#include "bsa_host.h"

namespace bsa {

namespace {
constexpr int kLshMaxBuckets = 64;
constexpr int kLshMaxCand = 256;
constexpr int kLshMaxDim = 256;

__device__ __forceinline__ float lsh_logsigmoid(float x) {
  return x < 0.f ? x - log1pf(expf(x)) : -log1pf(expf(-x));
}

struct LshWs {
  float *an, *bn;          // normalised summaries (G, nblk, dim)
  int32_t *qcode, *kcode;  // (G, nblk, rounds)
  int32_t *list;           // (G, rounds, NB, cap)
  int32_t *count;          // (G, rounds, NB)
};

int lsh_buckets(const bsa_lsh_args *a) {
  return a->hash_kind == BSA_HASH_SIGN ? (1 << a->n_planes) : a->n_planes;
}

size_t lsh_layout(const bsa_lsh_args *a, char *base, LshWs *w) {
  const size_t G = a->G, n = a->nblk, R = a->n_rounds, NB = lsh_buckets(a), cap = a->cap;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char *p = base ? base + off : nullptr;
    off += (bytes + 255) & ~size_t(255);
    return p;
  };
  char *an = take(G * n * a->dim * 4), *bn = take(G * n * a->dim * 4);
  char *qc = take(G * n * R * 4), *kc = take(G * n * R * 4);
  char *li = take(G * R * NB * cap * 4), *ct = take(G * R * NB * 4);
  if (w) {
    w->an = reinterpret_cast<float *>(an);
    w->bn = reinterpret_cast<float *>(bn);
    w->qcode = reinterpret_cast<int32_t *>(qc);
    w->kcode = reinterpret_cast<int32_t *>(kc);
    w->list = reinterpret_cast<int32_t *>(li);
    w->count = reinterpret_cast<int32_t *>(ct);
  }
  return off;
}
}  // namespace

// rows [0, G*nblk) are query summaries, [G*nblk, 2*G*nblk) key summaries
__global__ void lsh_hash_kernel(const bsa_lsh_args a, LshWs w) {
  const long long rows = (long long)a.G * a.nblk;
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= 2 * rows) return;
  const bool isk = t >= rows;
  const long long row = isk ? t - rows : t;
  const float *x = (isk ? a.b : a.a) + row * a.dim;
  float *y = (isk ? w.bn : w.an) + row * a.dim;
  float ss = 0.f;
  for (int d = 0; d < a.dim; ++d) ss = fmaf(x[d], x[d], ss);
  const float nrm = fmaxf(sqrtf(ss), 1e-12f);
  for (int d = 0; d < a.dim; ++d) y[d] = x[d] / nrm;
  int32_t *code = (isk ? w.kcode : w.qcode) + row * a.n_rounds;
  for (int r = 0; r < a.n_rounds; ++r) {
    int best = 0, bits = 0;
    float bv = 0.f;
    for (int c = 0; c < a.n_planes; ++c) {
      const float *pl = a.planes + (long long)r * a.n_planes + c;  // planes[d][r][c]
      const long long pstride = (long long)a.n_rounds * a.n_planes;
      float v = 0.f;
      for (int d = 0; d < a.dim; ++d) v = fmaf(y[d], pl[d * pstride], v);
      if (c == 0 || v > bv) {  // first maximum, as torch.argmax
        best = c;
        bv = v;
      }
      if (v > 0.f) bits |= 1 << c;
    }
    code[r] = a.hash_kind == BSA_HASH_SIGN ? bits : best;
  }
}

__global__ void lsh_bucket_kernel(const bsa_lsh_args a, LshWs w, int NB) {
  const int lane = threadIdx.x & 31;
  const long long gr = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gr >= (long long)a.G * a.n_rounds) return;
  const int g = (int)(gr / a.n_rounds), r = (int)(gr % a.n_rounds);
  __shared__ int cnt_sh[8][kLshMaxBuckets];
  int *cnt = cnt_sh[threadIdx.x >> 5];
  for (int c = lane; c < NB; c += 32) cnt[c] = 0;
  __syncwarp();
  int32_t *list = w.list + gr * NB * a.cap;
  for (int base = 0; base < a.nblk; base += 32) {
    const int j = base + lane;
    const bool live = j < a.nblk;
    const int code = live ? w.kcode[((long long)g * a.nblk + j) * a.n_rounds + r] : -1;
    const unsigned act = __ballot_sync(0xffffffffu, live);
    const unsigned peers = __match_any_sync(0xffffffffu, code);
    if (live) {
      const int rank = __popc(peers & act & ((1u << lane) - 1u));
      const int pos = cnt[code] + rank;
      if (pos < a.cap) list[(long long)code * a.cap + pos] = j;
    }
    __syncwarp();
    if (live && lane == __ffs(peers & act) - 1) cnt[code] += __popc(peers & act);
    __syncwarp();
  }
  for (int c = lane; c < NB; c += 32) w.count[gr * NB + c] = min(cnt[c], a.cap);
}

__device__ __forceinline__ bool lsh_better(float s1, int i1, float s2, int i2) {
  return s1 > s2 || (s1 == s2 && i1 < i2);
}

__global__ void __launch_bounds__(256) lsh_select_kernel(const bsa_lsh_args a, LshWs w, int NB,
                                                          int rk, int W) {
  constexpr int PER = kLshMaxCand / 32;
  const int lane = threadIdx.x & 31;
  const long long gi = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gi >= (long long)a.G * a.nblk) return;
  const int g = (int)(gi / a.nblk), i = (int)(gi % a.nblk);
  __shared__ float yq_sh[8][kLshMaxDim];
  float *yq = yq_sh[threadIdx.x >> 5];
  for (int d = lane; d < a.dim; d += 32) yq[d] = w.an[gi * a.dim + d];
  __syncwarp();
  const int P = a.n_rounds * a.cap;
  float sc[PER];
  int id[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int p = lane + 32 * k;
    sc[k] = -INFINITY;
    id[k] = -1;
    if (p < P) {
      const int r = p / a.cap, pos = p % a.cap;
      const int qb = w.qcode[gi * a.n_rounds + r];
      const long long lb = ((long long)g * a.n_rounds + r) * NB + qb;
      const int j = pos < w.count[lb] ? w.list[lb * a.cap + pos] : -1;
      // the reference dedups ids clamped at 0: an empty slot (-1) of an earlier
      // round removes block 0 (src/ssa_model.py:452-457)
      bool drop0 = false;
      if (j == 0)
        for (int r2 = 0; r2 < r && !drop0; ++r2) {
          const long long lb2 = ((long long)g * a.n_rounds + r2) * NB + w.qcode[gi * a.n_rounds + r2];
          drop0 = w.count[lb2] < a.cap;
        }
      if (j >= 0 && j != i && (!a.causal || j < i) && !drop0) {
        const float *yk = w.bn + ((long long)g * a.nblk + j) * a.dim;
        float s = 0.f;
        for (int d = 0; d < a.dim; ++d) s = fmaf(yq[d], yk[d], s);
        sc[k] = s * a.scale;
        id[k] = j;
      }
    }
  }
  float own = 0.f;
  if (lane == 0) {
    const float *yk = w.bn + gi * a.dim;
    float s = 0.f;
    for (int d = 0; d < a.dim; ++d) s = fmaf(yq[d], yk[d], s);
    own = s * a.scale;
  }
  const long long ob = gi * W;
  if (lane == 0) {
    a.sel[ob] = i;
    if (a.score_out) a.score_out[ob] = own;
    if (a.gate_out) a.gate_out[ob] = lsh_logsigmoid(own);
  }
  for (int t = 0; t < rk; ++t) {
    float bs = -INFINITY;
    int bi = -1;
#pragma unroll
    for (int k = 0; k < PER; ++k)
      if (id[k] >= 0 && (bi < 0 || lsh_better(sc[k], id[k], bs, bi))) bs = sc[k], bi = id[k];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || lsh_better(os, oi, bs, bi))) bs = os, bi = oi;
    }
    if (lane == 0) {
      const bool ok = bi >= 0;
      a.sel[ob + 1 + t] = ok ? bi : i;
      if (a.score_out) a.score_out[ob + 1 + t] = ok ? bs : 0.f;
      if (a.gate_out) a.gate_out[ob + 1 + t] = lsh_logsigmoid(ok ? bs : 0.f);
    }
#pragma unroll
    for (int k = 0; k < PER; ++k)
      if (id[k] == bi) id[k] = -1;  // retire the winner and its duplicates
  }
}

int32_t lsh_width(const bsa_lsh_args *a) {
  const int T = std::min(a->topk, std::max(1, a->nblk - 1));
  return 1 + std::min(T, a->n_rounds * a->cap);
}

static bsa_status lsh_check(const bsa_lsh_args *a) {
  if (a->G <= 0 || a->nblk <= 0 || a->dim <= 0 || a->dim > kLshMaxDim)
    return fail(BSA_ERR_SHAPE, "select_lsh: need G, nblk > 0 and dim in [1, 256]");
  if (a->hash_kind != BSA_HASH_ARGMAX && a->hash_kind != BSA_HASH_SIGN)
    return fail(BSA_ERR_ARG, "select_lsh: bad hash_kind");
  if (a->n_rounds <= 0 || a->n_planes <= 0 || a->cap <= 0)
    return fail(BSA_ERR_SHAPE, "select_lsh: n_rounds, n_planes and cap must be positive");
  if (a->hash_kind == BSA_HASH_SIGN ? a->n_planes > 6 : a->n_planes > kLshMaxBuckets)
    return fail(BSA_ERR_UNSUPPORTED, "select_lsh: at most 64 buckets");
  if (a->n_rounds * a->cap > kLshMaxCand)
    return fail(BSA_ERR_UNSUPPORTED, "select_lsh: n_rounds * cap must be <= 256");
  if (a->topk < 0 || a->topk > 64) return fail(BSA_ERR_UNSUPPORTED, "select_lsh: topk must be in [0, 64]");
  return BSA_OK;
}

size_t lsh_workspace(const bsa_lsh_args *a) {
  if (lsh_check(a) != BSA_OK) return 0;
  return lsh_layout(a, nullptr, nullptr);
}

bsa_status run_lsh(const bsa_lsh_args *a, void *ws, size_t ws_bytes, cudaStream_t st) {
  if (bsa_status s = lsh_check(a)) return s;
  if (!a->a || !a->b || !a->planes || !a->sel) return fail(BSA_ERR_ARG, "select_lsh: NULL input/output");
  const size_t need = lsh_layout(a, nullptr, nullptr);
  if (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255))
    return fail(BSA_ERR_ARG, "select_lsh: workspace too small or not 256-byte aligned");
  LshWs w;
  lsh_layout(a, static_cast<char *>(ws), &w);
  const int NB = lsh_buckets(a);
  const long long rows2 = 2LL * a->G * a->nblk;
  lsh_hash_kernel<<<(unsigned)((rows2 + 127) / 128), 128, 0, st>>>(*a, w);
  if (bsa_status s = check_launch("lsh_hash")) return s;
  const long long gr = (long long)a->G * a->n_rounds;
  lsh_bucket_kernel<<<(unsigned)((gr + 7) / 8), 256, 0, st>>>(*a, w, NB);
  if (bsa_status s = check_launch("lsh_bucket")) return s;
  const int W = lsh_width(a);
  const long long nq = (long long)a->G * a->nblk;
  lsh_select_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, st>>>(*a, w, NB, W - 1, W);
  return check_launch("lsh_select");
}

}  // namespace bsa
