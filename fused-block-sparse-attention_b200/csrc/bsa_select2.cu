// The remaining selectors of the reference's Qwen evaluation, on device
// (src/qwen_blocksparse.py:124-299), all ending in _finish (:87-99):
//
//   scores_topk_kernel  top-k of a caller-supplied score matrix (SelectOracle's
//                       per-block attention mass, SelectRandom's uniform draws):
//                       one warp per row, k rounds of a warp arg-max restricted
//                       to entries ranked after the previous pick, so nothing
//                       needs marking; then _finish (non-finite -> own, + own
//                       (+ sink), ascending).
//   qmax_kernel         per-token Quest bound, max over the query block's tokens
//                       (SelectMaxQMax :221-247, and the re-score of
//                       SelectTwoStage :270-299 over its stage-1 candidates):
//                       CTA per (group, query block); 32 query tokens at a time
//                       in shared memory, one warp per candidate with one token
//                       per lane, running maxima per candidate in shared memory;
//                       then the same top-k + _finish.
// Ranking: higher score first, ties to the lower block id (torch.topk leaves
// the tie order open); every score is one fp32 fma chain over d from 0.
#include <algorithm>

#include "bsa_common.cuh"
#include "bsa_host.h"

namespace bsa {

namespace {
constexpr int kS2MaxT = 64;

__device__ __forceinline__ bool s2_better(float s1, int i1, float s2, int i2) {
  return s1 > s2 || (s1 == s2 && i1 < i2);
}

// Warp-cooperative top-T of (score, id) pairs produced by get(m) for m < n,
// written as rank-ordered ids (-1 when fewer finite entries) into out[0..T).
template <typename Get>
__device__ void warp_topk(int n, int T, Get get, int *out) {
  const int lane = threadIdx.x & 31;
  float ps = INFINITY;  // previous pick: everything must rank after it
  int pi = -1;
  for (int t = 0; t < T; ++t) {
    float bs = -INFINITY;
    int bi = -1;
    for (int m = lane; m < n; m += 32) {
      float s;
      int id;
      get(m, s, id);
      if (id < 0 || !(s > -INFINITY)) continue;
      if (pi >= 0 && !s2_better(ps, pi, s, id)) continue;  // already picked (or better)
      if (bi < 0 || s2_better(s, id, bs, bi)) bs = s, bi = id;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || s2_better(os, oi, bs, bi))) bs = os, bi = oi;
    }
    if (lane == 0) out[t] = bi;
    if (bi < 0) {  // nothing left: the rest stays -1
      for (int u = t + 1 + lane; u < T; u += 32) out[u] = -1;
      break;
    }
    ps = bs;
    pi = bi;
  }
  __syncwarp();
}

// _finish: picks (missing -> own), own, optional sink 0, ascending.
__device__ void finish_row(const int *picks, int T, int own, int sink, int *scratch, int32_t *dst) {
  const int lane = threadIdx.x & 31;
  const int W = T + 1 + (sink ? 1 : 0);
  for (int l = lane; l < T; l += 32) scratch[l] = picks[l] >= 0 ? picks[l] : own;
  if (lane == 0) {
    scratch[T] = own;
    if (sink) scratch[T + 1] = 0;
  }
  __syncwarp();
  for (int l = lane; l < W; l += 32) {
    const int v = scratch[l];
    int rank = 0;
    for (int m = 0; m < W; ++m) {
      const int u = scratch[m];
      rank += (u < v) || (u == v && m < l);
    }
    dst[rank] = v;
  }
  __syncwarp();
}
}  // namespace

__global__ void __launch_bounds__(256) scores_topk_kernel(const bsa_scores_args a, int T, int W) {
  __shared__ int s_pick[8][kS2MaxT];
  __shared__ int s_scr[8][kS2MaxT + 2];
  const int warp = threadIdx.x >> 5;
  const long long row = blockIdx.x * 8LL + warp;
  if (row >= (long long)a.G * a.nblk) return;
  const int g = (int)(row / a.nblk), i = (int)(row % a.nblk);
  const float *sr = a.score + g * a.score_sg + (long long)i * a.score_si;
  auto get = [&](int m, float &s, int &id) {
    s = sr[m];
    id = m;
    if (s != s) s = -INFINITY;  // NaN ranks last and is not finite
  };
  warp_topk(i + 1, T, get, s_pick[warp]);  // causal: j <= i
  finish_row(s_pick[warp], T, i, a.sink, s_scr[warp], a.sel + row * W);
}

__global__ void __launch_bounds__(256) qmax_kernel(const bsa_qmax_args a, int T, int W) {
  extern __shared__ float qsm[];
  const int dim = a.dim, bsr = a.bs;
  const int g = blockIdx.y, i = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NC = a.cand ? a.M : i + 1;
  float *sq = qsm;                   // [32][dim] query tokens of this pass
  float *best = sq + 32 * dim;       // [NC] running max per candidate
  int *cid = reinterpret_cast<int *>(best + NC);  // [NC] candidate block ids (-1 invalid)
  __shared__ int s_pick[kS2MaxT];
  __shared__ int s_scr[kS2MaxT + 2];
  for (int m = tid; m < NC; m += 256) {
    int j = m;
    if (a.cand) {
      j = a.cand[((long long)g * a.nblk + i) * a.M + m];
      if (j > i || j >= a.nblk) j = -1;  // future or out of range: not a candidate
    }
    cid[m] = j;
    best[m] = -INFINITY;
  }
  const float *qrow = a.qtok + ((long long)g * a.nblk + i) * bsr * dim;
  const float *kmax = a.kmax + (long long)g * a.nblk * dim;
  const float *kmin = a.kmin + (long long)g * a.nblk * dim;
  for (int t0 = 0; t0 < bsr; t0 += 32) {
    const int nt = min(32, bsr - t0);
    __syncthreads();
    for (int e = tid; e < nt * dim; e += 256) sq[e] = qrow[(long long)t0 * dim + e];
    __syncthreads();
    for (int m = warp; m < NC; m += 8) {
      const int j = cid[m];
      if (j < 0) continue;
      const float *kx = kmax + (long long)j * dim, *kn = kmin + (long long)j * dim;
      float s = -INFINITY;
      if (lane < nt) {
        const float *q = sq + lane * dim;
        s = 0.f;
        for (int d = 0; d < dim; ++d) s = fmaf(q[d], q[d] >= 0.f ? kx[d] : kn[d], s);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, o));
      if (lane == 0) best[m] = fmaxf(best[m], s);
    }
  }
  __syncthreads();
  if (warp == 0) {
    auto get = [&](int m, float &s, int &id) {
      id = cid[m];
      s = best[m];
    };
    warp_topk(NC, T, get, s_pick);
    finish_row(s_pick, T, i, a.sink, s_scr, a.sel + ((long long)g * a.nblk + i) * W);
  }
}

int32_t scores_width(int nblk, int topk, int sink) {
  return std::max(0, std::min(topk, nblk)) + 1 + (sink ? 1 : 0);
}

bsa_status run_scores_topk(const bsa_scores_args *a, cudaStream_t st) {
  if (!a->score || !a->sel) return fail(BSA_ERR_ARG, "select_scores: NULL input/output");
  if (a->G <= 0 || a->nblk <= 0) return fail(BSA_ERR_SHAPE, "select_scores: sizes must be positive");
  if (a->topk < 0 || a->topk > kS2MaxT) return fail(BSA_ERR_UNSUPPORTED, "select_scores: topk must be in [0, 64]");
  const int T = std::min(a->topk, a->nblk), W = scores_width(a->nblk, a->topk, a->sink);
  const long long rows = (long long)a->G * a->nblk;
  scores_topk_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(*a, T, W);
  return check_launch("select_scores");
}

bsa_status run_qmax(const bsa_qmax_args *a, cudaStream_t st) {
  if (!a->qtok || !a->kmax || !a->kmin || !a->sel) return fail(BSA_ERR_ARG, "select_qmax: NULL input/output");
  if (a->G <= 0 || a->nblk <= 0 || a->bs <= 0 || a->dim <= 0 || a->dim > 512)
    return fail(BSA_ERR_SHAPE, "select_qmax: sizes must be positive (dim <= 512)");
  if (a->topk < 0 || a->topk > kS2MaxT) return fail(BSA_ERR_UNSUPPORTED, "select_qmax: topk must be in [0, 64]");
  if (a->cand && (a->M <= 0 || a->M > 4096)) return fail(BSA_ERR_SHAPE, "select_qmax: M must be in [1, 4096]");
  if (a->G > 65535) return fail(BSA_ERR_SHAPE, "select_qmax: G > 65535");
  const int NC = a->cand ? a->M : a->nblk;
  const size_t smem = (size_t)32 * a->dim * 4 + (size_t)NC * 8;
  if (smem > 200 * 1024) return fail(BSA_ERR_UNSUPPORTED, "select_qmax: too many candidates");
  const int T = std::min(a->topk, a->nblk), W = scores_width(a->nblk, a->topk, a->sink);
  cudaFuncSetAttribute(qmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  qmax_kernel<<<dim3(a->nblk, a->G), 256, smem, st>>>(*a, T, W);
  return check_launch("select_qmax");
}

}  // namespace bsa
