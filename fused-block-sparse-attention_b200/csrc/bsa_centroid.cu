// CentroidSSA's bucket routing on device (reference src/ssa_model.py:263-299):
// key block j sits in the bucket of its centroid key_cent[b, j]; each bucket
// keeps its first `cap` blocks by index; query block i reads the buckets of its
// top-cpq centroids top_c[b, i, :] (cpq-major, cap-minor, the reference's gather
// layout), its own block removed (-1); with refine, the rk candidates of largest
// q_blk_i . k_blk_j are kept, in descending score order (ties to the earlier
// candidate), invalid picks as -1.  No nblk x nblk tensor exists.
//
// Grid (ceil(nblk / 128), B), 128 threads.  Every CTA rebuilds the C x cap
// bucket table of its batch row in shared memory (one warp per centroid,
// ballot compaction in block order), then one thread per query block gathers
// (and optionally re-scores) its candidates.
#include <algorithm>

#include "bsa_common.cuh"
#include "bsa_host.h"

namespace bsa {

constexpr int kCrMaxTable = 8192;  // C * cap entries in shared memory
constexpr int kCrMaxCand = 128;    // cpq * cap candidates per query block

__global__ void __launch_bounds__(128) centroid_route_kernel(const bsa_centroid_args a, int m) {
  __shared__ int table[kCrMaxTable];
  const int b = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int32_t *kc = a.key_cent + (long long)b * a.nblk;
  for (int i = tid; i < a.C * a.cap; i += 128) table[i] = -1;
  __syncthreads();
  for (int c = warp; c < a.C; c += 4) {
    int n = 0;
    for (int j0 = 0; j0 < a.nblk && n < a.cap; j0 += 32) {
      const int j = j0 + lane;
      const bool hit = j < a.nblk && kc[j] == c;
      const unsigned bal = __ballot_sync(0xffffffffu, hit);
      const int r = n + __popc(bal & ((1u << lane) - 1u));
      if (hit && r < a.cap) table[c * a.cap + r] = j;
      n += __popc(bal);
    }
  }
  __syncthreads();
  const int i = blockIdx.x * 128 + tid;
  if (i >= a.nblk) return;
  const int m0 = a.cpq * a.cap;
  int cand[kCrMaxCand];
  for (int t = 0; t < a.cpq; ++t) {
    const int c = a.top_c[((long long)b * a.nblk + i) * a.cpq + t];
    for (int r = 0; r < a.cap; ++r) {
      int j = (c >= 0 && c < a.C) ? table[c * a.cap + r] : -1;
      if (j == i) j = -1;
      cand[t * a.cap + r] = j;
    }
  }
  int32_t *out = a.sel + ((long long)b * a.nblk + i) * (1 + m);
  out[0] = i;
  if (m == m0) {
    for (int x = 0; x < m0; ++x) out[1 + x] = cand[x];
    return;
  }
  // refine: exact fp32 fma chain per candidate, then the rk best by selection
  float sc[kCrMaxCand];
  const float *qb = a.q_blk + ((long long)b * a.nblk + i) * a.dim;
  for (int x = 0; x < m0; ++x) {
    float s = -INFINITY;
    if (cand[x] >= 0) {
      const float *kb = a.k_blk + ((long long)b * a.nblk + cand[x]) * a.dim;
      s = 0.f;
      for (int d = 0; d < a.dim; ++d) s = fmaf(qb[d], kb[d], s);
    }
    sc[x] = s;
  }
  for (int y = 0; y < m; ++y) {
    int best = -1;
    for (int x = 0; x < m0; ++x)
      if (cand[x] >= 0 && sc[x] > -INFINITY && (best < 0 || sc[x] > sc[best])) best = x;
    if (best >= 0) {
      out[1 + y] = cand[best];
      cand[best] = -1;
    } else {
      out[1 + y] = -1;
    }
  }
}

int32_t centroid_width(const bsa_centroid_args *a) {
  const int m0 = a->cpq * a->cap;
  return 1 + ((a->q_blk && a->rk > 0 && a->rk < m0) ? a->rk : m0);
}

bsa_status run_centroid_route(const bsa_centroid_args *a, cudaStream_t st) {
  if (!a->key_cent || !a->top_c || !a->sel) return fail(BSA_ERR_ARG, "centroid: NULL pointer");
  if (a->B <= 0 || a->nblk <= 0 || a->C <= 0 || a->cpq <= 0 || a->cap <= 0 || a->cpq > a->C)
    return fail(BSA_ERR_SHAPE, "centroid: need B, nblk, C, cap > 0 and 0 < cpq <= C");
  if ((long long)a->C * a->cap > kCrMaxTable || a->cpq * a->cap > kCrMaxCand)
    return fail(BSA_ERR_UNSUPPORTED, "centroid: C * cap <= 8192 and cpq * cap <= 128 supported");
  if (a->q_blk && (!a->k_blk || a->dim <= 0)) return fail(BSA_ERR_ARG, "centroid: refine needs k_blk, dim");
  const int m = centroid_width(a) - 1;
  dim3 grid((unsigned)((a->nblk + 127) / 128), (unsigned)a->B);
  centroid_route_kernel<<<grid, 128, 0, st>>>(*a, m);
  return check_launch("centroid_route");
}

}  // namespace bsa
