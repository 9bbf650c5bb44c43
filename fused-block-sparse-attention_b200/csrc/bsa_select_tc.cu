// Exact block selection with tensor-core scoring (DOT scores, top-k <= 16).
//
// The nblk x nblk scores are formed tile by tile on the tensor cores (tf32
// inputs, fp32 accumulation, mma.sync m16n8k8) and streamed through a per-row
// top-32 list in registers, so the score matrix never reaches memory.  The
// tf32 scores are approximations; the result is made exact by certification:
//  1. the 32 best candidates by approximate score (per half of the keys) are
//     re-scored with the exact
//     fp32 fma chain (the arithmetic of the SIMT kernel and the oracle), and the
//     top-T among them is taken by (score desc, block asc);
//  2. every candidate outside the list has an approximate score <= the list's
//     last one, and each approximate score is within E = delta * |a| * max|b| of
//     the exact one (tf32 rounding of both operands, 2^-11 each, plus fp32
//     accumulation: delta = 2^-9 covers both with a factor two to spare, for
//     dim <= 128); so if (last approximate score) + E < (T-th exact pick), no
//     outside candidate can enter the top-T and the row is exact;
//  3. rows that fail the test (near-ties at the list boundary; rare) are
//     recorded and re-selected by an exact warp-per-row scan.
// The result is bitwise the SIMT kernel's.
//
//   select_tc_kernel<DIM>  CTA per (group, 64 query rows); warp w scores rows
//                          16*(w&3).. against key half w>>2 of each 64-block key
//                          tile (each half keeps its own top-32 lists, merged by
//                          the exact re-score); causal tiles skipped; heaviest
//                          CTAs first.
//   select_fallback_kernel one warp per failed row.
#include <climits>

#include "bsa_common.cuh"
#include "bsa_host.h"

namespace bsa {

namespace {
constexpr int kTcRows = 64, kTcKeys = 64, kTcList = 32;
constexpr float kTcDelta = 1.0f / 512.0f;

__device__ __forceinline__ bool tc_better(float s1, int i1, float s2, int i2) {
  return s1 > s2 || (s1 == s2 && i1 < i2);
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float *c, const uint32_t *a, const uint32_t *b) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Streaming insertion of one candidate per lane into the warp's sorted list
// (lane l holds entry l, length TL <= 32), as in the SIMT selection kernel.
__device__ __forceinline__ void list_insert(float &es, int &ei, int TL, float cs, int ci) {
  const int lane = threadIdx.x & 31;
  float thr_s = __shfl_sync(0xffffffffu, es, TL - 1);
  int thr_i = __shfl_sync(0xffffffffu, ei, TL - 1);
  unsigned mask = __ballot_sync(0xffffffffu, cs > -INFINITY && tc_better(cs, ci, thr_s, thr_i));
  while (mask) {
    const int src = __ffs(mask) - 1;
    mask &= mask - 1;
    const float vs = __shfl_sync(0xffffffffu, cs, src);
    const int vi = __shfl_sync(0xffffffffu, ci, src);
    if (!tc_better(vs, vi, thr_s, thr_i)) continue;
    const int pos = __popc(__ballot_sync(0xffffffffu, lane < TL && tc_better(es, ei, vs, vi)));
    const float us = __shfl_up_sync(0xffffffffu, es, 1);
    const int ui = __shfl_up_sync(0xffffffffu, ei, 1);
    if (lane == pos) {
      es = vs;
      ei = vi;
    } else if (lane > pos && lane < TL) {
      es = us;
      ei = ui;
    }
    thr_s = __shfl_sync(0xffffffffu, es, TL - 1);
    thr_i = __shfl_sync(0xffffffffu, ei, TL - 1);
  }
}

__device__ __forceinline__ float dot_exact(const float *a, const float *b, int dim) {
  float s = 0.f;
  for (int d = 0; d < dim; ++d) s = fmaf(a[d], b[d], s);
  return s;
}

__device__ __forceinline__ float tc_logsigmoid(float x) {
  return x < 0.f ? x - log1pf(expf(x)) : -log1pf(expf(-x));
}

__device__ __forceinline__ bool cand_ok(const bsa_select_args &a, int j, int qi) {
  if (j < 0 || j >= a.nblk) return false;
  if (a.layout == BSA_SEL_SSA) return j != qi && (!a.causal || j < qi);
  return j <= qi;
}

// Writes one row from the final picks (lane l < T holds pick l: id or -1, exact score).
__device__ void tc_write_row(const bsa_select_args &a, int T, int W, long long ob, int row,
                             const float *arow, const float *Bg, int pick, float psc, int *scratch) {
  const int lane = threadIdx.x & 31;
  const bool valid = lane < T && pick >= 0;
  if (a.layout == BSA_SEL_SSA) {
    float own = 0.f;
    if (a.score_out || a.gate_out) own = dot_exact(arow, Bg + (long long)row * a.dim, a.dim);
    if (lane == 0) {
      a.sel[ob] = row;
      if (a.score_out) a.score_out[ob] = own;
      if (a.gate_out) a.gate_out[ob] = tc_logsigmoid(own);
    }
    if (lane < T) {
      a.sel[ob + 1 + lane] = valid ? pick : row;
      const float sc = valid ? psc : own;
      if (a.score_out) a.score_out[ob + 1 + lane] = sc;
      if (a.gate_out) a.gate_out[ob + 1 + lane] = tc_logsigmoid(sc);
    }
  } else if (a.layout == BSA_SEL_RAW) {
    if (lane < T) a.sel[ob + lane] = valid ? pick : -1;
  } else {
    if (lane < T) scratch[lane] = valid ? pick : row;
    if (lane == 0) {
      scratch[T] = row;
      if (a.sink) scratch[T + 1] = 0;
    }
    __syncwarp();
    for (int l = lane; l < W; l += 32) {
      const int v = scratch[l];
      int rank = 0;
      for (int m = 0; m < W; ++m) {
        const int u = scratch[m];
        rank += (u < v) || (u == v && m < l);
      }
      a.sel[ob + rank] = v;
    }
    __syncwarp();
  }
}

}  // namespace

__global__ void bnorm_max_kernel(const bsa_select_args a, unsigned *bmax) {
  const long long n = (long long)a.G * a.nblk;
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < n;
       r += (long long)gridDim.x * blockDim.x) {
    const float *b = a.b1 + r * a.dim;
    float s = 0.f;
    for (int d = 0; d < a.dim; ++d) s = fmaf(b[d], b[d], s);
    const float nb = sqrtf(s) * 1.0001f;
    atomicMax(bmax + r / a.nblk, __float_as_uint(nb));  // non-negative floats order as uints
  }
}

template <int DIM>
__global__ void __launch_bounds__(256) select_tc_kernel(const bsa_select_args a, int T, int W,
                                                        const unsigned *bmax, int *fail_rows,
                                                        int *fail_count, int max_fail) {
  constexpr int LD = DIM + 4;
  extern __shared__ float tsm[];
  float *As = tsm;                      // [64][LD] query summaries
  float *Bs = As + kTcRows * LD;        // [64][LD] key summaries of the tile
  float *Ss = Bs + kTcKeys * LD;        // per warp [16][33] masked scores
  float *Ls = Ss + 8 * 16 * 33;         // [64 rows][2 halves][32] list scores
  int *Li = reinterpret_cast<int *>(Ls + kTcRows * 2 * kTcList);  // list ids
  __shared__ int scratch_all[8][kTcList + 2];
  const int nq = a.nq > 0 ? a.nq : a.nblk, qb0 = a.q_blk0;
  const int ntiles = (nq + kTcRows - 1) / kTcRows;
  const int qt = ntiles - 1 - (int)blockIdx.x;  // heaviest causal tiles first
  const int g = blockIdx.y;
  const int q0 = qt * kTcRows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rg = warp & 3, kh = warp >> 2;  // 16-row group, 32-key half of each tile
  const bool causal_like = a.layout != BSA_SEL_SSA || a.causal;
  const float *A = a.a + (long long)g * nq * DIM;
  const float *Bg = a.b1 + (long long)g * a.nblk * DIM;
  float *Sw = Ss + warp * 16 * 33;

  for (int i = tid; i < kTcRows * DIM; i += 256) {
    const int r = i / DIM, d = i % DIM;
    As[r * LD + d] = q0 + r < nq ? A[(long long)(q0 + r) * DIM + d] : 0.f;
  }
  float es[16];
  int ei[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) es[r] = -INFINITY, ei[r] = INT_MAX;

  const int nkt = (a.nblk + kTcKeys - 1) / kTcKeys;
  const int kt_last = causal_like ? min(nkt - 1, (qb0 + min(q0 + kTcRows, nq) - 1) / kTcKeys) : nkt - 1;
  const int ra = rg * 16 + (lane >> 2);  // this lane's first accumulator row (and ra + 8)
  for (int kt = 0; kt <= kt_last; ++kt) {
    const int k0 = kt * kTcKeys;
    __syncthreads();
    for (int i = tid; i < kTcKeys * DIM / 4; i += 256) {
      const int r = i / (DIM / 4), c4 = i % (DIM / 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + r < a.nblk) v = *reinterpret_cast<const float4 *>(Bg + (long long)(k0 + r) * DIM + 4 * c4);
      *reinterpret_cast<float4 *>(Bs + r * LD + 4 * c4) = v;
    }
    __syncthreads();
    float acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
#pragma unroll
    for (int k8 = 0; k8 < DIM / 8; ++k8) {
      uint32_t af[4];
      const int c = k8 * 8 + (lane & 3);
      af[0] = to_tf32(As[ra * LD + c]);
      af[1] = to_tf32(As[(ra + 8) * LD + c]);
      af[2] = to_tf32(As[ra * LD + c + 4]);
      af[3] = to_tf32(As[(ra + 8) * LD + c + 4]);
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        uint32_t bf[2];
        const int kr = kh * 32 + n * 8 + (lane >> 2);
        bf[0] = to_tf32(Bs[kr * LD + c]);
        bf[1] = to_tf32(Bs[kr * LD + c + 4]);
        mma_tf32(acc[n], af, bf);
      }
    }
    // masked scores of this warp's 16 rows x 32 keys -> shared memory
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rl = (lane >> 2) + (e >= 2 ? 8 : 0);
        const int col = n * 8 + 2 * (lane & 3) + (e & 1);
        const int lrow = q0 + rg * 16 + rl, qi = qb0 + lrow, j = k0 + kh * 32 + col;
        Sw[rl * 33 + col] = (lrow < nq && cand_ok(a, j, qi)) ? acc[n][e] : -INFINITY;
      }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < 16; ++r) list_insert(es[r], ei[r], kTcList, Sw[r * 33 + lane], k0 + kh * 32 + lane);
    __syncwarp();
  }
  // both key halves' lists of every row -> shared memory
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    const int row = rg * 16 + r;
    Ls[(row * 2 + kh) * kTcList + lane] = es[r];
    Li[(row * 2 + kh) * kTcList + lane] = ei[r] == INT_MAX ? -1 : ei[r];
  }
  __syncthreads();

  // ---- per row (warp w: rows w, w + 8, ...): exact re-score of the 64 listed
  // candidates, exact top-T, certification, output
  const float bm = __uint_as_float(bmax[g]);
  int *scratch = scratch_all[warp];
  for (int rr = warp; rr < kTcRows; rr += 8) {
    const int lrow = q0 + rr;
    if (lrow >= nq) break;
    const int row = qb0 + lrow;
    const float *arow = A + (long long)lrow * DIM;
    const int id0 = Li[(rr * 2) * kTcList + lane], id1 = Li[(rr * 2 + 1) * kTcList + lane];
    const float x0 = id0 >= 0 ? dot_exact(arow, Bg + (long long)id0 * DIM, DIM) : -INFINITY;
    const float x1 = id1 >= 0 ? dot_exact(arow, Bg + (long long)id1 * DIM, DIM) : -INFINITY;
    int pick = -1;
    float psc = -INFINITY, ps = INFINITY;
    int pi = -1;
    for (int t = 0; t < T; ++t) {
      float bs = -INFINITY;
      int bi = -1;
      if (id0 >= 0 && (pi < 0 || tc_better(ps, pi, x0, id0))) bs = x0, bi = id0;
      if (id1 >= 0 && (pi < 0 || tc_better(ps, pi, x1, id1)) && (bi < 0 || tc_better(x1, id1, bs, bi)))
        bs = x1, bi = id1;
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float os = __shfl_xor_sync(0xffffffffu, bs, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || tc_better(os, oi, bs, bi))) bs = os, bi = oi;
      }
      if (lane == t) pick = bi, psc = bs;
      if (bi < 0) break;
      ps = bs;
      pi = bi;
    }
    // certification: a half whose list is full must end below the T-th exact pick by E
    bool ok = true;
    const bool full0 = __shfl_sync(0xffffffffu, id0, kTcList - 1) >= 0;
    const bool full1 = __shfl_sync(0xffffffffu, id1, kTcList - 1) >= 0;
    if ((full0 || full1) && T > 0) {
      float an = 0.f;
      for (int d = lane; d < DIM; d += 32) an = fmaf(arow[d], arow[d], an);
#pragma unroll
      for (int o = 16; o; o >>= 1) an += __shfl_xor_sync(0xffffffffu, an, o);
      const float E = kTcDelta * sqrtf(an) * 1.0001f * bm;
      const float tth = __shfl_sync(0xffffffffu, psc, T - 1);
      const int tthi = __shfl_sync(0xffffffffu, pick, T - 1);
      const float last0 = Ls[(rr * 2) * kTcList + kTcList - 1];
      const float last1 = Ls[(rr * 2 + 1) * kTcList + kTcList - 1];
      ok = tthi >= 0 && (!full0 || last0 + E < tth) && (!full1 || last1 + E < tth);
    }
    if (!ok && lane == 0) {
      const int f = atomicAdd(fail_count, 1);
      if (f < max_fail) fail_rows[f] = g * nq + lrow;
    }
    const long long ob = ((long long)g * nq + lrow) * W;
    tc_write_row(a, T, W, ob, row, arow, Bg, pick, psc, scratch);
  }
}

// Exact warp-per-row re-selection of the rows the certification rejected.
__global__ void select_fallback_kernel(const bsa_select_args a, int T, int W, const int *fail_rows,
                                       const int *fail_count, int max_fail) {
  __shared__ int scratch_all[8][kTcList + 2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = a.nq > 0 ? a.nq : a.nblk;
  const int nf = min(*fail_count, max_fail);
  const int TL = T > 0 ? T : 1;
  for (int f = blockIdx.x * 8 + warp; f < nf; f += gridDim.x * 8) {
    const int gr = fail_rows[f];
    const int g = gr / nq, lrow = gr % nq, row = a.q_blk0 + lrow;
    const float *arow = a.a + (long long)gr * a.dim;
    const float *Bg = a.b1 + (long long)g * a.nblk * a.dim;
    float es = -INFINITY;
    int ei = INT_MAX;
    const int jend = (a.layout != BSA_SEL_SSA || a.causal) ? min(a.nblk, row + 1) : a.nblk;
    for (int j0 = 0; j0 < jend; j0 += 32) {
      const int j = j0 + lane;
      float s = -INFINITY;
      if (j < jend && cand_ok(a, j, row)) s = dot_exact(arow, Bg + (long long)j * a.dim, a.dim);
      list_insert(es, ei, TL, s, j);
    }
    const int pick = (lane < T && ei != INT_MAX) ? ei : -1;
    tc_write_row(a, T, W, ((long long)g * nq + lrow) * W, row, arow, Bg, pick, es,
                 scratch_all[warp]);
  }
}

// Opt-in (BSA_SELECT_TC=1): exact, but measured slower than the fp32 SIMT kernel
// on this part (262k: 1.9 ms against 0.88 ms), so the SIMT kernel stays the default.
bool select_tc_applicable(const bsa_select_args *a, int T) {
  const char *on = getenv("BSA_SELECT_TC");
  return on && on[0] == '1' && a->score_kind == BSA_SCORE_DOT && T >= 1 && T <= 16 &&
         (a->dim == 64 || a->dim == 128);
}

// Scratch: bmax (G floats) + fail count + fail rows (one per query row).
size_t select_tc_workspace(const bsa_select_args *a) {
  const int nq = a->nq > 0 ? a->nq : a->nblk;
  return align_up((size_t)a->G * 4, 256) + 256 + align_up((size_t)a->G * nq * 4, 256);
}

bsa_status run_select_tc(const bsa_select_args *a, int T, int W, void *ws, cudaStream_t st) {
  const int nq = a->nq > 0 ? a->nq : a->nblk;
  uint8_t *base = static_cast<uint8_t *>(ws);
  unsigned *bmax = reinterpret_cast<unsigned *>(base);
  int *fcount = reinterpret_cast<int *>(base + align_up((size_t)a->G * 4, 256));
  int *frows = reinterpret_cast<int *>(base + align_up((size_t)a->G * 4, 256) + 256);
  const int max_fail = a->G * nq;
  cudaMemsetAsync(base, 0, align_up((size_t)a->G * 4, 256) + 256, st);
  const long long nb = (long long)a->G * a->nblk;
  bnorm_max_kernel<<<(unsigned)std::min<long long>((nb + 255) / 256, 148LL * 8), 256, 0, st>>>(*a, bmax);
  if (bsa_status s = check_launch("select_bnorm")) return s;
  dim3 grid((nq + kTcRows - 1) / kTcRows, a->G);
  const int LD = a->dim + 4;
  const size_t smem = ((size_t)kTcRows * LD + (size_t)kTcKeys * LD + 8 * 16 * 33 +
                       (size_t)kTcRows * 2 * kTcList * 2) * 4;
  if (a->dim == 64) {
    cudaFuncSetAttribute(select_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    select_tc_kernel<64><<<grid, 256, smem, st>>>(*a, T, W, bmax, frows, fcount, max_fail);
  } else {
    cudaFuncSetAttribute(select_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    select_tc_kernel<128><<<grid, 256, smem, st>>>(*a, T, W, bmax, frows, fcount, max_fail);
  }
  if (bsa_status s = check_launch("select_tc")) return s;
  select_fallback_kernel<<<148, 256, 0, st>>>(*a, T, W, frows, fcount, max_fail);
  return check_launch("select_fallback");
}

}  // namespace bsa
