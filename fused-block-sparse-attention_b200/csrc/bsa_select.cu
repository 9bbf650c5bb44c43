// Block-pair selection for sm_100a: block pooling, fused block-pair scoring
// with a streaming warp top-k (the nblk x nblk score matrix never reaches
// HBM), and the Qwen partial rotary embedding.
//
// Scores are exact fp32 fma chains in a fixed order (d = 0..dim-1) so the
// selected indices are bitwise reproducible and match the CPU oracle exactly;
// ranking is (score desc, block id asc).
#include "bsa_common.cuh"
#include "bsa_host.h"

namespace bsa {

// ------------------------------------------------------------------ pooling
template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ float tof(T x) {
  if constexpr (sizeof(T) == 4)
    return x;
  else
    return Mma<T>::to_f(x);
}

template <typename T>
__global__ void pool_kernel(const bsa_pool_args a, int Hout) {
  constexpr int V = Vec16<T>::N;
  const int ng = a.D / V;
  const long long n = (long long)a.B * Hout * a.nblk * ng;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < n;
       t += (long long)gridDim.x * blockDim.x) {
    const int dg = (int)(t % ng);
    long long r = t / ng;
    const int blk = (int)(r % a.nblk);
    r /= a.nblk;
    const int ho = (int)(r % Hout);
    const int b = (int)(r / Hout);
    float sum[V], mn[V], mx[V];
#pragma unroll
    for (int e = 0; e < V; ++e) {
      sum[e] = 0.f;
      mn[e] = INFINITY;
      mx[e] = -INFINITY;
    }
    const T *x = reinterpret_cast<const T *>(a.x.ptr) + b * a.x.sb + dg * V;
    // rope-aware pooling: this column group's rotated values need the partner
    // group half a rotation away (16-bit types; rope_rot % 16 == 0)
    const int half = a.rope_rot / 2;
    const bool rot = sizeof(T) == 2 && a.rope_cos && dg * V < a.rope_rot;
    const bool lowhalf = dg * V < half;
    const long long pofs = lowhalf ? half : -half;  // partner column offset
    // reads the 8 (or 4) values of head hh, row gr, rotated when needed
    auto load = [&](long long hh, long long gr, float *out) {
      const uint4 u = *reinterpret_cast<const uint4 *>(x + hh * a.x.sh + gr * a.x.sl);
      const T *ue = reinterpret_cast<const T *>(&u);
      if constexpr (sizeof(T) == 2) {
        if (rot) {
          const uint4 w = *reinterpret_cast<const uint4 *>(x + hh * a.x.sh + gr * a.x.sl + pofs);
          const T *we = reinterpret_cast<const T *>(&w);
          const T *cs = reinterpret_cast<const T *>(a.rope_cos) + b * a.rope_sb + gr * a.rope_sl;
          const T *sn = reinterpret_cast<const T *>(a.rope_sin) + b * a.rope_sb + gr * a.rope_sl;
          const int c0 = lowhalf ? dg * V : dg * V - half;  // the pair's low index
#pragma unroll
          for (int e = 0; e < V; ++e) {
            const T lo = lowhalf ? ue[e] : we[e], hi = lowhalf ? we[e] : ue[e];
            T y0, y1;
            rope_pair<T>(lo, hi, cs[c0 + e], sn[c0 + e], cs[c0 + half + e], sn[c0 + half + e], y0,
                         y1);
            out[e] = tof(lowhalf ? y0 : y1);
          }
          return;
        }
      }
#pragma unroll
      for (int e = 0; e < V; ++e) out[e] = tof(ue[e]);
    };
    if (!rot && a.grp == 1) {
      // plain rows: eight loads in flight per thread, then the same per-row
      // accumulation order as below (rows past L count as zeros)
      const T *xr = x + ho * a.x.sh;
      for (int row0 = 0; row0 < a.bs; row0 += 8) {
        uint4 u[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const long long gr = (long long)blk * a.bs + row0 + i;
          u[i] = (row0 + i < a.bs && gr < a.L) ? *reinterpret_cast<const uint4 *>(xr + gr * a.x.sl)
                                               : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (row0 + i >= a.bs) break;
          const T *ue = reinterpret_cast<const T *>(&u[i]);
#pragma unroll
          for (int e = 0; e < V; ++e) {
            const float val = tof(ue[e]);
            sum[e] = __fadd_rn(sum[e], val);
            mn[e] = fminf(mn[e], val);
            mx[e] = fmaxf(mx[e], val);
          }
        }
      }
    } else
    for (int row = 0; row < a.bs; ++row) {
      const long long gr = (long long)blk * a.bs + row;
      float val[V];
      if (gr < a.L) {
        if (a.grp == 1) {
          load(ho, gr, val);
        } else {
#pragma unroll
          for (int e = 0; e < V; ++e) val[e] = 0.f;
          for (int gi = 0; gi < a.grp; ++gi) {
            float ve[V];
            load((long long)(ho * a.grp + gi), gr, ve);
#pragma unroll
            for (int e = 0; e < V; ++e) val[e] = __fadd_rn(val[e], ve[e]);
          }
#pragma unroll
          for (int e = 0; e < V; ++e) val[e] = __fdiv_rn(val[e], (float)a.grp);
        }
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) val[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < V; ++e) {
        sum[e] = __fadd_rn(sum[e], val[e]);
        mn[e] = fminf(mn[e], val[e]);
        mx[e] = fmaxf(mx[e], val[e]);
      }
    }
    const long long o = (((long long)b * Hout + ho) * a.nblk + blk) * a.D + dg * V;
#pragma unroll
    for (int e = 0; e < V; ++e) {
      if (a.mean) a.mean[o + e] = __fdiv_rn(sum[e], (float)a.bs);
      if (a.vmin) a.vmin[o + e] = mn[e];
      if (a.vmax) a.vmax[o + e] = mx[e];
    }
  }
}

bsa_status run_pool(const bsa_pool_args *a, cudaStream_t st) {
  if (!a->x.ptr) return fail(BSA_ERR_ARG, "pool: x is NULL");
  if (a->B <= 0 || a->H <= 0 || a->L <= 0 || a->D <= 0 || a->bs <= 0 || a->grp <= 0 ||
      a->H % a->grp || a->nblk != (a->L + a->bs - 1) / a->bs)
    return fail(BSA_ERR_SHAPE, "pool: bad shape (need H % grp == 0, nblk == ceil(L/bs))");
  if (a->grp > 1 && (a->vmin || a->vmax))
    return fail(BSA_ERR_ARG, "pool: min/max need grp == 1");
  if (a->rope_cos && (!a->rope_sin || a->dtype == BSA_F32 || a->rope_rot <= 0 ||
                      a->rope_rot % 16 || a->rope_rot > a->D))
    return fail(BSA_ERR_ARG, "pool: rope needs cos/sin, a 16-bit dtype and rot % 16 == 0, rot <= D");
  const int V = a->dtype == BSA_F32 ? 4 : 8;
  if (a->D % V) return fail(BSA_ERR_SHAPE, "pool: D must be a multiple of 16 bytes");
  const size_t es = elem_size(a->dtype);
  if (reinterpret_cast<uintptr_t>(a->x.ptr) % 16 || (a->x.sb * es) % 16 || (a->x.sh * es) % 16 ||
      (a->x.sl * es) % 16)
    return fail(BSA_ERR_STRIDE, "pool: x needs 16-byte aligned rows");
  const int Hout = a->H / a->grp;
  const long long n = (long long)a->B * Hout * a->nblk * (a->D / V);
  const int threads = 256;
  const long long blocks = std::max<long long>(1, std::min<long long>((n + threads - 1) / threads, 1LL << 20));
  if (a->dtype == BSA_BF16)
    pool_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, st>>>(*a, Hout);
  else if (a->dtype == BSA_F16)
    pool_kernel<__half><<<(unsigned)blocks, threads, 0, st>>>(*a, Hout);
  else if (a->dtype == BSA_F32)
    pool_kernel<float><<<(unsigned)blocks, threads, 0, st>>>(*a, Hout);
  else
    return fail(BSA_ERR_DTYPE, "pool: bad dtype");
  return check_launch("pool");
}

// ------------------------------------------------------------------ selection
constexpr int kTile = 64;   // query rows / key columns per tile
constexpr int kLdA = 68;    // padded row stride (floats) of the transposed tiles
constexpr int kDC = 32;     // dims per key-summary chunk

__device__ __forceinline__ bool better(float s1, int i1, float s2, int i2) {
  return s1 > s2 || (s1 == s2 && i1 < i2);
}

__device__ __forceinline__ float logsigmoid(float x) {
  return x < 0.f ? x - log1pf(expf(x)) : -log1pf(expf(-x));
}

template <int KIND>
__global__ void __launch_bounds__(256) select_kernel(const bsa_select_args a, int T, int W) {
  // T = picks written per row (may be 0); TL >= 1 is the length of the
  // register-resident sorted list (lane l holds entry l).
  const int TL = T > 0 ? T : 1;
  extern __shared__ float ssm[];
  const int dim = a.dim;
  float *As = ssm;                           // [dim][kLdA]  query summaries, transposed
  float *B1 = As + dim * kLdA;               // [kDC][kLdA]
  float *B2 = B1 + kDC * kLdA;               // [kDC][kLdA]  (MAXDOT2 / QUEST)
  float *S = B2 + kDC * kLdA;                // [64][65]
  // query rows are local (nq of them, global block = qb0 + local); keys are global
  const int nq = a.nq > 0 ? a.nq : a.nblk, qb0 = a.q_blk0;
  const int ntiles = (nq + kTile - 1) / kTile, nktiles = (a.nblk + kTile - 1) / kTile;
  const int qt = ntiles - 1 - (int)blockIdx.x;  // heaviest causal tiles first
  const int g = blockIdx.y;
  const int q0 = qt * kTile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ty = tid >> 4, tx = tid & 15;
  const bool causal_like = a.layout == BSA_SEL_FINISH || a.causal;

  const float *A = a.a + (long long)g * nq * dim;
  const float *Bg1 = a.b1 + (long long)g * a.nblk * dim;
  const float *Bg2 = a.b2 ? a.b2 + (long long)g * a.nblk * dim : nullptr;
  for (int i = tid; i < kTile * dim; i += 256) {
    const int r = i / dim, d = i % dim;
    As[d * kLdA + r] = (q0 + r < nq) ? A[(long long)(q0 + r) * dim + d] : 0.f;
  }

  float es[8];
  int ei[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    es[r] = -INFINITY;
    ei[r] = INT_MAX;
  }

  const int kt_last = causal_like ? min(nktiles - 1, (qb0 + min(q0 + kTile, nq) - 1) / kTile)
                                  : nktiles - 1;
  for (int kt = 0; kt <= kt_last; ++kt) {
    const int k0 = kt * kTile;
    float acc[4][4], acc2[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = acc2[i][j] = 0.f;
    for (int dc = 0; dc < dim; dc += kDC) {
      __syncthreads();
      for (int i = tid; i < kTile * kDC; i += 256) {
        const int c = i / kDC, dd = i % kDC;
        const bool ok = k0 + c < a.nblk && dc + dd < dim;
        B1[dd * kLdA + c] = ok ? Bg1[(long long)(k0 + c) * dim + dc + dd] : 0.f;
        if (KIND != BSA_SCORE_DOT) B2[dd * kLdA + c] = ok ? Bg2[(long long)(k0 + c) * dim + dc + dd] : 0.f;
      }
      __syncthreads();
      const int dn = min(kDC, dim - dc);
      for (int dd = 0; dd < dn; ++dd) {
        const float4 av = *reinterpret_cast<const float4 *>(As + (dc + dd) * kLdA + ty * 4);
        const float4 bv = *reinterpret_cast<const float4 *>(B1 + dd * kLdA + tx * 4);
        const float ar[4] = {av.x, av.y, av.z, av.w};
        const float br[4] = {bv.x, bv.y, bv.z, bv.w};
        if (KIND == BSA_SCORE_DOT) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
        } else {
          const float4 cv = *reinterpret_cast<const float4 *>(B2 + dd * kLdA + tx * 4);
          const float cr[4] = {cv.x, cv.y, cv.z, cv.w};
          if (KIND == BSA_SCORE_MAXDOT2) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
                acc2[i][j] = fmaf(ar[i], cr[j], acc2[i][j]);
              }
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j)
                acc[i][j] = fmaf(ar[i], ar[i] >= 0.f ? br[j] : cr[j], acc[i][j]);
          }
        }
      }
    }
    // scores -> S with validity
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = qb0 + q0 + ty * 4 + i;  // global query block
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kj = k0 + tx * 4 + j;
        bool ok = q0 + ty * 4 + i < nq && kj < a.nblk;
        if (a.layout == BSA_SEL_SSA)
          ok = ok && kj != qi && (!a.causal || kj < qi);
        else
          ok = ok && kj <= qi;
        const float sc = KIND == BSA_SCORE_MAXDOT2 ? fmaxf(acc[i][j], acc2[i][j]) : acc[i][j];
        S[(ty * 4 + i) * 65 + tx * 4 + j] = ok ? sc : -INFINITY;
      }
    }
    __syncthreads();
    // streaming top-T merge: warp w owns rows w*8 .. w*8+7
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int lr = warp * 8 + r;
      float thr_s = __shfl_sync(0xffffffffu, es[r], TL - 1);
      int thr_i = __shfl_sync(0xffffffffu, ei[r], TL - 1);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const float cs = S[lr * 65 + lane + half * 32];
        const int ci = k0 + lane + half * 32;
        unsigned mask =
            __ballot_sync(0xffffffffu, cs > -INFINITY && better(cs, ci, thr_s, thr_i));
        while (mask) {
          const int src = __ffs(mask) - 1;
          mask &= mask - 1;
          const float vs = __shfl_sync(0xffffffffu, cs, src);
          const int vi = __shfl_sync(0xffffffffu, ci, src);
          if (!better(vs, vi, thr_s, thr_i)) continue;  // uniform across the warp
          const int pos =
              __popc(__ballot_sync(0xffffffffu, lane < TL && better(es[r], ei[r], vs, vi)));
          const float us = __shfl_up_sync(0xffffffffu, es[r], 1);
          const int ui = __shfl_up_sync(0xffffffffu, ei[r], 1);
          if (lane == pos) {
            es[r] = vs;
            ei[r] = vi;
          } else if (lane > pos) {
            es[r] = us;
            ei[r] = ui;
          }
          thr_s = __shfl_sync(0xffffffffu, es[r], TL - 1);
          thr_i = __shfl_sync(0xffffffffu, ei[r], TL - 1);
        }
      }
    }
  }
  __syncthreads();

  // ---- write rows
  int *scratch = reinterpret_cast<int *>(S) + warp * 128;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int lrow = q0 + warp * 8 + r;
    if (lrow >= nq) continue;  // warp-uniform
    const int row = qb0 + lrow;  // global query block
    const long long ob = ((long long)g * nq + lrow) * W;
    const bool valid = lane < T && ei[r] != INT_MAX;
    if (a.layout == BSA_SEL_SSA) {
      float own = 0.f;
      if ((a.score_out || a.gate_out) && lane == 0) {
        // the a-row of local row `lrow` is column (lrow - q0) of As
        float s = 0.f, s2 = 0.f;
        const float *b1r = Bg1 + (long long)row * dim;
        const float *b2r = Bg2 ? Bg2 + (long long)row * dim : nullptr;
        for (int d = 0; d < dim; ++d) {
          const float av = As[d * kLdA + (lrow - q0)];
          if (KIND == BSA_SCORE_QUEST)
            s = fmaf(av, av >= 0.f ? b1r[d] : b2r[d], s);
          else
            s = fmaf(av, b1r[d], s);
          if (KIND == BSA_SCORE_MAXDOT2) s2 = fmaf(av, b2r[d], s2);
        }
        own = KIND == BSA_SCORE_MAXDOT2 ? fmaxf(s, s2) : s;
      }
      own = __shfl_sync(0xffffffffu, own, 0);
      if (lane == 0) {
        a.sel[ob] = row;
        if (a.score_out) a.score_out[ob] = own;
        if (a.gate_out) a.gate_out[ob] = logsigmoid(own);
      }
      if (lane < T) {
        a.sel[ob + 1 + lane] = valid ? ei[r] : row;
        const float sc = valid ? es[r] : own;
        if (a.score_out) a.score_out[ob + 1 + lane] = sc;
        if (a.gate_out) a.gate_out[ob + 1 + lane] = logsigmoid(sc);
      }
    } else if (a.layout == BSA_SEL_RAW) {
      // RAW: the picks in rank order, -1 where fewer than T candidates exist
      if (lane < T) a.sel[ob + lane] = valid ? ei[r] : -1;
    } else {
      // FINISH: picks (invalid -> own), own, optional sink; ascending sort
      if (lane < T) scratch[lane] = valid ? ei[r] : row;
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
}

bool select_tc5_applicable(const bsa_select_args *a, int T);
bsa_status run_select_tc5(const bsa_select_args *a, int T, int W, cudaStream_t st);

int32_t select_width(const bsa_select_args *a) {
  if (a->layout == BSA_SEL_SSA) return 1 + std::max(0, std::min(a->topk, a->nblk - 1));
  if (a->layout == BSA_SEL_RAW) return std::max(0, std::min(a->topk, a->nblk));
  return std::max(0, std::min(a->topk, a->nblk)) + 1 + (a->sink ? 1 : 0);
}

bsa_status run_select(const bsa_select_args *a, cudaStream_t st) {
  if (!a->a || !a->b1 || !a->sel) return fail(BSA_ERR_ARG, "select: NULL input/output");
  if (a->G <= 0 || a->nblk <= 0 || a->dim <= 0 || a->dim > 256 || a->dim % 4)
    return fail(BSA_ERR_SHAPE, "select: need G, nblk > 0 and dim a multiple of 4 in [4, 256]");
  if (a->topk < 0 || a->topk > 32) return fail(BSA_ERR_UNSUPPORTED, "select: topk must be in [0, 32]");
  if (a->score_kind != BSA_SCORE_DOT && !a->b2)
    return fail(BSA_ERR_ARG, "select: MAXDOT2/QUEST need b2");
  if (a->layout != BSA_SEL_SSA && a->layout != BSA_SEL_FINISH && a->layout != BSA_SEL_RAW)
    return fail(BSA_ERR_ARG, "select: bad layout");
  if (a->layout != BSA_SEL_SSA && (a->score_out || a->gate_out))
    return fail(BSA_ERR_ARG, "select: score/gate outputs are SSA-layout only");
  if ((long long)a->G > 65535) return fail(BSA_ERR_SHAPE, "select: G > 65535");
  const int W = select_width(a);
  int T = a->layout == BSA_SEL_SSA ? W - 1 : std::min(a->topk, a->nblk);
  if (a->layout == BSA_SEL_RAW && T == 0) return BSA_OK;
  const int nq = a->nq > 0 ? a->nq : a->nblk;
  if (a->q_blk0 < 0 || a->nq < 0 || (long long)a->q_blk0 + nq > a->nblk)
    return fail(BSA_ERR_SHAPE, "select: query range outside [0, nblk)");
  // large DOT selections: tcgen05 approximate scores + exact re-scoring
  // (bsa_select_tc5.cu), bit-identical to the kernel below
  if (select_tc5_applicable(a, T)) return run_select_tc5(a, T, W, st);
  const int ntiles = (nq + kTile - 1) / kTile;
  const size_t smem = (size_t)(a->dim * kLdA + 2 * kDC * kLdA + kTile * 65) * 4;
  dim3 grid(ntiles, a->G);
  void (*kern)(const bsa_select_args, int, int) = nullptr;
  switch (a->score_kind) {
    case BSA_SCORE_DOT: kern = select_kernel<BSA_SCORE_DOT>; break;
    case BSA_SCORE_MAXDOT2: kern = select_kernel<BSA_SCORE_MAXDOT2>; break;
    case BSA_SCORE_QUEST: kern = select_kernel<BSA_SCORE_QUEST>; break;
    default: return fail(BSA_ERR_ARG, "select: bad score_kind");
  }
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<grid, 256, smem, st>>>(*a, T, W);
  return check_launch("select");
}

// ------------------------------------------------------------------ rope
template <typename T>
__global__ void rope_kernel(const bsa_rope_args a) {
  const int half = a.rot / 2;
  const int extra = a.D - a.rot;  // pass-through dims per row
  const int per_row = half + ((a.x.ptr != a.y.ptr) ? extra : 0);
  const long long n = (long long)a.B * a.H * a.L * per_row;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < n;
       t += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(t % per_row);
    long long r = t / per_row;
    const int l = (int)(r % a.L);
    r /= a.L;
    const int h = (int)(r % a.H);
    const int b = (int)(r / a.H);
    const T *x = reinterpret_cast<const T *>(a.x.ptr) + b * a.x.sb + h * a.x.sh + (long long)l * a.x.sl;
    T *y = reinterpret_cast<T *>(a.y.ptr) + b * a.y.sb + h * a.y.sh + (long long)l * a.y.sl;
    if (j >= half) {
      const int d = a.rot + (j - half);
      y[d] = x[d];
      continue;
    }
    const T *c = reinterpret_cast<const T *>(a.cos) + b * a.cs_sb + (long long)l * a.cs_sl;
    const T *s = reinterpret_cast<const T *>(a.sin) + b * a.cs_sb + (long long)l * a.cs_sl;
    const int i0 = j, i1 = j + half;
    const float x0 = tof(x[i0]), x1 = tof(x[i1]);
    if constexpr (sizeof(T) == 4) {
      const float y0 = __fadd_rn(__fmul_rn(x0, c[i0]), __fmul_rn(-x1, s[i0]));
      const float y1 = __fadd_rn(__fmul_rn(x1, c[i1]), __fmul_rn(x0, s[i1]));
      y[i0] = y0;
      y[i1] = y1;
    } else {
      // each product and the sum rounded to T, as torch does op by op
      auto rd = [](float v) { return Mma<T>::to_f(Mma<T>::from_f(v)); };
      const float t0 = rd(__fmul_rn(x0, tof(c[i0]))), u0 = rd(__fmul_rn(-x1, tof(s[i0])));
      const float t1 = rd(__fmul_rn(x1, tof(c[i1]))), u1 = rd(__fmul_rn(x0, tof(s[i1])));
      y[i0] = Mma<T>::from_f(__fadd_rn(t0, u0));
      y[i1] = Mma<T>::from_f(__fadd_rn(t1, u1));
    }
  }
}

// Vectorised form (16-bit types, rot % 16 == 0, 16-byte rows): one thread per
// (row, group of 8 pairs), plus pass-through groups of 8 when y is not x.
template <typename T>
__global__ void rope_vec_kernel(const bsa_rope_args a) {
  const int half = a.rot / 2;
  const int ng = half / 8, npass = (a.x.ptr != a.y.ptr) ? (a.D - a.rot) / 8 : 0;
  const int per_row = ng + npass;
  const long long n = (long long)a.B * a.H * a.L * per_row;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < n;
       t += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(t % per_row);
    long long r = t / per_row;
    const int l = (int)(r % a.L);
    r /= a.L;
    const int h = (int)(r % a.H);
    const int b = (int)(r / a.H);
    const T *x = reinterpret_cast<const T *>(a.x.ptr) + b * a.x.sb + h * a.x.sh + (long long)l * a.x.sl;
    T *y = reinterpret_cast<T *>(a.y.ptr) + b * a.y.sb + h * a.y.sh + (long long)l * a.y.sl;
    if (g >= ng) {
      const int d = a.rot + 8 * (g - ng);
      *reinterpret_cast<uint4 *>(y + d) = *reinterpret_cast<const uint4 *>(x + d);
      continue;
    }
    const int i0 = 8 * g, i1 = i0 + half;
    const T *c = reinterpret_cast<const T *>(a.cos) + b * a.cs_sb + (long long)l * a.cs_sl;
    const T *s = reinterpret_cast<const T *>(a.sin) + b * a.cs_sb + (long long)l * a.cs_sl;
    const uint4 ux0 = *reinterpret_cast<const uint4 *>(x + i0), ux1 = *reinterpret_cast<const uint4 *>(x + i1);
    const uint4 uc0 = *reinterpret_cast<const uint4 *>(c + i0), uc1 = *reinterpret_cast<const uint4 *>(c + i1);
    const uint4 us0 = *reinterpret_cast<const uint4 *>(s + i0), us1 = *reinterpret_cast<const uint4 *>(s + i1);
    const T *x0 = reinterpret_cast<const T *>(&ux0), *x1 = reinterpret_cast<const T *>(&ux1);
    const T *c0 = reinterpret_cast<const T *>(&uc0), *c1 = reinterpret_cast<const T *>(&uc1);
    const T *s0 = reinterpret_cast<const T *>(&us0), *s1 = reinterpret_cast<const T *>(&us1);
    uint4 uy0, uy1;
    T *y0 = reinterpret_cast<T *>(&uy0), *y1 = reinterpret_cast<T *>(&uy1);
#pragma unroll
    for (int e = 0; e < 8; ++e) rope_pair<T>(x0[e], x1[e], c0[e], s0[e], c1[e], s1[e], y0[e], y1[e]);
    *reinterpret_cast<uint4 *>(y + i0) = uy0;
    *reinterpret_cast<uint4 *>(y + i1) = uy1;
  }
}

bsa_status run_rope(const bsa_rope_args *a, cudaStream_t st) {
  if (!a->x.ptr || !a->y.ptr || !a->cos || !a->sin) return fail(BSA_ERR_ARG, "rope: NULL pointer");
  if (a->rot <= 0 || a->rot % 2 || a->rot > a->D || a->B <= 0 || a->H <= 0 || a->L <= 0)
    return fail(BSA_ERR_SHAPE, "rope: need 0 < rot <= D, rot even");
  const int half = a->rot / 2;
  {
    const size_t es = elem_size(a->dtype);
    auto al = [&](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
    const bool vec = a->dtype != BSA_F32 && a->rot % 16 == 0 && a->D % 8 == 0 && al(a->x.ptr) &&
                     al(a->y.ptr) && al(a->cos) && al(a->sin) && (a->x.sb * es) % 16 == 0 &&
                     (a->x.sh * es) % 16 == 0 && (a->x.sl * es) % 16 == 0 &&
                     (a->y.sb * es) % 16 == 0 && (a->y.sh * es) % 16 == 0 &&
                     (a->y.sl * es) % 16 == 0 && (a->cs_sb * es) % 16 == 0 && (a->cs_sl * es) % 16 == 0;
    if (vec) {
      const int per_row = half / 8 + ((a->x.ptr != a->y.ptr) ? (a->D - a->rot) / 8 : 0);
      const long long n = (long long)a->B * a->H * a->L * per_row;
      const long long blocks = std::max<long long>(1, std::min<long long>((n + 255) / 256, 1LL << 20));
      if (a->dtype == BSA_BF16)
        rope_vec_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(*a);
      else
        rope_vec_kernel<__half><<<(unsigned)blocks, 256, 0, st>>>(*a);
      return check_launch("rope");
    }
  }
  const int per_row = half + ((a->x.ptr != a->y.ptr) ? a->D - a->rot : 0);
  const long long n = (long long)a->B * a->H * a->L * per_row;
  const int threads = 256;
  const long long blocks = std::max<long long>(1, std::min<long long>((n + threads - 1) / threads, 1LL << 20));
  if (a->dtype == BSA_BF16)
    rope_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, st>>>(*a);
  else if (a->dtype == BSA_F16)
    rope_kernel<__half><<<(unsigned)blocks, threads, 0, st>>>(*a);
  else if (a->dtype == BSA_F32)
    rope_kernel<float><<<(unsigned)blocks, threads, 0, st>>>(*a);
  else
    return fail(BSA_ERR_DTYPE, "rope: bad dtype");
  return check_launch("rope");
}

}  // namespace bsa
