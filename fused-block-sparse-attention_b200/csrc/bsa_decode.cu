// Decode: the T newest tokens of a sequence attend to their selected blocks of
// a K/V cache (split-K over the selected blocks, then a merge).  The reference
// has no decode path; this is the consumer its selection feeds next.  The
// arithmetic is the forward's (scale, additive per-block gate, SLOT or TOKEN
// masks) restricted to query rows L-T .. L-1, which all lie in the last block.
//
//   decode_partial_kernel  CTA per (b, KV head, split); the query rows of the
//                          whole GQA group (grp heads x T tokens, <= 32 rows) sit
//                          in shared memory; the split's selected blocks are
//                          read once each (K rows by 16-byte loads, several
//                          threads per key; V by columns, coalesced), with an
//                          online softmax per row; writes (m, l, O) per row.
//   decode_merge_kernel    one warp per (b, query head, token): merges the splits.
// Memory-bound by design: every selected K/V byte is read once per step.
#include <algorithm>

#include "bsa_common.cuh"
#include "bsa_host.h"

namespace bsa {

namespace {
constexpr int kDecMaxRows = 32, kDecMaxD = 256, kDecMaxBs = 128, kDecThreads = 256;

template <typename T>
__device__ __forceinline__ float dec_f(T x) {
  return Mma<T>::to_f(x);
}
template <>
__device__ __forceinline__ float dec_f<float>(float x) {
  return x;
}
}  // namespace

// part: (B*Hkv, nsplit, R, D + 2) fp32 rows of (O[D], m, l)
template <typename T>
__global__ void __launch_bounds__(kDecThreads) decode_partial_kernel(const bsa_decode_args a, int R,
                                                                     int nsplit, float *part) {
  extern __shared__ float dsm[];
  const int D = a.D, bs = a.bs;
  float *sq = dsm;                          // [R][D]
  float *ss = sq + R * D;                   // [R][bs] scores, then probabilities
  float *sm = ss + R * bs;                  // [R] running max
  float *sl = sm + R;                       // [R] running sum
  float *sal = sl + R;                      // [R] rescale of this block
  const int grp = a.Hq / a.Hkv;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / a.Hkv, hk = bh % a.Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qb = (a.L - 1) / bs;  // the block holding every query row

  for (int i = tid; i < R * D; i += kDecThreads) {
    const int r = i / D, d = i % D;
    const int h = hk * grp + r / a.T, t = r % a.T;
    const T *qp = reinterpret_cast<const T *>(a.q.ptr) + b * a.q.sb + h * a.q.sh + t * a.q.sl;
    sq[i] = dec_f<T>(qp[d]);
  }
  for (int r = tid; r < R; r += kDecThreads) {
    sm[r] = -INFINITY;
    sl[r] = 0.f;
  }
  // output ownership: thread (rg, d) holds rows rg, rg + RG, ... of column d
  const int RG = kDecThreads / D;  // D divides 256
  const int od = tid % D, org = tid / D;
  float acc[kDecMaxRows];
#pragma unroll
  for (int i = 0; i < kDecMaxRows; ++i) acc[i] = 0.f;
  const int32_t *selrow = a.sel + b * a.sel_sb + hk * a.sel_sh;
  const float *gaterow = a.gate ? a.gate + b * a.gate_sb + hk * a.gate_sh : nullptr;
  const T *kbase = reinterpret_cast<const T *>(a.k.ptr) + b * a.k.sb + hk * a.k.sh;
  const T *vbase = reinterpret_cast<const T *>(a.v.ptr) + b * a.v.sb + hk * a.v.sh;
  const int tpk = kDecThreads / bs;  // threads per key in the score pass (bs divides 256)
  const int dchunk = D / tpk;
  __syncthreads();

  for (int slot = split; slot < a.kk; slot += nsplit) {
    const int kb = selrow[slot];
    if (kb < 0 || kb > qb) {  // outside the cache or after the query block
      if (kb < 0 || (long long)kb * bs >= a.L) report(a.status, BSA_DEVERR_INDEX);
      continue;
    }
    bool dup = false;
    if (a.mask_mode == BSA_MASK_TOKEN)
      for (int i = 0; i < slot && !dup; ++i) dup = selrow[i] == kb;
    if (dup) continue;
    if (a.mask_mode == BSA_MASK_SLOT && slot > 0 && kb >= qb) continue;
    const float g = gaterow ? gaterow[slot] : 0.f;
    // ---- scores: key k = tid / tpk, dims [dchunk * (tid % tpk), +dchunk)
    {
      const int k = tid / tpk, part_i = tid % tpk;
      const long long key = (long long)kb * bs + k;
      float dot[kDecMaxRows];
#pragma unroll
      for (int r = 0; r < kDecMaxRows; ++r) dot[r] = 0.f;
      if (key < a.L) {
        const T *kr = kbase + key * a.k.sl + part_i * dchunk;
        for (int d0 = 0; d0 < dchunk; d0 += 8) {
          float kv[8];
          if constexpr (sizeof(T) == 2) {
            const uint4 u = *reinterpret_cast<const uint4 *>(kr + d0);
            const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
            for (int i = 0; i < 8; ++i) kv[i] = dec_f<T>(e[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) kv[i] = dec_f<T>(kr[d0 + i]);
          }
#pragma unroll
          for (int r = 0; r < kDecMaxRows; ++r) {
            if (r < R) {
              const float *qr = sq + r * D + part_i * dchunk + d0;
#pragma unroll
              for (int i = 0; i < 8; ++i) dot[r] = fmaf(qr[i], kv[i], dot[r]);
            }
          }
        }
      }
      // sum the tpk partial dots (consecutive lanes)
#pragma unroll
      for (int r = 0; r < kDecMaxRows; ++r) {
        if (r >= R) break;
        for (int o = 1; o < tpk; o <<= 1) dot[r] += __shfl_xor_sync(0xffffffffu, dot[r], o);
        if (part_i == 0) {
          const long long qpos = (long long)a.L - a.T + (r % a.T);
          bool ok = key < a.L;
          if (a.mask_mode == BSA_MASK_TOKEN || slot == 0) ok = ok && key <= qpos;
          ss[r * bs + k] = ok ? fmaf(dot[r], a.scale, g) : -INFINITY;
        }
      }
    }
    __syncthreads();
    // ---- online softmax, one warp per row
    for (int r = warp; r < R; r += kDecThreads / 32) {
      float mx = -INFINITY;
      for (int k = lane; k < bs; k += 32) mx = fmaxf(mx, ss[r * bs + k]);
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mold = sm[r], mnew = fmaxf(mold, mx);
      float sum = 0.f;
      for (int k = lane; k < bs; k += 32) {
        const float p = mnew == -INFINITY ? 0.f : expf(ss[r * bs + k] - mnew);
        ss[r * bs + k] = p;
        sum += p;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      __syncwarp();
      if (lane == 0) {
        const float al = mold == -INFINITY ? 0.f : expf(mold - mnew);
        sal[r] = al;
        sm[r] = mnew;
        sl[r] = sl[r] * al + sum;
      }
    }
    __syncthreads();
    // ---- O += P V
    {
#pragma unroll
      for (int i = 0; i < kDecMaxRows; ++i) {
        const int r = org + i * RG;
        if (r < R) acc[i] *= sal[r];
      }
      for (int k = 0; k < bs; ++k) {
        const long long key = (long long)kb * bs + k;
        if (key >= a.L) break;
        const float vv = dec_f<T>(vbase[key * a.v.sl + od]);
#pragma unroll
        for (int i = 0; i < kDecMaxRows; ++i) {
          const int r = org + i * RG;
          if (r < R) acc[i] = fmaf(ss[r * bs + k], vv, acc[i]);
        }
      }
    }
    __syncthreads();
  }
  // ---- partial (O, m, l) of each row
  float *pb = part + ((long long)bh * nsplit + split) * R * (D + 2);
#pragma unroll
  for (int i = 0; i < kDecMaxRows; ++i) {
    const int r = org + i * RG;
    if (r < R) pb[r * (D + 2) + od] = acc[i];
  }
  for (int r = tid; r < R; r += kDecThreads) {
    pb[r * (D + 2) + D] = sm[r];
    pb[r * (D + 2) + D + 1] = sl[r];
  }
}

template <typename T>
__global__ void decode_merge_kernel(const bsa_decode_args a, int R, int nsplit, const float *part) {
  const int grp = a.Hq / a.Hkv;
  const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)a.B * a.Hkv * R) return;
  const int r = (int)(w % R);
  const long long bh = w / R;
  const int b = (int)(bh / a.Hkv), hk = (int)(bh % a.Hkv);
  const int h = hk * grp + r / a.T, t = r % a.T;
  const int D = a.D;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part[((bh * nsplit + s) * R + r) * (D + 2) + D]);
  float Lsum = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float *ps = part + ((bh * nsplit + s) * R + r) * (D + 2);
    if (ps[D] > -INFINITY) Lsum += ps[D + 1] * expf(ps[D] - M);
  }
  const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
  T *op = reinterpret_cast<T *>(a.o.ptr) + b * a.o.sb + h * a.o.sh + t * a.o.sl;
  for (int d = lane; d < D; d += 32) {
    float v = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float *ps = part + ((bh * nsplit + s) * R + r) * (D + 2);
      if (ps[D] > -INFINITY) v = fmaf(ps[d], expf(ps[D] - M), v);
    }
    if constexpr (sizeof(T) == 2)
      op[d] = Mma<T>::from_f(v * inv);
    else
      op[d] = v * inv;
  }
}

static int decode_nsplit(const bsa_decode_args *a) {
  const long long heads = (long long)a->B * a->Hkv;
  const long long want = std::max<long long>(1, (2LL * 148 + heads - 1) / heads);
  return (int)std::min<long long>(a->kk, want);
}

static bsa_status decode_check(const bsa_decode_args *a) {
  if (a->dtype != BSA_BF16 && a->dtype != BSA_F16 && a->dtype != BSA_F32)
    return fail(BSA_ERR_DTYPE, "decode: dtype must be bf16, f16 or f32");
  if (a->B <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->L <= 0 || a->T <= 0 || a->kk <= 0 ||
      a->Hq % a->Hkv)
    return fail(BSA_ERR_SHAPE, "decode: sizes must be positive and Hq a multiple of Hkv");
  if (a->T > a->L || (a->L - a->T) / a->bs != (a->L - 1) / a->bs)
    return fail(BSA_ERR_SHAPE, "decode: the T query rows must lie in the last block");
  const int R = (a->Hq / a->Hkv) * a->T;
  if (R > kDecMaxRows) return fail(BSA_ERR_UNSUPPORTED, "decode: (Hq/Hkv) * T must be <= 32");
  if (a->D > kDecMaxD || a->D < 8 || kDecThreads % a->D || a->D % 8)
    return fail(BSA_ERR_UNSUPPORTED, "decode: D must divide 256 (8..256)");
  if (a->bs > kDecMaxBs || kDecThreads % a->bs || (a->D / (kDecThreads / a->bs)) % 8)
    return fail(BSA_ERR_UNSUPPORTED, "decode: bs must divide 256, be <= 128 and D/(256/bs) a multiple of 8");
  if (!a->q.ptr || !a->k.ptr || !a->v.ptr || !a->o.ptr || !a->sel)
    return fail(BSA_ERR_ARG, "decode: NULL tensor");
  if (a->mask_mode != BSA_MASK_SLOT && a->mask_mode != BSA_MASK_TOKEN)
    return fail(BSA_ERR_ARG, "decode: bad mask_mode");
  if (!(a->scale > 0.f)) return fail(BSA_ERR_ARG, "decode: bad scale");
  if (a->dtype != BSA_F32 && ((reinterpret_cast<uintptr_t>(a->k.ptr) % 16) || (a->k.sl * 2) % 16))
    return fail(BSA_ERR_STRIDE, "decode: K rows must be 16-byte aligned");
  return BSA_OK;
}

size_t decode_workspace(const bsa_decode_args *a) {
  if (decode_check(a) != BSA_OK) return 0;
  const int R = (a->Hq / a->Hkv) * a->T;
  return (size_t)a->B * a->Hkv * decode_nsplit(a) * R * (a->D + 2) * 4;
}

bsa_status run_decode(const bsa_decode_args *a, void *ws, size_t ws_bytes, cudaStream_t st) {
  if (bsa_status s = decode_check(a)) return s;
  const size_t need = decode_workspace(a);
  if (!ws || ws_bytes < need) return fail(BSA_ERR_WORKSPACE, "decode: workspace too small");
  const int R = (a->Hq / a->Hkv) * a->T, nsplit = decode_nsplit(a);
  const size_t smem = ((size_t)R * a->D + (size_t)R * a->bs + 3 * R) * 4;
  dim3 grid(a->B * a->Hkv, nsplit);
  float *part = static_cast<float *>(ws);
  const long long warps = (long long)a->B * a->Hkv * R;
  const unsigned mblocks = (unsigned)((warps * 32 + 255) / 256);
#define BSA_DEC(T_)                                                                         \
  {                                                                                         \
    cudaFuncSetAttribute(decode_partial_kernel<T_>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                         (int)smem);                                                        \
    decode_partial_kernel<T_><<<grid, kDecThreads, smem, st>>>(*a, R, nsplit, part);        \
    if (bsa_status s = check_launch("decode_partial")) return s;                            \
    decode_merge_kernel<T_><<<mblocks, 256, 0, st>>>(*a, R, nsplit, part);                   \
  }
  if (a->dtype == BSA_BF16)
    BSA_DEC(__nv_bfloat16)
  else if (a->dtype == BSA_F16)
    BSA_DEC(__half)
  else
    BSA_DEC(float)
#undef BSA_DEC
  return check_launch("decode_merge");
}

}  // namespace bsa
