// Block-pair selection on the 5th-generation tensor cores (sm_100a), exact.
//
// Replaces the fp32 FMA scoring of select_kernel for the mean-pooled q.k
// selection (score kind DOT, the BASELINE configurations 1-3 and 5; reference
// src/ssa_model.py:118-119,151-162 with scores from mean pooling) when the block
// count is large.  The selected indices are bit-identical to select_kernel and
// the CPU oracle:
//
//  1. Approximate scores  S~ = A.B^T  per 128 x 128 tile, tcgen05.mma kind::tf32
//     (operands are the fp32 summaries, TMA-loaded with 128-byte swizzle; the
//     tensor core reads them as tf32), accumulated in TMEM (two buffers).
//  2. Per query row (one epilogue thread per TMEM lane) a sorted list of the
//     best KT >= T exact scores so far, in registers (KT = 8, 16 or 32).  A key block can only enter the list when its
//     exact score s >= thr (the T-th exact score, ties to the lower block id).
//     Since |S~ - s| <= eps = 2^-7 * |a| * |b| (tf32 operand rounding of at most
//     2^-10 relative per factor, fp32 accumulation, and the fp32 rounding of the
//     exact chain itself are all below 2^-8 * sum_d |a_d b_d| <= 2^-8 |a||b|,
//     with a factor 2 to spare), every key with S~ + eps < thr is skipped
//     without changing the result.
//  3. Keys that pass are re-scored with the exact fp32 chain
//     s = fma(a_d, b_d, s), d = 0..dim-1 (operands read back from the same
//     shared-memory tiles), cooperatively: the passing (row, key) pairs of a
//     warp are queued and scored one per lane, then every row inserts its own
//     results by (score desc, block id asc) with a fixed compare-exchange sweep.
//  After the first few tiles the threshold is high and almost every key is
//  rejected by one add and one compare, so the exact work is a small multiple
//  of T per row instead of one dot product per causal block pair; the
//  nblk x nblk score matrix never leaves TMEM.
//
// Work split: a cluster of C CTAs serves one 128-row query tile; CTA r takes
// the key tiles kt = r, r + C, ... .  At the end CTA 0 merges the C sorted
// lists of each row through distributed shared memory (an exact merge: the
// order is total) and writes the row.  C is chosen on the host so that small
// group counts (one head per GPU) still fill the SMs.  No TMA multicast.
//
// Warp roles (192 threads): warps 0-3 epilogue (thread t = query row t = TMEM
// lane t), warp 4 TMA producer, warp 5 TMEM allocator + single MMA issuer.
// Every mbarrier wait is bounded; a timeout sets BSA_DEVERR_TIMEOUT in the
// status word and the CTA finishes without writing its rows.
#include <algorithm>

#include "bsa_common.cuh"
#include "bsa_host.h"
#include "bsa_tc05.cuh"

namespace bsa {
namespace s5 {

constexpr int kM = 128;          // query rows per tile (TMEM lanes)
constexpr int kN = 128;          // key blocks per tile (TMEM columns per buffer)
constexpr int kTmemCols = 256;   // two accumulator buffers
constexpr int kMaxT = 32;
constexpr int kThreads = 192;
constexpr int kQueue = 1024;     // candidates of one 32-column chunk of one warp (32 x 32)

__host__ __device__ constexpr int chunks(int dim) { return dim / 32; }          // 128-byte K chunks
__host__ __device__ constexpr int tile_bytes(int dim) { return kM * dim * 4; }  // A or one B stage
__host__ __device__ constexpr int stages(int dim) { return dim <= 32 ? 6 : (dim <= 64 ? 4 : 2); }

struct Smem {
  // offsets (bytes) from the 1024-aligned dynamic shared memory base
  int a, b, ls, li, nb, q, bars, total;
};
__host__ __device__ constexpr Smem layout(int dim) {
  Smem s{};
  s.a = 0;
  s.b = tile_bytes(dim);
  s.ls = s.b + stages(dim) * tile_bytes(dim);
  s.li = s.ls + kMaxT * kM * 4;
  s.nb = s.li + kMaxT * kM * 4;
  s.q = s.nb + kM * 4 + kM * 4;     // column norms + per-row list lengths
  s.bars = s.q + 4 * kQueue * (2 + 4);  // per-warp candidate queues (u16 entry + fp32 score)
  s.total = s.bars + 8 * (1 + 2 * 6 + 2 * 2) + 16;
  return s;
}

__device__ __forceinline__ bool better(float s1, int i1, float s2, int i2) {
  return s1 > s2 || (s1 == s2 && i1 < i2);
}

__device__ __forceinline__ float logsigmoid(float x) {
  return x < 0.f ? x - log1pf(expf(x)) : -log1pf(expf(-x));
}

// byte offset of element (row, k) in a K-major, 128B-swizzled fp32 tile of kM rows
__device__ __forceinline__ uint32_t off(int row, int k) {
  const int c = k >> 5, u = (k & 31) >> 2;
  return (uint32_t)(c * kM * 128 + row * 128 + ((u ^ (row & 7)) << 4) + ((k & 3) << 2));
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::tf32 instruction descriptor: fp32 accumulator, tf32 A and B, both K-major
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ int ld_dsmem_s32(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

template <int DIM, int KT>
__global__ void __launch_bounds__(kThreads, 1)
    select_tc5_kernel(const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_b, const bsa_select_args a, int T,
                      int W, int C) {
  constexpr Smem L = layout(DIM);
  constexpr int NS = stages(DIM);
  constexpr int NCH = chunks(DIM);
  constexpr uint32_t TB = tile_bytes(DIM);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *ls = reinterpret_cast<float *>(sm + L.ls);
  int *li = reinterpret_cast<int *>(sm + L.li);
  float *nbs = reinterpret_cast<float *>(sm + L.nb);
  int *cnt = reinterpret_cast<int *>(sm + L.nb + kM * 4);
  uint16_t *qent = reinterpret_cast<uint16_t *>(sm + L.q);                  // [4][kQueue]
  float *qres = reinterpret_cast<float *>(sm + L.q + 4 * kQueue * 2);       // [4][kQueue]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + L.bars);
  uint64_t *a_full = bars;
  uint64_t *b_full = bars + 1;         // [NS]
  uint64_t *b_empty = bars + 1 + 6;    // [NS]
  uint64_t *acc_full = bars + 13;      // [2]
  uint64_t *acc_empty = bars + 15;     // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 17);
  __shared__ int s_err;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = C > 1 ? cluster_rank() : 0;
  const int cl = blockIdx.x / C;
  const int nq = a.nq > 0 ? a.nq : a.nblk, qb0 = a.q_blk0;
  const int nqt = (nq + kM - 1) / kM, nkt = (a.nblk + kN - 1) / kN;
  const int qt = nqt - 1 - cl;  // heaviest causal tiles first
  const int g = blockIdx.y;
  const int q0 = qt * kM;
  const bool causal_like = a.layout == BSA_SEL_FINISH || a.layout == BSA_SEL_RAW || a.causal;
  const int kt_last = causal_like ? min(nkt - 1, (qb0 + min(q0 + kM, nq) - 1) / kN) : nkt - 1;
  // this CTA's key tiles: rank, rank + C, ... <= kt_last
  const int ntile = kt_last >= (int)rank ? (kt_last - (int)rank) / C + 1 : 0;

  if (tid == 0) {
    s_err = 0;
    mbar_init(a_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 5) {
    tc05::alloc(tmem_slot, kTmemCols);
    tc05::relinquish();
  }
  tc05::fence_before();
  __syncthreads();
  tc05::fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    // (the warp waits together, one elected lane issues)
    if (ntile > 0) {
      if (tc05::elect_one()) {
        prefetch_tmap(&map_a);
        prefetch_tmap(&map_b);
        mbar_expect_tx(a_full, TB);
        for (int c = 0; c < NCH; ++c) tma_load_3d(sm + L.a + c * kM * 128, &map_a, a_full, c * 32, q0, g);
      }
      __syncwarp();
      int issued = 0;
      for (int t = 0; t < ntile; ++t) {
        const int s = t % NS;
        if (t >= NS && !mbar_wait_warp(&b_empty[s], ((t / NS) - 1) & 1)) {
          if (lane == 0) {
            report(a.status, BSA_DEVERR_TIMEOUT);
            atomicOr(&s_err, 1);
          }
          break;
        }
        const int k0 = ((int)rank + t * C) * kN;
        if (tc05::elect_one()) {
          mbar_expect_tx(&b_full[s], TB);
          for (int c = 0; c < NCH; ++c)
            tma_load_3d(sm + L.b + s * TB + c * kM * 128, &map_b, &b_full[s], c * 32, k0, g);
        }
        __syncwarp();
        issued = t + 1;
      }
      // every issued load has landed before the CTA can exit: the last NS
      // issued stages are waited for here (consumed ones complete at once)
      for (int t = max(0, issued - NS); t < issued; ++t)
        if (!mbar_wait_warp(&b_full[t % NS], (t / NS) & 1) && lane == 0)
          report(a.status, BSA_DEVERR_TIMEOUT);
      mbar_wait_warp(a_full, 0);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    // (the warp waits together, one elected lane issues the MMAs and commits)
    if (ntile > 0) {
      constexpr uint32_t idesc = idesc_tf32(kM, kN);
      bool ok = mbar_wait_warp(a_full, 0);
      const uint64_t adesc = tc05::sdesc(smem_u32(sm + L.a), 16, 1024);
      for (int t = 0; t < ntile && ok; ++t) {
        const int s = t % NS, b = t & 1;
        if (t >= 2 && !mbar_wait_warp(&acc_empty[b], ((t >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait_warp(&b_full[s], (t / NS) & 1)) {
          ok = false;
          break;
        }
        tc05::fence_after();
        const uint64_t bdesc = tc05::sdesc(smem_u32(sm + L.b + s * TB), 16, 1024);
        if (tc05::elect_one()) {
#pragma unroll
          for (int k = 0; k < DIM / 8; ++k) {
            const uint32_t koff = (uint32_t)((k >> 2) * kM * 128 + (k & 3) * 32);
            mma_tf32(tmem + b * kN, tc05::dadd(adesc, koff), tc05::dadd(bdesc, koff), idesc, k > 0);
          }
          tc05::commit(&acc_full[b]);
        }
        __syncwarp();
      }
      if (!ok && lane == 0) {
        report(a.status, BSA_DEVERR_TIMEOUT);
        atomicOr(&s_err, 1);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int row = tid;  // TMEM lane = local query row in the tile
    const int lrow = q0 + row;
    const bool live = lrow < nq;
    const int qi = qb0 + lrow;  // global query block
    // candidate key j is valid iff j < jend and j != jskip
    int jend, jskip = -1;
    if (a.layout == BSA_SEL_SSA) {
      jend = a.causal ? min(qi, a.nblk) : a.nblk;
      if (!a.causal) jskip = qi;
    } else {
      jend = min(qi + 1, a.nblk);
    }
    if (!live) jend = 0;
    const uint8_t *As = sm + L.a;
    float na = 0.f;
    // this row's best KT (the power of two >= T) exact scores so far, sorted by
    // (score desc, id asc), in registers; empty entries are (-inf, INT_MAX).  A
    // key that does not beat the last entry cannot be among the best T.
    float Ls[KT];
    int Li[KT];
#pragma unroll
    for (int l = 0; l < KT; ++l) {
      Ls[l] = -INFINITY;
      Li[l] = INT_MAX;
    }
    bool ok = ntile == 0 || mbar_wait(a_full, 0);
    if (live && ok) {
#pragma unroll 4
      for (int d = 0; d < DIM; d += 4) {
        const float4 x = *reinterpret_cast<const float4 *>(As + off(row, d));
        na = fmaf(x.x, x.x, na);
        na = fmaf(x.y, x.y, na);
        na = fmaf(x.z, x.z, na);
        na = fmaf(x.w, x.w, na);
      }
    }
    const float ka = 0.0078125f * sqrtf(na) * 1.0001f;  // 2^-7 |a| (rounded up)
    __shared__ int e_err;  // written by epilogue threads only, read after a barrier
    if (tid == 0) e_err = ok ? 0 : 1;
    named_bar_sync(1, 128);
    for (int t = 0; t < ntile; ++t) {
      const int s = t % NS, b = t & 1;
      const int k0 = ((int)rank + t * C) * kN;
      if (e_err == 0 && !mbar_wait(&acc_full[b], (t >> 1) & 1)) atomicOr(&e_err, 1);
      tc05::fence_after();
      const uint8_t *Bs = sm + L.b + s * TB;
      // column norms of this key tile (thread t: key row t of the stage)
      {
        // four independent chains (only an upper bound is needed: the 1.0001
        // factor covers any summation order's rounding)
        float n0 = 0.f, n1 = 0.f, n2 = 0.f, n3 = 0.f;
#pragma unroll
        for (int d = 0; d < DIM; d += 4) {
          const float4 x = *reinterpret_cast<const float4 *>(Bs + off(row, d));
          n0 = fmaf(x.x, x.x, n0);
          n1 = fmaf(x.y, x.y, n1);
          n2 = fmaf(x.z, x.z, n2);
          n3 = fmaf(x.w, x.w, n3);
        }
        // the tile's largest key norm: one bound for every column of the tile
        float nbm = sqrtf((n0 + n1) + (n2 + n3)) * 1.0001f;
#pragma unroll
        for (int o = 16; o; o >>= 1) nbm = fmaxf(nbm, __shfl_xor_sync(0xffffffffu, nbm, o));
        if (lane == 0) nbs[warp] = nbm;
      }
      named_bar_sync(1, 128);  // norms written; every epilogue warp sees the same e_err
      if (e_err) break;
      const int cend = min(kN, jend - k0);  // columns < cend may be valid for this row
      const float nbmax = fmaxf(fmaxf(nbs[0], nbs[1]), fmaxf(nbs[2], nbs[3]));
      float cut = __fsub_rd(Ls[KT - 1], __fmul_ru(ka, nbmax));
      if (__any_sync(0xffffffffu, Li[KT - 1] == INT_MAX)) {
        // a list of this warp is not full yet (its cut is -inf): bound the tile's
        // own KT-th best instead.  The minimum over KT disjoint column groups of
        // the group maxima of S~ is <= the KT-th largest S~ of the tile (t), and
        // a key among the tile's best KT exact scores has s >= t - E, so
        // S~ >= t - 2E (E = ka * max|b| >= eps of every key): exact to skip the rest.
        constexpr int GS = kN / KT;  // columns per group
        float tmin = INFINITY;
#pragma unroll
        for (int ch = 0; ch < kN / 32; ++ch) {
          const int cc = ch * 32;
          __syncwarp();
          float v[32];
          tc05::ld32(tc05::taddr(tmem, warp * 32, b * kN + cc), v);
          tc05::wait_ld();
          const int lim = min(max(cend - cc, 0), 32);
#pragma unroll
          for (int g0 = 0; g0 < 32; g0 += GS) {
            float gm = -INFINITY;
#pragma unroll
            for (int c = g0; c < g0 + GS; ++c) {
              const bool ok = c < lim && k0 + cc + c != jskip;
              gm = fmaxf(gm, ok ? v[c] : -INFINITY);
            }
            tmin = fminf(tmin, gm);
          }
        }
        const float e2 = 2.f * __fmul_ru(ka, nbmax);
        cut = fmaxf(cut, __fsub_rd(tmin, e2));
      }
      // 1. candidate masks of the four 32-column chunks, branch-free: valid
      //    columns, and the approximate score against the current threshold
      unsigned mk[kN / 32];
#pragma unroll
      for (int ch = 0; ch < kN / 32; ++ch) {
        const int cc = ch * 32;
        __syncwarp();
        float v[32];
        tc05::ld32(tc05::taddr(tmem, warp * 32, b * kN + cc), v);
        tc05::wait_ld();
        if (ch == kN / 32 - 1) {
          tc05::fence_before();
          __syncwarp();
          if (lane == 0) tc05::mbar_arrive(&acc_empty[b]);
        }
        const int lim = min(max(cend - cc, 0), 32);
        unsigned m = lim >= 32 ? 0xffffffffu : ((1u << lim) - 1u);
        if (jskip >= k0 + cc && jskip < k0 + cc + 32) m &= ~(1u << (jskip - k0 - cc));
        // S~ >= cut with cut = thr - ka * max|b|, rounded down (directed
        // rounding keeps the test a superset of S~ + eps >= thr)
        unsigned pass = 0;
#pragma unroll
        for (int c = 0; c < 32; ++c) pass |= (unsigned)(v[c] >= cut) << c;
        mk[ch] = m & pass;
      }
      // 2. The candidates of the whole warp are re-scored cooperatively (one per
      //    lane, so the exact dot products never run with idle lanes): each lane
      //    queues its (row, column) pairs at its exclusive prefix, the warp scores
      //    the queue 32 at a time, then every lane inserts its own results.  The
      //    whole tile forms one group unless its candidates overflow the queue
      //    (early tiles, whose threshold is still low): then chunk by chunk.
      uint16_t *wq = qent + warp * kQueue;
      float *wr = qres + warp * kQueue;
      auto group = [&](int c0, int c1) {
        int nc = 0;
#pragma unroll
        for (int ch = 0; ch < kN / 32; ++ch)
          if (ch >= c0 && ch < c1) nc += __popc(mk[ch]);
        int pre = nc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, pre, o);
          if (lane >= o) pre += y;
        }
        const int total = __shfl_sync(0xffffffffu, pre, 31);
        if (total == 0) return;
        pre -= nc;
        {
          int p = pre;
#pragma unroll
          for (int ch = 0; ch < kN / 32; ++ch) {
            if (ch < c0 || ch >= c1) continue;
            unsigned mm = mk[ch];
            while (mm) {
              wq[p++] = (uint16_t)((lane << 7) | (ch * 32 + __ffs(mm) - 1));
              mm &= mm - 1;
            }
          }
        }
        __syncwarp();
        for (int base = 0; base < total; base += 32) {
          const int idx = base + lane;
          if (idx < total) {
            const int ent = wq[idx];
            const int r = warp * 32 + (ent >> 7), col = ent & 127;
            float e = 0.f;
#pragma unroll 4
            for (int d = 0; d < DIM; d += 4) {
              const float4 x = *reinterpret_cast<const float4 *>(As + off(r, d));
              const float4 y = *reinterpret_cast<const float4 *>(Bs + off(col, d));
              e = fmaf(x.x, y.x, e);
              e = fmaf(x.y, y.y, e);
              e = fmaf(x.z, y.z, e);
              e = fmaf(x.w, y.w, e);
            }
            wr[idx] = e;
          }
        }
        __syncwarp();
        for (int x = pre; x < pre + nc; ++x) {
          const int j = k0 + (wq[x] & 127);
          float cs = wr[x];
          if (!(cs > -INFINITY)) continue;  // -inf / NaN never rank
          if (!better(cs, j, Ls[KT - 1], Li[KT - 1])) continue;
          int ci = j;
          // insertion by a fixed compare-exchange sweep (no data-dependent indexing)
#pragma unroll
          for (int l = 0; l < KT; ++l) {
            const bool bt = better(cs, ci, Ls[l], Li[l]);
            const float ts = Ls[l];
            const int ti = Li[l];
            Ls[l] = bt ? cs : ts;
            Li[l] = bt ? ci : ti;
            cs = bt ? ts : cs;
            ci = bt ? ti : ci;
          }
        }
        __syncwarp();  // the queue is reused by the next group
      };
      int tile_n = 0;
#pragma unroll
      for (int ch = 0; ch < kN / 32; ++ch) tile_n += __popc(mk[ch]);
      const int tile_total = __reduce_add_sync(0xffffffffu, tile_n);
      if (tile_total <= kQueue) {
        group(0, kN / 32);
      } else {
#pragma unroll 1
        for (int ch = 0; ch < kN / 32; ++ch) group(ch, ch + 1);
      }
      named_bar_sync(1, 128);  // nbs is rewritten by the next tile
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&b_empty[s]);
    }
    if (tid == 0 && e_err) atomicOr(&s_err, 1);
    if (tid == 0 && e_err) report(a.status, BSA_DEVERR_TIMEOUT);
    int n = 0;
#pragma unroll
    for (int l = 0; l < KT; ++l) {
      ls[l * kM + row] = Ls[l];
      li[l * kM + row] = Li[l];
      n += Li[l] != INT_MAX;
    }
    cnt[row] = min(n, T);
  }

  // ---------------------------------------------------------------- merge + write
  tc05::fence_before();
  __syncthreads();
  if (C > 1) cluster_sync();  // every CTA's lists are final
  const bool err = s_err != 0;
  if (rank == 0 && warp < 4) {
    const int row = tid;
    const int lrow = q0 + row;
    if (lrow < nq && !err) {
      const int qi = qb0 + lrow;
      const long long ob = ((long long)g * nq + lrow) * W;
      // C-way merge of the sorted lists (list r lives in CTA r of the cluster)
      int head[8], len[8];
      float hs[8];
      int hi[8];
      const uint32_t ls_addr = smem_u32(ls), li_addr = smem_u32(li), cnt_addr = smem_u32(cnt);
      for (int r = 0; r < 8; ++r) {
        head[r] = 0;
        len[r] = 0;
        hs[r] = -INFINITY;
        hi[r] = INT_MAX;
        if (r < C) {
          len[r] = C > 1 ? ld_dsmem_s32(map_rank(cnt_addr + row * 4, r)) : cnt[row];
          if (len[r] > 0) {
            hs[r] = C > 1 ? ld_dsmem_f32(map_rank(ls_addr + row * 4, r)) : ls[row];
            hi[r] = C > 1 ? ld_dsmem_s32(map_rank(li_addr + row * 4, r)) : li[row];
          }
        }
      }
      float own = 0.f;
      if (a.layout == BSA_SEL_SSA && (a.score_out || a.gate_out)) {
        const float *b1r = a.b1 + ((long long)g * a.nblk + qi) * DIM;
        const uint8_t *As = sm + L.a;
        for (int d = 0; d < DIM; ++d)
          own = fmaf(*reinterpret_cast<const float *>(As + off(row, d)), b1r[d], own);
      }
      int scratch[kMaxT + 2];
      for (int l = 0; l < T; ++l) {
        int best = -1;
        for (int r = 0; r < C; ++r)
          if (head[r] < len[r] && (best < 0 || better(hs[r], hi[r], hs[best], hi[best]))) best = r;
        float sc = own;
        int id = -1;
        if (best >= 0) {
          sc = hs[best];
          id = hi[best];
          const int h = ++head[best];
          if (h < len[best]) {
            const uint32_t o = (uint32_t)(h * kM + row) * 4;
            hs[best] = C > 1 ? ld_dsmem_f32(map_rank(ls_addr + o, best)) : ls[h * kM + row];
            hi[best] = C > 1 ? ld_dsmem_s32(map_rank(li_addr + o, best)) : li[h * kM + row];
          }
        }
        if (a.layout == BSA_SEL_SSA) {
          a.sel[ob + 1 + l] = id >= 0 ? id : qi;
          if (a.score_out) a.score_out[ob + 1 + l] = sc;
          if (a.gate_out) a.gate_out[ob + 1 + l] = logsigmoid(sc);
        } else if (a.layout == BSA_SEL_RAW) {
          a.sel[ob + l] = id;
        } else {
          scratch[l] = id >= 0 ? id : qi;
        }
      }
      if (a.layout == BSA_SEL_SSA) {
        a.sel[ob] = qi;
        if (a.score_out) a.score_out[ob] = own;
        if (a.gate_out) a.gate_out[ob] = logsigmoid(own);
      } else if (a.layout == BSA_SEL_FINISH) {
        scratch[T] = qi;
        if (a.sink) scratch[T + 1] = 0;
        // insertion sort ascending (W <= 34)
        for (int x = 1; x < W; ++x) {
          const int v = scratch[x];
          int y = x - 1;
          while (y >= 0 && scratch[y] > v) {
            scratch[y + 1] = scratch[y];
            --y;
          }
          scratch[y + 1] = v;
        }
        for (int x = 0; x < W; ++x) a.sel[ob + x] = scratch[x];
      }
    }
  }
  __syncthreads();
  if (C > 1) cluster_sync();  // CTA 0 has finished reading the other lists
  if (warp == 5) {
    tc05::fence_after();
    tc05::dealloc(tmem, kTmemCols);
  }
}

}  // namespace s5

// Used by run_select: the tensor-core path serves DOT scores with dim 32 or 64, 1 <= T <= 32, and enough key blocks for the tensor cores to pay off.
bool select_tc5_applicable(const bsa_select_args *a, int T) {
  if (getenv("BSA_SELECT_SIMT")) return false;
  // measured against the fp32 SIMT kernel: ahead from 4096 key blocks (262k
  // tokens of block 64: 0.18 against 0.45 ms for one head, 0.67 against 0.72 for
  // eight); BSA_SELECT_TC5=1 forces this path from 512 key blocks up
  const int min_nblk = getenv("BSA_SELECT_TC5") ? 512 : 4096;
  return a->score_kind == BSA_SCORE_DOT && (a->dim == 32 || a->dim == 64) &&
         T >= 1 && T <= s5::kMaxT && a->nblk >= min_nblk &&
         reinterpret_cast<uintptr_t>(a->a) % 16 == 0 && reinterpret_cast<uintptr_t>(a->b1) % 16 == 0;
}

bsa_status run_select_tc5(const bsa_select_args *a, int T, int W, cudaStream_t st) {
  using namespace s5;
  const int nq = a->nq > 0 ? a->nq : a->nblk;
  CUtensorMap ma, mb;
  if (bsa_status s = make_tmap_f32_rows(&ma, a->a, a->G, nq, a->dim, kM, "select a")) return s;
  if (bsa_status s = make_tmap_f32_rows(&mb, a->b1, a->G, a->nblk, a->dim, kN, "select b")) return s;
  const int nqt = (nq + kM - 1) / kM, nkt = (a->nblk + kN - 1) / kN;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  // split the key tiles of a query tile over C CTAs when there are too few
  // query tiles to fill the SMs (one resident CTA per SM); measured on B200:
  // clusters of 4 fill best, clusters of 8 schedule worse than 4
  int C = 1;
  while (C < 4 && (long long)nqt * a->G * C * 2 <= nsm && C * 2 <= std::max(1, nkt / 2)) C *= 2;
  if (const char *e = getenv("BSA_SELECT_SPLIT")) C = std::max(1, std::min(8, atoi(e)));
  const int smem = layout(a->dim).total + 1024;
  void (*kern)(const CUtensorMap, const CUtensorMap, const bsa_select_args, int, int, int) = nullptr;
  const int kt = T <= 8 ? 8 : (T <= 16 ? 16 : 32);
#define BSA_S5_PICK(D_)                                        \
  kern = kt == 8 ? select_tc5_kernel<D_, 8>                    \
                 : (kt == 16 ? select_tc5_kernel<D_, 16> : select_tc5_kernel<D_, 32>);
  if (a->dim == 32) {
    BSA_S5_PICK(32)
  } else {
    BSA_S5_PICK(64)
  }
#undef BSA_S5_PICK
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(nqt * C), (unsigned)a->G, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, ma, mb, *a, T, W, C) != cudaSuccess)
    return check_launch("select_tc5");
  return check_launch("select_tc5");
}

}  // namespace bsa
