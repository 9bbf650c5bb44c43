// Block-sparse attention backward, dK/dV part, on tcgen05 for block 64,
// head dim 64.
//
// One CTA processes two dK/dV work items (tiles A and B): consecutive chunks of
// the key-block CSR plan, each a key block of one KV head with up to 32 listed
// (query block, slot) entries.  The key block's K and V stay in shared memory
// as the stationary A operands; the listed query blocks stream through a
// 5-stage ring (Q, dO by TMA, lse and Dvec rows by bulk copy).
//
// Per step j (one entry and query head of each tile):
//   S^T  = K  Q_j^T    dP^T = V dO_j^T         (tcgen05, fp32 in TMEM, 3 buffers)
//   P^T  = 2^(S^T*scale*log2e + gate - lse_j)  dS^T = P^T (dP^T - Dvec_j)
//   dV  += P^T dO_j    dK  += dS^T Q_j          (tcgen05, A operand in TMEM)
// P^T and dS^T (16-bit pairs) are written back over the step's own S^T and dP^T
// columns, so they are double-buffered with them and need no shared memory.
// The two tiles run as independent pipelines: each has its own S/dP buffers,
// hand-off barriers, dK/dV accumulators and MMA-issuing thread; they share
// only the ring stage and the K/V buffer.
//
// Warp roles (352 threads, one CTA per SM):
//   warps 0-3  elementwise for tile A, warps 4-7 for tile B: each warp owns the
//              tile's 16 TMEM lanes of its quadrant (16x32bx2 loads and
//              stores), writes P^T / dS^T to TMEM, dS^T rows to global memory
//              for the dQ pass, and the final dK / dV.
//   warp 8     TMA producer: the warp reads a unit's CSR entries and gate values
//              at once, then one thread publishes the unit to the other warps
//              and issues the ring loads.
//   warp 9     TMEM allocation (512 columns) and tile A's MMA-issuing thread,
//   warp 10    tile B's MMA-issuing thread; each polls its tile's S/dP queue
//              and dV/dK queue.  (One thread for both tiles was the bottleneck:
//              issuing 32 MMAs and polling took ~3.7k cycles per step.)
// TMEM columns: S^T [0,192) and dP^T [192,384) in three 64-column buffers, dV
// [384,448), dK [448,512); tile B at lane offset 16.
#include <algorithm>
#include <type_traits>

#include "bsa_attn.cuh"
#include "bsa_host.h"
#include "bsa_tc05.cuh"

namespace bsa {

namespace {
constexpr int B5_BS = 64, B5_D = 64;
constexpr int B5_TILE = B5_BS * B5_D * 2;            // 8 KB
constexpr int B5_ROWB = B5_BS * 4;                   // one lse / Dvec row chunk
// NKV K/V buffers, NST ring stages
constexpr int b5_smem(int NST, int NKV) {
  return 1024 + NKV * 4 * B5_TILE    // K, V of both tiles
         + NST * 4 * B5_TILE         // ring: (stage, tile) Q, dO
         + NST * 2 * 2 * B5_ROWB;    // ring: (stage, tile) lse, Dvec
}
constexpr uint32_t B5_TMEM_COLS = 512;
// TMEM: NSB buffers of S^T (P^T) and of dP^T (dS^T), NAB dV/dK accumulator pairs
constexpr int B5_NSB = 3, B5_NAB = 1;
static_assert(128 * B5_NSB + 128 * B5_NAB == (int)B5_TMEM_COLS, "TMEM columns");
constexpr int B5_SCOL = 0, B5_DPCOL = 64 * B5_NSB, B5_DVCOL = 128 * B5_NSB, B5_DKCOL = B5_DVCOL + 64;
}  // namespace

// Work unit u -> (two chunks of the plan, KV head within the bin group).
struct B5Unit {
  int n[2], kb[2], b[2], hk[2], ebeg[2], nch[2], cidx[2], poff[2];
  bool valid[2];
};

__device__ __forceinline__ void b5_unit(const BwdPlan &pl, const AttnParams &p, unsigned total,
                                        int u, B5Unit &w) {
  const unsigned x0 = 2u * (unsigned)(u / pl.Y);
  const int y = u % pl.Y;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const unsigned xs = x0 + t;
    w.valid[t] = xs < total;
    w.n[t] = 0;
    w.kb[t] = w.b[t] = w.hk[t] = w.ebeg[t] = w.cidx[t] = w.poff[t] = 0;
    w.nch[t] = 1;
    if (!w.valid[t]) continue;
    const unsigned x = pl.chunk_ord ? (unsigned)pl.chunk_ord[xs] : xs;
    const int bin = pl.chunk_bin[x];
    const unsigned coff = (unsigned)(pl.plan[bin] >> 32);
    w.poff[t] = (int)(pl.plan[bin] & 0xffffffffu);
    w.nch[t] = (int)((unsigned)(pl.plan[bin + 1] >> 32) - coff);
    w.cidx[t] = (int)(x - coff);
    w.ebeg[t] = pl.row_ptr[bin] + w.cidx[t] * pl.C;
    const int ee = min(pl.row_ptr[bin + 1], w.ebeg[t] + pl.C);
    w.n[t] = (ee - w.ebeg[t]) * p.grp;
    w.kb[t] = bin % p.nblk;
    w.b[t] = bin / (p.nblk * pl.Hs);
    w.hk[t] = ((bin / p.nblk) % pl.Hs) * pl.Y + y;
  }
}

// GATE: a gate tensor is present (without one the exponent's offset is -lse, which
// folds into the FMA)
template <typename T, int B5_NST, int NKV, bool GATE>
__global__ void __launch_bounds__(352, 1)
    attn_dkdv_sm100_kernel(const __grid_constant__ CUtensorMap tq,
                           const __grid_constant__ CUtensorMap tdo,
                           const __grid_constant__ CUtensorMap tk,
                           const __grid_constant__ CUtensorMap tv, const int perm_q,
                           const int perm_do, const int perm_k, const int perm_v,
                           const AttnParams p, const BwdPlan pl) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_KK = tc05::idesc_f16(kBF16, 64, 64, false);  // both K-major
  constexpr uint32_t IDESC_KM = tc05::idesc_f16(kBF16, 64, B5_D, true);  // B MN-major
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sKV = smem;                       // (buffer, tile): K, V
  uint8_t *sR = sKV + NKV * 4 * B5_TILE;     // (stage, tile): Q, dO
  float *sRow = reinterpret_cast<float *>(sR + B5_NST * 4 * B5_TILE);  // (stage, tile): lse[64], Dvec[64]
  // per tile and TMEM buffer b (the step's parity): s_full (S^T, dP^T computed),
  // p_full (P^T, dS^T written over them), s_empty (the step's dV/dK MMAs, the
  // last readers of the buffer, are done)
  __shared__ __align__(8) uint64_t kv_full[NKV], kv_empty[NKV], r_full[B5_NST], r_empty[B5_NST],
      s_full[2][B5_NSB], s_empty[2][B5_NSB], p_full[2][B5_NSB], acc_empty[2][B5_NAB];
  __shared__ uint32_t tmem_base_sh;
  // per ring stage and tile: (local query block, slot, query head) and the gate
  // value of the step, written by the producer before it arrives on r_full
  __shared__ int s_meta[B5_NST][2][3];
  // per non-empty work unit (ring of 8, indexed by the unit's ordinal): the two
  // tiles' step counts and max(n0, n1), -1 after the last unit; written by the
  // producer before it arms the unit's K/V barrier, read by the MMA issuer
  __shared__ int s_unit[8][3];
  // every work unit (ring of 8, indexed by the unit's position in this CTA's
  // sequence) for the elementwise warps, per tile: steps, key block, batch,
  // KV head, valid, chunks of the bin, partial index base; and (u mod Y)
  __shared__ int s_eu[8][2][7];
  __shared__ int s_euy[8];
  __shared__ __align__(8) uint64_t eu_full[8], eu_empty[8];
  __shared__ float s_g2[B5_NST][2];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned total = (unsigned)(pl.plan[pl.nbins] >> 32);
  const int nunits = (int)((total + 1) / 2) * pl.Y;

  if (tid == 0) {
    // descriptors fetched ahead of the first TMA load
    prefetch_tmap(&tq);
    prefetch_tmap(&tdo);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    // per tile t: s_full/p_full/s_empty (S^T, dP^T buffers and the P^T, dS^T
    // written over them), acc_empty (dK/dV accumulators); the ring stage and the K/V buffer are
    // released by both tiles' MMAs (two commits each)
    for (int s = 0; s < NKV; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 2);
    }
    for (int t = 0; t < 2; ++t) {
      for (int s = 0; s < B5_NSB; ++s) {
        mbar_init(&s_full[t][s], 1);
        mbar_init(&s_empty[t][s], 1);
        mbar_init(&p_full[t][s], 128);
      }
      for (int s = 0; s < B5_NAB; ++s) mbar_init(&acc_empty[t][s], 128);
    }
    for (int s = 0; s < B5_NST; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], 2);
    }
    for (int s = 0; s < 8; ++s) {
      mbar_init(&eu_full[s], 1);
      mbar_init(&eu_empty[s], 8);  // lane 0 of each elementwise warp
    }
    fence_mbar_init();
  }
  if (warp == 9) {
    tc05::alloc(&tmem_base_sh, B5_TMEM_COLS);
    tc05::relinquish();
  }
  tc05::fence_before();
  __syncthreads();
  tc05::fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 8) {
    // ================= producer: K/V per unit (2 buffers), Q/dO/lse/Dvec per step (ring).
    // The whole warp reads a unit's CSR entries (<= 32 per tile) and gate values
    // at once; one elected lane then issues the loads step by step from shared
    // memory while the warp waits with it.
    __shared__ int s_pq[2][32], s_ps[2][32];
    __shared__ float s_pg[2][32];
    int gs = 0, ne = 0, iu = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++iu) {
      B5Unit w;
      b5_unit(pl, p, total, u, w);
      const int ns = max(w.n[0], w.n[1]);
      if (w.b[0] < 0 || w.b[0] >= p.B || w.b[1] < 0 || w.b[1] >= p.B) {
        report(p.status, BSA_DEVERR_INDEX);  // self-check: keep every address in range
        w.b[0] = w.b[1] = 0;
      }
      if (lane == 0) {
        // publish the unit to the elementwise warps (every unit, empty ones too:
        // their valid tiles still write zero dK / dV)
        const int eb = iu & 7;
        if (iu >= 8 && !mbar_wait(&eu_empty[eb], ((iu >> 3) - 1) & 1))
          report(p.status, BSA_DEVERR_TIMEOUT);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          s_eu[eb][t][0] = w.n[t];
          s_eu[eb][t][1] = w.kb[t];
          s_eu[eb][t][2] = w.b[t];
          s_eu[eb][t][3] = w.hk[t];
          s_eu[eb][t][4] = w.valid[t];
          s_eu[eb][t][5] = w.nch[t];
          s_eu[eb][t][6] = w.poff[t] + w.cidx[t];
        }
        s_euy[eb] = u % pl.Y;
        tc05::mbar_arrive(&eu_full[eb]);
      }
      if (ns == 0) continue;
      __syncwarp();  // lane 0 is done with the previous unit's entries
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (lane < w.n[t] / p.grp) {
          int ci = w.ebeg[t] + lane;
          if (ci < 0 || ci >= pl.ncol) {  // self-check: never read outside the CSR list
            report(p.status, BSA_DEVERR_INDEX);
            ci = 0;
          }
          const int e = pl.col[ci];
          int qblk = e / p.kk, slot = e - (e / p.kk) * p.kk;
          if (qblk < 0 || qblk >= p.nq) {
            report(p.status, BSA_DEVERR_INDEX);
            qblk = slot = 0;
          }
          s_pq[t][lane] = qblk;
          s_ps[t][lane] = slot;
          s_pg[t][lane] = p.gate ? __ldg(p.gate + w.b[t] * p.gate_sb + w.hk[t] * p.gate_sh +
                                         (long long)qblk * p.gate_sn + slot) * kLog2e
                                 : 0.f;
        }
      }
      __syncwarp();
      // the loads are issued by one elected lane (lane 0); the warp stays
      // converged so that the waits and addresses are warp-uniform
      const int kvb = ne % NKV;
      // K/V buffer: the earlier unit's last S/dP MMAs on it must be done
      if (ne >= NKV && !mbar_wait_warp(&kv_empty[kvb], ((ne / NKV) - 1) & 1))
        report(p.status, BSA_DEVERR_TIMEOUT);
      if (tc05::elect_one()) {
        s_unit[ne & 7][0] = w.n[0];
        s_unit[ne & 7][1] = w.n[1];
        s_unit[ne & 7][2] = ns;
        mbar_expect_tx(&kv_full[kvb], ((w.n[0] > 0) + (w.n[1] > 0)) * 2 * B5_TILE);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (w.n[t] == 0) continue;
          uint8_t *dst = sKV + (kvb * 2 + t) * 2 * B5_TILE;
          tma_load_rhb(dst, &tk, &kv_full[kvb], perm_k, 0, w.kb[t] * p.bs, w.hk[t], w.b[t]);
          tma_load_rhb(dst + B5_TILE, &tv, &kv_full[kvb], perm_v, 0, w.kb[t] * p.bs, w.hk[t], w.b[t]);
        }
      }
      __syncwarp();
      ++ne;
      for (int j = 0; j < ns; ++j, ++gs) {
        const int st = gs % B5_NST;
        if (gs >= B5_NST && !mbar_wait_warp(&r_empty[st], ((gs / B5_NST) - 1) & 1))
          report(p.status, BSA_DEVERR_TIMEOUT);
        if (tc05::elect_one()) {
          const int act = (j < w.n[0]) + (j < w.n[1]);
          int mq[2], mh[2];
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (j >= w.n[t]) continue;
            const int en = j / p.grp;
            const int qblk = s_pq[t][en], h = w.hk[t] * p.grp + (j - en * p.grp);
            mq[t] = qblk;
            mh[t] = h;
            s_meta[st][t][0] = qblk;
            s_meta[st][t][1] = s_ps[t][en];
            s_meta[st][t][2] = h;
            s_g2[st][t] = s_pg[t][en];
          }
          // the arrive below releases the metadata stores to the r_full waiters
          mbar_expect_tx(&r_full[st], act * (2 * B5_TILE + 2 * B5_ROWB));
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (j >= w.n[t]) continue;
            const int qblk = mq[t], h = mh[t];
            const int row = qblk * p.bs;
            uint8_t *dst = sR + (st * 2 + t) * 2 * B5_TILE;
            tma_load_rhb(dst, &tq, &r_full[st], perm_q, 0, row, h, w.b[t]);
            tma_load_rhb(dst + B5_TILE, &tdo, &r_full[st], perm_do, 0, row, h, w.b[t]);
            const long long rb = ((long long)w.b[t] * p.Hq + h) * p.Lp + row;
            float *rw = sRow + (st * 2 + t) * 2 * B5_BS;
            bulk_load(rw, p.lse + rb, B5_ROWB, &r_full[st]);
            bulk_load(rw + B5_BS, p.dvec + rb, B5_ROWB, &r_full[st]);
          }
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      // end of the unit sequence for the MMA issuer
      const int kvb = ne % NKV;
      if (ne >= NKV && !mbar_wait(&kv_empty[kvb], ((ne / NKV) - 1) & 1))
        report(p.status, BSA_DEVERR_TIMEOUT);
      s_unit[ne & 7][0] = s_unit[ne & 7][1] = 0;
      s_unit[ne & 7][2] = -1;
      tc05::mbar_arrive(&kv_full[kvb]);
    }
  } else if (warp >= 9) {
    // ================= MMA issuers: warp 9 for tile A, warp 10 for tile B, each
    // polling the tile's S/dP queue and its dV/dK queue (tcgen05.commit tracks
    // the issuing thread's own MMAs; the shared ring stage and K/V buffer are
    // released by one commit of each).  The whole warp runs the loop, so the
    // descriptors stay warp-uniform; barrier tests are made uniform by a vote and
    // one elected lane (always lane 0) issues the MMAs and commits.
    {
      const int t = warp - 9;
      auto test = [&](uint64_t *bar, uint32_t par) {
        return __any_sync(0xffffffffu, mbar_test(bar, par));
      };
      // descriptors built once; per MMA only a 64-bit add
      const uint64_t dkv0 = tc05::sdesc(smem_u32(sKV), 16, 1024);          // K, V (A, K-major)
      const uint64_t drk0 = tc05::sdesc(smem_u32(sR), 16, 1024);           // Q, dO as K-major B
      const uint64_t drm0 = tc05::sdesc(smem_u32(sR), B5_BS * 128, 1024);  // Q, dO as MN-major B
      // S queue (js, gss, nes) and G queue (jg, gsg, neg); the units (ordinals
      // ne = 0, 1, ...) come from the producer's s_unit ring: the S queue opens
      // unit nes once its K/V barrier has completed
      int js = 0, gss = 0, nes = 0, jg = 0, gsg = 0, neg = 0;
      int sn = 0, gn = 0, sns = 0, gns = 0;  // tile length and unit length of the current units
      bool s_open = false, have_s = true, have_g = true;
      uint32_t idle = 0;
      while (have_g) {
        bool progress = false;
        // ---- open the next unit of the S queue once its K/V have landed
        if (have_s && !s_open && test(&kv_full[nes % NKV], (nes / NKV) & 1)) {
          sns = s_unit[nes & 7][2];
          sn = s_unit[nes & 7][t];
          if (sns < 0) {
            have_s = false;
          } else {
            s_open = true;
          }
          progress = true;
        }
        // ---- dV += P^T dO, dK += dS^T Q, step gsg (its unit neg was opened by
        // the S queue, which runs ahead)
        if (gsg < gss && test(&p_full[t][gsg % B5_NSB], (gsg / B5_NSB) & 1) &&
            (jg > 0 || neg < B5_NAB ||
             test(&acc_empty[t][neg % B5_NAB], ((neg / B5_NAB) - 1) & 1))) {
          if (jg == 0) {
            gns = s_unit[neg & 7][2];
            gn = s_unit[neg & 7][t];
          }
          const int st = gsg % B5_NST, ab = neg % B5_NAB, bb = gsg % B5_NSB;
          tc05::fence_after();
          if (jg < gn) {
            const uint32_t roff = (st * 2 + t) * 2 * B5_TILE;  // Q; dO at + TILE
            const uint64_t bdo = tc05::dadd(drm0, roff + B5_TILE), bq = tc05::dadd(drm0, roff);
            // P^T and dS^T (16-bit pairs) over the step's S^T and dP^T columns
            const uint32_t ap = tc05::taddr(tmem, 16 * t, B5_SCOL + 64 * bb);
            const uint32_t ads = tc05::taddr(tmem, 16 * t, B5_DPCOL + 64 * bb);
            const uint32_t dv = tc05::taddr(tmem, 16 * t, B5_DVCOL + 128 * ab);
            const uint32_t dk = tc05::taddr(tmem, 16 * t, B5_DKCOL + 128 * ab);
            if (tc05::elect_one()) {
#pragma unroll
              for (int ks = 0; ks < B5_BS / 16; ++ks) {
                const uint32_t acc = (jg > 0 || ks > 0) ? 1u : 0u;
                tc05::mma_f16_ts(dv, ap + ks * 8, tc05::dadd(bdo, ks * 2048), IDESC_KM, acc);
                tc05::mma_f16_ts(dk, ads + ks * 8, tc05::dadd(bq, ks * 2048), IDESC_KM, acc);
              }
            }
            __syncwarp();
          }
          if (tc05::elect_one()) {
            tc05::commit(&r_empty[st]);  // count 2: the stage is free once both tiles are done
            tc05::commit(&s_empty[t][bb]);
          }
          __syncwarp();
          ++gsg;
          if (++jg == gns) {
            jg = 0;
            ++neg;
          }
          progress = true;
        } else if (!have_s && gsg == gss) {
          have_g = false;  // every opened step is done and no unit follows
        }
        // ---- S^T = K Q^T, dP^T = V dO^T, step gss
        if (s_open && test(&r_full[gss % B5_NST], (gss / B5_NST) & 1) &&
            (gss < B5_NSB || test(&s_empty[t][gss % B5_NSB], ((gss / B5_NSB) - 1) & 1))) {
          const int st = gss % B5_NST, bb = gss % B5_NSB;
          tc05::fence_after();
          if (js < sn) {
            const uint32_t roff = (st * 2 + t) * 2 * B5_TILE;           // Q; dO at + TILE
            const uint32_t koff = ((nes % NKV) * 2 + t) * 2 * B5_TILE;  // K; V at + TILE
            const uint64_t ak = tc05::dadd(dkv0, koff), av = tc05::dadd(dkv0, koff + B5_TILE);
            const uint64_t bq = tc05::dadd(drk0, roff), bdo = tc05::dadd(drk0, roff + B5_TILE);
            const uint32_t ds = tc05::taddr(tmem, 16 * t, B5_SCOL + 64 * bb);
            const uint32_t ddp = tc05::taddr(tmem, 16 * t, B5_DPCOL + 64 * bb);
            if (tc05::elect_one()) {
#pragma unroll
              for (int ks = 0; ks < B5_D / 16; ++ks) {
                tc05::mma_f16(ds, tc05::dadd(ak, ks * 32), tc05::dadd(bq, ks * 32), IDESC_KK, ks > 0);
                tc05::mma_f16(ddp, tc05::dadd(av, ks * 32), tc05::dadd(bdo, ks * 32), IDESC_KK, ks > 0);
              }
            }
            __syncwarp();
          }
          const bool last = js + 1 == sns;
          if (tc05::elect_one()) {
            tc05::commit(&s_full[t][bb]);
            if (last) tc05::commit(&kv_empty[nes % NKV]);  // count 2: last readers of the K/V buffer
          }
          __syncwarp();
          ++gss;
          if (++js == sns) {
            js = 0;
            ++nes;
            s_open = false;
          }
          progress = true;
        }
        if (progress) {
          idle = 0;
        } else {
          if (++idle > kSpinLimit) {
            report(p.status, BSA_DEVERR_TIMEOUT);
            break;
          }
          __nanosleep(20);
        }
      }
    }
  } else {
    // ================= elementwise warps 0-7: warps 0-3 tile A, warps 4-7 tile B,
    // so that the two tiles' steps run as independent pipelines.  Each warp
    // reads its tile's 16 TMEM lanes of its quadrant (16x32bx2 loads): thread
    // (lane) = key row quad*16 + (lane & 15), 16 query columns at
    // 32*g + 16*(lane >> 4) for g = 0, 1.
    const int quad = warp & 3, t = warp >> 2, hh = lane >> 4;
    const int kr = quad * 16 + (lane & 15);  // key row within the block
    const uint32_t lane_base = (uint32_t)(quad * 32 + 16 * t) << 16;
    int gs = 0, ne = 0, iu = 0;
    uint64_t evict_first;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(evict_first));
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++iu) {
      // the unit as the producer published it
      const int eb = iu & 7;
      if (!mbar_wait(&eu_full[eb], (iu >> 3) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
      const int ns = max(s_eu[eb][0][0], s_eu[eb][1][0]);
      const int nmine = s_eu[eb][t][0], kb = s_eu[eb][t][1];
      const int b = s_eu[eb][t][2], hk = s_eu[eb][t][3];
      const bool wvalid = s_eu[eb][t][4] != 0;
      const int wnch = s_eu[eb][t][5];
      const int wpc = s_eu[eb][t][6];
      const int uy = s_euy[eb];
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&eu_empty[eb]);
      const bool key_ok = (long long)kb * p.bs + kr < p.L;
      for (int j = 0; j < ns; ++j, ++gs) {
        const int bb = gs % B5_NSB, st = gs % B5_NST;
        if (!mbar_wait(&s_full[t][bb], (gs / B5_NSB) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        // acquire the stage's TMA / bulk data and the producer's metadata
        if (!mbar_wait(&r_full[st], (gs / B5_NST) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
        uint32_t wp[16], wd[16];
        const bool active = j < nmine;
        const int qblk = s_meta[st][t][0], slot = s_meta[st][t][1];
        // qblk is the local query block; kb is global
        const bool triu = p.causal && ((p.mask_mode == BSA_MASK_SLOT) ? slot == 0 : kb == p.q0 + qblk);
        const float g2 = GATE ? s_g2[st][t] : 0.f;
        const float *lsep = sRow + (st * 2 + t) * 2 * B5_BS;
        float sv[2][16], dp[2][16];
        // all four TMEM loads in flight before one wait
        tc05::ld16x2(tmem + lane_base + B5_SCOL + 64 * bb, sv[0]);
        tc05::ld16x2(tmem + lane_base + B5_DPCOL + 64 * bb, dp[0]);
        tc05::ld16x2(tmem + lane_base + B5_SCOL + 64 * bb + 32, sv[1]);
        tc05::ld16x2(tmem + lane_base + B5_DPCOL + 64 * bb + 32, dp[1]);
        tc05::wait_ld();
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const int cg = 32 * g + 16 * hh;  // first query column of this group
          if (active) {
            const long long q0 = (long long)qblk * p.bs + cg;
            if (triu || !key_ok || q0 + 16 > p.Lq) {  // diagonal / padded steps: explicit masks
#pragma unroll
              for (int c = 0; c < 16; ++c)
                if (!key_ok || (triu && kr > cg + c) || q0 + c >= p.Lq) sv[g][c] = -INFINITY;
            }
            // pairs of columns through the packed f32x2 pipe (same per-element
            // rounding as the scalar sequence)
            const float2 s22 = make_float2(p.scale2, p.scale2), g22 = make_float2(g2, g2);
#pragma unroll
            for (int c = 0; c < 16; c += 4) {
              const float4 a4 = *reinterpret_cast<const float4 *>(lsep + cg + c);
              const float4 d4 = *reinterpret_cast<const float4 *>(lsep + B5_BS + cg + c);
              const float *x = sv[g], *y = dp[g];
              const float2 e01 = fma2(make_float2(x[c], x[c + 1]), s22,
                                      sub2(g22, make_float2(a4.x, a4.y)));
              const float2 e23 = fma2(make_float2(x[c + 2], x[c + 3]), s22,
                                      sub2(g22, make_float2(a4.z, a4.w)));
              const float2 p01 = make_float2(ex2(e01.x), ex2(e01.y));
              const float2 p23 = make_float2(ex2(e23.x), ex2(e23.y));
              const float2 d01 = mul2(p01, sub2(make_float2(y[c], y[c + 1]), make_float2(d4.x, d4.y)));
              const float2 d23 = mul2(p23, sub2(make_float2(y[c + 2], y[c + 3]), make_float2(d4.z, d4.w)));
              const int o = 8 * g + (c >> 1);
              wp[o] = Mma<T>::pack(p01.x, p01.y);
              wp[o + 1] = Mma<T>::pack(p23.x, p23.y);
              wd[o] = Mma<T>::pack(d01.x, d01.y);
              wd[o + 1] = Mma<T>::pack(d23.x, d23.y);
            }
          }
        }
        if (active) {
          // P^T / dS^T over the S^T / dP^T columns just read (this warp's loads of
          // all 64 columns have completed): query column c -> column c / 2
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            tc05::st16x2_8(tmem + lane_base + B5_SCOL + 64 * bb + 16 * g, wp + 8 * g);
            tc05::st16x2_8(tmem + lane_base + B5_DPCOL + 64 * bb + 16 * g, wd + 8 * g);
          }
          tc05::wait_st();
        }
        tc05::fence_before();
        tc05::mbar_arrive(&p_full[t][bb]);
        if (p.ds && active) {
          // dS^T row of this key for the dQ pass (2 x 16 query columns), after the
          // MMA hand-off; evict-first so that the stream of dS tiles does not
          // push the gathered Q / dO rows out of L2
          const int hq = s_meta[st][t][2];
          T *dst = reinterpret_cast<T *>(p.ds) +
                   (((((long long)b * p.Hq + hq) * p.nq + qblk) * p.kk + slot) * B5_BS + kr) * B5_BS;
#pragma unroll
          for (int g = 0; g < 2; ++g)
#pragma unroll
            for (int c8 = 0; c8 < 2; ++c8) {
              const int o = 8 * g + 4 * c8;
              asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1,%2,%3,%4}, %5;" ::"l"(
                               dst + 32 * g + 16 * hh + 8 * c8),
                           "r"(wd[o]), "r"(wd[o + 1]), "r"(wd[o + 2]), "r"(wd[o + 3]),
                           "l"(evict_first)
                           : "memory");
            }
        }
      }
      // ---- dK (scaled) and dV of this unit: this thread's row, its two 16-column
      // groups, one accumulator at a time
      const int ab = ne % B5_NAB;
      if (ns > 0) {
        const int gl = gs - 1;  // last step of this unit
        if (!mbar_wait(&s_empty[t][gl % B5_NSB], (gl / B5_NSB) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
      }
      long long pidx = -1;
      if (wvalid && wnch > 1) {
        pidx = (long long)wpc * pl.Y + uy;
        if (pidx < 0 || pidx >= pl.npart * pl.Y) {  // self-check: partial tile in range
          report(p.status, BSA_DEVERR_INDEX);
          pidx = -2;
        }
      }
#pragma unroll 1
      for (int m = 0; m < 2; ++m) {  // 0: dK, 1: dV
        float acc[2][16];
        if (ns > 0) {
          tc05::ld16x2(tmem + lane_base + (m ? B5_DVCOL : B5_DKCOL) + 128 * ab, acc[0]);
          tc05::ld16x2(tmem + lane_base + (m ? B5_DVCOL : B5_DKCOL) + 128 * ab + 32, acc[1]);
          tc05::wait_ld();
          if (m == 1) {
            tc05::fence_before();
            tc05::mbar_arrive(&acc_empty[t][ab]);
          }
        }
        if (!wvalid) continue;
        if (nmine == 0) {
#pragma unroll
          for (int c = 0; c < 16; ++c) acc[0][c] = acc[1][c] = 0.f;
        }
        if (wnch == 1) {
          const long long gk = (long long)kb * p.bs + kr;
          if (gk < p.L) {
            const float sc = m ? 1.f : p.scale;
            T *dst = m ? reinterpret_cast<T *>(p.dv) + b * p.dv_sb + hk * p.dv_sh + gk * p.dv_sl
                       : reinterpret_cast<T *>(p.dk) + b * p.dk_sb + hk * p.dk_sh + gk * p.dk_sl;
#pragma unroll
            for (int g = 0; g < 2; ++g)
#pragma unroll
              for (int c = 0; c < 16; c += 8) {
                uint4 a4;
                a4.x = Mma<T>::pack(acc[g][c] * sc, acc[g][c + 1] * sc);
                a4.y = Mma<T>::pack(acc[g][c + 2] * sc, acc[g][c + 3] * sc);
                a4.z = Mma<T>::pack(acc[g][c + 4] * sc, acc[g][c + 5] * sc);
                a4.w = Mma<T>::pack(acc[g][c + 6] * sc, acc[g][c + 7] * sc);
                *reinterpret_cast<uint4 *>(dst + 32 * g + 16 * hh + c) = a4;
              }
          }
        } else if (pidx >= 0) {
          float *part = pl.part + pidx * (2LL * B5_BS * B5_D) + m * (B5_BS * B5_D);
#pragma unroll
          for (int g = 0; g < 2; ++g)
#pragma unroll
            for (int c = 0; c < 16; c += 4)
              *reinterpret_cast<float4 *>(part + kr * B5_D + 32 * g + 16 * hh + c) =
                  make_float4(acc[g][c], acc[g][c + 1], acc[g][c + 2], acc[g][c + 3]);
        }
      }
      if (ns > 0) ++ne;
    }
  }
  tc05::fence_before();
  __syncthreads();
  if (warp == 9) {
    tc05::fence_after();
    tc05::dealloc(tmem, B5_TMEM_COLS);
  }
}

// ------------------------------------------------------------------ launcher
bool dkdv_sm100_applicable(int dtype, int bs, int D) {
  return dtype != BSA_F32 && bs == 64 && D == 64 && !getenv("BSA_BWD_LEGACY");
}

bsa_status launch_dkdv_sm100(int dtype, const CUtensorMap &mq, const CUtensorMap &mdo,
                             const CUtensorMap &mk, const CUtensorMap &mv, int pq, int pdo, int pk,
                             int pv, const AttnParams &p, const BwdPlan &pl, long long dkv_grid,
                             cudaStream_t st) {
  // persistent: one CTA per SM (the unit count is only known on the device)
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const long long units_max = ((dkv_grid + 1) / 2) * pl.Y;
  const unsigned grid = (unsigned)std::max<long long>(1, std::min<long long>(nsm, units_max));
  // ring stages: 5 by default, BSA_DKDV_STAGES=4 for 4
  const char *cfg = getenv("BSA_DKDV_STAGES");
  const int variant = cfg ? atoi(cfg) : 5;
#define BSA_B5_LAUNCH(T_, N_, KV_)                                                          \
  {                                                                                         \
    auto kern = p.gate ? attn_dkdv_sm100_kernel<T_, N_, KV_, true>                          \
                       : attn_dkdv_sm100_kernel<T_, N_, KV_, false>;                        \
    constexpr int sm = b5_smem(N_, KV_);                                                    \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);            \
    kern<<<grid, 352, sm, st>>>(mq, mdo, mk, mv, pq, pdo, pk, pv, p, pl);                   \
  }
#define BSA_B5_PICK(T_)                                      \
  if (variant == 4) BSA_B5_LAUNCH(T_, 4, 1)                  \
  else if (variant == 42) BSA_B5_LAUNCH(T_, 4, 2)            \
  else BSA_B5_LAUNCH(T_, 5, 1)
  if (dtype == BSA_BF16) {
    BSA_B5_PICK(__nv_bfloat16)
  } else {
    BSA_B5_PICK(__half)
  }
#undef BSA_B5_PICK
#undef BSA_B5_LAUNCH
  return check_launch("attn_dkdv_sm100");
}

}  // namespace bsa
