// Block-sparse attention backward, dQ part, on tcgen05 for block 64, head dim
// 64, organised like the forward kernel: one CTA per pair of adjacent query
// blocks (tiles A and B) of one head, two CTAs per SM.
//
// Per live slot j of each tile (tiles advance together; a tile with fewer live
// slots idles on its last steps):
//   S_j  = Q K_j^T,  dP_j = dO V_j^T        (tcgen05 64x64x16 chains into TMEM)
//   P    = 2^(S_j * scale * log2e + gate - lse)   (lse of the forward, per row)
//   dS   = P (dP_j - Dvec)                   (Dvec = rowsum(dO * O), per row)
//   dQ  += dS K_j                            (tcgen05, dQ accumulated in TMEM)
//   dgate[slot] += sum(dS)                   (fp32, fixed reduction order)
// TMEM: S [0,64), dP [64,128), dQ [128,192) with tile B at lane offset 16
// (256 columns allocated).  Shared memory: Q, dO of both tiles, a 2-stage K
// ring (K_j is read by S_j and by dQ_j), a 1-stage V ring (V_j only by dP_j),
// dS of both tiles.
//
// Warp roles (192 threads):
//   warps 0-3  elementwise: one query row per thread (lanes 0-15 tile A, 16-31
//              tile B), 32 columns at a time; dS (bf16) -> shared memory in the
//              128B-swizzled K-major layout; final dQ * scale and dgate.
//   warp 4     TMA producer (one thread, polls both rings).
//   warp 5     TMEM owner and MMA-issuing thread (polls the S/dP and dQ queues).
// Every wait is bounded; a timeout sets BSA_DEVERR_TIMEOUT.
#include <type_traits>

#include "bsa_attn.cuh"
#include "bsa_host.h"
#include "bsa_tc05.cuh"

namespace bsa {

namespace {
constexpr int D5_BS = 64, D5_D = 64, D5_KST = 2;
constexpr int D5_TILE = D5_BS * D5_D * 2;  // 8 KB
constexpr int D5_MAXN = 64;
constexpr int D5_SMEM = 1024 + 4 * D5_TILE + D5_KST * 2 * D5_TILE + 2 * D5_TILE + 2 * D5_TILE;
constexpr uint32_t D5_TMEM_COLS = 256;
constexpr int D5_SCOL = 0, D5_DPCOL = 64, D5_DQCOL = 128;
}  // namespace

template <typename T>
__global__ void __launch_bounds__(192, 2)
    attn_dq_f5_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                      const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                      const int perm_q, const int perm_do, const int perm_k, const int perm_v,
                      const AttnParams p) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = tc05::idesc_f16(kBF16, 64, 64, false);
  constexpr uint32_t IDESC_DQ = tc05::idesc_f16(kBF16, 64, D5_D, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sQ = smem;                          // tile t at sQ + t*TILE
  uint8_t *sDO = sQ + 2 * D5_TILE;             // tile t at sDO + t*TILE
  uint8_t *sK = sDO + 2 * D5_TILE;             // K ring: (stage, tile)
  uint8_t *sV = sK + D5_KST * 2 * D5_TILE;     // V: (tile)
  uint8_t *sS = sV + 2 * D5_TILE;              // dS: (tile)
  __shared__ __align__(8) uint64_t bar_q, k_full[D5_KST], k_empty[D5_KST], v_full, v_empty,
      sd_full, sd_empty, ds_full, dq_done;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int s_item[2][D5_MAXN];
  __shared__ int s_islot[2][D5_MAXN];
  __shared__ float s_gv[2][D5_MAXN];  // gate value of the j-th live slot
  __shared__ int s_n[2];
  __shared__ float s_dg[2][D5_MAXN][4];  // dgate partials: (tile, step, warp)

  const int npairs = (p.nq + 1) >> 1;
  long long id = blockIdx.x;
  const int gi = (int)(id % p.grp);
  id /= p.grp;
  const int pair = (int)(id % npairs);
  id /= npairs;
  const int hk = (int)(id % p.Hkv);
  const int b = (int)(id / p.Hkv);
  const int h = hk * p.grp + gi;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qb0 = 2 * pair;
  const bool validB = qb0 + 1 < p.nq;

  if (warp < 2) {  // live-slot lists (warp 0: tile A, warp 1: tile B)
    const int t = warp;
    const int qi = qb0 + t, qblk = p.q0 + qi;
    int n = 0;
    if (t == 0 || validB) {
      const int32_t *selrow = p.sel + b * p.sel_sb + hk * p.sel_sh + (long long)qi * p.sel_sn;
      const float *grow = p.gate ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn
                                 : nullptr;
      n = warp_live_slots(selrow, p.kk, D5_MAXN, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal,
                          p.status, [&](int pos, int kb, int kind, int slot) {
                            s_item[t][pos] = (kb << 3) | kind;
                            s_islot[t][pos] = slot;
                            s_gv[t][pos] = grow ? __ldg(grow + slot) : 0.f;
                          });
    }
    if (lane == 0) s_n[t] = n;
  }
  if (tid == 0) {
    // descriptors fetched ahead of the first TMA load
    prefetch_tmap(&tq);
    prefetch_tmap(&tdo);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    mbar_init(&bar_q, 1);
    for (int s = 0; s < D5_KST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    mbar_init(&v_full, 1);
    mbar_init(&v_empty, 1);
    mbar_init(&sd_full, 1);
    mbar_init(&sd_empty, 128);
    mbar_init(&ds_full, 128);
    mbar_init(&dq_done, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tc05::alloc(&tmem_base_sh, D5_TMEM_COLS);
    tc05::relinquish();
  }
  tc05::fence_before();
  __syncthreads();
  tc05::fence_after();
  const uint32_t tmem = tmem_base_sh;
  const int nA = s_n[0], nB = s_n[1];
  const int nsteps = nA > nB ? nA : nB;

  if (warp == 4) {
    // ================= TMA producer: the warp polls together (voted tests), one
    // elected lane (lane 0) issues the loads
    {
      auto test = [&](uint64_t *bar, uint32_t par) {
        return __any_sync(0xffffffffu, mbar_test(bar, par));
      };
      if (tc05::elect_one()) {
        mbar_expect_tx(&bar_q, (validB ? 4 : 2) * D5_TILE);
        tma_load_rhb(sQ, &tq, &bar_q, perm_q, 0, qb0 * p.bs, h, b);
        tma_load_rhb(sDO, &tdo, &bar_q, perm_do, 0, qb0 * p.bs, h, b);
        if (validB) {
          tma_load_rhb(sQ + D5_TILE, &tq, &bar_q, perm_q, 0, (qb0 + 1) * p.bs, h, b);
          tma_load_rhb(sDO + D5_TILE, &tdo, &bar_q, perm_do, 0, (qb0 + 1) * p.bs, h, b);
        }
      }
      __syncwarp();
      int jk = 0, jv = 0;
      uint32_t idle = 0;
      auto issue = [&](bool isv, int j) {
        const int st = isv ? 0 : j % D5_KST;
        uint64_t *full = isv ? &v_full : &k_full[st];
        uint8_t *ring = isv ? sV : sK + st * 2 * D5_TILE;
        const int act = (j < nA ? 1 : 0) + (j < nB ? 1 : 0);
        if (tc05::elect_one()) {
          mbar_expect_tx(full, act * D5_TILE);
          for (int t = 0; t < 2; ++t) {
            if (j >= (t ? nB : nA)) continue;
            tma_load_rhb(ring + t * D5_TILE, isv ? &tv : &tk, full, isv ? perm_v : perm_k, 0,
                         (s_item[t][j] >> 3) * p.bs, hk, b);
          }
        }
        __syncwarp();
      };
      while (jk < nsteps || jv < nsteps) {
        bool progress = false;
        if (jk < nsteps &&
            (jk < D5_KST || test(&k_empty[jk % D5_KST], ((jk / D5_KST) - 1) & 1))) {
          issue(false, jk++);
          progress = true;
        }
        if (jv < nsteps && (jv < 1 || test(&v_empty, (jv - 1) & 1))) {
          issue(true, jv++);
          progress = true;
        }
        if (progress) {
          idle = 0;
        } else {
          if (++idle > kSpinLimit) {
            report(p.status, BSA_DEVERR_TIMEOUT);
            break;
          }
          __nanosleep(32);
        }
      }
    }
  } else if (warp == 5) {
    // ================= MMA issuer: S/dP queue and dQ queue, polled by the whole
    // warp (warp-uniform descriptors; barrier tests made uniform by a vote); one
    // elected lane, always lane 0, issues the MMAs and commits
    {
      auto test = [&](uint64_t *bar, uint32_t par) {
        return __any_sync(0xffffffffu, mbar_test(bar, par));
      };
      if (!mbar_wait_warp(&bar_q, 0)) report(p.status, BSA_DEVERR_TIMEOUT);
      // descriptors built once; per MMA only a 64-bit add
      const uint64_t dq0 = tc05::sdesc(smem_u32(sQ), 16, 1024);
      const uint64_t ddo0 = tc05::sdesc(smem_u32(sDO), 16, 1024);
      const uint64_t dds0 = tc05::sdesc(smem_u32(sS), 16, 1024);
      const uint64_t dk0 = tc05::sdesc(smem_u32(sK), 16, 1024);
      const uint64_t dkm0 = tc05::sdesc(smem_u32(sK), D5_BS * 128, 1024);  // K as MN-major B
      const uint64_t dv0 = tc05::sdesc(smem_u32(sV), 16, 1024);
      int js = 0, jg = 0;
      uint32_t idle = 0;
      while (jg < nsteps) {
        bool progress = false;
        // dQ += dS_jg K_jg once the elementwise warps have written dS_jg
        if (jg < js && test(&ds_full, jg & 1)) {
          const int st = jg % D5_KST;
          tc05::fence_after();
          for (int t = 0; t < 2; ++t) {
            if (jg >= (t ? nB : nA)) continue;
            const uint64_t da = tc05::dadd(dds0, t * D5_TILE);
            const uint64_t db = tc05::dadd(dkm0, (st * 2 + t) * D5_TILE);
            const uint32_t d = tc05::taddr(tmem, 16 * t, D5_DQCOL);
            // a tile's first live step starts its accumulator
            if (tc05::elect_one()) {
#pragma unroll
              for (int ks = 0; ks < D5_BS / 16; ++ks)
                tc05::mma_f16(d, tc05::dadd(da, ks * 32), tc05::dadd(db, ks * 2048), IDESC_DQ,
                              (jg > 0 || ks > 0) ? 1u : 0u);
            }
            __syncwarp();
          }
          if (tc05::elect_one()) {
            tc05::commit(&k_empty[st]);
            tc05::commit(&dq_done);
          }
          __syncwarp();
          ++jg;
          progress = true;
        }
        // S_js, dP_js once K_js, V_js have landed and S/dP of js-1 have been read
        if (js < nsteps && test(&k_full[js % D5_KST], (js / D5_KST) & 1) &&
            test(&v_full, js & 1) && (js < 1 || test(&sd_empty, (js - 1) & 1))) {
          const int st = js % D5_KST;
          tc05::fence_after();
          for (int t = 0; t < 2; ++t) {
            if (js >= (t ? nB : nA)) continue;
            const uint64_t aq = tc05::dadd(dq0, t * D5_TILE), ado = tc05::dadd(ddo0, t * D5_TILE);
            const uint64_t bk = tc05::dadd(dk0, (st * 2 + t) * D5_TILE), bv = tc05::dadd(dv0, t * D5_TILE);
            const uint32_t ds = tc05::taddr(tmem, 16 * t, D5_SCOL);
            const uint32_t ddp = tc05::taddr(tmem, 16 * t, D5_DPCOL);
            if (tc05::elect_one()) {
#pragma unroll
              for (int ks = 0; ks < D5_D / 16; ++ks) {
                tc05::mma_f16(ds, tc05::dadd(aq, ks * 32), tc05::dadd(bk, ks * 32), IDESC_S, ks > 0);
                tc05::mma_f16(ddp, tc05::dadd(ado, ks * 32), tc05::dadd(bv, ks * 32), IDESC_S, ks > 0);
              }
            }
            __syncwarp();
          }
          if (tc05::elect_one()) {
            tc05::commit(&sd_full);
            tc05::commit(&v_empty);
          }
          __syncwarp();
          ++js;
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
    // ================= elementwise warps 0-3
    const int t = lane >> 4;
    const int r = warp * 16 + (lane & 15);  // query row within its block
    const int qi = qb0 + t;
    const int nmine = t ? nB : nA;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const long long bh = (long long)b * p.Hq + h;
    const bool row_ok = qi < p.nq;
    const long long grow = (long long)qi * p.bs + r;
    const float lse = row_ok ? p.lse[bh * p.Lp + grow] : 0.f;
    const float dv = row_ok ? p.dvec[bh * p.Lp + grow] : 0.f;
    const float *gaterow =
        (p.gate && row_ok) ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn
                           : nullptr;
    const uint32_t sa = smem_u32(sS + t * D5_TILE);
    for (int j = 0; j < nsteps; ++j) {
      if (!mbar_wait(&sd_full, j & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
      tc05::fence_after();
      const bool active = j < nmine && row_ok;
      int kind = 0, kb = 0;
      float g2 = 0.f;
      if (j < nmine) {
        const int item = s_item[t][j];
        kind = item & 7;
        kb = item >> 3;
        g2 = gaterow ? s_gv[t][j] * kLog2e : 0.f;
      }
      const float off = g2 - lse;  // exponent offset of this row and step
      uint32_t w[32];
      float dgs = 0.f;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float s[32], dp[32];
        tc05::ld32(tmem + lane_base + D5_SCOL + 32 * hf, s);
        tc05::ld32(tmem + lane_base + D5_DPCOL + 32 * hf, dp);
        tc05::wait_ld();
        if (active && !(kind & (KIND_TRIU | KIND_PAD))) {  // common case: no masks
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float d0 = ex2(fmaf(s[c], p.scale2, off)) * (dp[c] - dv);
            const float d1 = ex2(fmaf(s[c + 1], p.scale2, off)) * (dp[c + 1] - dv);
            dgs += d0;
            dgs += d1;
            w[16 * hf + (c >> 1)] = Mma<T>::pack(d0, d1);
          }
        } else {  // diagonal / padded block, or an idle tile (its TMEM is stale)
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float d2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int col = 32 * hf + c + e;
              const bool masked = !active || ((kind & KIND_TRIU) && col > r) ||
                                  ((kind & KIND_PAD) && kb * p.bs + col >= p.L);
              const float pr = masked ? 0.f : ex2(fmaf(s[c + e], p.scale2, off));
              d2[e] = pr * (dp[c + e] - dv);
              dgs += d2[e];
            }
            w[16 * hf + (c >> 1)] = Mma<T>::pack(d2[0], d2[1]);
          }
        }
      }
      tc05::fence_before();
      tc05::mbar_arrive(&sd_empty);
      // dgate partial of this step: rows of this warp's 16 lanes of the tile
#pragma unroll
      for (int o = 8; o; o >>= 1) dgs += __shfl_xor_sync(0xffffffffu, dgs, o);
      if ((lane & 15) == 0 && j < D5_MAXN) s_dg[t][j][warp] = dgs;
      // dQ_{j-1} must have read the dS buffer
      if (j >= 1) {
        if (!mbar_wait(&dq_done, (j - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
      }
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(swz(sa, D5_BS, r, c8 * 8)),
                     "r"(w[4 * c8]), "r"(w[4 * c8 + 1]), "r"(w[4 * c8 + 2]), "r"(w[4 * c8 + 3])
                     : "memory");
      fence_proxy_async_smem();
      tc05::fence_before();
      tc05::mbar_arrive(&ds_full);
    }
    // ---- epilogue: dQ * scale, dgate per slot
    if (nsteps > 0) {
      if (!mbar_wait(&dq_done, (nsteps - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
      tc05::fence_after();
    }
    float o[64];
    tc05::ld32(tmem + lane_base + D5_DQCOL, o);
    tc05::ld32(tmem + lane_base + D5_DQCOL + 32, o + 32);
    tc05::wait_ld();
    if (nmine == 0) {  // never accumulated: the TMEM columns hold stale data
#pragma unroll
      for (int c = 0; c < 64; ++c) o[c] = 0.f;
    }
    if (row_ok && grow < p.Lq) {
      T *dqrow = reinterpret_cast<T *>(p.dq) + b * p.dq_sb + h * p.dq_sh + grow * p.dq_sl;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        uint4 wv;
        wv.x = Mma<T>::pack(o[c8 * 8 + 0] * p.scale, o[c8 * 8 + 1] * p.scale);
        wv.y = Mma<T>::pack(o[c8 * 8 + 2] * p.scale, o[c8 * 8 + 3] * p.scale);
        wv.z = Mma<T>::pack(o[c8 * 8 + 4] * p.scale, o[c8 * 8 + 5] * p.scale);
        wv.w = Mma<T>::pack(o[c8 * 8 + 6] * p.scale, o[c8 * 8 + 7] * p.scale);
        *reinterpret_cast<uint4 *>(dqrow + c8 * 8) = wv;
      }
    }
    named_bar_sync(1, 128);  // all dgate partials written
    if (p.dgate) {
      for (int i = tid; i < 2 * p.kk; i += 128) {
        const int tt = i / p.kk, slot = i % p.kk;
        const int qq = qb0 + tt;
        if (qq >= p.nq) continue;
        float v = 0.f;
        const int n = tt ? nB : nA;
        for (int jj = 0; jj < n; ++jj)
          if (s_islot[tt][jj] == slot) {
            v = (s_dg[tt][jj][0] + s_dg[tt][jj][1]) + (s_dg[tt][jj][2] + s_dg[tt][jj][3]);
            break;
          }
        p.dgate[(bh * p.nq + qq) * (long long)p.kk + slot] = v;
      }
    }
  }
  tc05::fence_before();
  __syncthreads();
  if (warp == 5) {
    tc05::fence_after();
    tc05::dealloc(tmem, D5_TMEM_COLS);
  }
}

// On by default; BSA_DQ_F5=0 selects the mma.sync dQ kernel instead.
bool dq_f5_applicable(const AttnParams &p, int dtype, int D) {
  const char *env = getenv("BSA_DQ_F5");
  if (env && env[0] == '0') return false;
  return dtype != BSA_F32 && p.bs == 64 && D == 64 && p.sel && p.kk <= D5_MAXN &&
         !getenv("BSA_BWD_LEGACY");
}

bsa_status launch_dq_f5(int dtype, const CUtensorMap &mq, const CUtensorMap &mdo,
                        const CUtensorMap &mk, const CUtensorMap &mv, int pq, int pdo, int pk,
                        int pv, const AttnParams &p, cudaStream_t st) {
  const long long grid = (long long)p.B * p.Hq * ((p.nq + 1) / 2);
  if (dtype == BSA_BF16) {
    cudaFuncSetAttribute(attn_dq_f5_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, D5_SMEM);
    attn_dq_f5_kernel<__nv_bfloat16><<<(unsigned)grid, 192, D5_SMEM, st>>>(mq, mdo, mk, mv, pq, pdo,
                                                                           pk, pv, p);
  } else {
    cudaFuncSetAttribute(attn_dq_f5_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, D5_SMEM);
    attn_dq_f5_kernel<__half><<<(unsigned)grid, 192, D5_SMEM, st>>>(mq, mdo, mk, mv, pq, pdo, pk,
                                                                   pv, p);
  }
  return check_launch("attn_dq_f5");
}

}  // namespace bsa
