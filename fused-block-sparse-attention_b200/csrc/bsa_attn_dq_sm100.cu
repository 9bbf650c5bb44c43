// Block-sparse attention backward, dQ part, on tcgen05 for block 64, head
// dim 64, plus the Dvec = rowsum(dO * O) pre-pass.
//
// Persistent: one CTA per SM loops over work units; a unit is two adjacent
// query blocks (tiles A and B) of one (batch, query head).  Q and dO of the
// unit stay in shared memory; the selected K/V blocks of both tiles stream
// through a 3-stage ring.  Per step j (the j-th live slot of each tile):
//   S  = Q K_j^T      dP = dO V_j^T                (tcgen05, TMEM, 2 buffers)
//   P  = 2^(S*scale*log2e + gate - lse)   dS = P (dP - Dvec)
//   dQ += dS K_j                                   (tcgen05, TMEM accumulator)
//   dgate[slot] = sum(dS)  (per tile, reduced in a fixed order: deterministic)
// Warp roles (320 threads): warps 0-7 elementwise (two per TMEM quadrant,
// 32 columns each), warp 8 TMA producer, warp 9 TMEM allocation + MMA issuer
// (polls the S/dP and dQ queues).  TMEM: S [0,128), dP [128,256), dQ
// accumulators [256,320) and [320,384) by unit parity; tile B at lane 16.
#include <algorithm>
#include <type_traits>

#include "bsa_attn.cuh"
#include "bsa_host.h"
#include "bsa_tc05.cuh"

namespace bsa {

namespace {
constexpr int Q5_BS = 64, Q5_D = 64, Q5_NST = 3, Q5_MAXN = 64;
constexpr int Q5_TILE = Q5_BS * Q5_D * 2;
constexpr int Q5_SMEM = 1024 + 4 * Q5_TILE       // Q, dO of both tiles
                        + Q5_NST * 4 * Q5_TILE   // ring: (stage, tile) K, V
                        + 4 * Q5_TILE;           // dS: (buffer, tile)
constexpr uint32_t Q5_TMEM_COLS = 512;
constexpr int Q5_SCOL = 0, Q5_DPCOL = 128, Q5_DQCOL = 256;
}  // namespace

// rowsum(dO * O) per row, fp32, for every (b, h, row < Lp); rows >= L get 0.
template <typename T>
__global__ void dvec_kernel(const AttnParams p, int D) {
  const long long nrows = (long long)p.B * p.Hq * p.Lp;
  const int lane = threadIdx.x & 7;  // 8 threads per row
  for (long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 3; r < nrows;
       r += ((long long)gridDim.x * blockDim.x) >> 3) {
    const int row = (int)(r % p.Lp);
    const long long bh = r / p.Lp;
    const int h = (int)(bh % p.Hq), b = (int)(bh / p.Hq);
    float acc = 0.f;
    if (row < p.Lq) {
      const T *po = reinterpret_cast<const T *>(p.oin) + b * p.oi_sb + h * p.oi_sh + (long long)row * p.oi_sl;
      const T *pd = reinterpret_cast<const T *>(p.dout) + b * p.do_sb + h * p.do_sh + (long long)row * p.do_sl;
      for (int c = lane * 8; c < D; c += 64) {
        const uint4 ov = *reinterpret_cast<const uint4 *>(po + c);
        const uint4 dv = *reinterpret_cast<const uint4 *>(pd + c);
        const T *oe = reinterpret_cast<const T *>(&ov);
        const T *de = reinterpret_cast<const T *>(&dv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(Mma<T>::to_f(oe[e]), Mma<T>::to_f(de[e]), acc);
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    if (lane == 0) p.dvec[r] = acc;
  }
}

// Live slots of one query block, walked in slot order.
struct Q5Cursor {
  const int32_t *selrow;
  int slot;
};

__device__ __forceinline__ int q5_kind(const AttnParams &p, const int32_t *selrow, int slot,
                                       int qblk, int &kb) {
  kb = __ldg(selrow + slot);
  bool dup = false;
  if (p.mask_mode == BSA_MASK_TOKEN)
    for (int i = 0; i < slot && !dup; ++i) dup = __ldg(selrow + i) == kb;
  return slot_kind(kb, slot, dup, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal, nullptr);
}

// Advances `c` to the next live slot; returns its packed (kb << 3 | kind), or -1.
__device__ __forceinline__ int q5_next(const AttnParams &p, Q5Cursor &c, int qblk, int &slot) {
  while (c.slot < p.kk) {
    int kb;
    const int s = c.slot++;
    const int kind = q5_kind(p, c.selrow, s, qblk, kb);
    if (kind != KIND_SKIP) {
      slot = s;
      return (kb << 3) | kind;
    }
  }
  return -1;
}

struct Q5Unit {
  int b, h, hk, qb0;
  int n[2];
  bool valid[2];
  const int32_t *selrow[2];
};

__device__ __forceinline__ void q5_unit(const AttnParams &p, int u, Q5Unit &w) {
  const int npairs = (p.nq + 1) >> 1;
  const int pair = u % npairs;
  const int bh = u / npairs;
  w.h = bh % p.Hq;
  w.b = bh / p.Hq;
  w.hk = w.h / p.grp;
  w.qb0 = 2 * pair;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qi = w.qb0 + t, qblk = p.q0 + qi;  // local / global query block
    w.valid[t] = qi < p.nq;
    w.n[t] = 0;
    w.selrow[t] = p.sel + w.b * p.sel_sb + w.hk * p.sel_sh + (long long)(w.valid[t] ? qi : 0) * p.sel_sn;
    if (!w.valid[t]) continue;
    int n = 0;
    for (int s = 0; s < p.kk; ++s) {
      int kb;
      if (q5_kind(p, w.selrow[t], s, qblk, kb) != KIND_SKIP) ++n;
    }
    w.n[t] = n;
  }
}

template <typename T>
__global__ void __launch_bounds__(320, 1)
    attn_dq_sm100_kernel(const __grid_constant__ CUtensorMap tq,
                         const __grid_constant__ CUtensorMap tdo,
                         const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const int perm_q,
                         const int perm_do, const int perm_k, const int perm_v,
                         const AttnParams p) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_KK = tc05::idesc_f16(kBF16, 64, 64, false);
  constexpr uint32_t IDESC_KM = tc05::idesc_f16(kBF16, 64, Q5_D, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sQD = smem;                       // tile t: Q, dO
  uint8_t *sR = sQD + 4 * Q5_TILE;           // (stage, tile): K, V
  uint8_t *sDS = sR + Q5_NST * 4 * Q5_TILE;  // (buffer, tile): dS
  // p_full[b] / g_done[b]: dS of a step with parity b written / consumed (one
  // barrier per buffer so the phase tracking stays exact).
  __shared__ __align__(8) uint64_t qd_full, qd_empty, r_full[Q5_NST], r_empty[Q5_NST],
      s_full[2], s_empty[2], p_full[2], g_done[2], acc_empty[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ float s_dg[Q5_MAXN][2][8];  // per (step, tile, warp) sums of dS

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int npairs = (p.nq + 1) >> 1;
  const int nunits = p.B * p.Hq * npairs;
  if (tid == 0) {
    mbar_init(&qd_full, 1);
    mbar_init(&qd_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 256);
      mbar_init(&p_full[s], 256);
      mbar_init(&g_done[s], 1);
      mbar_init(&acc_empty[s], 256);
    }
    for (int s = 0; s < Q5_NST; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], 1);
    }
    fence_mbar_init();
  }
  if (warp == 9) {
    tc05::alloc(&tmem_base_sh, Q5_TMEM_COLS);
    tc05::relinquish();
  }
  tc05::fence_before();
  __syncthreads();
  tc05::fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 8) {
    // ================= producer
    if (lane == 0) {
      int gs = 0, ne = 0;
      uint32_t idle = 0;
      for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
        Q5Unit w;
        q5_unit(p, u, w);
        const int ns = max(w.n[0], w.n[1]);
        if (ns == 0) continue;
        if (ne >= 1 && !mbar_wait(&qd_empty, (ne - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        mbar_expect_tx(&qd_full, ((w.n[0] > 0) + (w.n[1] > 0)) * 2 * Q5_TILE);
        for (int t = 0; t < 2; ++t) {
          if (w.n[t] == 0) continue;
          const int row = (w.qb0 + t) * p.bs;
          tma_load_rhb(sQD + 2 * t * Q5_TILE, &tq, &qd_full, perm_q, 0, row, w.h, w.b);
          tma_load_rhb(sQD + (2 * t + 1) * Q5_TILE, &tdo, &qd_full, perm_do, 0, row, w.h, w.b);
        }
        ++ne;
        Q5Cursor cur[2] = {{w.selrow[0], 0}, {w.selrow[1], 0}};
        for (int j = 0; j < ns; ++j, ++gs) {
          const int st = gs % Q5_NST;
          while (gs >= Q5_NST && !mbar_test(&r_empty[st], ((gs / Q5_NST) - 1) & 1)) {
            if (++idle > kSpinLimit) {
              report(p.status, BSA_DEVERR_TIMEOUT);
              break;
            }
            __nanosleep(32);
          }
          idle = 0;
          mbar_expect_tx(&r_full[st], ((j < w.n[0]) + (j < w.n[1])) * 2 * Q5_TILE);
          for (int t = 0; t < 2; ++t) {
            if (j >= w.n[t]) continue;
            int slot;
            const int it = q5_next(p, cur[t], p.q0 + w.qb0 + t, slot);
            const int kb = it >> 3;
            uint8_t *dst = sR + (st * 2 + t) * 2 * Q5_TILE;
            tma_load_rhb(dst, &tk, &r_full[st], perm_k, 0, kb * p.bs, w.hk, w.b);
            tma_load_rhb(dst + Q5_TILE, &tv, &r_full[st], perm_v, 0, kb * p.bs, w.hk, w.b);
          }
        }
      }
    }
  } else if (warp == 9) {
    // ================= MMA issuer
    if (lane == 0) {
      int us = blockIdx.x, js = 0, gss = 0, nes = -1;
      int ug = blockIdx.x, jg = 0, gsg = 0, neg = -1;
      Q5Unit ws, wg;
      uint32_t idle = 0;
      auto next_unit = [&](int &u, Q5Unit &w, int &ne) -> bool {
        for (; u < nunits; u += gridDim.x) {
          q5_unit(p, u, w);
          if (max(w.n[0], w.n[1]) > 0) {
            ++ne;
            return true;
          }
        }
        return false;
      };
      bool have_s = next_unit(us, ws, nes);
      bool have_g = next_unit(ug, wg, neg);
      const uint32_t qd_addr = smem_u32(sQD);
      while (have_g) {
        bool progress = false;
        // ---- dQ += dS K for step (ug, jg)
        if (gsg < gss && mbar_test(&p_full[gsg & 1], (gsg >> 1) & 1) &&
            (jg > 0 || neg < 2 || mbar_test(&acc_empty[neg & 1], ((neg >> 1) - 1) & 1))) {
          const int st = gsg % Q5_NST, ab = neg & 1;
          tc05::fence_after();
          for (int t = 0; t < 2; ++t) {
            if (jg >= wg.n[t]) continue;
            const uint32_t k_addr = smem_u32(sR + (st * 2 + t) * 2 * Q5_TILE);
            const uint32_t ds_addr = smem_u32(sDS + ((gsg & 1) * 2 + t) * Q5_TILE);
            const uint32_t dq = tc05::taddr(tmem, 16 * t, Q5_DQCOL + 64 * ab);
#pragma unroll
            for (int ks = 0; ks < Q5_BS / 16; ++ks)
              tc05::mma_f16(dq, tc05::sdesc(ds_addr + ks * 32, 16, 1024),
                            tc05::sdesc(k_addr + ks * 2048, Q5_BS * 128, 1024), IDESC_KM,
                            (jg > 0 || ks > 0) ? 1u : 0u);
          }
          tc05::commit(&r_empty[st]);
          tc05::commit(&g_done[gsg & 1]);
          ++gsg;
          if (++jg == max(wg.n[0], wg.n[1])) {
            jg = 0;
            ug += gridDim.x;
            have_g = next_unit(ug, wg, neg);
          }
          progress = true;
        }
        // ---- S = Q K^T, dP = dO V^T for step (us, js)
        if (have_s && mbar_test(&r_full[gss % Q5_NST], (gss / Q5_NST) & 1) &&
            (gss < 2 || mbar_test(&s_empty[gss & 1], ((gss >> 1) - 1) & 1)) &&
            (js > 0 || mbar_test(&qd_full, nes & 1))) {
          const int st = gss % Q5_NST, bb = gss & 1;
          tc05::fence_after();
          for (int t = 0; t < 2; ++t) {
            if (js >= ws.n[t]) continue;
            const uint32_t q_addr = qd_addr + 2 * t * Q5_TILE, do_addr = q_addr + Q5_TILE;
            const uint32_t k_addr = smem_u32(sR + (st * 2 + t) * 2 * Q5_TILE);
            const uint32_t v_addr = k_addr + Q5_TILE;
            const uint32_t ds = tc05::taddr(tmem, 16 * t, Q5_SCOL + 64 * bb);
            const uint32_t ddp = tc05::taddr(tmem, 16 * t, Q5_DPCOL + 64 * bb);
#pragma unroll
            for (int ks = 0; ks < Q5_D / 16; ++ks) {
              tc05::mma_f16(ds, tc05::sdesc(q_addr + ks * 32, 16, 1024),
                            tc05::sdesc(k_addr + ks * 32, 16, 1024), IDESC_KK, ks > 0);
              tc05::mma_f16(ddp, tc05::sdesc(do_addr + ks * 32, 16, 1024),
                            tc05::sdesc(v_addr + ks * 32, 16, 1024), IDESC_KK, ks > 0);
            }
          }
          tc05::commit(&s_full[bb]);
          ++gss;
          if (++js == max(ws.n[0], ws.n[1])) {
            tc05::commit(&qd_empty);  // last reader of this unit's Q / dO
            js = 0;
            us += gridDim.x;
            have_s = next_unit(us, ws, nes);
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
    // ================= elementwise warps 0-7
    const int quad = warp & 3, hf = warp >> 2;
    const int t = lane >> 4;
    const int r = quad * 16 + (lane & 15);  // query row within its block
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    int gs = 0, ne = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
      Q5Unit w;
      q5_unit(p, u, w);
      const int ns = max(w.n[0], w.n[1]);
      const int qi = w.qb0 + t, qblk = p.q0 + qi, nmine = w.n[t];
      const long long bh = (long long)w.b * p.Hq + w.h;
      const long long grow = (long long)qi * p.bs + r;
      float lse2 = 0.f, dv = 0.f;
      if (w.valid[t]) {
        lse2 = p.lse[bh * p.Lp + grow];
        dv = p.dvec[bh * p.Lp + grow];
      }
      const float *gaterow =
          (p.gate && w.valid[t]) ? p.gate + w.b * p.gate_sb + w.hk * p.gate_sh + (long long)qi * p.gate_sn
                                 : nullptr;
      Q5Cursor cur = {w.selrow[t], 0};
      for (int j = 0; j < ns; ++j, ++gs) {
        const int bb = gs & 1;
        if (!mbar_wait(&s_full[bb], (gs >> 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
        float sv[32], dp[32];
        tc05::ld32(tmem + lane_base + Q5_SCOL + 64 * bb + 32 * hf, sv);
        tc05::ld32(tmem + lane_base + Q5_DPCOL + 64 * bb + 32 * hf, dp);
        tc05::wait_ld();
        tc05::fence_before();
        tc05::mbar_arrive(&s_empty[bb]);
        uint32_t wd[16];
        float dgs = 0.f;
        const bool active = j < nmine;
        if (active) {
          int slot;
          const int it = q5_next(p, cur, qblk, slot);
          const int kind = it & 7, kb = it >> 3;
          const float off = (gaterow ? __ldg(gaterow + slot) * kLog2e : 0.f) - lse2;
          if (kind & (KIND_TRIU | KIND_PAD)) {
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const int key = 32 * hf + c;
              if (((kind & KIND_TRIU) && key > r) || ((kind & KIND_PAD) && kb * p.bs + key >= p.L))
                sv[c] = -INFINITY;
            }
          }
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float p0 = ex2(fmaf(sv[c], p.scale2, off));
            const float p1 = ex2(fmaf(sv[c + 1], p.scale2, off));
            const float d0 = p0 * (dp[c] - dv), d1 = p1 * (dp[c + 1] - dv);
            dgs += d0 + d1;
            wd[c >> 1] = Mma<T>::pack(d0, d1);
          }
          if (grow >= p.Lq) dgs = 0.f;
        }
        if (p.dgate) {  // per-warp, per-tile partial of sum(dS) for this step
#pragma unroll
          for (int o = 8; o; o >>= 1) dgs += __shfl_xor_sync(0xffffffffu, dgs, o);
          if ((lane & 15) == 0 && j < Q5_MAXN) s_dg[j][t][warp] = dgs;
        }
        if (gs >= 2) {  // dQ MMAs of step gs-2 read dS buffer gs & 1
          if (!mbar_wait(&g_done[bb], ((gs >> 1) - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
          tc05::fence_after();
        }
        if (active) {
          const uint32_t da = smem_u32(sDS + (bb * 2 + t) * Q5_TILE);
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8)
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(swz(da, Q5_BS, r, 32 * hf + 8 * c8)),
                         "r"(wd[4 * c8]), "r"(wd[4 * c8 + 1]), "r"(wd[4 * c8 + 2]), "r"(wd[4 * c8 + 3])
                         : "memory");
        }
        fence_proxy_async_smem();
        tc05::fence_before();
        tc05::mbar_arrive(&p_full[bb]);
      }
      // ---- dQ of this unit (scaled), dgate of its slots
      float dq[32];
      if (ns > 0) {
        const int gl = gs - 1;
        if (!mbar_wait(&g_done[gl & 1], (gl >> 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
        const int ab = ne & 1;
        tc05::ld32(tmem + lane_base + Q5_DQCOL + 64 * ab + 32 * hf, dq);
        tc05::wait_ld();
        tc05::fence_before();
        tc05::mbar_arrive(&acc_empty[ab]);
        ++ne;
      }
      if (p.dgate) {
        asm volatile("bar.sync 1, 256;" ::: "memory");
        // thread i < 2*kk writes slot (i % kk) of tile (i / kk)
        for (int i = warp * 32 + lane; i < 2 * p.kk; i += 256) {
          const int tt = i / p.kk, slot = i % p.kk;
          const int qb = w.qb0 + tt;  // local
          if (qb >= p.nq) continue;
          // live slots of tile tt in order: its j-th live slot is `slot`?
          Q5Cursor c2 = {w.selrow[tt], 0};
          float v = 0.f;
          for (int jj = 0; jj < Q5_MAXN; ++jj) {
            int sl;
            if (q5_next(p, c2, p.q0 + qb, sl) < 0) break;
            if (sl == slot) {
#pragma unroll
              for (int wv = 0; wv < 8; ++wv) v += s_dg[jj][tt][wv];
              break;
            }
          }
          p.dgate[(((long long)w.b * p.Hq + w.h) * p.nq + qb) * p.kk + slot] = v;
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
      }
      if (!w.valid[t] || grow >= p.Lq) continue;
      if (nmine == 0) {
#pragma unroll
        for (int c = 0; c < 32; ++c) dq[c] = 0.f;
      }
      T *dqp = reinterpret_cast<T *>(p.dq) + w.b * p.dq_sb + w.h * p.dq_sh + grow * p.dq_sl + 32 * hf;
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        uint4 v4;
        v4.x = Mma<T>::pack(dq[c] * p.scale, dq[c + 1] * p.scale);
        v4.y = Mma<T>::pack(dq[c + 2] * p.scale, dq[c + 3] * p.scale);
        v4.z = Mma<T>::pack(dq[c + 4] * p.scale, dq[c + 5] * p.scale);
        v4.w = Mma<T>::pack(dq[c + 6] * p.scale, dq[c + 7] * p.scale);
        *reinterpret_cast<uint4 *>(dqp + c) = v4;
      }
    }
  }
  tc05::fence_before();
  __syncthreads();
  if (warp == 9) {
    tc05::fence_after();
    tc05::dealloc(tmem, Q5_TMEM_COLS);
  }
}

// ------------------------------------------------------------------ launchers
// Opt-in (BSA_DQ_TC05=1): on the 262k benchmark this kernel is slower than
// the mma.sync dQ kernel (4.2 ms against 3.45 ms), so the latter stays the
// default until the tcgen05 version overtakes it.
bool dq_sm100_applicable(const AttnParams &p, int dtype, int D) {
  const char *on = getenv("BSA_DQ_TC05");
  return on && on[0] == '1' && dtype != BSA_F32 && p.bs == 64 && D == 64 && p.kk <= Q5_MAXN &&
         !getenv("BSA_BWD_LEGACY");
}

bsa_status launch_dvec(int dtype, const AttnParams &p, int D, cudaStream_t st) {
  const long long rows = (long long)p.B * p.Hq * p.Lp;
  const unsigned blocks = (unsigned)std::min<long long>((rows * 8 + 255) / 256, 148LL * 32);
  if (dtype == BSA_BF16)
    dvec_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(p, D);
  else
    dvec_kernel<__half><<<blocks, 256, 0, st>>>(p, D);
  return check_launch("dvec");
}

bsa_status launch_dq_sm100(int dtype, const CUtensorMap &mq, const CUtensorMap &mdo,
                           const CUtensorMap &mk, const CUtensorMap &mv, int pq, int pdo, int pk,
                           int pv, const AttnParams &p, cudaStream_t st) {
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const long long units = (long long)p.B * p.Hq * ((p.nq + 1) / 2);
  const unsigned grid = (unsigned)std::max<long long>(1, std::min<long long>(nsm, units));
  if (dtype == BSA_BF16) {
    auto kern = attn_dq_sm100_kernel<__nv_bfloat16>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Q5_SMEM);
    kern<<<grid, 320, Q5_SMEM, st>>>(mq, mdo, mk, mv, pq, pdo, pk, pv, p);
  } else {
    auto kern = attn_dq_sm100_kernel<__half>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Q5_SMEM);
    kern<<<grid, 320, Q5_SMEM, st>>>(mq, mdo, mk, mv, pq, pdo, pk, pv, p);
  }
  return check_launch("attn_dq_sm100");
}

}  // namespace bsa
