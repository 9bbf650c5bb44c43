// Block-sparse attention forward on the 5th-generation tensor cores (tcgen05,
// accumulators in tensor memory) for block 64, head dim 64.
//
// One CTA computes two adjacent query blocks (tiles A and B) of one head.  A
// 64-row UMMA accumulator occupies TMEM lanes 0-15 of each 32-lane quadrant,
// so tile B's accumulators are placed at lane offset 16: every one of the 128
// softmax threads then owns one full query row (no shuffles for row max / sum).
//
// Warp roles (192 threads; 6 warps x <=168 registers keeps two CTAs resident
// per SM, since each SM sub-partition holds 16K registers):
//   warps 0-3  softmax: TMEM -> registers (32x32b loads), scale, gate, masks,
//              lazy-rescaled online softmax, P (16-bit pairs) written back over
//              the row's own S columns, final O / l.
//   warp 4     TMA producer (one thread): Q tiles once, then K blocks into a
//              ring that is freed as soon as S_j completes and V blocks into a
//              ring freed when PV_j completes; it polls both rings without
//              blocking so neither stream waits behind the other.
//   warp 5     TMEM allocation (256 columns); lane 0 issues the MMAs, polling
//              two queues without blocking: PV_j = P_j V_j into the TMEM O
//              accumulator as soon as P_j is ready (first priority; P_j is the
//              A operand, read from TMEM), and S_j = Q K_j^T into a
//              double-buffered TMEM S as soon as K_j has landed and PV_{j-2}
//              (the last reader of that buffer) is done.  Completions are
//              signalled by tcgen05.commit.
// TMEM columns: S / P buffers [0,64) and [64,128), O [128,192).  Since P lives in
// the S buffers, the softmax of step j+1 never waits for PV_j; only a rescale
// of O does.
//
// The running max is only raised (and O, l rescaled) when a row's new maximum
// exceeds the one in use by more than 2^8, so the rescale of O in TMEM is rare;
// the final O / l uses the same maximum as every P, so the result is exact.
#include <type_traits>

#include "bsa_attn.cuh"
#include "bsa_host.h"
#include "bsa_tc05.cuh"

namespace bsa {



namespace {
constexpr int F5_BS = 64, F5_D = 64;
constexpr int F5_TILE = F5_BS * F5_D * 2;  // 8 KB
constexpr int F5_MAXN = 64;                // live slots per tile kept in shared memory
// Q of both tiles, NK K stages and NV V stages (each stage both tiles)
template <int NK, int NV>
constexpr int f5_smem() { return 1024 + 2 * F5_TILE + (NK + NV) * 2 * F5_TILE; }
constexpr uint32_t F5_TMEM_COLS = 256;
constexpr int F5_SCOL0 = 0, F5_OCOL = 128;
constexpr float F5_RESCALE = 8.f;  // log2 units
}  // namespace

template <typename T, int NK, int NV>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tq,
                          const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, const int perm_q,
                          const int perm_k, const int perm_v, const AttnParams p) {
  constexpr bool kBF16 = sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = tc05::idesc_f16(kBF16, 64, 64, false);
  constexpr uint32_t IDESC_PV = tc05::idesc_f16(kBF16, 64, F5_D, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sQ = smem;                          // tile t at sQ + t*TILE
  uint8_t *sK = smem + 2 * F5_TILE;              // K ring: (stage, tile)
  uint8_t *sV = sK + NK * 2 * F5_TILE;           // V ring: (stage, tile)
  // per TMEM buffer b (the step's parity): s_full (S computed), p_full (P written
  // over S), s_empty (PV, the last reader of P, done)
  __shared__ __align__(8) uint64_t bar_q, k_full[NK], k_empty[NK], v_full[NV], v_empty[NV],
      s_full[2], s_empty[2], p_full[2], o_done, o_final;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int s_item[2][F5_MAXN];  // (kb << 3) | kind of the j-th live slot
  __shared__ float s_gv[2][F5_MAXN];  // its gate value (read with the list)
  __shared__ int s_n[2];

  // ---- CTA coordinates: (b, kv head, query-block pair, head in group)
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
  const int qb0 = 2 * pair;  // local index of tile A's query block
  const bool validB = qb0 + 1 < p.nq;

  // ---- live-slot lists of both tiles (warp 0: tile A, warp 1: tile B)
  if (warp < 2) {
    const int t = warp;
    const int qi = qb0 + t, qblk = p.q0 + qi;
    int n = 0;
    if (t == 0 || validB) {
      const int32_t *selrow = p.sel + b * p.sel_sb + hk * p.sel_sh + (long long)qi * p.sel_sn;
      const float *grow = p.gate ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn
                                 : nullptr;
      n = warp_live_slots(selrow, p.kk, F5_MAXN, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal,
                          p.status, [&](int pos, int kb, int kind, int slot) {
                            s_item[t][pos] = (kb << 3) | kind;
                            s_gv[t][pos] = grow ? __ldg(grow + slot) : 0.f;
                          });
    }
    if (lane == 0) s_n[t] = n;
  }
  if (tid == 0) {
    // descriptors fetched ahead of the first TMA load
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    mbar_init(&bar_q, 1);
    for (int s = 0; s < NK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < NV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 1);
      mbar_init(&p_full[s], 128);
    }
    mbar_init(&o_done, 1);
    mbar_init(&o_final, 1);  // one phase: the last PV has completed
    fence_mbar_init();
  }
  if (warp == 5) {
    tc05::alloc(&tmem_base_sh, F5_TMEM_COLS);
    tc05::relinquish();
  }
  tc05::fence_before();
  __syncthreads();
  tc05::fence_after();
  const uint32_t tmem = tmem_base_sh;
  const int nA = s_n[0], nB = s_n[1];
  const int nsteps = nA > nB ? nA : nB;

  if (warp == 4) {
    // ================= TMA producer: the warp polls both rings together (voted
    // tests), one elected lane (lane 0) issues the loads
    if (tc05::elect_one()) {
      mbar_expect_tx(&bar_q, (validB ? 2 : 1) * F5_TILE);
      tma_load_rhb(sQ, &tq, &bar_q, perm_q, 0, qb0 * p.bs, h, b);
      if (validB) tma_load_rhb(sQ + F5_TILE, &tq, &bar_q, perm_q, 0, (qb0 + 1) * p.bs, h, b);
    }
    __syncwarp();
    {
      auto test = [&](uint64_t *bar, uint32_t par) {
        return __any_sync(0xffffffffu, mbar_test(bar, par));
      };
      int jk = 0, jv = 0;
      uint32_t idle = 0;
      auto issue = [&](bool isv, int j) {
        const int st = isv ? j % NV : j % NK;
        uint64_t *full = isv ? &v_full[st] : &k_full[st];
        uint8_t *ring = isv ? sV : sK;
        const int act = (j < nA ? 1 : 0) + (j < nB ? 1 : 0);
        if (tc05::elect_one()) {
          mbar_expect_tx(full, act * F5_TILE);
          for (int t = 0; t < 2; ++t) {
            if (j >= (t ? nB : nA)) continue;
            const int kb = s_item[t][j] >> 3;
            tma_load_rhb(ring + (st * 2 + t) * F5_TILE, isv ? &tv : &tk, full, isv ? perm_v : perm_k,
                         0, kb * p.bs, hk, b);
          }
        }
        __syncwarp();
      };
      while (jk < nsteps || jv < nsteps) {
        bool progress = false;
        if (jk < nsteps && (jk < NK || test(&k_empty[jk % NK], ((jk / NK) - 1) & 1))) {
          issue(false, jk++);
          progress = true;
        }
        if (jv < nsteps && (jv < NV || test(&v_empty[jv % NV], ((jv / NV) - 1) & 1))) {
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
    // ================= MMA issuer (S and PV queues, polled).  The whole warp runs
    // the loop, so the descriptors stay warp-uniform; barrier tests are made
    // uniform by a vote and one elected lane (always lane 0) issues the MMAs and
    // commits.
    {
      auto test = [&](uint64_t *bar, uint32_t par) {
        return __any_sync(0xffffffffu, mbar_test(bar, par));
      };
      if (!mbar_wait(&bar_q, 0)) report(p.status, BSA_DEVERR_TIMEOUT);
      // descriptors built once; per MMA only a 64-bit add (the issuing thread's
      // scalar work is on the critical path of every step)
      const uint64_t dq0 = tc05::sdesc(smem_u32(sQ), 16, 1024);
      const uint64_t dk0 = tc05::sdesc(smem_u32(sK), 16, 1024);
      const uint64_t dv0 = tc05::sdesc(smem_u32(sV), F5_BS * 128, 1024);
      int js = 0, jp = 0;
      uint32_t idle = 0;
      while (js < nsteps || jp < nsteps) {
        bool progress = false;
        if (jp < js && test(&p_full[jp & 1], (jp >> 1) & 1) && test(&v_full[jp % NV], (jp / NV) & 1)) {
          const int st = jp % NV, bb = jp & 1;
          tc05::fence_after();
          for (int t = 0; t < 2; ++t) {
            if (jp >= (t ? nB : nA)) continue;
            // P (16-bit pairs) over the step's S columns is the A operand
            const uint32_t ta = tc05::taddr(tmem, 16 * t, F5_SCOL0 + 64 * bb);
            const uint64_t db = tc05::dadd(dv0, (st * 2 + t) * F5_TILE);
            const uint32_t d = tc05::taddr(tmem, 16 * t, F5_OCOL);
            if (tc05::elect_one()) {
#pragma unroll
              for (int ks = 0; ks < F5_BS / 16; ++ks)
                tc05::mma_f16_ts(d, ta + ks * 8, tc05::dadd(db, ks * 2048), IDESC_PV,
                                 (jp > 0 || ks > 0) ? 1u : 0u);
            }
            __syncwarp();
          }
          if (tc05::elect_one()) {
            tc05::commit(&v_empty[st]);
            tc05::commit(&s_empty[bb]);
            tc05::commit(&o_done);
            if (jp == nsteps - 1) tc05::commit(&o_final);
          }
          __syncwarp();
          ++jp;
          progress = true;
        }
        if (js < nsteps && test(&k_full[js % NK], (js / NK) & 1) &&
            (js < 2 || test(&s_empty[js & 1], ((js >> 1) - 1) & 1))) {
          const int st = js % NK, bb = js & 1;
          tc05::fence_after();
          for (int t = 0; t < 2; ++t) {
            if (js >= (t ? nB : nA)) continue;
            const uint64_t da = tc05::dadd(dq0, t * F5_TILE);
            const uint64_t db = tc05::dadd(dk0, (st * 2 + t) * F5_TILE);
            const uint32_t d = tc05::taddr(tmem, 16 * t, F5_SCOL0 + 64 * bb);
            if (tc05::elect_one()) {
#pragma unroll
              for (int ks = 0; ks < F5_D / 16; ++ks)
                tc05::mma_f16(d, tc05::dadd(da, ks * 32), tc05::dadd(db, ks * 32), IDESC_S, ks > 0);
            }
            __syncwarp();
          }
          if (tc05::elect_one()) {
            tc05::commit(&s_full[bb]);
            tc05::commit(&k_empty[st]);
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
    // ================= softmax warps 0-3
    const int t = lane >> 4;            // tile of this thread
    const int r = warp * 16 + (lane & 15);  // query row within its block
    const int qi = qb0 + t;                   // local query block (global p.q0 + qi)
    const int nmine = t ? nB : nA;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float *gaterow =
        (p.gate && qi < p.nq)
            ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn
            : nullptr;
    float m_used = -INFINITY, l = 0.f;
    float s[64];
    for (int j = 0; j < nsteps; ++j) {
      const int bb = j & 1;
      if (!mbar_wait(&s_full[bb], (j >> 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
      tc05::fence_after();
      tc05::ld32(tmem + lane_base + F5_SCOL0 + 64 * bb, s);
      tc05::ld32(tmem + lane_base + F5_SCOL0 + 64 * bb + 32, s + 32);
      tc05::wait_ld();
      const bool active = j < nmine;
      float mx = -INFINITY, g2 = 0.f;
      if (active) {
        const int item = s_item[t][j];
        const int kind = item & 7, kb = item >> 3;
        g2 = gaterow ? s_gv[t][j] * kLog2e : 0.f;
        if (kind & (KIND_TRIU | KIND_PAD)) {  // diagonal / padded block only
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (((kind & KIND_TRIU) && c > r) || ((kind & KIND_PAD) && kb * p.bs + c >= p.L))
              s[c] = -INFINITY;
        }
        // row max of the raw scores (scale2 > 0)
        const float mr = max64(s);
        mx = mr == -INFINITY ? -INFINITY : fmaf(mr, p.scale2, g2);
      }
      const bool need = active && mx > -INFINITY && (m_used == -INFINITY || mx > m_used + F5_RESCALE);
      float alpha = 1.f;
      if (need) {
        alpha = m_used == -INFINITY ? 0.f : ex2(m_used - mx);
        m_used = mx;
        l *= alpha;
      }
      // p = 2^(s*scale2 + g2 - m_used): one fma + one ex2 per element, packed to T
      uint32_t w[32];
      if (active) {
        const float off = g2 - (m_used == -INFINITY ? 0.f : m_used);
        float sum8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) sum8[i] = 0.f;
        // column pairs through the packed f32x2 pipe (same rounding per element)
        const float2 s22 = make_float2(p.scale2, p.scale2), off2 = make_float2(off, off);
        float2 acc2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) acc2[i] = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const float2 e = fma2(make_float2(s[c], s[c + 1]), s22, off2);
          const float2 pp = make_float2(ex2(e.x), ex2(e.y));
          acc2[(c >> 1) & 3] = add2(acc2[(c >> 1) & 3], pp);
          w[c >> 1] = Mma<T>::pack(pp.x, pp.y);
        }
        sum8[0] = acc2[0].x; sum8[1] = acc2[0].y; sum8[2] = acc2[1].x; sum8[3] = acc2[1].y;
        sum8[4] = acc2[2].x; sum8[5] = acc2[2].y; sum8[6] = acc2[3].x; sum8[7] = acc2[3].y;
        l += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      }
      // a rescale of O needs PV_{j-1} complete (S_j was issued after PV_{j-2}
      // completed, so the barrier is at most one phase behind: no ambiguity)
      if (__any_sync(0xffffffffu, need) && j >= 1) {
        if (!mbar_wait(&o_done, (j - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
        float o[32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t ta = tmem + lane_base + F5_OCOL + 32 * half;
          tc05::ld32(ta, o);
          tc05::wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] *= alpha;
          tc05::st32(ta, o);
        }
        tc05::wait_st();
      }
      // P over this row's S columns (all 64 were read above)
      tc05::st32(tmem + lane_base + F5_SCOL0 + 64 * bb, reinterpret_cast<const float *>(w));
      tc05::wait_st();
      tc05::fence_before();
      tc05::mbar_arrive(&p_full[bb]);
    }
    // ---- epilogue: O / l
    if (nsteps > 0) {
      // the last PV: a barrier with a single phase, since o_done may be anywhere
      // between PV_{n-3} and PV_{n-1} here (two parity waits on it could miss)
      if (!mbar_wait(&o_final, 0)) report(p.status, BSA_DEVERR_TIMEOUT);
      tc05::fence_after();
    }
    float o[64];
    tc05::ld32(tmem + lane_base + F5_OCOL, o);
    tc05::ld32(tmem + lane_base + F5_OCOL + 32, o + 32);
    tc05::wait_ld();
    if (nmine == 0) {  // never accumulated: the TMEM columns hold stale data
#pragma unroll
      for (int c = 0; c < 64; ++c) o[c] = 0.f;
    }
    const long long grow = (long long)qi * p.bs + r;
    if (qi < p.nq) {
      const long long bh = (long long)b * p.Hq + h;
      if (p.lse) p.lse[bh * p.Lp + grow] = l > 0.f ? m_used + __log2f(l) : INFINITY;
      if (grow < p.Lq) {
        const float inv = (nmine > 0 && l > 0.f) ? 1.f / l : 0.f;
        T *orow = reinterpret_cast<T *>(p.o) + b * p.o_sb + h * p.o_sh + grow * p.o_sl;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          uint4 w;
          w.x = Mma<T>::pack(o[c8 * 8 + 0] * inv, o[c8 * 8 + 1] * inv);
          w.y = Mma<T>::pack(o[c8 * 8 + 2] * inv, o[c8 * 8 + 3] * inv);
          w.z = Mma<T>::pack(o[c8 * 8 + 4] * inv, o[c8 * 8 + 5] * inv);
          w.w = Mma<T>::pack(o[c8 * 8 + 6] * inv, o[c8 * 8 + 7] * inv);
          *reinterpret_cast<uint4 *>(orow + c8 * 8) = w;
        }
      }
    }
  }
  tc05::fence_before();
  __syncthreads();
  if (warp == 5) {
    tc05::fence_after();
    tc05::dealloc(tmem, F5_TMEM_COLS);
  }
}

// ------------------------------------------------------------------ launcher
bool fwd_sm100_applicable(const bsa_attn_args *a) {
  return a->dtype != BSA_F32 && a->bs == 64 && a->D == 64 && a->sel && a->kk <= F5_MAXN &&
         !a->out_gate.ptr && !getenv("BSA_FWD_LEGACY");
}

bsa_status launch_fwd_sm100(const bsa_attn_args *a, const AttnParams &p, cudaStream_t st) {
  TensorMap4 mq, mk, mv;
  bsa_status s;
  if ((s = make_tmap(&mq, a->q.ptr, a->dtype, a->B, a->Hq, p.Lq, 64, a->q.sb, a->q.sh, a->q.sl, 64, "q")))
    return s;
  if ((s = make_tmap(&mk, a->k.ptr, a->dtype, a->B, a->Hkv, a->L, 64, a->k.sb, a->k.sh, a->k.sl, 64, "k")))
    return s;
  if ((s = make_tmap(&mv, a->v.ptr, a->dtype, a->B, a->Hkv, a->L, 64, a->v.sb, a->v.sh, a->v.sl, 64, "v")))
    return s;
  auto pk = [](const TensorMap4 &m) { return m.perm[0] | (m.perm[1] << 2) | (m.perm[2] << 4); };
  const long long grid = (long long)a->B * a->Hq * ((p.nq + 1) / 2);
  // K / V ring stages: 2 / 2 by default; BSA_FWD_STAGES="KV" (two digits) overrides
  const char *env = getenv("BSA_FWD_STAGES");
  const int cfg = env ? atoi(env) : 22;
#define BSA_F5_LAUNCH(T_, K_, V_)                                                                \
  {                                                                                             \
    auto kern = attn_fwd_sm100_kernel<T_, K_, V_>;                                              \
    constexpr int sm = f5_smem<K_, V_>();                                                       \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);                \
    kern<<<(unsigned)grid, 192, sm, st>>>(mq.map, mk.map, mv.map, pk(mq), pk(mk), pk(mv), p);   \
  }
#define BSA_F5_PICK(T_)                                   \
  if (cfg == 32) BSA_F5_LAUNCH(T_, 3, 2)                  \
  else if (cfg == 23) BSA_F5_LAUNCH(T_, 2, 3)             \
  else BSA_F5_LAUNCH(T_, 2, 2)
  if (a->dtype == BSA_BF16) {
    BSA_F5_PICK(__nv_bfloat16)
  } else {
    BSA_F5_PICK(__half)
  }
#undef BSA_F5_PICK
#undef BSA_F5_LAUNCH
  return check_launch("attn_fwd_sm100");
}

}  // namespace bsa
