// Block-sparse attention forward for sm_100a.
//
// One CTA per (batch, query head, query block); the CTA index puts the query
// heads of one KV group next to each other so their shared K/V tiles are
// served from L2.  Selected K/V blocks are streamed through shared memory by
// TMA (128B-swizzled boxes, mbarrier completion, NST-deep ring), each warp owns
// 16 query rows and runs QK^T and PV on bf16/f16 mma.sync tiles with the
// online-softmax state in registers.  The selection slot table (block id +
// mask kind, duplicates removed in TOKEN mode) is built once per CTA in shared
// memory so the producer thread only issues loads for live slots.
//
// Math follows the reference forward (src/triton_kernel.py:41-74): per slot,
// S = Q K^T * scale (+ gate), causal masks, online max / sum, O = acc / l.
// Internally exponentials are base 2 with scale*log2(e) folded in; the row
// log-sum-exp is written in that domain for the backward.
#include "bsa_attn.cuh"
#include "bsa_host.h"

namespace bsa {

template <int BS, int D>
struct FwdCfg : TileCfg<BS, D> {
  using B_ = TileCfg<BS, D>;
  static constexpr int NST = D >= 128 ? 2 : 3;  // K/V ring depth
  static constexpr bool QREG = D <= 128;        // Q fragments kept in registers
  static constexpr int SMEM = 1024 + B_::TILE + NST * 2 * B_::CH;
};

// Item word: (slot << 8) | (chunk << 3) | kind, -1 = end of work.
template <typename T, int BS, int D>
__global__ void __launch_bounds__(TileCfg<BS, D>::NT)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const int perm_q, const int perm_k,
                    const int perm_v, const AttnParams p) {
  using Cfg = FwdCfg<BS, D>;
  constexpr int NST = Cfg::NST, KC = Cfg::KC, NCH = Cfg::NCH, NT = Cfg::NT;
  constexpr int NT8 = KC / 8;  // 8-key n-tiles per chunk
  constexpr int DK = D / 16;   // 16-wide k-steps over D
  constexpr int DN = D / 8;    // 8-wide n-tiles over D
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sQ = smem;
  uint8_t *sKV = smem + Cfg::TILE;
  __shared__ __align__(8) uint64_t bar[NST + 1];
  __shared__ int s_slot[kMaxKK];
  __shared__ int s_item[NST];
  __shared__ int s_kblk[NST];

  // ---- CTA coordinates
  long long id = blockIdx.x;
  const int gi = (int)(id % p.grp);
  id /= p.grp;
  const int qi = (int)(id % p.nq);  // local query block; qblk is its global index
  id /= p.nq;
  const int qblk = p.q0 + qi;
  const int hk = (int)(id % p.Hkv);
  const int b = (int)(id / p.Hkv);
  const int h = hk * p.grp + gi;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int32_t *selrow =
      p.sel ? p.sel + b * p.sel_sb + hk * p.sel_sh + (long long)qi * p.sel_sn : nullptr;
  const float *gaterow =
      p.gate ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn : nullptr;

  if (selrow)
    build_slot_table(s_slot, selrow, p.kk, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal,
                     p.status);
  if (tid == 0) {
    for (int s = 0; s <= NST; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
  }
  __syncthreads();

  // ---- producer state (thread 0 only)
  int cur_slot = 0, cur_chunk = 0;
  auto next_item = [&](int &kb_out) -> int {
    while (cur_slot < p.kk) {
      int kind, kb;
      if (selrow) {
        const int w = s_slot[cur_slot];
        kind = w & 7;
        kb = w >> 3;
      } else {
        kb = cur_slot;
        kind = slot_kind(kb, cur_slot, false, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal,
                         p.status);
      }
      if (kind == KIND_SKIP || ((kind & KIND_PAD) && kb * p.bs + cur_chunk * KC >= p.L)) {
        ++cur_slot;
        cur_chunk = 0;
        continue;
      }
      const int item = (cur_slot << 8) | (cur_chunk << 3) | kind;
      if (++cur_chunk == NCH) {
        cur_chunk = 0;
        ++cur_slot;
      }
      kb_out = kb;
      return item;
    }
    return -1;
  };
  auto issue = [&](int st, int item, int kb) {
    const int chunk = (item >> 3) & 31;
    uint8_t *dk = sKV + st * 2 * Cfg::CH;
    uint8_t *dv = dk + Cfg::CH;
    mbar_expect_tx(&bar[st], 2 * Cfg::CH);
    const int row = kb * p.bs + chunk * KC;
#pragma unroll
    for (int r = 0; r < D / 64; ++r) {
      tma_load_rhb(dk + r * KC * 128, &tk, &bar[st], perm_k, r * 64, row, hk, b);
      tma_load_rhb(dv + r * KC * 128, &tv, &bar[st], perm_v, r * 64, row, hk, b);
    }
  };

  if (tid == 0) {
    mbar_expect_tx(&bar[NST], Cfg::TILE);
#pragma unroll
    for (int r = 0; r < D / 64; ++r)
      tma_load_rhb(sQ + r * BS * 128, &tq, &bar[NST], perm_q, r * 64, qi * p.bs, h, b);
    for (int s = 0; s < NST; ++s) {
      int kb = 0;
      const int item = next_item(kb);
      s_item[s] = item;
      s_kblk[s] = kb;
      if (item >= 0) issue(s, item, kb);
    }
  }
  __syncthreads();

  const uint32_t q_base = smem_u32(sQ);
  if (!mbar_wait(&bar[NST], 0)) report(p.status, BSA_DEVERR_TIMEOUT);
  uint32_t qf[Cfg::QREG ? DK : 1][4];
  if constexpr (Cfg::QREG) {
#pragma unroll
    for (int ks = 0; ks < DK; ++ks)
      ldsm_x4(swz(q_base, BS, warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), qf[ks][0],
              qf[ks][1], qf[ks][2], qf[ks][3]);
  }

  float acc[DN][4];
#pragma unroll
  for (int n = 0; n < DN; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int r0 = warp * 16 + (lane >> 2);  // query rows of this lane within the block
  const int r1 = r0 + 8;

  for (int it = 0;; ++it) {
    const int st = it % NST;
    const int item = s_item[st];
    if (item < 0) break;
    const int kb = s_kblk[st];
    if (!mbar_wait(&bar[st], (it / NST) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
    const int slot = item >> 8, chunk = (item >> 3) & 31, kind = item & 7;
    // Warp-uniform skip: every key of this chunk lies above the warp's rows.
    const bool dead = (kind & KIND_TRIU) && chunk * KC > warp * 16 + 15;
    if (!dead) {
      const uint32_t k_base = smem_u32(sKV + st * 2 * Cfg::CH);
      const uint32_t v_base = k_base + Cfg::CH;
      float s[NT8][4];
#pragma unroll
      for (int n = 0; n < NT8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < DK; ++ks) {
        uint32_t a[4];
        if constexpr (Cfg::QREG) {
          a[0] = qf[ks][0];
          a[1] = qf[ks][1];
          a[2] = qf[ks][2];
          a[3] = qf[ks][3];
        } else {
          ldsm_x4(swz(q_base, BS, warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), a[0], a[1],
                  a[2], a[3]);
        }
#pragma unroll
        for (int np = 0; np < KC / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(swz(k_base, KC, np * 16 + (lane & 7) + ((lane >> 4) << 3),
                      ks * 16 + ((lane >> 3) & 1) * 8),
                  b0, b1, b2, b3);
          Mma<T>::run(s[2 * np], a, b0, b1);
          Mma<T>::run(s[2 * np + 1], a, b2, b3);
        }
      }
      // scale, gate, masks (log2 domain)
      const float g2 = gaterow ? __ldg(gaterow + slot) * kLog2e : 0.f;
      const int key0 = chunk * KC + (lane & 3) * 2;  // key index within the block
#pragma unroll
      for (int n = 0; n < NT8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + n * 8 + (e & 1);
          const int row = e < 2 ? r0 : r1;
          float x = fmaf(s[n][e], p.scale2, g2);
          if ((kind & KIND_TRIU) && key > row) x = -INFINITY;
          if ((kind & KIND_PAD) && kb * p.bs + key >= p.L) x = -INFINITY;
          s[n][e] = x;
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < NT8; ++n) {
        mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
        mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float base0 = mn0 == -INFINITY ? 0.f : mn0;
      const float base1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = ex2(m0 - base0), al1 = ex2(m1 - base1);
      m0 = mn0;
      m1 = mn1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int n = 0; n < NT8; ++n) {
        s[n][0] = ex2(s[n][0] - base0);
        s[n][1] = ex2(s[n][1] - base0);
        s[n][2] = ex2(s[n][2] - base1);
        s[n][3] = ex2(s[n][3] - base1);
        ps0 += s[n][0] + s[n][1];
        ps1 += s[n][2] + s[n][3];
      }
      l0 = l0 * al0 + ps0;
      l1 = l1 * al1 + ps1;
#pragma unroll
      for (int n = 0; n < DN; ++n) {
        acc[n][0] *= al0;
        acc[n][1] *= al0;
        acc[n][2] *= al1;
        acc[n][3] *= al1;
      }
      // O += P V
#pragma unroll
      for (int ks = 0; ks < KC / 16; ++ks) {
        uint32_t a[4];
        a[0] = Mma<T>::pack(s[2 * ks][0], s[2 * ks][1]);
        a[1] = Mma<T>::pack(s[2 * ks][2], s[2 * ks][3]);
        a[2] = Mma<T>::pack(s[2 * ks + 1][0], s[2 * ks + 1][1]);
        a[3] = Mma<T>::pack(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(swz(v_base, KC, ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                        dp * 16 + ((lane >> 4) << 3)),
                    b0, b1, b2, b3);
          Mma<T>::run(acc[2 * dp], a, b0, b1);
          Mma<T>::run(acc[2 * dp + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();  // stage st fully consumed
    if (tid == 0) {
      int kb2 = 0;
      const int nxt = next_item(kb2);
      s_item[st] = nxt;
      s_kblk[st] = kb2;
      if (nxt >= 0) issue(st, nxt, kb2);
    }
  }

  // ---- epilogue
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const long long bh = (long long)b * p.Hq + h;
  if (p.lse && (lane & 3) == 0) {
    p.lse[bh * p.Lp + (long long)qi * p.bs + r0] = l0 > 0.f ? m0 + __log2f(l0) : INFINITY;
    p.lse[bh * p.Lp + (long long)qi * p.bs + r1] = l1 > 0.f ? m1 + __log2f(l1) : INFINITY;
  }
  // stage O (rounded to T) in the Q region, then 16-byte coalesced stores
#pragma unroll
  for (int n = 0; n < DN; ++n) {
    const int col = n * 8 + (lane & 3) * 2;
    const uint32_t w0 = Mma<T>::pack(acc[n][0] * inv0, acc[n][1] * inv0);
    const uint32_t w1 = Mma<T>::pack(acc[n][2] * inv1, acc[n][3] * inv1);
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(swz(q_base, BS, r0, col)), "r"(w0));
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(swz(q_base, BS, r1, col)), "r"(w1));
  }
  __syncthreads();
  T *obase = reinterpret_cast<T *>(p.o) + b * p.o_sb + h * p.o_sh;
  const T *gbase = p.og ? reinterpret_cast<const T *>(p.og) + b * p.og_sb + h * p.og_sh : nullptr;
  for (int idx = tid; idx < BS * (D / 8); idx += NT) {
    const int row = idx / (D / 8), c8 = idx % (D / 8);
    const long long grow = (long long)qi * p.bs + row;
    if (grow >= p.Lq) continue;
    uint4 val;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                 : "r"(swz(q_base, BS, row, c8 * 8)));
    if (gbase) {
      const uint4 g = *reinterpret_cast<const uint4 *>(gbase + grow * p.og_sl + c8 * 8);
      T *ov = reinterpret_cast<T *>(&val);
      const T *gv = reinterpret_cast<const T *>(&g);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float sg = Mma<T>::to_f(Mma<T>::from_f(1.f / (1.f + expf(-Mma<T>::to_f(gv[e])))));
        ov[e] = Mma<T>::from_f(Mma<T>::to_f(ov[e]) * sg);
      }
    }
    *reinterpret_cast<uint4 *>(obase + grow * p.o_sl + c8 * 8) = val;
  }
}

// ------------------------------------------------------------------ fp32 path
// Exact-fp32 SIMT forward used for fp32 inputs (the parity mode of the
// reference's fp32 configuration).  One CTA of 256 threads per (b, h, qblk);
// S, P and the accumulator live in shared memory; 32-key chunks.
template <int BS, int D>
struct F32Cfg {
  static constexpr int KC = 32;
  static constexpr int LD = D + 1;
  static constexpr int SMEM =
      (BS * LD /*q*/ + 2 * KC * LD /*k,v*/ + BS * (KC + 1) /*S*/ + BS * LD /*acc*/ + 3 * BS) * 4 +
      kMaxKK * 4;
};

template <int BS, int D>
__global__ void __launch_bounds__(256) attn_fwd_f32_kernel(const AttnParams p) {
  using Cfg = F32Cfg<BS, D>;
  constexpr int KC = Cfg::KC, LD = Cfg::LD;
  extern __shared__ float fsm[];
  float *sq = fsm;
  float *sk = sq + BS * LD;
  float *sv = sk + KC * LD;
  float *sS = sv + KC * LD;
  float *sacc = sS + BS * (KC + 1);
  float *sm = sacc + BS * LD;
  float *sl = sm + BS;
  float *sal = sl + BS;
  int *s_slot = reinterpret_cast<int *>(sal + BS);

  long long id = blockIdx.x;
  const int gi = (int)(id % p.grp);
  id /= p.grp;
  const int qi = (int)(id % p.nq);  // local query block; qblk is its global index
  id /= p.nq;
  const int qblk = p.q0 + qi;
  const int hk = (int)(id % p.Hkv);
  const int b = (int)(id / p.Hkv);
  const int h = hk * p.grp + gi;
  const int tid = threadIdx.x;
  const int32_t *selrow =
      p.sel ? p.sel + b * p.sel_sb + hk * p.sel_sh + (long long)qi * p.sel_sn : nullptr;
  const float *gaterow =
      p.gate ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn : nullptr;
  if (selrow)
    build_slot_table(s_slot, selrow, p.kk, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal,
                     p.status);
  const float *q = reinterpret_cast<const float *>(p.q) + b * p.q_sb + h * p.q_sh;
  const float *k = reinterpret_cast<const float *>(p.k) + b * p.k_sb + hk * p.k_sh;
  const float *v = reinterpret_cast<const float *>(p.v) + b * p.v_sb + hk * p.v_sh;
  for (int i = tid; i < BS * D; i += 256) {
    const int r = i / D, d = i % D;
    const long long gr = (long long)qi * p.bs + r;
    sq[r * LD + d] = gr < p.Lq ? q[gr * p.q_sl + d] : 0.f;
    sacc[r * LD + d] = 0.f;
  }
  for (int r = tid; r < BS; r += 256) {
    sm[r] = -INFINITY;
    sl[r] = 0.f;
  }
  __syncthreads();
  for (int slot = 0; slot < p.kk; ++slot) {
    int kind, kb;
    if (selrow) {
      kind = s_slot[slot] & 7;
      kb = s_slot[slot] >> 3;
    } else {
      kb = slot;
      kind = slot_kind(kb, slot, false, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal, p.status);
    }
    if (kind == KIND_SKIP) continue;
    const float g = gaterow ? gaterow[slot] : 0.f;
    for (int c0 = 0; c0 < BS; c0 += KC) {
      for (int i = tid; i < KC * D; i += 256) {
        const int r = i / D, d = i % D;
        const long long gr = (long long)kb * p.bs + c0 + r;
        const bool ok = (c0 + r < p.bs) && gr < p.L;
        sk[r * LD + d] = ok ? k[gr * p.k_sl + d] : 0.f;
        sv[r * LD + d] = ok ? v[gr * p.v_sl + d] : 0.f;
      }
      __syncthreads();
      for (int i = tid; i < BS * KC; i += 256) {
        const int r = i / KC, c = i % KC;
        float s = 0.f;
        for (int d = 0; d < D; ++d) s = fmaf(sq[r * LD + d], sk[c * LD + d], s);
        s = s * p.scale + g;
        const int key = c0 + c;
        if (key >= p.bs) s = -INFINITY;
        if ((kind & KIND_TRIU) && key > r) s = -INFINITY;
        if ((kind & KIND_PAD) && (long long)kb * p.bs + key >= p.L) s = -INFINITY;
        sS[r * (KC + 1) + c] = s;
      }
      __syncthreads();
      for (int r = tid; r < BS; r += 256) {
        float mx = -INFINITY;
        for (int c = 0; c < KC; ++c) mx = fmaxf(mx, sS[r * (KC + 1) + c]);
        const float mn = fmaxf(sm[r], mx);
        const float base = mn == -INFINITY ? 0.f : mn;
        const float al = expf(sm[r] - base);
        float sum = 0.f;
        for (int c = 0; c < KC; ++c) {
          const float e = expf(sS[r * (KC + 1) + c] - base);
          sS[r * (KC + 1) + c] = e;
          sum += e;
        }
        sl[r] = sl[r] * al + sum;
        sm[r] = mn;
        sal[r] = al;
      }
      __syncthreads();
      for (int i = tid; i < BS * D; i += 256) {
        const int r = i / D, d = i % D;
        float a = sacc[r * LD + d] * sal[r];
        for (int c = 0; c < KC; ++c) a = fmaf(sS[r * (KC + 1) + c], sv[c * LD + d], a);
        sacc[r * LD + d] = a;
      }
      __syncthreads();
    }
  }
  float *o = reinterpret_cast<float *>(p.o) + b * p.o_sb + h * p.o_sh;
  const float *og = p.og ? reinterpret_cast<const float *>(p.og) + b * p.og_sb + h * p.og_sh : nullptr;
  for (int i = tid; i < BS * D; i += 256) {
    const int r = i / D, d = i % D;
    const long long gr = (long long)qi * p.bs + r;
    if (gr >= p.Lq) continue;
    float val = sl[r] > 0.f ? sacc[r * LD + d] / sl[r] : 0.f;
    if (og) val = val * (1.f / (1.f + expf(-og[gr * p.og_sl + d])));
    o[gr * p.o_sl + d] = val;
  }
  if (p.lse) {
    const long long bh = (long long)b * p.Hq + h;
    for (int r = tid; r < BS; r += 256)
      p.lse[bh * p.Lp + (long long)qi * p.bs + r] =
          sl[r] > 0.f ? (sm[r] + logf(sl[r])) * kLog2e : INFINITY;
  }
}

// ------------------------------------------------------------------ launchers
template <typename T, int BS, int D>
static bsa_status launch_fwd_tc(const bsa_attn_args *a, const AttnParams &p, cudaStream_t st) {
  using Cfg = FwdCfg<BS, D>;
  TensorMap4 mq, mk, mv;
  bsa_status s;
  if ((s = make_tmap(&mq, a->q.ptr, a->dtype, a->B, a->Hq, p.Lq, D, a->q.sb, a->q.sh, a->q.sl, BS,
                     "q")))
    return s;
  if ((s = make_tmap(&mk, a->k.ptr, a->dtype, a->B, a->Hkv, a->L, D, a->k.sb, a->k.sh, a->k.sl,
                     Cfg::KC, "k")))
    return s;
  if ((s = make_tmap(&mv, a->v.ptr, a->dtype, a->B, a->Hkv, a->L, D, a->v.sb, a->v.sh, a->v.sl,
                     Cfg::KC, "v")))
    return s;
  auto pk = [](const TensorMap4 &m) { return m.perm[0] | (m.perm[1] << 2) | (m.perm[2] << 4); };
  auto kern = attn_fwd_kernel<T, BS, D>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  const long long grid = (long long)a->B * a->Hq * p.nq;
  kern<<<(unsigned)grid, Cfg::NT, Cfg::SMEM, st>>>(mq.map, mk.map, mv.map, pk(mq), pk(mk), pk(mv),
                                                    p);
  return check_launch("attn_fwd");
}

template <int BS, int D>
static bsa_status launch_fwd_f32(const AttnParams &p, long long grid, cudaStream_t st) {
  auto kern = attn_fwd_f32_kernel<BS, D>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, F32Cfg<BS, D>::SMEM);
  kern<<<(unsigned)grid, 256, F32Cfg<BS, D>::SMEM, st>>>(p);
  return check_launch("attn_fwd_f32");
}

template <typename T>
static bsa_status dispatch_fwd_tc(const bsa_attn_args *a, const AttnParams &p, cudaStream_t st) {
#define BSA_FWD_CASE(BS_, D_) \
  if (a->bs == BS_ && a->D == D_) return launch_fwd_tc<T, BS_, D_>(a, p, st);
  BSA_FWD_CASE(16, 64)
  BSA_FWD_CASE(32, 64)
  BSA_FWD_CASE(64, 64)
  BSA_FWD_CASE(128, 64)
  BSA_FWD_CASE(32, 128)
  BSA_FWD_CASE(64, 128)
  BSA_FWD_CASE(128, 128)
  BSA_FWD_CASE(64, 256)
  BSA_FWD_CASE(128, 256)
#undef BSA_FWD_CASE
  return fail(BSA_ERR_UNSUPPORTED, "attn_fwd: no bf16/f16 kernel for (bs, D) = (" +
                                       std::to_string(a->bs) + ", " + std::to_string(a->D) + ")");
}

bsa_status fill_attn_params(const bsa_attn_args *a, AttnParams *p, bool bwd);
bool fwd_sm100_applicable(const bsa_attn_args *a);
bool fwd_b128_applicable(const bsa_attn_args *a);
bsa_status launch_fwd_b128(const bsa_attn_args *a, const AttnParams &p, cudaStream_t st);
bsa_status launch_fwd_sm100(const bsa_attn_args *a, const AttnParams &p, cudaStream_t st);

bsa_status run_attn_fwd(const bsa_attn_args *a, cudaStream_t st) {
  AttnParams p;
  bsa_status s = fill_attn_params(a, &p, false);
  if (s) return s;
  if (a->dtype == BSA_F32) {
    const long long grid = (long long)a->B * a->Hq * p.nq;
#define BSA_F32_CASE(BS_, D_) \
  if (a->bs == BS_ && a->D == D_) return launch_fwd_f32<BS_, D_>(p, grid, st);
    BSA_F32_CASE(16, 64)
    BSA_F32_CASE(32, 64)
    BSA_F32_CASE(64, 64)
    BSA_F32_CASE(32, 128)
    BSA_F32_CASE(64, 128)
    BSA_F32_CASE(16, 32)
    BSA_F32_CASE(32, 32)
    BSA_F32_CASE(64, 32)
#undef BSA_F32_CASE
    return fail(BSA_ERR_UNSUPPORTED, "attn_fwd: no fp32 kernel for (bs, D) = (" +
                                         std::to_string(a->bs) + ", " + std::to_string(a->D) + ")");
  }
  if (a->rope_cos) {
    // the in-kernel rotation of q lives in the block-128 tcgen05 kernel
    if (!fwd_b128_applicable(a) || a->D != 256)
      return fail(BSA_ERR_UNSUPPORTED,
                  "attn_fwd: rope inside the kernel needs block 128, D 256, 16-bit types");
    return launch_fwd_b128(a, p, st);
  }
  if (fwd_sm100_applicable(a)) return launch_fwd_sm100(a, p, st);
  if (fwd_b128_applicable(a)) return launch_fwd_b128(a, p, st);
  if (a->dtype == BSA_BF16) return dispatch_fwd_tc<__nv_bfloat16>(a, p, st);
  return dispatch_fwd_tc<__half>(a, p, st);
}

}  // namespace bsa
