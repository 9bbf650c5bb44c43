// Block-sparse attention forward on tcgen05 for block 128, head dim 64 (the
// long-context configuration) or 256 (the Qwen GQA configuration).
//
// One CTA computes one query block (128 rows = one M=128 UMMA tile) of one
// query head.  K and V move through shared memory in 64-column chunks
// (16 KB each), so D = 256 needs no more buffer than D = 64 per ring slot.
// Per live slot j (a selected key block):
//   S_j  = Q K_j^T      per 64-column chunk 4 x tcgen05.mma 128x128x16 (fp32, TMEM)
//   P_j  = 2^(S_j * scale * log2e + gate - m)   (bf16 pairs, TMEM)
//   O   += P_j V_j      per 64-column chunk 8 x tcgen05.mma 128x64x16 into TMEM,
//                       P_j as the A operand from TMEM
// TMEM: S columns [0, 128), P [128, 192), O [192, 192 + D) (D = 64: 256
// allocated, two CTAs per SM; D = 256: 512, one).  Row m of every tile lives in
// lane m.
// An optional sigmoid output gate (Qwen) is applied in the epilogue.
//
// Warp roles (320 threads; <= 96 registers per thread keeps two CTAs per SM):
//   warps 0-7  softmax: warp w reads rows 32*(w&3).. and key columns
//              64*(w>>2)..+63; the two warps of a row quarter exchange their
//              half-row maxima through shared memory (named barrier 1 + (w&3));
//              the maximum in use is raised only when the block exceeds it by
//              more than 2^8 (lazy rescaling; O is then rescaled in TMEM); the
//              exponentials go to registers while PV_{j-1} may still run, and P
//              is written to its TMEM columns once PV_{j-1} has released them;
//              final O / l.
//   warp 8     TMA producer (one thread): Q once, then the K and V chunks into
//              ONE ring of 64-column slots, in the order the MMAs consume them
//              (K of step 0; then K of step j + 1 and V of step j for each j),
//              so a slot is freed by whichever MMAs read it (S for K, PV for V)
//              and both kinds share the buffering.
//   warp 9     TMEM owner and MMA-issuing thread: S_{j+1} as soon as all
//              softmax warps have read S_j, PV_j as soon as P_j is complete.
// Every mbarrier wait is bounded; a timeout sets BSA_DEVERR_TIMEOUT.
#include <type_traits>

#include "bsa_attn.cuh"
#include "bsa_host.h"
#include "bsa_tc05.cuh"

namespace bsa {

namespace {
constexpr int G8_BS = 128;
constexpr int G8_TILE = G8_BS * 64 * 2;  // 16 KB: a 128-row block of 64 columns
constexpr int G8_WPROD = 8, G8_WMMA = 9, G8_THREADS = 320;
constexpr int G8_SCOL = 0, G8_PCOL = 128, G8_OCOL = 192;
constexpr float G8_RESCALE = 8.f;  // log2 units
template <int D>
struct G8 {
  static constexpr int NCH = D / 64;                 // 64-column chunks per row
  // ring slots shared by K and V chunks (D = 64: 5 x 16 KB keeps two CTAs per SM)
  static constexpr int NSL = D == 64 ? 5 : 8;
  static constexpr int SMEM = 1024 + NCH * G8_TILE + NSL * G8_TILE;
  static constexpr uint32_t TMEM_COLS = D == 64 ? 256 : 512;
  static constexpr int MINB = D == 64 ? 2 : 1;       // CTAs per SM
  // live slots kept in shared memory (D = 256 also runs the identity selection,
  // every causal block, for up to 512 blocks)
  static constexpr int MAXN = D == 64 ? 64 : 512;
};
}  // namespace

template <typename T, int D>
__global__ void __launch_bounds__(G8_THREADS, G8<D>::MINB)
    attn_fwd_b128_kernel(const __grid_constant__ CUtensorMap tq,
                         const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const int perm_q,
                         const int perm_k, const int perm_v, const AttnParams p) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = tc05::idesc_f16(kBF16, 128, 128, false);
  constexpr uint32_t IDESC_PV = tc05::idesc_f16(kBF16, 128, 64, true);
  constexpr int NCH = G8<D>::NCH, NSL = G8<D>::NSL;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sQ = smem;                       // Q chunk c at sQ + c * TILE
  uint8_t *sR = sQ + NCH * G8_TILE;         // K/V ring: NSL chunk slots
  __shared__ __align__(8) uint64_t bar_q, r_full[NSL], r_empty[NSL], s_full, s_empty, p_full,
      o_done, q_ready;
  __shared__ uint32_t tmem_base_sh;
  constexpr int MAXN = G8<D>::MAXN;
  __shared__ int s_item[MAXN];   // (kb << 3) | kind of the j-th live slot
  __shared__ float s_gv[MAXN];  // its gate value (read with the list)
  __shared__ int s_n;
  __shared__ float s_xch[3][4][2][32];  // half-row maxima (by step parity), row sums

  long long id = blockIdx.x;
  const int gi = (int)(id % p.grp);
  id /= p.grp;
  const int qi = (int)(id % p.nq);  // local query block (global p.q0 + qi)
  id /= p.nq;
  const int hk = (int)(id % p.Hkv);
  const int b = (int)(id / p.Hkv);
  const int h = hk * p.grp + gi;
  const int qblk = p.q0 + qi;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {  // live-slot list, built by the whole warp
    const int32_t *selrow =
        p.sel ? p.sel + b * p.sel_sb + hk * p.sel_sh + (long long)qi * p.sel_sn : nullptr;
    const float *grow = (p.gate && p.sel)
                            ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn
                            : nullptr;
    const int n = warp_live_slots(selrow, p.sel ? p.kk : p.nblk, MAXN, qblk, p.nblk, p.bs, p.L,
                                  p.mask_mode, p.causal, p.status,
                                  [&](int pos, int kb, int kind, int slot) {
                                    s_item[pos] = (kb << 3) | kind;
                                    s_gv[pos] = grow ? __ldg(grow + slot) : 0.f;
                                  });
    if (lane == 0) s_n = n;
  }
  if (tid == 0) {
    // descriptors fetched ahead of the first TMA load
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    mbar_init(&bar_q, 1);
    for (int s = 0; s < NSL; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&s_empty, 8);  // one arrive per softmax warp
    mbar_init(&p_full, 8);
    mbar_init(&o_done, 1);
    mbar_init(&q_ready, 8);  // one arrive per softmax warp once q is rotated (rope)
    fence_mbar_init();
  }
  if (warp == G8_WMMA) {
    tc05::alloc(&tmem_base_sh, G8<D>::TMEM_COLS);
    tc05::relinquish();
  }
  tc05::fence_before();
  __syncthreads();
  tc05::fence_after();
  const uint32_t tmem = tmem_base_sh;
  const int nsteps = s_n;

  // Ring sequence: K chunks of step 0, then per step j the K chunks of step
  // j + 1 (if any) and the V chunks of step j; item number n uses slot n % NSL.
  // Producer and MMA issuer walk the same sequence with their own counters.
  if (warp == G8_WPROD) {
    // ================= TMA producer: the warp waits together (voted), one
    // elected lane (lane 0) issues the loads
    {
      if (tc05::elect_one()) {
        mbar_expect_tx(&bar_q, NCH * G8_TILE);
        for (int c = 0; c < NCH; ++c)
          tma_load_rhb(sQ + c * G8_TILE, &tq, &bar_q, perm_q, 64 * c, qi * p.bs, h, b);
      }
      __syncwarp();
      int n = 0;
      auto load = [&](bool isv, int j) {
        for (int c = 0; c < NCH; ++c, ++n) {
          const int sl = n % NSL;
          if (n >= NSL && !mbar_wait_warp(&r_empty[sl], ((n / NSL) - 1) & 1))
            report(p.status, BSA_DEVERR_TIMEOUT);
          if (tc05::elect_one()) {
            mbar_expect_tx(&r_full[sl], G8_TILE);
            tma_load_rhb(sR + sl * G8_TILE, isv ? &tv : &tk, &r_full[sl], isv ? perm_v : perm_k,
                         64 * c, (s_item[j] >> 3) * p.bs, hk, b);
          }
          __syncwarp();
        }
      };
      if (nsteps > 0) load(false, 0);
      for (int j = 0; j < nsteps; ++j) {
        if (j + 1 < nsteps) load(false, j + 1);
        load(true, j);
      }
    }
  } else if (warp == G8_WMMA) {
    // ================= MMA issuer: the whole warp runs the sequence (warp-uniform
    // descriptors and waits); one elected lane, always lane 0, issues the MMAs
    // and commits
    {
      if (!mbar_wait_warp((D == 256 && p.rope_cos) ? &q_ready : &bar_q, 0))
        report(p.status, BSA_DEVERR_TIMEOUT);
      const uint64_t dq = tc05::sdesc(smem_u32(sQ), 16, 1024);
      int n = 0;
      auto issue_s = [&](int js) {
        if (js >= 1 && !mbar_wait_warp(&s_empty, (js - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        for (int c = 0; c < NCH; ++c, ++n) {
          const int sl = n % NSL;
          if (!mbar_wait_warp(&r_full[sl], (n / NSL) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
          tc05::fence_after();
          const uint64_t dk = tc05::sdesc(smem_u32(sR + sl * G8_TILE), 16, 1024);
          const uint64_t dqc = dq + c * (G8_TILE >> 4);
          if (tc05::elect_one()) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              tc05::mma_f16(tc05::taddr(tmem, 0, G8_SCOL), dqc + 2 * ks, dk + 2 * ks, IDESC_S,
                            (c > 0 || ks > 0) ? 1u : 0u);
            tc05::commit(&r_empty[sl]);
          }
          __syncwarp();
        }
        if (tc05::elect_one()) tc05::commit(&s_full);
        __syncwarp();
      };
      if (nsteps > 0) issue_s(0);
      for (int jp = 0; jp < nsteps; ++jp) {
        if (jp + 1 < nsteps) issue_s(jp + 1);
        if (!mbar_wait_warp(&p_full, jp & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        for (int c = 0; c < NCH; ++c, ++n) {
          const int sl = n % NSL;
          if (!mbar_wait_warp(&r_full[sl], (n / NSL) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
          tc05::fence_after();
          const uint64_t dv = tc05::sdesc(smem_u32(sR + sl * G8_TILE), G8_TILE, 1024);
          if (tc05::elect_one()) {
#pragma unroll
            for (int ks = 0; ks < G8_BS / 16; ++ks)  // keys 16*ks: P columns 8*ks (16-bit pairs)
              tc05::mma_f16_ts(tc05::taddr(tmem, 0, G8_OCOL + 64 * c),
                               tc05::taddr(tmem, 0, G8_PCOL + 8 * ks), dv + 128 * ks, IDESC_PV,
                               (jp > 0 || ks > 0) ? 1u : 0u);
            tc05::commit(&r_empty[sl]);
          }
          __syncwarp();
        }
        if (tc05::elect_one()) tc05::commit(&o_done);
        __syncwarp();
      }
    }
  } else {
    // ================= softmax warps 0-7
    const int quad = warp & 3, hf = warp >> 2;
    const int r = quad * 32 + lane;  // query row within the block
    const int cb = 64 * hf;          // first key column of this warp
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const float *gaterow = (p.gate && p.sel)
                               ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn
                               : nullptr;
    if constexpr (D == 256) if (p.rope_cos) {
      // partial rotary embedding of q in shared memory, before the first S MMA:
      // the rotary dims (< rope_rot <= 64) all lie in Q's first 64-column chunk;
      // item = (row, group of 8 pairs), 16-byte loads of the swizzled tile
      if (!mbar_wait(&bar_q, 0)) report(p.status, BSA_DEVERR_TIMEOUT);
      const int half = p.rope_rot / 2, ng = half / 8;
      for (int it = warp * 32 + lane; it < G8_BS * ng; it += 256) {
        const int row = it / ng, i0 = 8 * (it % ng), i1 = i0 + half;
        const long long pos = (long long)qblk * p.bs + row;
        if (pos >= p.L) continue;
        uint4 *a0 = reinterpret_cast<uint4 *>(sQ + swz(0, G8_BS, row, i0));
        uint4 *a1 = reinterpret_cast<uint4 *>(sQ + swz(0, G8_BS, row, i1));
        const T *cs = reinterpret_cast<const T *>(p.rope_cos) + b * p.rope_sb + pos * p.rope_sl;
        const T *sn = reinterpret_cast<const T *>(p.rope_sin) + b * p.rope_sb + pos * p.rope_sl;
        const uint4 ux0 = *a0, ux1 = *a1;
        const uint4 uc0 = *reinterpret_cast<const uint4 *>(cs + i0), uc1 = *reinterpret_cast<const uint4 *>(cs + i1);
        const uint4 us0 = *reinterpret_cast<const uint4 *>(sn + i0), us1 = *reinterpret_cast<const uint4 *>(sn + i1);
        const T *x0 = reinterpret_cast<const T *>(&ux0), *x1 = reinterpret_cast<const T *>(&ux1);
        const T *c0 = reinterpret_cast<const T *>(&uc0), *c1 = reinterpret_cast<const T *>(&uc1);
        const T *s0 = reinterpret_cast<const T *>(&us0), *s1 = reinterpret_cast<const T *>(&us1);
        uint4 uy0, uy1;
        T *y0 = reinterpret_cast<T *>(&uy0), *y1 = reinterpret_cast<T *>(&uy1);
#pragma unroll
        for (int e = 0; e < 8; ++e) rope_pair<T>(x0[e], x1[e], c0[e], s0[e], c1[e], s1[e], y0[e], y1[e]);
        *a0 = uy0;
        *a1 = uy1;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&q_ready);
    }
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; j < nsteps; ++j) {
      if (!mbar_wait(&s_full, j & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
      tc05::fence_after();
      float s[64];
      tc05::ld32(tmem + lane_base + G8_SCOL + cb, s);
      tc05::ld32(tmem + lane_base + G8_SCOL + cb + 32, s + 32);
      tc05::wait_ld();
      tc05::fence_before();
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&s_empty);
      const int item = s_item[j];
      const int kind = item & 7, kb = item >> 3;
      const float g2 = gaterow ? s_gv[j] * kLog2e : 0.f;
      if (kind & (KIND_TRIU | KIND_PAD)) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (((kind & KIND_TRIU) && cb + c > r) || ((kind & KIND_PAD) && kb * p.bs + cb + c >= p.L))
            s[c] = -INFINITY;
      }
      // block row maximum (both halves of the row, through shared memory), then
      // the exponentials into registers while PV_{j-1} may still be running
      const float mh = max64(s);
      s_xch[j & 1][quad][hf][lane] = mh;
      named_bar_sync(1 + quad, 64);
      const float mr = fmaxf(mh, s_xch[j & 1][quad][hf ^ 1][lane]);
      const float mx = mr == -INFINITY ? -INFINITY : fmaf(mr, p.scale2, g2);
      bool need = false;
      float alpha = 1.f;
      if (mx > -INFINITY && (m_used == -INFINITY || mx > m_used + G8_RESCALE)) {
        alpha = m_used == -INFINITY ? 0.f : ex2(m_used - mx);
        m_used = mx;
        l *= alpha;
        need = true;
      }
      const float off = g2 - (m_used == -INFINITY ? 0.f : m_used);
      uint32_t w[32];
      float sum8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum8[i] = 0.f;
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float p0 = ex2(fmaf(s[c], p.scale2, off)), p1 = ex2(fmaf(s[c + 1], p.scale2, off));
        sum8[c & 7] += p0;
        sum8[(c & 7) + 1] += p1;
        w[c >> 1] = Mma<T>::pack(p0, p1);
      }
      l += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      // PV_{j-1} must be complete before P is overwritten (and before O is rescaled)
      if (j >= 1) {
        if (!mbar_wait(&o_done, (j - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
      }
      if (__any_sync(0xffffffffu, need) && j >= 1) {
        // O columns [hf * D/2, +D/2) of this warp's rows, 32 at a time
#pragma unroll 1
        for (int c32 = 0; c32 < D / 64; ++c32) {
          float o[32];
          const uint32_t ta = tmem + lane_base + G8_OCOL + hf * (D / 2) + 32 * c32;
          tc05::ld32(ta, o);
          tc05::wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] *= alpha;
          tc05::st32(ta, o);
        }
        tc05::wait_st();
      }
      // P of keys cb..cb+63 -> TMEM columns PCOL + cb/2 .. +31 of this row
      tc05::st32(tmem + lane_base + G8_PCOL + 32 * hf, reinterpret_cast<const float *>(w));
      tc05::wait_st();
      tc05::fence_before();
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&p_full);
    }
    // ---- epilogue: O / l, l summed over the two halves of the row
    s_xch[2][quad][hf][lane] = l;
    named_bar_sync(1 + quad, 64);
    const float lt = l + s_xch[2][quad][hf ^ 1][lane];
    if (nsteps > 0) {
      if (!mbar_wait(&o_done, (nsteps - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
      tc05::fence_after();
    }
    const long long grow = (long long)qi * p.bs + r;
    const long long bh = (long long)b * p.Hq + h;
    if (p.lse && hf == 0) p.lse[bh * p.Lp + grow] = lt > 0.f ? m_used + __log2f(lt) : INFINITY;
    const float inv = (nsteps > 0 && lt > 0.f) ? 1.f / lt : 0.f;
    T *orow = reinterpret_cast<T *>(p.o) + b * p.o_sb + h * p.o_sh + grow * p.o_sl + hf * (D / 2);
    const T *grow_g = p.og ? reinterpret_cast<const T *>(p.og) + b * p.og_sb + h * p.og_sh +
                                 grow * p.og_sl + hf * (D / 2)
                           : nullptr;
#pragma unroll 1
    for (int c32 = 0; c32 < D / 64; ++c32) {
      float o[32];
      tc05::ld32(tmem + lane_base + G8_OCOL + hf * (D / 2) + 32 * c32, o);
      tc05::wait_ld();
      if (grow >= p.Lq) continue;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint4 wv;
        uint32_t *w = reinterpret_cast<uint32_t *>(&wv);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          w[e] = Mma<T>::pack(o[c8 * 8 + 2 * e] * inv, o[c8 * 8 + 2 * e + 1] * inv);
        if (grow_g) {  // sigmoid output gate, rounded as the reference's bf16 ops
          const uint4 gq = *reinterpret_cast<const uint4 *>(grow_g + 32 * c32 + c8 * 8);
          T *ov = reinterpret_cast<T *>(&wv);
          const T *gv = reinterpret_cast<const T *>(&gq);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float sg = Mma<T>::to_f(Mma<T>::from_f(1.f / (1.f + expf(-Mma<T>::to_f(gv[e])))));
            ov[e] = Mma<T>::from_f(Mma<T>::to_f(ov[e]) * sg);
          }
        }
        *reinterpret_cast<uint4 *>(orow + 32 * c32 + c8 * 8) = wv;
      }
    }
  }
  tc05::fence_before();
  __syncthreads();
  if (warp == G8_WMMA) {
    tc05::fence_after();
    tc05::dealloc(tmem, G8<D>::TMEM_COLS);
  }
}

bool fwd_b128_applicable(const bsa_attn_args *a) {
  if (a->dtype == BSA_F32 || a->bs != 128 || (a->D != 64 && a->D != 256) || getenv("BSA_FWD_LEGACY"))
    return false;
  const int maxn = a->D == 64 ? G8<64>::MAXN : G8<256>::MAXN;
  return a->sel ? a->kk <= maxn : (a->D == 256 && a->nblk <= maxn);
}

bsa_status launch_fwd_b128(const bsa_attn_args *a, const AttnParams &p, cudaStream_t st) {
  TensorMap4 mq, mk, mv;
  bsa_status s;
  if ((s = make_tmap(&mq, a->q.ptr, a->dtype, a->B, a->Hq, p.Lq, a->D, a->q.sb, a->q.sh, a->q.sl, 128, "q")))
    return s;
  if ((s = make_tmap(&mk, a->k.ptr, a->dtype, a->B, a->Hkv, a->L, a->D, a->k.sb, a->k.sh, a->k.sl, 128, "k")))
    return s;
  if ((s = make_tmap(&mv, a->v.ptr, a->dtype, a->B, a->Hkv, a->L, a->D, a->v.sb, a->v.sh, a->v.sl, 128, "v")))
    return s;
  auto pk = [](const TensorMap4 &m) { return m.perm[0] | (m.perm[1] << 2) | (m.perm[2] << 4); };
  const long long grid = (long long)a->B * a->Hq * p.nq;
#define BSA_G8(T_, D_)                                                                         \
  {                                                                                            \
    auto kern = attn_fwd_b128_kernel<T_, D_>;                                                  \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G8<D_>::SMEM);     \
    kern<<<(unsigned)grid, G8_THREADS, G8<D_>::SMEM, st>>>(mq.map, mk.map, mv.map, pk(mq),     \
                                                            pk(mk), pk(mv), p);                \
  }
  if (a->dtype == BSA_BF16) {
    if (a->D == 64) BSA_G8(__nv_bfloat16, 64) else BSA_G8(__nv_bfloat16, 256)
  } else {
    if (a->D == 64) BSA_G8(__half, 64) else BSA_G8(__half, 256)
  }
#undef BSA_G8
  return check_launch("attn_fwd_b128");
}

}  // namespace bsa
