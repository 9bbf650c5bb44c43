// Block-sparse attention forward on tcgen05 for block 128, head dim 64 (the
// long-context configuration).
//
// One CTA computes one query block (128 rows = one M=128 UMMA tile) of one
// head.  Per live slot j (a selected key block):
//   S_j  = Q K_j^T      4 x tcgen05.mma 128x128x16 into TMEM (fp32)
//   P_j  = 2^(S_j * scale * log2e + gate - m)   (bf16, shared memory)
//   O   += P_j V_j      8 x tcgen05.mma 128x64x16, O accumulated in TMEM
// TMEM: S columns [0, 128), O columns [128, 192) (256 allocated: two CTAs per SM).
// Row m of every tile lives in TMEM lane m.
//
// Warp roles (320 threads; <= 96 registers per thread keeps two CTAs per SM):
//   warps 0-7  softmax: warp w reads rows 32*(w&3).. and key columns
//              64*(w>>2)..+63; the two warps of a row quarter exchange their
//              half-row maxima through shared memory (named barrier 1 + (w&3));
//              exponentials use the maximum in use and are redone (rarely)
//              when the block raises it by more than 2^8 (lazy rescaling; O is
//              rescaled in TMEM); P is written 128B-swizzled K-major in two
//              64-key regions; final O / l.
//   warp 8     TMA producer (one thread): Q once, then K and V blocks into two
//              rings of two stages (K freed by S_j's completion, V by PV_j's).
//   warp 9     TMEM owner and MMA-issuing thread: S_{j+1} as soon as all
//              softmax warps have read S_j, PV_j as soon as P_j is complete.
// Every mbarrier wait is bounded; a timeout sets BSA_DEVERR_TIMEOUT.
#include <type_traits>

#include "bsa_attn.cuh"
#include "bsa_host.h"
#include "bsa_tc05.cuh"

namespace bsa {

namespace {
constexpr int G8_BS = 128, G8_D = 64, G8_NST = 2;
constexpr int G8_TILE = G8_BS * G8_D * 2;  // 16 KB: a 128-row block of 64 dims
constexpr int G8_MAXN = 64;                // live slots kept in shared memory
constexpr int G8_SMEM = 1024 + G8_TILE + 2 * G8_NST * G8_TILE + 2 * G8_TILE;  // Q, K, V rings, P
constexpr int G8_WPROD = 8, G8_WMMA = 9, G8_THREADS = 320;
constexpr uint32_t G8_TMEM_COLS = 256;
constexpr int G8_SCOL = 0, G8_OCOL = 128;
constexpr float G8_RESCALE = 8.f;  // log2 units
}  // namespace

template <typename T>
__global__ void __launch_bounds__(G8_THREADS, 2)
    attn_fwd_b128_kernel(const __grid_constant__ CUtensorMap tq,
                         const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const int perm_q,
                         const int perm_k, const int perm_v, const AttnParams p) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = tc05::idesc_f16(kBF16, 128, 128, false);
  constexpr uint32_t IDESC_PV = tc05::idesc_f16(kBF16, 128, G8_D, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sQ = smem;
  uint8_t *sK = sQ + G8_TILE;               // K ring
  uint8_t *sV = sK + G8_NST * G8_TILE;      // V ring
  uint8_t *sP = sV + G8_NST * G8_TILE;      // P: keys 0-63 at sP, 64-127 at sP + TILE
  __shared__ __align__(8) uint64_t bar_q, k_full[G8_NST], k_empty[G8_NST], v_full[G8_NST],
      v_empty[G8_NST], s_full, s_empty, p_full, o_done;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int s_item[G8_MAXN];   // (kb << 3) | kind of the j-th live slot
  __shared__ int s_islot[G8_MAXN];
  __shared__ int s_n;
  __shared__ float s_xch[2][4][2][32];  // half-row maxima (by step parity), then sums

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

  if (tid == 0) {
    const int32_t *selrow = p.sel + b * p.sel_sb + hk * p.sel_sh + (long long)qi * p.sel_sn;
    int n = 0;
    for (int slot = 0; slot < p.kk; ++slot) {
      const int kb = __ldg(selrow + slot);
      bool dup = false;
      if (p.mask_mode == BSA_MASK_TOKEN)
        for (int i = 0; i < slot && !dup; ++i) dup = __ldg(selrow + i) == kb;
      const int kind =
          slot_kind(kb, slot, dup, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal, p.status);
      if (kind != KIND_SKIP && n < G8_MAXN) {
        s_item[n] = (kb << 3) | kind;
        s_islot[n] = slot;
        ++n;
      }
    }
    s_n = n;
    mbar_init(&bar_q, 1);
    for (int s = 0; s < G8_NST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&s_empty, 8);  // one arrive per softmax warp
    mbar_init(&p_full, 8);
    mbar_init(&o_done, 1);
    fence_mbar_init();
  }
  if (warp == G8_WMMA) {
    tc05::alloc(&tmem_base_sh, G8_TMEM_COLS);
    tc05::relinquish();
  }
  tc05::fence_before();
  __syncthreads();
  tc05::fence_after();
  const uint32_t tmem = tmem_base_sh;
  const int nsteps = s_n;

  if (warp == G8_WPROD) {
    // ================= TMA producer: Q once; K_{j+1} before waiting for V_j's slot
    if (lane == 0) {
      mbar_expect_tx(&bar_q, G8_TILE);
      tma_load_rhb(sQ, &tq, &bar_q, perm_q, 0, qi * p.bs, h, b);
      auto load = [&](bool isv, int j) {
        const int st = j % G8_NST;
        uint64_t *full = isv ? &v_full[st] : &k_full[st];
        uint64_t *empty = isv ? &v_empty[st] : &k_empty[st];
        if (j >= G8_NST && !mbar_wait(empty, ((j / G8_NST) - 1) & 1))
          report(p.status, BSA_DEVERR_TIMEOUT);
        mbar_expect_tx(full, G8_TILE);
        tma_load_rhb((isv ? sV : sK) + st * G8_TILE, isv ? &tv : &tk, full, isv ? perm_v : perm_k,
                     0, (s_item[j] >> 3) * p.bs, hk, b);
      };
      if (nsteps > 0) load(false, 0);
      for (int j = 0; j < nsteps; ++j) {
        if (j + 1 < nsteps) load(false, j + 1);
        load(true, j);
      }
    }
  } else if (warp == G8_WMMA) {
    // ================= MMA issuer
    if (lane == 0) {
      if (!mbar_wait(&bar_q, 0)) report(p.status, BSA_DEVERR_TIMEOUT);
      const uint64_t dq = tc05::sdesc(smem_u32(sQ), 16, 1024);
      auto issue_s = [&](int js) {
        const int st = js % G8_NST;
        if (!mbar_wait(&k_full[st], (js / G8_NST) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        if (js >= 1 && !mbar_wait(&s_empty, (js - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
        const uint64_t dk = tc05::sdesc(smem_u32(sK + st * G8_TILE), 16, 1024);
#pragma unroll
        for (int ks = 0; ks < G8_D / 16; ++ks)
          tc05::mma_f16(tc05::taddr(tmem, 0, G8_SCOL), dq + 2 * ks, dk + 2 * ks, IDESC_S, ks > 0);
        tc05::commit(&s_full);
        tc05::commit(&k_empty[st]);
      };
      if (nsteps > 0) issue_s(0);
      for (int jp = 0; jp < nsteps; ++jp) {
        if (jp + 1 < nsteps) issue_s(jp + 1);
        const int st = jp % G8_NST;
        if (!mbar_wait(&p_full, jp & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        if (!mbar_wait(&v_full[st], (jp / G8_NST) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
        const uint64_t dv = tc05::sdesc(smem_u32(sV + st * G8_TILE), G8_TILE, 1024);
        const uint64_t dp = tc05::sdesc(smem_u32(sP), 16, 1024);
#pragma unroll
        for (int ks = 0; ks < G8_BS / 16; ++ks)  // keys 16*ks: region ks/4, +32 B per 16 keys
          tc05::mma_f16(tc05::taddr(tmem, 0, G8_OCOL), dp + (ks >> 2) * (G8_TILE >> 4) + 2 * (ks & 3),
                        dv + 128 * ks, IDESC_PV, (jp > 0 || ks > 0) ? 1u : 0u);
        tc05::commit(&v_empty[st]);
        tc05::commit(&o_done);
      }
    }
  } else {
    // ================= softmax warps 0-7
    const int quad = warp & 3, hf = warp >> 2;
    const int r = quad * 32 + lane;  // query row within the block
    const int cb = 64 * hf;          // first key column of this warp
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t pbase = smem_u32(sP + hf * G8_TILE);
    const float *gaterow =
        p.gate ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn : nullptr;
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
      const float g2 = gaterow ? __ldg(gaterow + s_islot[j]) * kLog2e : 0.f;
      if (kind & (KIND_TRIU | KIND_PAD)) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (((kind & KIND_TRIU) && cb + c > r) || ((kind & KIND_PAD) && kb * p.bs + cb + c >= p.L))
            s[c] = -INFINITY;
      }
      // PV_{j-1} must be complete before P is overwritten (and before O is rescaled)
      if (j >= 1) {
        if (!mbar_wait(&o_done, (j - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
        tc05::fence_after();
      }
      // exponentials with the maximum in use, written to P 8 columns at a time,
      // the block maximum formed alongside
      float sum8[8], m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum8[i] = 0.f, m8[i] = -INFINITY;
      auto write_p = [&](float off, bool track) {
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          uint32_t w4[4];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const int c = c8 * 8 + e;
            const float p0 = ex2(fmaf(s[c], p.scale2, off)), p1 = ex2(fmaf(s[c + 1], p.scale2, off));
            if (track) {
              m8[e] = fmaxf(m8[e], s[c]);
              m8[e + 1] = fmaxf(m8[e + 1], s[c + 1]);
            }
            sum8[e] += p0;
            sum8[e + 1] += p1;
            w4[e >> 1] = Mma<T>::pack(p0, p1);
          }
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(swz(pbase, 128, r, c8 * 8)),
                       "r"(w4[0]), "r"(w4[1]), "r"(w4[2]), "r"(w4[3])
                       : "memory");
        }
      };
      write_p(g2 - (m_used == -INFINITY ? 0.f : m_used), true);
      const float mh = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      s_xch[j & 1][quad][hf][lane] = mh;
      named_bar_sync(1 + quad, 64);
      const float mr = fmaxf(mh, s_xch[j & 1][quad][hf ^ 1][lane]);
      const float mx = mr == -INFINITY ? -INFINITY : fmaf(mr, p.scale2, g2);
      bool need = false;
      float alpha = 1.f;
      if (mx > -INFINITY && (m_used == -INFINITY || mx > m_used + G8_RESCALE)) {
        // rare: the block raised the maximum past the slack; redo P with it
        alpha = m_used == -INFINITY ? 0.f : ex2(m_used - mx);
        m_used = mx;
        l *= alpha;
        need = true;
#pragma unroll
        for (int i = 0; i < 8; ++i) sum8[i] = 0.f;
        write_p(g2 - m_used, false);
      }
      l += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      if (__any_sync(0xffffffffu, need) && j >= 1) {
        // O columns [32*hf, +32) of this warp's rows
        float o[32];
        const uint32_t ta = tmem + lane_base + G8_OCOL + 32 * hf;
        tc05::ld32(ta, o);
        tc05::wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] *= alpha;
        tc05::st32(ta, o);
        tc05::wait_st();
      }
      fence_proxy_async_smem();
      tc05::fence_before();
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(&p_full);
    }
    // ---- epilogue: O / l, l summed over the two halves of the row
    s_xch[0][quad][hf][lane] = l;
    named_bar_sync(1 + quad, 64);
    const float lt = l + s_xch[0][quad][hf ^ 1][lane];
    if (nsteps > 0) {
      if (!mbar_wait(&o_done, (nsteps - 1) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
      tc05::fence_after();
    }
    float o[32];
    tc05::ld32(tmem + lane_base + G8_OCOL + 32 * hf, o);
    tc05::wait_ld();
    if (nsteps == 0) {
#pragma unroll
      for (int c = 0; c < 32; ++c) o[c] = 0.f;
    }
    const long long grow = (long long)qi * p.bs + r;
    const long long bh = (long long)b * p.Hq + h;
    if (p.lse && hf == 0) p.lse[bh * p.Lp + grow] = lt > 0.f ? m_used + __log2f(lt) : INFINITY;
    if (grow < p.Lq) {
      const float inv = (nsteps > 0 && lt > 0.f) ? 1.f / lt : 0.f;
      T *orow = reinterpret_cast<T *>(p.o) + b * p.o_sb + h * p.o_sh + grow * p.o_sl + 32 * hf;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint4 wv;
        wv.x = Mma<T>::pack(o[c8 * 8 + 0] * inv, o[c8 * 8 + 1] * inv);
        wv.y = Mma<T>::pack(o[c8 * 8 + 2] * inv, o[c8 * 8 + 3] * inv);
        wv.z = Mma<T>::pack(o[c8 * 8 + 4] * inv, o[c8 * 8 + 5] * inv);
        wv.w = Mma<T>::pack(o[c8 * 8 + 6] * inv, o[c8 * 8 + 7] * inv);
        *reinterpret_cast<uint4 *>(orow + c8 * 8) = wv;
      }
    }
  }
  tc05::fence_before();
  __syncthreads();
  if (warp == G8_WMMA) {
    tc05::fence_after();
    tc05::dealloc(tmem, G8_TMEM_COLS);
  }
}

bool fwd_b128_applicable(const bsa_attn_args *a) {
  return a->dtype != BSA_F32 && a->bs == 128 && a->D == 64 && a->sel && a->kk <= G8_MAXN &&
         !a->out_gate.ptr && !getenv("BSA_FWD_LEGACY");
}

bsa_status launch_fwd_b128(const bsa_attn_args *a, const AttnParams &p, cudaStream_t st) {
  TensorMap4 mq, mk, mv;
  bsa_status s;
  if ((s = make_tmap(&mq, a->q.ptr, a->dtype, a->B, a->Hq, p.Lq, 64, a->q.sb, a->q.sh, a->q.sl, 128, "q")))
    return s;
  if ((s = make_tmap(&mk, a->k.ptr, a->dtype, a->B, a->Hkv, a->L, 64, a->k.sb, a->k.sh, a->k.sl, 128, "k")))
    return s;
  if ((s = make_tmap(&mv, a->v.ptr, a->dtype, a->B, a->Hkv, a->L, 64, a->v.sb, a->v.sh, a->v.sl, 128, "v")))
    return s;
  auto pk = [](const TensorMap4 &m) { return m.perm[0] | (m.perm[1] << 2) | (m.perm[2] << 4); };
  const long long grid = (long long)a->B * a->Hq * p.nq;
  auto kern = a->dtype == BSA_BF16 ? attn_fwd_b128_kernel<__nv_bfloat16> : attn_fwd_b128_kernel<__half>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G8_SMEM);
  kern<<<(unsigned)grid, G8_THREADS, G8_SMEM, st>>>(mq.map, mk.map, mv.map, pk(mq), pk(mk), pk(mv), p);
  return check_launch("attn_fwd_b128");
}

}  // namespace bsa
