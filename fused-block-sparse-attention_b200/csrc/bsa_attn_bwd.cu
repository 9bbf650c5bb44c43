// Block-sparse attention backward for sm_100a.
//
//  1. CSR transpose of the selection (bsa_sel_csr): an entry e = qi*kk + slot
//     is "active" under the same mask rules as the forward; its key block is
//     its bin.  Counts -> exclusive scan -> stable radix sort of (bin, e), so
//     every bin lists its entries in ascending e (deterministic).
//  2. dQ kernel, one CTA per (b, h, qblk): recomputes P from the forward's
//     row log-sum-exp, dP = dO V^T, dS = P (dP - Dvec), dQ = scale * dS K;
//     also writes Dvec = rowsum(dO * O) for step 3 and the per-slot gate
//     gradient sum(dS).
//  3. dK/dV kernel, one CTA per (bin, chunk of C entries, KV head): the key
//     block's K and V stay in registers; Q and dO chunks of each listed query
//     block are streamed by TMA; dV += P^T dO, dK += scale * dS^T Q.  Bins with
//     more than C entries write fp32 partial tiles that a second kernel sums
//     in chunk order, so no float atomics are used anywhere.
//
// The reference computes the same gradients with a 3-pass recompute per query
// block and float atomics for dK/dV (src/triton_kernel.py:77-181).
#include <cub/cub.cuh>

#include "bsa_attn.cuh"
#include "bsa_host.h"

namespace bsa {

// ------------------------------------------------------------------ CSR build
static inline int csr_nq(const bsa_csr_args *a) { return a->nq > 0 ? a->nq : a->nblk; }

__global__ void csr_count_kernel(bsa_csr_args a, int nq, int32_t *cnt, uint32_t *keys,
                                 int32_t *vals, int nbins) {
  // one thread per (b, hs, local query block, slot); bins are global key blocks
  const long long n = (long long)a.B * a.Hs * nq * a.kk;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < n;
       t += (long long)gridDim.x * blockDim.x) {
    const int slot = (int)(t % a.kk);
    long long r = t / a.kk;
    const int qi = (int)(r % nq), qblk = a.q_blk0 + qi;
    r /= nq;
    const int hs = (int)(r % a.Hs);
    const int b = (int)(r / a.Hs);
    const int32_t *selrow = a.sel + b * a.sel_sb + hs * a.sel_sh + (long long)qi * a.sel_sn;
    const int kb = selrow[slot];
    bool dup = false;
    if (a.mask_mode == BSA_MASK_TOKEN)
      for (int i = 0; i < slot && !dup; ++i) dup = selrow[i] == kb;
    const int kind =
        slot_kind(kb, slot, dup, qblk, a.nblk, a.bs, a.L, a.mask_mode, a.causal, a.status);
    if (kind != KIND_SKIP) {
      const int bin = (b * a.Hs + hs) * a.nblk + kb;
      atomicAdd(cnt + bin, 1);
      keys[t] = (uint32_t)bin;
    } else {
      keys[t] = (uint32_t)nbins;  // sorts after every real bin
    }
    vals[t] = qi * a.kk + slot;
  }
}

struct CsrWs {
  int32_t *cnt;
  uint32_t *keys_in, *keys_out;
  int32_t *vals_in;
  void *cub_tmp;
  size_t cub_bytes;
  size_t total;
};

static int bits_for(long long v) {
  int b = 1;
  while ((1LL << b) <= v) ++b;
  return b;
}

static size_t csr_layout(const bsa_csr_args *a, CsrWs *w, uint8_t *base) {
  const long long nbins = (long long)a->B * a->Hs * a->nblk;
  const long long n = (long long)a->B * a->Hs * csr_nq(a) * a->kk;
  size_t sort_bytes = 0, scan_bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, (uint32_t *)nullptr, (uint32_t *)nullptr,
                                  (int32_t *)nullptr, (int32_t *)nullptr, (int)n, 0,
                                  bits_for(nbins));
  cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, (int32_t *)nullptr, (int32_t *)nullptr,
                                (int)(nbins + 1));
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t *p = base ? base + off : nullptr;
    off += align_up(bytes, 256);
    return p;
  };
  w->cnt = (int32_t *)take((nbins + 1) * 4);
  w->keys_in = (uint32_t *)take(n * 4);
  w->keys_out = (uint32_t *)take(n * 4);
  w->vals_in = (int32_t *)take(n * 4);
  w->cub_bytes = std::max(sort_bytes, scan_bytes);
  w->cub_tmp = take(w->cub_bytes);
  w->total = off;
  return off;
}

bsa_status run_sel_csr(const bsa_csr_args *a, void *ws, size_t ws_bytes, cudaStream_t st) {
  CsrWs w;
  const size_t need = csr_layout(a, &w, nullptr);
  if (!ws || ws_bytes < need) return fail(BSA_ERR_WORKSPACE, "sel_csr: workspace too small");
  csr_layout(a, &w, reinterpret_cast<uint8_t *>(ws));
  const long long nbins = (long long)a->B * a->Hs * a->nblk;
  const long long n = (long long)a->B * a->Hs * csr_nq(a) * a->kk;
  // the counts must start at zero (the allocation-free entry point reuses its
  // scratch across calls, so this clear is what keeps a call from seeing the last one's)
  if (cudaMemsetAsync(w.cnt, 0, (nbins + 1) * 4, st) != cudaSuccess)
    return fail(BSA_ERR_LAUNCH, "sel_csr: clearing the bin counts failed");
  const int threads = 256;
  const long long blocks = std::min<long long>((n + threads - 1) / threads, 148LL * 64);
  csr_count_kernel<<<(unsigned)std::max<long long>(blocks, 1), threads, 0, st>>>(
      *a, csr_nq(a), w.cnt, w.keys_in, w.vals_in, (int)nbins);
  if (bsa_status s = check_launch("csr_count")) return s;
  size_t tb = w.cub_bytes;
  if (cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.keys_in, w.keys_out, w.vals_in, a->col,
                                      (int)n, 0, bits_for(nbins), st) != cudaSuccess)
    return fail(BSA_ERR_LAUNCH, "sel_csr: radix sort failed");
  tb = w.cub_bytes;
  if (cub::DeviceScan::ExclusiveSum(w.cub_tmp, tb, w.cnt, a->row_ptr, (int)(nbins + 1), st) !=
      cudaSuccess)
    return fail(BSA_ERR_LAUNCH, "sel_csr: scan failed");
  return check_launch("sel_csr");
}

size_t sel_csr_workspace(const bsa_csr_args *a) {
  CsrWs w;
  return csr_layout(a, &w, nullptr);
}

// ------------------------------------------------------------------ chunk plan
__global__ void plan_kernel(const int32_t *row_ptr, unsigned long long *plan_in, int nbins, int C) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i <= nbins; i += gridDim.x * blockDim.x) {
    unsigned long long v = 0;
    if (i < nbins) {
      const int c = row_ptr[i + 1] - row_ptr[i];
      const unsigned nch = c <= C ? 1u : (unsigned)((c + C - 1) / C);
      v = ((unsigned long long)nch << 32) | (nch > 1 ? nch : 0u);
    }
    plan_in[i] = v;
  }
}

// chunk x -> its bin, for every chunk of the plan (consumers look bins up in O(1))
__global__ void chunk_bin_kernel(const unsigned long long *plan, int nbins, int32_t *chunk_bin) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nbins; i += gridDim.x * blockDim.x) {
    const unsigned c0 = (unsigned)(plan[i] >> 32), c1 = (unsigned)(plan[i + 1] >> 32);
    for (unsigned x = c0; x < c1; ++x) chunk_bin[x] = i;
  }
}

// Sort keys of the chunks for the tcgen05 dK/dV kernel: (head group, then
// C - entries), slots past the chunk count last.  Within one (batch, selection
// head) group the chunks run largest first, so the two chunks of a work unit
// have equal size and both tiles stay busy on every step; the groups run one
// after another, so the query rows that the concurrently running units gather
// (Q, dO, lse, Dvec of one head: 64 MB at 262k tokens) stay in L2 instead of
// spanning every head at once.
__global__ void chunk_key_kernel(const unsigned long long *plan, const int32_t *row_ptr,
                                 const int32_t *chunk_bin, int nbins, int nblk, int C, int ncap,
                                 int32_t *key, int32_t *val) {
  const unsigned total = (unsigned)(plan[nbins] >> 32);
  const int ngroups = nbins / nblk;
  for (int x = blockIdx.x * blockDim.x + threadIdx.x; x < ncap; x += gridDim.x * blockDim.x) {
    int k = ngroups * (C + 2);
    if ((unsigned)x < total) {
      const int bin = chunk_bin[x];
      const int cidx = x - (int)(plan[bin] >> 32);
      const int e0 = row_ptr[bin] + cidx * C;
      k = (bin / nblk) * (C + 2) + C - (min(row_ptr[bin + 1], e0 + C) - e0);
    }
    key[x] = k;
    val[x] = x;
  }
}

// ------------------------------------------------------------------ dQ (tensor cores)
template <int BS, int D>
struct DqCfg : TileCfg<BS, D> {
  using B_ = TileCfg<BS, D>;
  static constexpr int NST = 2;
  static constexpr int SMEM = 1024 + 2 * B_::TILE + NST * 2 * B_::CH;
};

template <typename T, int BS, int D>
__global__ void __launch_bounds__(TileCfg<BS, D>::NT)
    attn_dq_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                   const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                   const int perm_q, const int perm_do, const int perm_k, const int perm_v,
                   const AttnParams p) {
  using Cfg = DqCfg<BS, D>;
  constexpr int NST = Cfg::NST, KC = Cfg::KC, NCH = Cfg::NCH, NT = Cfg::NT, NW = Cfg::NW;
  constexpr int NT8 = KC / 8, DK = D / 16, DN = D / 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sQ = smem;
  uint8_t *sdO = smem + Cfg::TILE;
  uint8_t *sKV = sdO + Cfg::TILE;
  __shared__ __align__(8) uint64_t bar[NST + 1];
  __shared__ int s_slot[kMaxKK];
  __shared__ float s_dg[kMaxKK];
  __shared__ float s_dgw[NST][NW];
  __shared__ int s_item[NST];
  __shared__ int s_kblk[NST];
  __shared__ float s_lse[BS], s_D[BS];

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
  const long long bh = (long long)b * p.Hq + h;

  const int32_t *selrow =
      p.sel ? p.sel + b * p.sel_sb + hk * p.sel_sh + (long long)qi * p.sel_sn : nullptr;
  const float *gaterow =
      p.gate ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn : nullptr;
  if (selrow)
    build_slot_table(s_slot, selrow, p.kk, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal,
                     p.status);
  for (int j = tid; j < kMaxKK; j += NT) s_dg[j] = 0.f;
  if (tid == 0) {
    for (int s = 0; s <= NST; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  // Dvec = rowsum(dO * O) for this block's rows: two threads per row.
  {
    const int row = tid >> 1, half = tid & 1;
    const long long grow = (long long)qi * p.bs + row;
    float acc = 0.f;
    if (grow < p.Lq) {
      const T *po = reinterpret_cast<const T *>(p.oin) + b * p.oi_sb + h * p.oi_sh + grow * p.oi_sl +
                    half * (D / 2);
      const T *pd = reinterpret_cast<const T *>(p.dout) + b * p.do_sb + h * p.do_sh +
                    grow * p.do_sl + half * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 2; c += 8) {
        const uint4 ov = *reinterpret_cast<const uint4 *>(po + c);
        const uint4 dv = *reinterpret_cast<const uint4 *>(pd + c);
        const T *oe = reinterpret_cast<const T *>(&ov);
        const T *de = reinterpret_cast<const T *>(&dv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(Mma<T>::to_f(oe[e]), Mma<T>::to_f(de[e]), acc);
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if (half == 0) {
      s_D[row] = acc;
      p.dvec[bh * p.Lp + grow] = acc;
      s_lse[row] = p.lse[bh * p.Lp + grow];
    }
  }
  __syncthreads();

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
    mbar_expect_tx(&bar[NST], 2 * Cfg::TILE);
#pragma unroll
    for (int r = 0; r < D / 64; ++r) {
      tma_load_rhb(sQ + r * BS * 128, &tq, &bar[NST], perm_q, r * 64, qi * p.bs, h, b);
      tma_load_rhb(sdO + r * BS * 128, &tdo, &bar[NST], perm_do, r * 64, qi * p.bs, h, b);
    }
    for (int s = 0; s < NST; ++s) {
      int kb = 0;
      const int item = next_item(kb);
      s_item[s] = item;
      s_kblk[s] = kb;
      if (item >= 0) issue(s, item, kb);
    }
  }
  __syncthreads();

  const uint32_t q_base = smem_u32(sQ), do_base = smem_u32(sdO);
  if (!mbar_wait(&bar[NST], 0)) report(p.status, BSA_DEVERR_TIMEOUT);
  uint32_t qf[DK][4], df[DK][4];
#pragma unroll
  for (int ks = 0; ks < DK; ++ks) {
    ldsm_x4(swz(q_base, BS, warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), qf[ks][0],
            qf[ks][1], qf[ks][2], qf[ks][3]);
    ldsm_x4(swz(do_base, BS, warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), df[ks][0],
            df[ks][1], df[ks][2], df[ks][3]);
  }
  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8;
  const float lse0 = s_lse[r0], lse1 = s_lse[r1];
  const float D0 = s_D[r0], D1 = s_D[r1];
  float dq[DN][4];
#pragma unroll
  for (int n = 0; n < DN; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.f;

  for (int it = 0;; ++it) {
    const int st = it % NST;
    const int item = s_item[st];
    if (item < 0) break;
    const int kb = s_kblk[st];
    if (!mbar_wait(&bar[st], (it / NST) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
    const int slot = item >> 8, chunk = (item >> 3) & 31, kind = item & 7;
    const bool dead = (kind & KIND_TRIU) && chunk * KC > warp * 16 + 15;
    float dgs = 0.f;
    if (!dead) {
      const uint32_t k_base = smem_u32(sKV + st * 2 * Cfg::CH);
      const uint32_t v_base = k_base + Cfg::CH;
      float s[NT8][4], dp[NT8][4];
#pragma unroll
      for (int n = 0; n < NT8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < DK; ++ks) {
#pragma unroll
        for (int np = 0; np < KC / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          const int row = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int col = ks * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(swz(k_base, KC, row, col), b0, b1, b2, b3);
          Mma<T>::run(s[2 * np], qf[ks], b0, b1);
          Mma<T>::run(s[2 * np + 1], qf[ks], b2, b3);
          ldsm_x4(swz(v_base, KC, row, col), b0, b1, b2, b3);
          Mma<T>::run(dp[2 * np], df[ks], b0, b1);
          Mma<T>::run(dp[2 * np + 1], df[ks], b2, b3);
        }
      }
      const float g2 = gaterow ? __ldg(gaterow + slot) * kLog2e : 0.f;
      const int key0 = chunk * KC + (lane & 3) * 2;
#pragma unroll
      for (int n = 0; n < NT8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + n * 8 + (e & 1);
          const int row = e < 2 ? r0 : r1;
          bool masked = ((kind & KIND_TRIU) && key > row) ||
                        ((kind & KIND_PAD) && kb * p.bs + key >= p.L);
          const float pr = masked ? 0.f : ex2(fmaf(s[n][e], p.scale2, g2) - (e < 2 ? lse0 : lse1));
          const float ds = pr * (dp[n][e] - (e < 2 ? D0 : D1));
          s[n][e] = ds;
          dgs += ds;
        }
      }
      // dQ += dS K
#pragma unroll
      for (int ks = 0; ks < KC / 16; ++ks) {
        uint32_t a[4];
        a[0] = Mma<T>::pack(s[2 * ks][0], s[2 * ks][1]);
        a[1] = Mma<T>::pack(s[2 * ks][2], s[2 * ks][3]);
        a[2] = Mma<T>::pack(s[2 * ks + 1][0], s[2 * ks + 1][1]);
        a[3] = Mma<T>::pack(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
        for (int dp2 = 0; dp2 < D / 16; ++dp2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(swz(k_base, KC, ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                        dp2 * 16 + ((lane >> 4) << 3)),
                    b0, b1, b2, b3);
          Mma<T>::run(dq[2 * dp2], a, b0, b1);
          Mma<T>::run(dq[2 * dp2 + 1], a, b2, b3);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) dgs += __shfl_xor_sync(0xffffffffu, dgs, o);
    if (lane == 0) s_dgw[st][warp] = dgs;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) t += s_dgw[st][w];
      if (slot < kMaxKK) s_dg[slot] += t;
      int kb2 = 0;
      const int nxt = next_item(kb2);
      s_item[st] = nxt;
      s_kblk[st] = kb2;
      if (nxt >= 0) issue(st, nxt, kb2);
    }
  }
  __syncthreads();
  if (p.dgate) {
    float *dg = p.dgate + (bh * p.nq + qi) * (long long)p.kk;
    for (int j = tid; j < p.kk; j += NT) dg[j] = j < kMaxKK ? s_dg[j] : 0.f;
  }
  // stage dQ * scale (rounded to T) in the Q region, then 16-byte stores
#pragma unroll
  for (int n = 0; n < DN; ++n) {
    const int col = n * 8 + (lane & 3) * 2;
    const uint32_t w0 = Mma<T>::pack(dq[n][0] * p.scale, dq[n][1] * p.scale);
    const uint32_t w1 = Mma<T>::pack(dq[n][2] * p.scale, dq[n][3] * p.scale);
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(swz(q_base, BS, r0, col)), "r"(w0));
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(swz(q_base, BS, r1, col)), "r"(w1));
  }
  __syncthreads();
  T *dqb = reinterpret_cast<T *>(p.dq) + b * p.dq_sb + h * p.dq_sh;
  for (int idx = tid; idx < BS * (D / 8); idx += NT) {
    const int row = idx / (D / 8), c8 = idx % (D / 8);
    const long long grow = (long long)qi * p.bs + row;
    if (grow >= p.Lq) continue;
    uint4 val;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                 : "r"(swz(q_base, BS, row, c8 * 8)));
    *reinterpret_cast<uint4 *>(dqb + grow * p.dq_sl + c8 * 8) = val;
  }
}

// ------------------------------------------------------------------ dK/dV (tensor cores)
template <int BS, int D>
struct DkvCfg : TileCfg<BS, D> {
  using B_ = TileCfg<BS, D>;
  static constexpr int NST = 2;
  static constexpr bool KREG = D <= 64;  // K/V fragments kept in registers
  static constexpr int ROWB = B_::KC * 4;  // bytes of one lse / Dvec chunk
  // stage stride rounded to 1024 B: swizzled TMA destinations need 1024-B alignment
  static constexpr int STAGE = (2 * B_::CH + 2 * ROWB + 1023) / 1024 * 1024;
  static constexpr int SMEM = 1024 + 2 * B_::TILE + NST * STAGE;
};

template <typename T, int BS, int D>
__global__ void __launch_bounds__(TileCfg<BS, D>::NT)
    attn_dkdv_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                     const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                     const int perm_q, const int perm_do, const int perm_k, const int perm_v,
                     const AttnParams p, const BwdPlan pl) {
  using Cfg = DkvCfg<BS, D>;
  constexpr int NST = Cfg::NST, KC = Cfg::KC, NCH = Cfg::NCH, NT = Cfg::NT;
  constexpr int NT8 = KC / 8, DK = D / 16, DN = D / 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sK = smem;
  uint8_t *sV = smem + Cfg::TILE;
  uint8_t *sST = sV + Cfg::TILE;  // stages: Q chunk, dO chunk, lse chunk, Dvec chunk
  __shared__ __align__(8) uint64_t bar[NST + 1];
  __shared__ int s_item[NST];  // entry index into col (relative), -1 end

  const unsigned x = blockIdx.x;
  const unsigned total = (unsigned)(pl.plan[pl.nbins] >> 32);
  if (x >= total) return;
  const int bin = pl.chunk_bin[x];
  const unsigned chunk_off = (unsigned)(pl.plan[bin] >> 32);
  const unsigned part_off = (unsigned)(pl.plan[bin] & 0xffffffffu);
  const unsigned nch = (unsigned)(pl.plan[bin + 1] >> 32) - chunk_off;
  const int cidx = (int)(x - chunk_off);
  const int e_beg = pl.row_ptr[bin] + cidx * pl.C;
  const int e_end = min(pl.row_ptr[bin + 1], e_beg + pl.C);
  const int kb = bin % p.nblk;
  const int hs = (bin / p.nblk) % pl.Hs;
  const int b = bin / (p.nblk * pl.Hs);
  const int hk = hs * pl.Y + blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float *gbase = p.gate ? p.gate + b * p.gate_sb + hk * p.gate_sh : nullptr;

  if (tid == 0) {
    for (int s = 0; s <= NST; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // items: (entry, query head g, chunk c) in that nesting order
  const int nitems = (e_end - e_beg) * p.grp * NCH;
  auto issue = [&](int st, int it) {
    const int c = it % NCH;
    const int g = (it / NCH) % p.grp;
    const int e = pl.col[e_beg + it / (NCH * p.grp)];
    const int qi = e / p.kk;  // local query block
    const int h = hk * p.grp + g;
    uint8_t *base = sST + st * Cfg::STAGE;
    mbar_expect_tx(&bar[st], 2 * Cfg::CH + 2 * Cfg::ROWB);
    const int row = qi * p.bs + c * KC;
#pragma unroll
    for (int r = 0; r < D / 64; ++r) {
      tma_load_rhb(base + r * KC * 128, &tq, &bar[st], perm_q, r * 64, row, h, b);
      tma_load_rhb(base + Cfg::CH + r * KC * 128, &tdo, &bar[st], perm_do, r * 64, row, h, b);
    }
    const long long rb = ((long long)b * p.Hq + h) * p.Lp + row;
    bulk_load(base + 2 * Cfg::CH, p.lse + rb, Cfg::ROWB, &bar[st]);
    bulk_load(base + 2 * Cfg::CH + Cfg::ROWB, p.dvec + rb, Cfg::ROWB, &bar[st]);
  };
  if (tid == 0) {
    mbar_expect_tx(&bar[NST], 2 * Cfg::TILE);
#pragma unroll
    for (int r = 0; r < D / 64; ++r) {
      tma_load_rhb(sK + r * BS * 128, &tk, &bar[NST], perm_k, r * 64, kb * p.bs, hk, b);
      tma_load_rhb(sV + r * BS * 128, &tv, &bar[NST], perm_v, r * 64, kb * p.bs, hk, b);
    }
    for (int s = 0; s < NST && s < nitems; ++s) issue(s, s);
  }
  const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
  if (!mbar_wait(&bar[NST], 0)) report(p.status, BSA_DEVERR_TIMEOUT);
  uint32_t kf[Cfg::KREG ? DK : 1][4], vf[Cfg::KREG ? DK : 1][4];
  if constexpr (Cfg::KREG) {
#pragma unroll
    for (int ks = 0; ks < DK; ++ks) {
      ldsm_x4(swz(k_base, BS, warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), kf[ks][0],
              kf[ks][1], kf[ks][2], kf[ks][3]);
      ldsm_x4(swz(v_base, BS, warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), vf[ks][0],
              vf[ks][1], vf[ks][2], vf[ks][3]);
    }
  }
  float dk[DN][4], dv[DN][4];
#pragma unroll
  for (int n = 0; n < DN; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[n][e] = dv[n][e] = 0.f;
  const int kr0 = warp * 16 + (lane >> 2), kr1 = kr0 + 8;  // key rows of this lane

  for (int it = 0; it < nitems; ++it) {
    const int st = it % NST;
    if (!mbar_wait(&bar[st], (it / NST) & 1)) report(p.status, BSA_DEVERR_TIMEOUT);
    const int c = it % NCH;
    const int e = pl.col[e_beg + it / (NCH * p.grp)];
    const int qi = e / p.kk, slot = e % p.kk, qblk = p.q0 + qi;
    // the slot kind as recorded by the CSR build: TRIU only for causal slot 0
    // (SLOT mode) or the own block (TOKEN mode)
    const bool triu = p.causal && ((p.mask_mode == BSA_MASK_SLOT) ? slot == 0 : kb == qblk);
    const bool dead = triu && warp * 16 > c * KC + KC - 1;
    if (!dead) {
      const uint8_t *base = sST + st * Cfg::STAGE;
      const uint32_t qc = smem_u32(base), dc = qc + Cfg::CH;
      const float *slse = reinterpret_cast<const float *>(base + 2 * Cfg::CH);
      const float *sdv = slse + KC;
      const float g2 = gbase ? __ldg(gbase + (long long)qi * p.gate_sn + slot) * kLog2e : 0.f;
      float s[NT8][4], dp[NT8][4];
#pragma unroll
      for (int n = 0; n < NT8; ++n)
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) s[n][e2] = dp[n][e2] = 0.f;
#pragma unroll
      for (int ks = 0; ks < DK; ++ks) {
        uint32_t ka[4], va[4];
        if constexpr (Cfg::KREG) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            ka[i] = kf[ks][i];
            va[i] = vf[ks][i];
          }
        } else {
          ldsm_x4(swz(k_base, BS, warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), ka[0], ka[1],
                  ka[2], ka[3]);
          ldsm_x4(swz(v_base, BS, warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), va[0], va[1],
                  va[2], va[3]);
        }
#pragma unroll
        for (int np = 0; np < KC / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          const int row = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int col = ks * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(swz(qc, KC, row, col), b0, b1, b2, b3);
          Mma<T>::run(s[2 * np], ka, b0, b1);
          Mma<T>::run(s[2 * np + 1], ka, b2, b3);
          ldsm_x4(swz(dc, KC, row, col), b0, b1, b2, b3);
          Mma<T>::run(dp[2 * np], va, b0, b1);
          Mma<T>::run(dp[2 * np + 1], va, b2, b3);
        }
      }
      // P^T and dS^T; columns are query rows c*KC + n*8 + (lane&3)*2 + (e&1)
#pragma unroll
      for (int n = 0; n < NT8; ++n) {
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          const int qc_ = n * 8 + (lane & 3) * 2 + (e2 & 1);
          const int qrow = c * KC + qc_;
          const int krow = e2 < 2 ? kr0 : kr1;
          const bool masked = (triu && krow > qrow) ||
                              ((long long)qi * p.bs + qrow >= p.Lq) ||
                              ((long long)kb * p.bs + krow >= p.L);
          const float pr = masked ? 0.f : ex2(fmaf(s[n][e2], p.scale2, g2) - slse[qc_]);
          s[n][e2] = pr;
          dp[n][e2] = pr * (dp[n][e2] - sdv[qc_]);
        }
      }
      // dV += P^T dO ; dK += dS^T Q
#pragma unroll
      for (int ks = 0; ks < KC / 16; ++ks) {
        uint32_t pa[4], sa[4];
        pa[0] = Mma<T>::pack(s[2 * ks][0], s[2 * ks][1]);
        pa[1] = Mma<T>::pack(s[2 * ks][2], s[2 * ks][3]);
        pa[2] = Mma<T>::pack(s[2 * ks + 1][0], s[2 * ks + 1][1]);
        pa[3] = Mma<T>::pack(s[2 * ks + 1][2], s[2 * ks + 1][3]);
        sa[0] = Mma<T>::pack(dp[2 * ks][0], dp[2 * ks][1]);
        sa[1] = Mma<T>::pack(dp[2 * ks][2], dp[2 * ks][3]);
        sa[2] = Mma<T>::pack(dp[2 * ks + 1][0], dp[2 * ks + 1][1]);
        sa[3] = Mma<T>::pack(dp[2 * ks + 1][2], dp[2 * ks + 1][3]);
#pragma unroll
        for (int d2 = 0; d2 < D / 16; ++d2) {
          uint32_t b0, b1, b2, b3;
          const int row = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int col = d2 * 16 + ((lane >> 4) << 3);
          ldsm_x4_t(swz(dc, KC, row, col), b0, b1, b2, b3);
          Mma<T>::run(dv[2 * d2], pa, b0, b1);
          Mma<T>::run(dv[2 * d2 + 1], pa, b2, b3);
          ldsm_x4_t(swz(qc, KC, row, col), b0, b1, b2, b3);
          Mma<T>::run(dk[2 * d2], sa, b0, b1);
          Mma<T>::run(dk[2 * d2 + 1], sa, b2, b3);
        }
      }
    }
    __syncthreads();
    if (tid == 0 && it + NST < nitems) issue(st, it + NST);
  }

  // ---- write out
  if (nch == 1) {
    T *dkp = reinterpret_cast<T *>(p.dk) + b * p.dk_sb + hk * p.dk_sh;
    T *dvp = reinterpret_cast<T *>(p.dv) + b * p.dv_sb + hk * p.dv_sh;
#pragma unroll
    for (int n = 0; n < DN; ++n) {
      const int col = n * 8 + (lane & 3) * 2;
      const long long g0 = (long long)kb * p.bs + kr0, g1 = (long long)kb * p.bs + kr1;
      if (g0 < p.L) {
        *reinterpret_cast<uint32_t *>(dkp + g0 * p.dk_sl + col) =
            Mma<T>::pack(dk[n][0] * p.scale, dk[n][1] * p.scale);
        *reinterpret_cast<uint32_t *>(dvp + g0 * p.dv_sl + col) = Mma<T>::pack(dv[n][0], dv[n][1]);
      }
      if (g1 < p.L) {
        *reinterpret_cast<uint32_t *>(dkp + g1 * p.dk_sl + col) =
            Mma<T>::pack(dk[n][2] * p.scale, dk[n][3] * p.scale);
        *reinterpret_cast<uint32_t *>(dvp + g1 * p.dv_sl + col) = Mma<T>::pack(dv[n][2], dv[n][3]);
      }
    }
  } else {
    float *part = pl.part + ((long long)(part_off + cidx) * pl.Y + blockIdx.y) * (2LL * BS * D);
#pragma unroll
    for (int n = 0; n < DN; ++n) {
      const int col = n * 8 + (lane & 3) * 2;
      *reinterpret_cast<float2 *>(part + kr0 * D + col) = make_float2(dk[n][0], dk[n][1]);
      *reinterpret_cast<float2 *>(part + kr1 * D + col) = make_float2(dk[n][2], dk[n][3]);
      *reinterpret_cast<float2 *>(part + BS * D + kr0 * D + col) = make_float2(dv[n][0], dv[n][1]);
      *reinterpret_cast<float2 *>(part + BS * D + kr1 * D + col) = make_float2(dv[n][2], dv[n][3]);
    }
  }
}

// Sums the partial dK/dV tiles of multi-chunk bins in chunk order.
template <typename T>
__global__ void dkdv_reduce_kernel(const AttnParams p, const BwdPlan pl, int BS, int D) {
  const int bin = blockIdx.x;
  const unsigned chunk_off = (unsigned)(pl.plan[bin] >> 32);
  const unsigned nch = (unsigned)(pl.plan[bin + 1] >> 32) - chunk_off;
  if (nch <= 1) return;
  const unsigned part_off = (unsigned)(pl.plan[bin] & 0xffffffffu);
  const int kb = bin % p.nblk;
  const int hs = (bin / p.nblk) % pl.Hs;
  const int b = bin / (p.nblk * pl.Hs);
  const int hk = hs * pl.Y + blockIdx.y;
  T *dkp = reinterpret_cast<T *>(p.dk) + b * p.dk_sb + hk * p.dk_sh;
  T *dvp = reinterpret_cast<T *>(p.dv) + b * p.dv_sb + hk * p.dv_sh;
  if constexpr (sizeof(T) == 2) if ((D & 3) == 0 && (p.dk_sl & 3) == 0 && (p.dv_sl & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(dkp) & 7) == 0 && (reinterpret_cast<uintptr_t>(dvp) & 7) == 0) {
    // four columns per thread: float4 partial loads, 8-byte stores (same
    // summation order per element as below)
    for (int i = 4 * threadIdx.x; i < BS * D; i += 4 * blockDim.x) {
      const int r = i / D, d = i % D;
      float4 sk = make_float4(0.f, 0.f, 0.f, 0.f), sv = sk;
      for (unsigned c = 0; c < nch; ++c) {
        const float *part =
            pl.part + ((long long)(part_off + c) * pl.Y + blockIdx.y) * (2LL * BS * D);
        const float4 a = *reinterpret_cast<const float4 *>(part + i);
        const float4 v = *reinterpret_cast<const float4 *>(part + BS * D + i);
        sk.x += a.x; sk.y += a.y; sk.z += a.z; sk.w += a.w;
        sv.x += v.x; sv.y += v.y; sv.z += v.z; sv.w += v.w;
      }
      const long long g = (long long)kb * p.bs + r;
      if (g >= p.L) continue;
      uint2 wk, wv;
      wk.x = Mma<T>::pack(sk.x * p.scale, sk.y * p.scale);
      wk.y = Mma<T>::pack(sk.z * p.scale, sk.w * p.scale);
      wv.x = Mma<T>::pack(sv.x, sv.y);
      wv.y = Mma<T>::pack(sv.z, sv.w);
      *reinterpret_cast<uint2 *>(dkp + g * p.dk_sl + d) = wk;
      *reinterpret_cast<uint2 *>(dvp + g * p.dv_sl + d) = wv;
    }
    return;
  }
  for (int i = threadIdx.x; i < BS * D; i += blockDim.x) {
    const int r = i / D, d = i % D;
    float sk = 0.f, sv = 0.f;
    for (unsigned c = 0; c < nch; ++c) {
      const float *part =
          pl.part + ((long long)(part_off + c) * pl.Y + blockIdx.y) * (2LL * BS * D);
      sk += part[i];
      sv += part[BS * D + i];
    }
    const long long g = (long long)kb * p.bs + r;
    if (g >= p.L) continue;
    if constexpr (sizeof(T) == 4) {
      dkp[g * p.dk_sl + d] = sk * p.scale;
      dvp[g * p.dv_sl + d] = sv;
    } else {
      dkp[g * p.dk_sl + d] = Mma<T>::from_f(sk * p.scale);
      dvp[g * p.dv_sl + d] = Mma<T>::from_f(sv);
    }
  }
}

// ------------------------------------------------------------------ fp32 SIMT backward
template <int BS, int D>
struct F32BwdCfg {
  static constexpr int LD = D + 1;
  static constexpr int KC = 32;
  // dQ: q, dO, k, v chunks, S/dS
  static constexpr int DQ_SMEM =
      (2 * BS * LD + 2 * KC * LD + BS * (KC + 1) + BS * LD + 2 * BS) * 4 + kMaxKK * 8;
  // dKdV: k, v, q, dO, P, dS, dk, dv accumulators, lse, D
  static constexpr int DKV_SMEM = (6 * BS * LD + 2 * BS * (BS + 1) + 2 * BS) * 4;
};

template <int BS, int D>
__global__ void __launch_bounds__(256) attn_dq_f32_kernel(const AttnParams p) {
  using Cfg = F32BwdCfg<BS, D>;
  constexpr int LD = Cfg::LD, KC = Cfg::KC;
  extern __shared__ float fsm[];
  float *sq = fsm;
  float *sdo = sq + BS * LD;
  float *sk = sdo + BS * LD;
  float *sv = sk + KC * LD;
  float *sS = sv + KC * LD;
  float *sdq = sS + BS * (KC + 1);
  float *slse = sdq + BS * LD;
  float *sD = slse + BS;
  int *s_slot = reinterpret_cast<int *>(sD + BS);
  float *s_dg = reinterpret_cast<float *>(s_slot + kMaxKK);

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
  const long long bh = (long long)b * p.Hq + h;
  const int32_t *selrow =
      p.sel ? p.sel + b * p.sel_sb + hk * p.sel_sh + (long long)qi * p.sel_sn : nullptr;
  const float *gaterow =
      p.gate ? p.gate + b * p.gate_sb + hk * p.gate_sh + (long long)qi * p.gate_sn : nullptr;
  if (selrow)
    build_slot_table(s_slot, selrow, p.kk, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal,
                     p.status);
  for (int j = tid; j < kMaxKK; j += 256) s_dg[j] = 0.f;
  const float *q = reinterpret_cast<const float *>(p.q) + b * p.q_sb + h * p.q_sh;
  const float *dO = reinterpret_cast<const float *>(p.dout) + b * p.do_sb + h * p.do_sh;
  const float *o = reinterpret_cast<const float *>(p.oin) + b * p.oi_sb + h * p.oi_sh;
  const float *k = reinterpret_cast<const float *>(p.k) + b * p.k_sb + hk * p.k_sh;
  const float *v = reinterpret_cast<const float *>(p.v) + b * p.v_sb + hk * p.v_sh;
  for (int i = tid; i < BS * D; i += 256) {
    const int r = i / D, d = i % D;
    const long long gr = (long long)qi * p.bs + r;
    const bool ok = gr < p.Lq;
    sq[r * LD + d] = ok ? q[gr * p.q_sl + d] : 0.f;
    sdo[r * LD + d] = ok ? dO[gr * p.do_sl + d] : 0.f;
    sdq[r * LD + d] = 0.f;
  }
  __syncthreads();
  for (int r = tid; r < BS; r += 256) {
    const long long gr = (long long)qi * p.bs + r;
    float acc = 0.f;
    if (gr < p.Lq)
      for (int d = 0; d < D; ++d) acc = fmaf(o[gr * p.oi_sl + d], sdo[r * LD + d], acc);
    sD[r] = acc;
    p.dvec[bh * p.Lp + gr] = acc;
    slse[r] = p.lse[bh * p.Lp + gr] / kLog2e;  // natural-log domain
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
        float s = 0.f, dp = 0.f;
        for (int d = 0; d < D; ++d) {
          s = fmaf(sq[r * LD + d], sk[c * LD + d], s);
          dp = fmaf(sdo[r * LD + d], sv[c * LD + d], dp);
        }
        const int key = c0 + c;
        const bool masked = key >= p.bs || ((kind & KIND_TRIU) && key > r) ||
                            ((kind & KIND_PAD) && (long long)kb * p.bs + key >= p.L);
        const float pr = masked ? 0.f : expf(s * p.scale + g - slse[r]);
        sS[r * (KC + 1) + c] = pr * (dp - sD[r]);
      }
      __syncthreads();
      for (int i = tid; i < BS * D; i += 256) {
        const int r = i / D, d = i % D;
        float a = sdq[r * LD + d];
        for (int c = 0; c < KC; ++c) a = fmaf(sS[r * (KC + 1) + c], sk[c * LD + d], a);
        sdq[r * LD + d] = a;
      }
      if (tid == 0 && slot < kMaxKK) {
        float t = 0.f;
        for (int i = 0; i < BS * KC; ++i) t += sS[(i / KC) * (KC + 1) + (i % KC)];
        s_dg[slot] += t;
      }
      __syncthreads();
    }
  }
  if (p.dgate) {
    float *dg = p.dgate + (bh * p.nq + qi) * (long long)p.kk;
    for (int j = tid; j < p.kk; j += 256) dg[j] = j < kMaxKK ? s_dg[j] : 0.f;
  }
  float *dq = reinterpret_cast<float *>(p.dq) + b * p.dq_sb + h * p.dq_sh;
  for (int i = tid; i < BS * D; i += 256) {
    const int r = i / D, d = i % D;
    const long long gr = (long long)qi * p.bs + r;
    if (gr < p.Lq) dq[gr * p.dq_sl + d] = sdq[r * LD + d] * p.scale;
  }
}

template <int BS, int D>
__global__ void __launch_bounds__(256) attn_dkdv_f32_kernel(const AttnParams p, const BwdPlan pl) {
  using Cfg = F32BwdCfg<BS, D>;
  constexpr int LD = Cfg::LD, LP = BS + 1;
  extern __shared__ float fsm[];
  float *sk = fsm;
  float *sv = sk + BS * LD;
  float *sq = sv + BS * LD;
  float *sdo = sq + BS * LD;
  float *sdk = sdo + BS * LD;
  float *sdv = sdk + BS * LD;
  float *sP = sdv + BS * LD;  // [query r][key c]
  float *sdS = sP + BS * LP;
  float *slse = sdS + BS * LP;
  float *sD = slse + BS;

  const unsigned x = blockIdx.x;
  const unsigned total = (unsigned)(pl.plan[pl.nbins] >> 32);
  if (x >= total) return;
  const int bin = pl.chunk_bin[x];
  const unsigned chunk_off = (unsigned)(pl.plan[bin] >> 32);
  const unsigned part_off = (unsigned)(pl.plan[bin] & 0xffffffffu);
  const unsigned nch = (unsigned)(pl.plan[bin + 1] >> 32) - chunk_off;
  const int cidx = (int)(x - chunk_off);
  const int e_beg = pl.row_ptr[bin] + cidx * pl.C;
  const int e_end = min(pl.row_ptr[bin + 1], e_beg + pl.C);
  const int kb = bin % p.nblk;
  const int hs = (bin / p.nblk) % pl.Hs;
  const int b = bin / (p.nblk * pl.Hs);
  const int hk = hs * pl.Y + blockIdx.y;
  const int tid = threadIdx.x;
  const float *k = reinterpret_cast<const float *>(p.k) + b * p.k_sb + hk * p.k_sh;
  const float *v = reinterpret_cast<const float *>(p.v) + b * p.v_sb + hk * p.v_sh;
  for (int i = tid; i < BS * D; i += 256) {
    const int r = i / D, d = i % D;
    const long long gr = (long long)kb * p.bs + r;
    const bool ok = gr < p.L;
    sk[r * LD + d] = ok ? k[gr * p.k_sl + d] : 0.f;
    sv[r * LD + d] = ok ? v[gr * p.v_sl + d] : 0.f;
    sdk[r * LD + d] = 0.f;
    sdv[r * LD + d] = 0.f;
  }
  for (int ei = e_beg; ei < e_end; ++ei) {
    const int e = pl.col[ei];
    const int qi = e / p.kk, slot = e % p.kk, qblk = p.q0 + qi;
    const bool triu = p.causal && ((p.mask_mode == BSA_MASK_SLOT) ? slot == 0 : kb == qblk);
    for (int g = 0; g < p.grp; ++g) {
      const int h = hk * p.grp + g;
      const long long bh = (long long)b * p.Hq + h;
      const float gv = p.gate ? p.gate[b * p.gate_sb + hk * p.gate_sh +
                                       (long long)qi * p.gate_sn + slot]
                              : 0.f;
      const float *q = reinterpret_cast<const float *>(p.q) + b * p.q_sb + h * p.q_sh;
      const float *dO = reinterpret_cast<const float *>(p.dout) + b * p.do_sb + h * p.do_sh;
      __syncthreads();
      for (int i = tid; i < BS * D; i += 256) {
        const int r = i / D, d = i % D;
        const long long gr = (long long)qi * p.bs + r;
        const bool ok = gr < p.Lq;
        sq[r * LD + d] = ok ? q[gr * p.q_sl + d] : 0.f;
        sdo[r * LD + d] = ok ? dO[gr * p.do_sl + d] : 0.f;
      }
      for (int r = tid; r < BS; r += 256) {
        slse[r] = p.lse[bh * p.Lp + (long long)qi * p.bs + r] / kLog2e;
        sD[r] = p.dvec[bh * p.Lp + (long long)qi * p.bs + r];
      }
      __syncthreads();
      for (int i = tid; i < BS * BS; i += 256) {
        const int r = i / BS, c = i % BS;  // query r, key c
        float s = 0.f, dp = 0.f;
        for (int d = 0; d < D; ++d) {
          s = fmaf(sq[r * LD + d], sk[c * LD + d], s);
          dp = fmaf(sdo[r * LD + d], sv[c * LD + d], dp);
        }
        const bool masked = (triu && c > r) || ((long long)qi * p.bs + r >= p.Lq) ||
                            ((long long)kb * p.bs + c >= p.L);
        const float pr = masked ? 0.f : expf(s * p.scale + gv - slse[r]);
        sP[r * LP + c] = pr;
        sdS[r * LP + c] = pr * (dp - sD[r]);
      }
      __syncthreads();
      for (int i = tid; i < BS * D; i += 256) {
        const int c = i / D, d = i % D;
        float ak = sdk[c * LD + d], av = sdv[c * LD + d];
        for (int r = 0; r < BS; ++r) {
          av = fmaf(sP[r * LP + c], sdo[r * LD + d], av);
          ak = fmaf(sdS[r * LP + c], sq[r * LD + d], ak);
        }
        sdk[c * LD + d] = ak;
        sdv[c * LD + d] = av;
      }
    }
  }
  __syncthreads();
  if (nch == 1) {
    float *dkp = reinterpret_cast<float *>(p.dk) + b * p.dk_sb + hk * p.dk_sh;
    float *dvp = reinterpret_cast<float *>(p.dv) + b * p.dv_sb + hk * p.dv_sh;
    for (int i = tid; i < BS * D; i += 256) {
      const int r = i / D, d = i % D;
      const long long g = (long long)kb * p.bs + r;
      if (g < p.L) {
        dkp[g * p.dk_sl + d] = sdk[r * LD + d] * p.scale;
        dvp[g * p.dv_sl + d] = sdv[r * LD + d];
      }
    }
  } else {
    float *part = pl.part + ((long long)(part_off + cidx) * pl.Y + blockIdx.y) * (2LL * BS * D);
    for (int i = tid; i < BS * D; i += 256) {
      const int r = i / D, d = i % D;
      part[i] = sdk[r * LD + d];
      part[BS * D + i] = sdv[r * LD + d];
    }
  }
}

// ------------------------------------------------------------------ host side
static constexpr int kChunkEntries = 32;

struct BwdWs {
  float *dvec;
  int32_t *row_ptr, *col;
  unsigned long long *plan_in, *plan;
  int32_t *chunk_bin;
  int32_t *ord_key_in, *ord_key_out, *ord_in, *ord;
  void *sort_tmp;
  size_t sort_bytes;
  void *csr_ws;
  size_t csr_bytes;
  void *scan_tmp;
  size_t scan_bytes;
  float *part;
  void *ds;  // dS tiles for the stored-dS dQ pass (null when it does not apply)
  size_t total;
};

// local query blocks of an attention call (its query range; all blocks unsharded)
static int attn_nq(const bsa_attn_args *a) {
  const int Lq = a->Lq > 0 ? a->Lq : a->L;
  return (Lq + a->bs - 1) / a->bs;
}

static void csr_args_from(const bsa_attn_args *a, bsa_csr_args *c) {
  *c = bsa_csr_args{};
  c->B = a->B;
  c->Hs = a->sel_sh == 0 ? 1 : a->Hkv;
  c->nblk = a->nblk;
  c->kk = a->kk;
  c->bs = a->bs;
  c->L = a->L;
  c->mask_mode = a->mask_mode;
  c->causal = a->causal;
  c->sel = a->sel;
  c->sel_sb = a->sel_sb;
  c->sel_sh = a->sel_sh;
  c->sel_sn = a->sel_sn;
  c->status = a->status;
  c->q_blk0 = a->q_blk0;
  c->nq = attn_nq(a);
}

size_t dq_ds_bytes(const bsa_attn_args *a, int nq);
bsa_status launch_dq_ds(int dtype, const CUtensorMap &mk, int pk, const AttnParams &p,
                        cudaStream_t st);

static size_t bwd_layout(const bsa_attn_args *a, BwdWs *w, uint8_t *base) {
  bsa_csr_args c;
  csr_args_from(a, &c);
  const long long Lp = (long long)attn_nq(a) * a->bs;
  const long long nbins = (long long)a->B * c.Hs * a->nblk;
  const long long E = (long long)a->B * c.Hs * attn_nq(a) * a->kk;
  const int Y = a->Hkv / c.Hs;
  const long long pmax = 2 * ((E + kChunkEntries - 1) / kChunkEntries) + 1;
  size_t scan_bytes = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, (unsigned long long *)nullptr,
                                (unsigned long long *)nullptr, (int)(nbins + 1));
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t *p = base ? base + off : nullptr;
    off += align_up(bytes, 256);
    return p;
  };
  w->dvec = (float *)take((size_t)a->B * a->Hq * Lp * 4);
  w->row_ptr = (int32_t *)take((nbins + 1) * 4);
  w->col = (int32_t *)take(E * 4);
  w->plan_in = (unsigned long long *)take((nbins + 1) * 8);
  w->plan = (unsigned long long *)take((nbins + 1) * 8);
  const long long ncap = nbins + (E + kChunkEntries - 1) / kChunkEntries + 1;
  w->chunk_bin = (int32_t *)take(ncap * 4);
  size_t sort_bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, (int32_t *)nullptr, (int32_t *)nullptr,
                                  (int32_t *)nullptr, (int32_t *)nullptr, (int)ncap, 0,
                                  bits_for((long long)(nbins / a->nblk + 1) * (kChunkEntries + 2)));
  w->ord_key_in = (int32_t *)take(ncap * 4);
  w->ord_key_out = (int32_t *)take(ncap * 4);
  w->ord_in = (int32_t *)take(ncap * 4);
  w->ord = (int32_t *)take(ncap * 4);
  w->sort_bytes = sort_bytes;
  w->sort_tmp = take(sort_bytes);
  w->csr_bytes = sel_csr_workspace(&c);
  w->csr_ws = take(w->csr_bytes);
  w->scan_bytes = scan_bytes;
  w->scan_tmp = take(scan_bytes);
  w->part = (float *)take((size_t)pmax * Y * 2 * a->bs * a->D * 4);
  const size_t ds_bytes = dq_ds_bytes(a, attn_nq(a));
  w->ds = ds_bytes ? take(ds_bytes) : nullptr;
  w->total = off;
  return off;
}

size_t attn_bwd_workspace(const bsa_attn_args *a) {
  BwdWs w;
  return bwd_layout(a, &w, nullptr);
}

bsa_status fill_attn_params(const bsa_attn_args *a, AttnParams *p, bool bwd);
bool dkdv_sm100_applicable(int dtype, int bs, int D);
bool dq_sm100_applicable(const AttnParams &p, int dtype, int D);
bsa_status launch_dvec(int dtype, const AttnParams &p, int D, cudaStream_t st);
bool dq_f5_applicable(const AttnParams &p, int dtype, int D);
bsa_status launch_dq_f5(int dtype, const CUtensorMap &mq, const CUtensorMap &mdo,
                        const CUtensorMap &mk, const CUtensorMap &mv, int pq, int pdo, int pk,
                        int pv, const AttnParams &p, cudaStream_t st);
bsa_status launch_dq_sm100(int dtype, const CUtensorMap &mq, const CUtensorMap &mdo,
                           const CUtensorMap &mk, const CUtensorMap &mv, int pq, int pdo, int pk,
                           int pv, const AttnParams &p, cudaStream_t st);
bsa_status launch_dkdv_sm100(int dtype, const CUtensorMap &mq, const CUtensorMap &mdo,
                             const CUtensorMap &mk, const CUtensorMap &mv, int pq, int pdo, int pk,
                             int pv, const AttnParams &p, const BwdPlan &pl, long long dkv_grid,
                             cudaStream_t st);

template <typename T, int BS, int D>
static bsa_status launch_bwd_tc(const bsa_attn_args *a, const AttnParams &p, const BwdPlan &pl,
                                long long dkv_grid, cudaStream_t st) {
  using Q = DqCfg<BS, D>;
  using K = DkvCfg<BS, D>;
  TensorMap4 mq, mdo, mk, mv, mqc, mdoc;
  bsa_status s;
  if ((s = make_tmap(&mq, a->q.ptr, a->dtype, a->B, a->Hq, p.Lq, D, a->q.sb, a->q.sh, a->q.sl, BS, "q")))
    return s;
  if ((s = make_tmap(&mdo, a->dout.ptr, a->dtype, a->B, a->Hq, p.Lq, D, a->dout.sb, a->dout.sh,
                     a->dout.sl, BS, "dout")))
    return s;
  if ((s = make_tmap(&mqc, a->q.ptr, a->dtype, a->B, a->Hq, p.Lq, D, a->q.sb, a->q.sh, a->q.sl,
                     Q::KC, "q")))
    return s;
  if ((s = make_tmap(&mdoc, a->dout.ptr, a->dtype, a->B, a->Hq, p.Lq, D, a->dout.sb, a->dout.sh,
                     a->dout.sl, Q::KC, "dout")))
    return s;
  // K/V: chunk boxes for dQ, full-block boxes for dK/dV
  TensorMap4 mkc, mvc;
  if ((s = make_tmap(&mkc, a->k.ptr, a->dtype, a->B, a->Hkv, a->L, D, a->k.sb, a->k.sh, a->k.sl,
                     Q::KC, "k")))
    return s;
  if ((s = make_tmap(&mvc, a->v.ptr, a->dtype, a->B, a->Hkv, a->L, D, a->v.sb, a->v.sh, a->v.sl,
                     Q::KC, "v")))
    return s;
  if ((s = make_tmap(&mk, a->k.ptr, a->dtype, a->B, a->Hkv, a->L, D, a->k.sb, a->k.sh, a->k.sl, BS,
                     "k")))
    return s;
  if ((s = make_tmap(&mv, a->v.ptr, a->dtype, a->B, a->Hkv, a->L, D, a->v.sb, a->v.sh, a->v.sl, BS,
                     "v")))
    return s;
  auto pk = [](const TensorMap4 &m) { return m.perm[0] | (m.perm[1] << 2) | (m.perm[2] << 4); };
  if (BS == 64 && D == 64 && p.ds && dkdv_sm100_applicable(a->dtype, BS, D)) {
    // dK/dV first (it stores the dS tiles), then dQ from the stored tiles
    if ((s = launch_dvec(a->dtype, p, D, st))) return s;
    if ((s = launch_dkdv_sm100(a->dtype, mqc.map, mdoc.map, mk.map, mv.map, pk(mqc), pk(mdoc),
                               pk(mk), pk(mv), p, pl, dkv_grid, st)))
      return s;
    if ((s = launch_dq_ds(a->dtype, mk.map, pk(mk), p, st))) return s;
    dkdv_reduce_kernel<T><<<dim3(pl.nbins, pl.Y), 256, 0, st>>>(p, pl, BS, D);
    return check_launch("dkdv_reduce");
  }
  if (BS == 64 && D == 64 && dq_f5_applicable(p, a->dtype, D)) {
    if ((s = launch_dvec(a->dtype, p, D, st))) return s;
    if ((s = launch_dq_f5(a->dtype, mq.map, mdo.map, mk.map, mv.map, pk(mq), pk(mdo), pk(mk),
                          pk(mv), p, st)))
      return s;
  } else if (dq_sm100_applicable(p, a->dtype, D) && a->sel) {
    if ((s = launch_dvec(a->dtype, p, D, st))) return s;
    if ((s = launch_dq_sm100(a->dtype, mq.map, mdo.map, mkc.map, mvc.map, pk(mq), pk(mdo), pk(mkc),
                             pk(mvc), p, st)))
      return s;
  } else {
    auto kq = attn_dq_kernel<T, BS, D>;
    cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, Q::SMEM);
    const long long grid = (long long)a->B * a->Hq * p.nq;
    kq<<<(unsigned)grid, Q::NT, Q::SMEM, st>>>(mq.map, mdo.map, mkc.map, mvc.map, pk(mq), pk(mdo),
                                                pk(mkc), pk(mvc), p);
    if ((s = check_launch("attn_dq"))) return s;
  }
  if (dkdv_sm100_applicable(a->dtype, BS, D)) {
    if ((s = launch_dkdv_sm100(a->dtype, mqc.map, mdoc.map, mk.map, mv.map, pk(mqc), pk(mdoc),
                               pk(mk), pk(mv), p, pl, dkv_grid, st)))
      return s;
  } else {
    auto kk = attn_dkdv_kernel<T, BS, D>;
    cudaFuncSetAttribute(kk, cudaFuncAttributeMaxDynamicSharedMemorySize, K::SMEM);
    kk<<<dim3((unsigned)dkv_grid, pl.Y), K::NT, K::SMEM, st>>>(mqc.map, mdoc.map, mk.map, mv.map,
                                                               pk(mqc), pk(mdoc), pk(mk), pk(mv), p,
                                                               pl);
    if ((s = check_launch("attn_dkdv"))) return s;
  }
  dkdv_reduce_kernel<T><<<dim3(pl.nbins, pl.Y), 256, 0, st>>>(p, pl, BS, D);
  return check_launch("dkdv_reduce");
}

template <int BS, int D>
static bsa_status launch_bwd_f32(const AttnParams &p, const BwdPlan &pl, long long dkv_grid,
                                 cudaStream_t st) {
  using C = F32BwdCfg<BS, D>;
  auto kq = attn_dq_f32_kernel<BS, D>;
  cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, C::DQ_SMEM);
  const long long grid = (long long)p.B * p.Hq * p.nq;
  kq<<<(unsigned)grid, 256, C::DQ_SMEM, st>>>(p);
  if (bsa_status s = check_launch("attn_dq_f32")) return s;
  auto kk = attn_dkdv_f32_kernel<BS, D>;
  cudaFuncSetAttribute(kk, cudaFuncAttributeMaxDynamicSharedMemorySize, C::DKV_SMEM);
  kk<<<dim3((unsigned)dkv_grid, pl.Y), 256, C::DKV_SMEM, st>>>(p, pl);
  if (bsa_status s = check_launch("attn_dkdv_f32")) return s;
  dkdv_reduce_kernel<float><<<dim3(pl.nbins, pl.Y), 256, 0, st>>>(p, pl, BS, D);
  return check_launch("dkdv_reduce");
}

bsa_status run_attn_bwd(const bsa_attn_args *a, void *ws, size_t ws_bytes, cudaStream_t st) {
  AttnParams p;
  bsa_status s = fill_attn_params(a, &p, true);
  if (s) return s;
  if (!a->sel) return fail(BSA_ERR_UNSUPPORTED, "attn_bwd: needs an explicit selection");
  BwdWs w;
  const size_t need = bwd_layout(a, &w, nullptr);
  if (!ws || ws_bytes < need)
    return fail(BSA_ERR_WORKSPACE, "attn_bwd: workspace too small (need " + std::to_string(need) +
                                       " bytes)");
  if (reinterpret_cast<uintptr_t>(ws) % 256) return fail(BSA_ERR_WORKSPACE, "attn_bwd: workspace not 256-byte aligned");
  bwd_layout(a, &w, reinterpret_cast<uint8_t *>(ws));
  p.dvec = w.dvec;
  p.ds = w.ds;

  bsa_csr_args c;
  csr_args_from(a, &c);
  c.row_ptr = w.row_ptr;
  c.col = w.col;
  if ((s = run_sel_csr(&c, w.csr_ws, w.csr_bytes, st))) return s;
  const int nbins = a->B * c.Hs * a->nblk;
  plan_kernel<<<(nbins + 256) / 256, 256, 0, st>>>(w.row_ptr, w.plan_in, nbins, kChunkEntries);
  if ((s = check_launch("plan"))) return s;
  size_t tb = w.scan_bytes;
  if (cub::DeviceScan::ExclusiveSum(w.scan_tmp, tb, w.plan_in, w.plan, nbins + 1, st) !=
      cudaSuccess)
    return fail(BSA_ERR_LAUNCH, "attn_bwd: plan scan failed");
  chunk_bin_kernel<<<(nbins + 255) / 256, 256, 0, st>>>(w.plan, nbins, w.chunk_bin);
  if ((s = check_launch("chunk_bin"))) return s;
  BwdPlan pl;
  pl.Hs = c.Hs;
  pl.Y = a->Hkv / c.Hs;
  pl.nbins = nbins;
  pl.C = kChunkEntries;
  pl.row_ptr = w.row_ptr;
  pl.col = w.col;
  pl.plan = w.plan;
  pl.chunk_bin = w.chunk_bin;
  pl.chunk_ord = nullptr;
  pl.part = w.part;
  const long long E = (long long)a->B * c.Hs * attn_nq(a) * a->kk;
  pl.npart = 2 * ((E + kChunkEntries - 1) / kChunkEntries) + 1;
  pl.ncol = (int)E;
  const long long dkv_grid = nbins + (E + kChunkEntries - 1) / kChunkEntries;
  if (a->dtype != BSA_F32 && dkdv_sm100_applicable(a->dtype, a->bs, a->D) &&
      !getenv("BSA_DKDV_NOSORT")) {
    const int ncap = (int)(dkv_grid + 1);
    chunk_key_kernel<<<(ncap + 255) / 256, 256, 0, st>>>(w.plan, w.row_ptr, w.chunk_bin, nbins,
                                                        a->nblk, kChunkEntries, ncap, w.ord_key_in,
                                                        w.ord_in);
    if ((s = check_launch("chunk_key"))) return s;
    size_t sb = w.sort_bytes;
    const int key_bits = bits_for((long long)(nbins / a->nblk + 1) * (kChunkEntries + 2));
    if (cub::DeviceRadixSort::SortPairs(w.sort_tmp, sb, w.ord_key_in, w.ord_key_out, w.ord_in,
                                        w.ord, ncap, 0, key_bits, st) != cudaSuccess)
      return fail(BSA_ERR_LAUNCH, "attn_bwd: chunk order sort failed");
    pl.chunk_ord = w.ord;
  }

  if (a->dtype == BSA_F32) {
#define BSA_BF32(BS_, D_) \
  if (a->bs == BS_ && a->D == D_) return launch_bwd_f32<BS_, D_>(p, pl, dkv_grid, st);
    BSA_BF32(16, 64)
    BSA_BF32(32, 64)
    BSA_BF32(64, 64)
    BSA_BF32(16, 32)
    BSA_BF32(32, 32)
    BSA_BF32(64, 32)
#undef BSA_BF32
    return fail(BSA_ERR_UNSUPPORTED, "attn_bwd: no fp32 kernel for this (bs, D)");
  }
#define BSA_BTC(T_, BS_, D_) \
  if (a->bs == BS_ && a->D == D_) return launch_bwd_tc<T_, BS_, D_>(a, p, pl, dkv_grid, st);
  if (a->dtype == BSA_BF16) {
    BSA_BTC(__nv_bfloat16, 16, 64)
    BSA_BTC(__nv_bfloat16, 32, 64)
    BSA_BTC(__nv_bfloat16, 64, 64)
    BSA_BTC(__nv_bfloat16, 128, 64)
    BSA_BTC(__nv_bfloat16, 64, 128)
  } else {
    BSA_BTC(__half, 16, 64)
    BSA_BTC(__half, 32, 64)
    BSA_BTC(__half, 64, 64)
    BSA_BTC(__half, 128, 64)
    BSA_BTC(__half, 64, 128)
  }
#undef BSA_BTC
  return fail(BSA_ERR_UNSUPPORTED, "attn_bwd: no bf16/f16 kernel for (bs, D) = (" +
                                       std::to_string(a->bs) + ", " + std::to_string(a->D) + ")");
}

}  // namespace bsa
