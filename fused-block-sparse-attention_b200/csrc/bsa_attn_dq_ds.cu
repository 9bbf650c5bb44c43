// Block-sparse attention backward, dQ from the stored dS tiles, on tcgen05
// (block 64, head dim 64).
//
// The dK/dV kernel already forms dS^T = P^T (dP^T - Dvec) for every active
// (query block, slot, query head) entry; with p.ds set it also writes each
// 64 x 64 tile (bf16/f16, rows = keys) to the workspace.  dQ is then one more
// GEMM per entry instead of a second recomputation of S and dP:
//
//   dQ_i = scale * sum over the live slots j of query block i of  dS_ij K_j
//
// which reads each dS tile once (8 KB per entry) and the selected K blocks
// (through L2), and runs two of the seven per-pair GEMMs of the recomputing
// design fewer.  Rounding is unchanged: the recomputing dQ kernel also
// multiplies the dS rounded to the input type by K.
//
// One CTA per pair of adjacent query blocks (tiles A, B) of one query head,
// two CTAs per SM.  Per live slot j of each tile: TMA loads of dS_j (the
// stored tile is MN-major for this product: rows are keys = the K dimension)
// and K_j (MN-major B: rows are keys) into a 3-stage ring, then 4 chained
// 64x64x16 MMAs into the tile's TMEM accumulator (tile B at lane offset 16).
// Warps 0-3 write dQ * scale; warp 4 is the producer; warp 5 owns TMEM and
// issues the MMAs.  Every wait is bounded (timeout -> BSA_DEVERR_TIMEOUT).
#include <type_traits>

#include "bsa_attn.cuh"
#include "bsa_host.h"
#include "bsa_tc05.cuh"

namespace bsa {

namespace {
constexpr int DS_BS = 64, DS_D = 64, DS_NST = 3;
constexpr int DS_TILE = DS_BS * DS_D * 2;  // 8 KB
constexpr int DS_MAXN = 64;
constexpr int DS_SMEM = 1024 + DS_NST * 4 * DS_TILE;  // (stage, {dS_A, dS_B, K_A, K_B})
constexpr uint32_t DS_TMEM_COLS = 64;

// kind::f16 instruction descriptor with both operands MN-major
__host__ __device__ constexpr uint32_t idesc_f16_mn(bool bf16, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | (1u << 15) | (1u << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
}  // namespace

template <typename T>
__global__ void __launch_bounds__(192, 2)
    attn_dq_ds_kernel(const __grid_constant__ CUtensorMap tds, const __grid_constant__ CUtensorMap tk,
                      const int perm_ds, const int perm_k, const AttnParams p) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC = idesc_f16_mn(kBF16, 64, DS_D);
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[DS_NST], empty[DS_NST], done;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int s_kb[2][DS_MAXN];    // key block of the j-th live slot
  __shared__ int s_slot[2][DS_MAXN];  // its slot
  __shared__ int s_n[2];

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

  // live slots: the entries the dK/dV kernel processed (same classification)
  if (warp < 2) {  // warp 0: tile A, warp 1: tile B
    const int t = warp;
    const int qi = qb0 + t, qblk = p.q0 + qi;
    int n = 0;
    if (t == 0 || validB) {
      const int32_t *selrow = p.sel + b * p.sel_sb + hk * p.sel_sh + (long long)qi * p.sel_sn;
      n = warp_live_slots(selrow, p.kk, DS_MAXN, qblk, p.nblk, p.bs, p.L, p.mask_mode, p.causal,
                          p.status, [&](int pos, int kb, int, int slot) {
                            s_kb[t][pos] = kb;
                            s_slot[t][pos] = slot;
                          });
    }
    if (lane == 0) s_n[t] = n;
  }
  if (tid == 0) {
    // descriptors fetched ahead of the first TMA load
    prefetch_tmap(&tds);
    prefetch_tmap(&tk);
    for (int s = 0; s < DS_NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tc05::alloc(&tmem_base_sh, DS_TMEM_COLS);
    tc05::relinquish();
  }
  tc05::fence_before();
  __syncthreads();
  tc05::fence_after();
  const uint32_t tmem = tmem_base_sh;
  const int nA = s_n[0], nB = s_n[1];
  const int nsteps = nA > nB ? nA : nB;

  if (warp == 4) {
    // ================= TMA producer: the warp waits together (voted), one
    // elected lane (lane 0) issues the loads
    {
      for (int j = 0; j < nsteps; ++j) {
        const int st = j % DS_NST;
        if (j >= DS_NST && !mbar_wait_warp(&empty[st], ((j / DS_NST) - 1) & 1)) {
          report(p.status, BSA_DEVERR_TIMEOUT);
          break;
        }
        if (tc05::elect_one()) {
          const int act = (j < nA ? 1 : 0) + (j < nB ? 1 : 0);
          mbar_expect_tx(&full[st], act * 2 * DS_TILE);
          uint8_t *ring = smem + st * 4 * DS_TILE;
          for (int t = 0; t < 2; ++t) {
            if (j >= (t ? nB : nA)) continue;
            const long long e =
                (((long long)b * p.Hq + h) * p.nq + (qb0 + t)) * p.kk + s_slot[t][j];
            tma_load_rhb(ring + t * DS_TILE, &tds, &full[st], perm_ds, 0, (int)(e * DS_BS), 0, 0);
            tma_load_rhb(ring + (2 + t) * DS_TILE, &tk, &full[st], perm_k, 0, s_kb[t][j] * p.bs,
                         hk, b);
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == 5) {
    // ================= MMA issuer: the whole warp walks the steps (warp-uniform
    // descriptors and waits); one elected lane, always lane 0, issues the MMAs
    // and commits
    {
      // both operands MN-major: rows are keys (the K dimension), 128 B of M/N
      const uint64_t d0 = tc05::sdesc(smem_u32(smem), DS_BS * 128, 1024);
      for (int j = 0; j < nsteps; ++j) {
        const int st = j % DS_NST;
        if (!mbar_wait_warp(&full[st], (j / DS_NST) & 1)) {
          report(p.status, BSA_DEVERR_TIMEOUT);
          break;
        }
        tc05::fence_after();
        for (int t = 0; t < 2; ++t) {
          if (j >= (t ? nB : nA)) continue;
          const uint64_t da = tc05::dadd(d0, (st * 4 + t) * DS_TILE);
          const uint64_t db = tc05::dadd(d0, (st * 4 + 2 + t) * DS_TILE);
          const uint32_t d = tc05::taddr(tmem, 16 * t, 0);
          if (tc05::elect_one()) {
#pragma unroll
            for (int ks = 0; ks < DS_BS / 16; ++ks)
              tc05::mma_f16(d, tc05::dadd(da, ks * 2048), tc05::dadd(db, ks * 2048), IDESC,
                            (j > 0 || ks > 0) ? 1u : 0u);
          }
          __syncwarp();
        }
        if (tc05::elect_one()) tc05::commit(&empty[st]);
        __syncwarp();
      }
      if (tc05::elect_one()) tc05::commit(&done);  // arrives once every MMA issued above has completed
      __syncwarp();
    }
  } else {
    // ================= epilogue warps 0-3: dQ * scale
    const int t = lane >> 4;
    const int r = warp * 16 + (lane & 15);  // query row within its block
    const int qi = qb0 + t;
    const int nmine = t ? nB : nA;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    if (!mbar_wait(&done, 0)) report(p.status, BSA_DEVERR_TIMEOUT);
    tc05::fence_after();
    float o[64];
    tc05::ld32(tmem + lane_base, o);
    tc05::ld32(tmem + lane_base + 32, o + 32);
    tc05::wait_ld();
    if (nmine == 0) {  // never accumulated: the TMEM columns hold stale data
#pragma unroll
      for (int c = 0; c < 64; ++c) o[c] = 0.f;
    }
    const long long grow = (long long)qi * p.bs + r;
    if (qi < p.nq && grow < p.Lq) {
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
  }
  tc05::fence_before();
  __syncthreads();
  if (warp == 5) {
    tc05::fence_after();
    tc05::dealloc(tmem, DS_TMEM_COLS);
  }
}

// The stored-dS dQ pass: block 64, head dim 64, 16-bit inputs, no gate
// gradient requested (the recomputing dQ kernel sums dgate from its own dS), and
// a workspace of at most 24 GB for the tiles; BSA_DQ_DS=0 turns it off.
size_t dq_ds_bytes(const bsa_attn_args *a, int nq) {
  const char *env = getenv("BSA_DQ_DS");
  if (env && env[0] == '0') return 0;
  if (a->dtype == BSA_F32 || a->bs != 64 || a->D != 64 || !a->sel || a->dgate || a->kk > DS_MAXN ||
      getenv("BSA_BWD_LEGACY"))
    return 0;
  const long long rows = (long long)a->B * a->Hq * nq * a->kk * DS_BS;
  if (rows >= (1LL << 31)) return 0;
  const size_t bytes = (size_t)rows * DS_D * 2;
  return bytes <= (size_t(24) << 30) ? bytes : 0;
}

bsa_status launch_dq_ds(int dtype, const CUtensorMap &mk, int pk, const AttnParams &p,
                        cudaStream_t st) {
  TensorMap4 mds;
  const long long rows = (long long)p.B * p.Hq * p.nq * p.kk * DS_BS;
  if (bsa_status s = make_tmap(&mds, p.ds, dtype, 1, 1, (int)rows, DS_D, rows * DS_D, rows * DS_D,
                               DS_D, DS_BS, "ds"))
    return s;
  const int pds = mds.perm[0] | (mds.perm[1] << 2) | (mds.perm[2] << 4);
  const long long grid = (long long)p.B * p.Hq * ((p.nq + 1) / 2);
  if (dtype == BSA_BF16) {
    cudaFuncSetAttribute(attn_dq_ds_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, DS_SMEM);
    attn_dq_ds_kernel<__nv_bfloat16><<<(unsigned)grid, 192, DS_SMEM, st>>>(mds.map, mk, pds, pk, p);
  } else {
    cudaFuncSetAttribute(attn_dq_ds_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, DS_SMEM);
    attn_dq_ds_kernel<__half><<<(unsigned)grid, 192, DS_SMEM, st>>>(mds.map, mk, pds, pk, p);
  }
  return check_launch("attn_dq_ds");
}

}  // namespace bsa
