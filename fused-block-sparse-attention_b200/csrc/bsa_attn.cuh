// Parameter blocks and tile traits shared by the attention kernels and their
// host launchers.
#pragma once
#include "bsa_common.cuh"

namespace bsa {

struct AttnParams {
  int B, Hq, Hkv, grp, L, nblk, kk, bs, mask_mode, causal;
  int q0, nq, Lq;  // local query blocks [q0, q0 + nq) of Lq rows (q0 = 0, nq = nblk, Lq = L unsharded)
  int Lp;        // nq * bs (row count of lse / Dvec)
  float scale;   // softmax scale
  float scale2;  // scale * log2(e)
  const int32_t *sel;
  int64_t sel_sb, sel_sh, sel_sn;
  const float *gate;
  int64_t gate_sb, gate_sh, gate_sn;
  // forward
  void *o;
  int64_t o_sb, o_sh, o_sl;
  const void *og;
  int64_t og_sb, og_sh, og_sl;
  float *lse;
  // backward
  const void *q, *k, *v, *dout;  // used by the fp32 SIMT kernels (no TMA)
  int64_t q_sb, q_sh, q_sl, k_sb, k_sh, k_sl, v_sb, v_sh, v_sl, do_sb, do_sh, do_sl;
  const void *oin;
  int64_t oi_sb, oi_sh, oi_sl;
  void *dq, *dk, *dv;
  int64_t dq_sb, dq_sh, dq_sl, dk_sb, dk_sh, dk_sl, dv_sb, dv_sh, dv_sl;
  float *dgate;
  float *dvec;  // (B,Hq,Lp) rowsum(dO * O)
  // dS tiles of the active (query block, slot) entries, written by the dK/dV
  // kernel and read back by the dQ kernel that consumes them (null: dQ
  // recomputes S and dP itself): bf16/f16 [B][Hq][nq][kk][64 keys][64 rows]
  void *ds;
  // partial rotary embedding of q applied inside the forward (null: none)
  const void *rope_cos, *rope_sin;
  int64_t rope_sb, rope_sl;
  int rope_rot;
  int32_t *status;
};

// Backward CSR / chunk plan (device pointers into the workspace).
struct BwdPlan {
  int Hs;        // selection heads
  int Y;         // KV heads per selection head
  int nbins;     // B * Hs * nblk
  int C;         // entries per dK/dV chunk
  const int32_t *row_ptr;  // nbins + 1
  const int32_t *col;      // entries qblk*kk + slot
  const unsigned long long *plan;  // nbins + 1: (chunk_off << 32) | part_off (exclusive)
  const int32_t *chunk_bin;        // chunk -> bin
  const int32_t *chunk_ord;        // processing order of the chunks (largest first); may be null
  float *part;             // partial dK/dV tiles
  long long npart;         // capacity of part, in tiles (per KV head of a bin group)
  int ncol;                // capacity of col
};

template <int BS, int D>
struct TileCfg {
  static constexpr int NW = BS / 16;          // warps, 16 rows each
  static constexpr int NT = NW * 32;
  static constexpr int KC = BS < 64 ? BS : 64;  // rows per streamed chunk
  static constexpr int NCH = BS / KC;         // chunks per block
  static constexpr int TILE = BS * D * 2;     // bytes of a full 16-bit block tile
  static constexpr int CH = KC * D * 2;       // bytes of one 16-bit chunk
};

}  // namespace bsa
