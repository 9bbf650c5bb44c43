// extern "C" entry points of libbsa_b200.so: argument validation, then the
// launchers in bsa_attn_fwd.cu / bsa_attn_bwd.cu / bsa_select.cu.
#include <cmath>

#include "bsa_attn.cuh"
#include "bsa_host.h"

namespace bsa {

bsa_status run_attn_fwd(const bsa_attn_args *a, cudaStream_t st);
bsa_status run_attn_bwd(const bsa_attn_args *a, void *ws, size_t ws_bytes, cudaStream_t st);
size_t attn_bwd_workspace(const bsa_attn_args *a);
bsa_status run_sel_csr(const bsa_csr_args *a, void *ws, size_t ws_bytes, cudaStream_t st);
size_t sel_csr_workspace(const bsa_csr_args *a);
bsa_status run_pool(const bsa_pool_args *a, cudaStream_t st);
bsa_status run_select(const bsa_select_args *a, cudaStream_t st);
int32_t select_width(const bsa_select_args *a);
int32_t lsh_width(const bsa_lsh_args *a);
size_t lsh_workspace(const bsa_lsh_args *a);
bsa_status run_lsh(const bsa_lsh_args *a, void *ws, size_t ws_bytes, cudaStream_t st);
bsa_status run_rope(const bsa_rope_args *a, cudaStream_t st);
int32_t centroid_width(const bsa_centroid_args *a);
bsa_status run_centroid_route(const bsa_centroid_args *a, cudaStream_t st);
int32_t scores_width(int nblk, int topk, int sink);
bsa_status run_scores_topk(const bsa_scores_args *a, cudaStream_t st);
bsa_status run_qmax(const bsa_qmax_args *a, cudaStream_t st);
size_t decode_workspace(const bsa_decode_args *a);
bsa_status run_decode(const bsa_decode_args *a, void *ws, size_t ws_bytes, cudaStream_t st);

static bsa_status check_view(const bsa_view &v, int dtype, const char *name, bool vec16) {
  if (!v.ptr) return fail(BSA_ERR_ARG, std::string(name) + " is NULL");
  if (!vec16) return BSA_OK;
  const size_t es = elem_size(dtype);
  if (reinterpret_cast<uintptr_t>(v.ptr) % 16 || (v.sb * (int64_t)es) % 16 ||
      (v.sh * (int64_t)es) % 16 || (v.sl * (int64_t)es) % 16)
    return fail(BSA_ERR_STRIDE,
                std::string(name) + ": base and B/H/L strides must be 16-byte multiples");
  return BSA_OK;
}

bsa_status fill_attn_params(const bsa_attn_args *a, AttnParams *p, bool bwd) {
  if (!a) return fail(BSA_ERR_ARG, "args is NULL");
  if (a->dtype != BSA_BF16 && a->dtype != BSA_F16 && a->dtype != BSA_F32)
    return fail(BSA_ERR_DTYPE, "attn: dtype must be bf16, f16 or f32");
  if (a->B <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->L <= 0 || a->D <= 0 || a->bs <= 0 ||
      a->nblk <= 0 || a->kk <= 0)
    return fail(BSA_ERR_SHAPE, "attn: sizes must be positive");
  if (a->Hq % a->Hkv) return fail(BSA_ERR_SHAPE, "attn: Hq must be a multiple of Hkv");
  if ((long long)a->nblk * a->bs < a->L || (long long)(a->nblk - 1) * a->bs >= a->L)
    return fail(BSA_ERR_SHAPE, "attn: nblk must equal ceil(L / bs)");
  if ((long long)a->B * a->Hq * a->nblk >= (1LL << 31))
    return fail(BSA_ERR_SHAPE, "attn: B*Hq*nblk too large");
  if (a->mask_mode != BSA_MASK_SLOT && a->mask_mode != BSA_MASK_TOKEN)
    return fail(BSA_ERR_ARG, "attn: bad mask_mode");
  if (!a->sel && a->kk != a->nblk)
    return fail(BSA_ERR_SHAPE, "attn: identity selection (sel NULL) needs kk == nblk");
  if (a->sel && a->kk > kMaxKK)
    return fail(BSA_ERR_UNSUPPORTED, "attn: kk > 512 needs the identity selection");
  if (!(a->scale > 0.f) || !std::isfinite(a->scale)) return fail(BSA_ERR_ARG, "attn: bad scale");
  const int Lq = a->Lq > 0 ? a->Lq : a->L;
  if (a->q_blk0 < 0 || a->Lq < 0 || (long long)a->q_blk0 * a->bs + Lq > a->L ||
      (Lq % a->bs && (long long)a->q_blk0 * a->bs + Lq != a->L))
    return fail(BSA_ERR_SHAPE, "attn: query range must lie in [0, L) and end on a block or at L");
  if (!a->sel && (a->q_blk0 || a->Lq))
    return fail(BSA_ERR_UNSUPPORTED, "attn: a query range needs an explicit selection");
  const bool tc = a->dtype != BSA_F32;
  bsa_status s;
  if ((s = check_view(a->q, a->dtype, "q", tc)) || (s = check_view(a->k, a->dtype, "k", tc)) ||
      (s = check_view(a->v, a->dtype, "v", tc)) || (s = check_view(a->o, a->dtype, "o", tc)))
    return s;
  if (a->out_gate.ptr && (s = check_view(a->out_gate, a->dtype, "out_gate", tc))) return s;
  if (bwd) {
    if ((s = check_view(a->dout, a->dtype, "dout", tc)) ||
        (s = check_view(a->dq, a->dtype, "dq", tc)) ||
        (s = check_view(a->dk, a->dtype, "dk", false)) ||
        (s = check_view(a->dv, a->dtype, "dv", false)))
      return s;
    if (tc && ((a->dk.sl % 2) || (a->dv.sl % 2) || reinterpret_cast<uintptr_t>(a->dk.ptr) % 4 ||
               reinterpret_cast<uintptr_t>(a->dv.ptr) % 4))
      return fail(BSA_ERR_STRIDE, "attn_bwd: dk/dv rows must be 4-byte aligned");
    if (!a->lse) return fail(BSA_ERR_ARG, "attn_bwd: lse is NULL");
  }
  AttnParams &P = *p;
  P = AttnParams{};
  P.B = a->B;
  P.Hq = a->Hq;
  P.Hkv = a->Hkv;
  P.grp = a->Hq / a->Hkv;
  P.L = a->L;
  P.nblk = a->nblk;
  P.kk = a->kk;
  P.bs = a->bs;
  P.mask_mode = a->mask_mode;
  P.causal = a->causal ? 1 : 0;
  P.q0 = a->q_blk0;
  P.Lq = Lq;
  P.nq = (Lq + a->bs - 1) / a->bs;
  P.Lp = P.nq * a->bs;
  P.scale = a->scale;
  P.scale2 = a->scale * 1.4426950408889634f;
  P.sel = a->sel;
  P.sel_sb = a->sel_sb;
  P.sel_sh = a->sel_sh;
  P.sel_sn = a->sel_sn;
  P.gate = a->gate;
  P.gate_sb = a->gate_sb;
  P.gate_sh = a->gate_sh;
  P.gate_sn = a->gate_sn;
  P.o = a->o.ptr;
  P.o_sb = a->o.sb;
  P.o_sh = a->o.sh;
  P.o_sl = a->o.sl;
  P.og = a->out_gate.ptr;
  P.og_sb = a->out_gate.sb;
  P.og_sh = a->out_gate.sh;
  P.og_sl = a->out_gate.sl;
  P.lse = a->lse;
  if (a->rope_cos) {
    if (bwd) return fail(BSA_ERR_ARG, "attn_bwd: rope is forward-only (pass the rotated q)");
    if (!a->rope_sin || a->rope_rot <= 0 || a->rope_rot % 16 || a->rope_rot > 64 ||
        a->rope_rot > a->D)
      return fail(BSA_ERR_ARG, "attn_fwd: rope needs cos and sin and 16 <= rot <= 64, rot % 16 == 0");
    P.rope_cos = a->rope_cos;
    P.rope_sin = a->rope_sin;
    P.rope_sb = a->rope_sb;
    P.rope_sl = a->rope_sl;
    P.rope_rot = a->rope_rot;
  }
  P.q = a->q.ptr;
  P.q_sb = a->q.sb;
  P.q_sh = a->q.sh;
  P.q_sl = a->q.sl;
  P.k = a->k.ptr;
  P.k_sb = a->k.sb;
  P.k_sh = a->k.sh;
  P.k_sl = a->k.sl;
  P.v = a->v.ptr;
  P.v_sb = a->v.sb;
  P.v_sh = a->v.sh;
  P.v_sl = a->v.sl;
  P.dout = a->dout.ptr;
  P.do_sb = a->dout.sb;
  P.do_sh = a->dout.sh;
  P.do_sl = a->dout.sl;
  P.oin = a->o.ptr;
  P.oi_sb = a->o.sb;
  P.oi_sh = a->o.sh;
  P.oi_sl = a->o.sl;
  P.dq = a->dq.ptr;
  P.dq_sb = a->dq.sb;
  P.dq_sh = a->dq.sh;
  P.dq_sl = a->dq.sl;
  P.dk = a->dk.ptr;
  P.dk_sb = a->dk.sb;
  P.dk_sh = a->dk.sh;
  P.dk_sl = a->dk.sl;
  P.dv = a->dv.ptr;
  P.dv_sb = a->dv.sb;
  P.dv_sh = a->dv.sh;
  P.dv_sl = a->dv.sl;
  P.dgate = a->dgate;
  P.status = a->status;
  return BSA_OK;
}

static bsa_status check_csr(const bsa_csr_args *a) {
  if (!a || !a->sel) return fail(BSA_ERR_ARG, "sel_csr: NULL selection");
  if (a->B <= 0 || a->Hs <= 0 || a->nblk <= 0 || a->kk <= 0 || a->bs <= 0 || a->L <= 0)
    return fail(BSA_ERR_SHAPE, "sel_csr: sizes must be positive");
  if ((long long)a->B * a->Hs * a->nblk * a->kk >= (1LL << 31))
    return fail(BSA_ERR_SHAPE, "sel_csr: too many entries");
  if ((long long)a->nblk * a->kk >= (1LL << 31)) return fail(BSA_ERR_SHAPE, "sel_csr: nblk*kk too large");
  if (a->mask_mode != BSA_MASK_SLOT && a->mask_mode != BSA_MASK_TOKEN)
    return fail(BSA_ERR_ARG, "sel_csr: bad mask_mode");
  return BSA_OK;
}

}  // namespace bsa

using namespace bsa;

extern "C" {

bsa_status bsa_attn_fwd(const bsa_attn_args *a, bsa_stream_t stream) {
  return run_attn_fwd(a, reinterpret_cast<cudaStream_t>(stream));
}

size_t bsa_attn_bwd_workspace(const bsa_attn_args *a) {
  AttnParams p;
  if (fill_attn_params(a, &p, true) != BSA_OK || !a->sel) return 0;
  return attn_bwd_workspace(a);
}

bsa_status bsa_attn_bwd(const bsa_attn_args *a, void *workspace, size_t workspace_bytes,
                        bsa_stream_t stream) {
  return run_attn_bwd(a, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

bsa_status bsa_pool(const bsa_pool_args *a, bsa_stream_t stream) {
  if (!a) return fail(BSA_ERR_ARG, "pool: args is NULL");
  return run_pool(a, reinterpret_cast<cudaStream_t>(stream));
}

int32_t bsa_select_width(const bsa_select_args *a) { return a ? select_width(a) : 0; }

bsa_status bsa_select(const bsa_select_args *a, bsa_stream_t stream) {
  if (!a) return fail(BSA_ERR_ARG, "select: args is NULL");
  return run_select(a, reinterpret_cast<cudaStream_t>(stream));
}

int32_t bsa_select_lsh_width(const bsa_lsh_args *a) { return a ? lsh_width(a) : 0; }

size_t bsa_select_lsh_workspace(const bsa_lsh_args *a) { return a ? lsh_workspace(a) : 0; }

bsa_status bsa_select_lsh(const bsa_lsh_args *a, void *workspace, size_t workspace_bytes,
                          bsa_stream_t stream) {
  if (!a) return fail(BSA_ERR_ARG, "select_lsh: args is NULL");
  return run_lsh(a, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t bsa_csr_workspace(const bsa_csr_args *a) {
  if (check_csr(a) != BSA_OK) return 0;
  return sel_csr_workspace(a);
}

bsa_status bsa_sel_csr(const bsa_csr_args *a, void *workspace, size_t workspace_bytes,
                       bsa_stream_t stream) {
  if (bsa_status s = check_csr(a)) return s;
  if (!a->row_ptr || !a->col) return fail(BSA_ERR_ARG, "sel_csr: NULL output");
  return run_sel_csr(a, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t bsa_decode_workspace(const bsa_decode_args *a) { return a ? decode_workspace(a) : 0; }

bsa_status bsa_decode(const bsa_decode_args *a, void *workspace, size_t workspace_bytes,
                      bsa_stream_t stream) {
  if (!a) return fail(BSA_ERR_ARG, "decode: args is NULL");
  return run_decode(a, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int32_t bsa_select_scores_width(const bsa_scores_args *a) {
  return a ? scores_width(a->nblk, a->topk, a->sink) : 0;
}

bsa_status bsa_select_scores(const bsa_scores_args *a, bsa_stream_t stream) {
  if (!a) return fail(BSA_ERR_ARG, "select_scores: args is NULL");
  return run_scores_topk(a, reinterpret_cast<cudaStream_t>(stream));
}

bsa_status bsa_select_qmax(const bsa_qmax_args *a, bsa_stream_t stream) {
  if (!a) return fail(BSA_ERR_ARG, "select_qmax: args is NULL");
  return run_qmax(a, reinterpret_cast<cudaStream_t>(stream));
}

bsa_status bsa_rope(const bsa_rope_args *a, bsa_stream_t stream) {
  if (!a) return fail(BSA_ERR_ARG, "rope: args is NULL");
  return run_rope(a, reinterpret_cast<cudaStream_t>(stream));
}

int32_t bsa_centroid_width(const bsa_centroid_args *a) { return a ? centroid_width(a) : 0; }

bsa_status bsa_centroid_route(const bsa_centroid_args *a, bsa_stream_t stream) {
  if (!a) return fail(BSA_ERR_ARG, "centroid_route: args is NULL");
  return run_centroid_route(a, reinterpret_cast<cudaStream_t>(stream));
}

bsa_status bsa_status_decode(int32_t w) {
  if (w & BSA_DEVERR_TIMEOUT) return BSA_ERR_TIMEOUT;
  if (w & BSA_DEVERR_INDEX) return BSA_ERR_INDEX;
  return BSA_OK;
}

int32_t bsa_version(void) { return 100; }

}  // extern "C"
