"""ctypes binding of libbsa_b200.so (include/bsa.h) for torch tensors.

This module is the only place that touches the C ABI.  Every call enqueues
work on torch's current CUDA stream and never falls back to a CPU path: when
the library is missing, or a tensor is not on a CUDA device, it raises.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "csrc", "libbsa_b200.so")

# ---------------------------------------------------------------- enums
OK, ERR_SHAPE, ERR_DTYPE, ERR_STRIDE, ERR_UNSUPPORTED, ERR_INDEX, ERR_LAUNCH, ERR_TIMEOUT, \
    ERR_WORKSPACE, ERR_ARG = range(10)
DEVERR_INDEX, DEVERR_TIMEOUT = 1, 2
BF16, F16, F32 = 0, 1, 2
MASK_SLOT, MASK_TOKEN = 0, 1
SCORE_DOT, SCORE_MAXDOT2, SCORE_QUEST = 0, 1, 2
SEL_SSA, SEL_FINISH, SEL_RAW = 0, 1, 2
HASH_ARGMAX, HASH_SIGN = 0, 1

_STATUS_NAMES = {ERR_SHAPE: "shape", ERR_DTYPE: "dtype", ERR_STRIDE: "stride",
                 ERR_UNSUPPORTED: "unsupported", ERR_INDEX: "index", ERR_LAUNCH: "launch",
                 ERR_TIMEOUT: "timeout", ERR_WORKSPACE: "workspace", ERR_ARG: "argument"}

_DTYPES = {torch.bfloat16: BF16, torch.float16: F16, torch.float32: F32}


class BsaError(RuntimeError):
    """A bsa_status other than BSA_OK; `.status` holds the code."""

    def __init__(self, status, msg):
        super().__init__("bsa %s error: %s" % (_STATUS_NAMES.get(status, status), msg))
        self.status = status


class BsaShapeError(BsaError, ValueError):
    pass


# ---------------------------------------------------------------- structs
class View(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("sb", ctypes.c_int64), ("sh", ctypes.c_int64),
                ("sl", ctypes.c_int64)]


class AttnArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("dtype", "B", "Hq", "Hkv", "L", "D", "bs", "nblk", "kk", "mask_mode", "causal")] + [
        ("scale", ctypes.c_float)] + [(n, View) for n in
                                      ("q", "k", "v", "o", "dout", "dq", "dk", "dv", "out_gate")] + [
        ("sel", ctypes.c_void_p), ("sel_sb", ctypes.c_int64), ("sel_sh", ctypes.c_int64),
        ("sel_sn", ctypes.c_int64),
        ("gate", ctypes.c_void_p), ("gate_sb", ctypes.c_int64), ("gate_sh", ctypes.c_int64),
        ("gate_sn", ctypes.c_int64),
        ("lse", ctypes.c_void_p), ("dgate", ctypes.c_void_p), ("status", ctypes.c_void_p),
        ("q_blk0", ctypes.c_int32), ("Lq", ctypes.c_int32),
        ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p), ("rope_sb", ctypes.c_int64),
        ("rope_sl", ctypes.c_int64), ("rope_rot", ctypes.c_int32)]


class PoolArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("dtype", "B", "H", "L", "D", "bs", "nblk", "grp")] + [
        ("x", View), ("mean", ctypes.c_void_p), ("vmin", ctypes.c_void_p),
        ("vmax", ctypes.c_void_p), ("status", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p), ("rope_sb", ctypes.c_int64),
        ("rope_sl", ctypes.c_int64), ("rope_rot", ctypes.c_int32)]


class SelectArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("G", "nblk", "dim", "score_kind", "layout", "causal", "topk", "sink")] + [
        ("a", ctypes.c_void_p), ("b1", ctypes.c_void_p), ("b2", ctypes.c_void_p),
        ("sel", ctypes.c_void_p), ("score_out", ctypes.c_void_p), ("gate_out", ctypes.c_void_p),
        ("status", ctypes.c_void_p), ("q_blk0", ctypes.c_int32), ("nq", ctypes.c_int32)]


class LshArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("G", "nblk", "dim", "hash_kind", "n_rounds", "n_planes", "cap", "causal", "topk")] + [
        ("scale", ctypes.c_float), ("a", ctypes.c_void_p), ("b", ctypes.c_void_p),
        ("planes", ctypes.c_void_p), ("sel", ctypes.c_void_p), ("score_out", ctypes.c_void_p),
        ("gate_out", ctypes.c_void_p), ("status", ctypes.c_void_p)]


class DecodeArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("dtype", "B", "Hq", "Hkv", "L", "D", "bs", "T", "kk", "mask_mode")] + [
        ("scale", ctypes.c_float)] + [(n, View) for n in ("q", "k", "v", "o")] + [
        ("sel", ctypes.c_void_p), ("sel_sb", ctypes.c_int64), ("sel_sh", ctypes.c_int64),
        ("gate", ctypes.c_void_p), ("gate_sb", ctypes.c_int64), ("gate_sh", ctypes.c_int64),
        ("status", ctypes.c_void_p)]


class ScoresArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("G", "nblk", "topk", "sink")] + [
        ("score", ctypes.c_void_p), ("score_sg", ctypes.c_int64), ("score_si", ctypes.c_int64),
        ("sel", ctypes.c_void_p), ("status", ctypes.c_void_p)]


class QmaxArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("G", "nblk", "bs", "dim", "topk", "sink", "M")] + [
        ("qtok", ctypes.c_void_p), ("kmax", ctypes.c_void_p), ("kmin", ctypes.c_void_p),
        ("cand", ctypes.c_void_p), ("sel", ctypes.c_void_p), ("status", ctypes.c_void_p)]


class CsrArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("B", "Hs", "nblk", "kk", "bs", "L", "mask_mode", "causal")] + [
        ("sel", ctypes.c_void_p), ("sel_sb", ctypes.c_int64), ("sel_sh", ctypes.c_int64),
        ("sel_sn", ctypes.c_int64), ("row_ptr", ctypes.c_void_p), ("col", ctypes.c_void_p),
        ("status", ctypes.c_void_p), ("q_blk0", ctypes.c_int32), ("nq", ctypes.c_int32)]


class CentroidArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("B", "nblk", "C", "cpq", "cap", "dim", "rk")] + [
        ("key_cent", ctypes.c_void_p), ("top_c", ctypes.c_void_p), ("q_blk", ctypes.c_void_p),
        ("k_blk", ctypes.c_void_p), ("sel", ctypes.c_void_p)]


class RopeArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("dtype", "B", "H", "L", "D", "rot")] + [
        ("x", View), ("y", View), ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p),
        ("cs_sb", ctypes.c_int64), ("cs_sl", ctypes.c_int64)]


# C symbols and their signatures; tests check that every one is exported.
SYMBOLS = {
    "bsa_attn_fwd": (ctypes.c_int, [ctypes.POINTER(AttnArgs), ctypes.c_void_p]),
    "bsa_attn_bwd_workspace": (ctypes.c_size_t, [ctypes.POINTER(AttnArgs)]),
    "bsa_attn_bwd": (ctypes.c_int, [ctypes.POINTER(AttnArgs), ctypes.c_void_p, ctypes.c_size_t,
                                    ctypes.c_void_p]),
    "bsa_pool": (ctypes.c_int, [ctypes.POINTER(PoolArgs), ctypes.c_void_p]),
    "bsa_select_width": (ctypes.c_int32, [ctypes.POINTER(SelectArgs)]),
    "bsa_select": (ctypes.c_int, [ctypes.POINTER(SelectArgs), ctypes.c_void_p]),
    "bsa_select_lsh_width": (ctypes.c_int32, [ctypes.POINTER(LshArgs)]),
    "bsa_select_lsh_workspace": (ctypes.c_size_t, [ctypes.POINTER(LshArgs)]),
    "bsa_select_lsh": (ctypes.c_int, [ctypes.POINTER(LshArgs), ctypes.c_void_p, ctypes.c_size_t,
                                      ctypes.c_void_p]),
    "bsa_select_scores_width": (ctypes.c_int32, [ctypes.POINTER(ScoresArgs)]),
    "bsa_select_scores": (ctypes.c_int, [ctypes.POINTER(ScoresArgs), ctypes.c_void_p]),
    "bsa_select_qmax": (ctypes.c_int, [ctypes.POINTER(QmaxArgs), ctypes.c_void_p]),
    "bsa_csr_workspace": (ctypes.c_size_t, [ctypes.POINTER(CsrArgs)]),
    "bsa_sel_csr": (ctypes.c_int, [ctypes.POINTER(CsrArgs), ctypes.c_void_p, ctypes.c_size_t,
                                   ctypes.c_void_p]),
    "bsa_sel_csr_noalloc": (ctypes.c_int, [ctypes.POINTER(CsrArgs), ctypes.c_void_p]),
    "bsa_rope": (ctypes.c_int, [ctypes.POINTER(RopeArgs), ctypes.c_void_p]),
    "bsa_centroid_width": (ctypes.c_int32, [ctypes.POINTER(CentroidArgs)]),
    "bsa_centroid_route": (ctypes.c_int, [ctypes.POINTER(CentroidArgs), ctypes.c_void_p]),
    "bsa_decode_workspace": (ctypes.c_size_t, [ctypes.POINTER(DecodeArgs)]),
    "bsa_decode": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), ctypes.c_void_p, ctypes.c_size_t,
                                  ctypes.c_void_p]),
    "bsa_status_decode": (ctypes.c_int, [ctypes.c_int32]),
    "bsa_last_error": (ctypes.c_char_p, []),
    "bsa_version": (ctypes.c_int32, []),
}

_lib = None


def lib():
    """Loads the library once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libbsa_b200.so not found at %s: run "
                               "`python fused-block-sparse-attention_b200/build.py`" % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SYMBOLS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(st):
    if st != OK:
        msg = lib().bsa_last_error().decode()
        if st in (ERR_SHAPE, ERR_ARG):
            raise BsaShapeError(st, msg)
        raise BsaError(st, msg)


# ---------------------------------------------------------------- helpers
def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("bsa kernels run on CUDA tensors only (got a %s tensor); "
                               "there is no CPU path" % t.device)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dtype(t):
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise BsaError(ERR_DTYPE, "unsupported dtype %s" % t.dtype)


def _view4(t):
    """bsa_view of a (B,H,L,D) tensor (last dim must be unit-stride)."""
    assert t.stride(-1) == 1
    return View(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _tma_ok(t):
    es = t.element_size()
    return (t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and
            all((s * es) % 16 == 0 for s in t.stride()[:-1]))


def _prep(t):
    """Makes a (B,H,L,D) operand acceptable to the kernels (copies only if needed)."""
    if t.stride(-1) != 1 or (t.dtype != torch.float32 and not _tma_ok(t)):
        t = t.contiguous()
    return t


_status = {}


def status_tensor(device):
    """The persistent device status word of `device` (int32, cleared by check_status)."""
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    if key not in _status:
        _status[key] = torch.zeros(1, dtype=torch.int32, device="cuda:%d" % key)
    return _status[key]


def check_status(device=None):
    """Synchronises, decodes and clears the device status word; raises on error bits."""
    st = status_tensor(device if device is not None else torch.cuda.current_device())
    w = int(st.item())
    st.zero_()
    if w:
        code = lib().bsa_status_decode(w)
        raise BsaError(code, "device status word 0x%x" % w)


def _sel_fields(a, sel, B, Hkv, nblk):
    """Fills sel / sel strides.  sel: None (identity), (B,nblk,kk) shared over heads,
    or (B,Hs,nblk,kk) with Hs in (1, Hkv).  Returns (sel tensor kept alive, kk)."""
    if sel is None:
        a.sel = None
        return None, nblk
    if sel.dtype != torch.int32 or sel.stride(-1) != 1:
        sel = sel.to(torch.int32).contiguous()
    if sel.dim() == 3:
        if sel.shape[0] != B or sel.shape[1] != nblk:
            raise BsaShapeError(ERR_SHAPE, "sel must be (B, nblk, kk); got %s" % (tuple(sel.shape),))
        a.sel, a.sel_sb, a.sel_sh, a.sel_sn = sel.data_ptr(), sel.stride(0), 0, sel.stride(1)
    elif sel.dim() == 4:
        if sel.shape[0] != B or sel.shape[1] not in (1, Hkv) or sel.shape[2] != nblk:
            raise BsaShapeError(ERR_SHAPE, "sel must be (B, Hkv, nblk, kk); got %s" % (tuple(sel.shape),))
        a.sel, a.sel_sb, a.sel_sn = sel.data_ptr(), sel.stride(0), sel.stride(2)
        a.sel_sh = sel.stride(1) if sel.shape[1] > 1 else 0
    else:
        raise BsaShapeError(ERR_SHAPE, "sel must be 3-D or 4-D")
    return sel, sel.shape[-1]


def _gate_fields(a, gate, sel):
    gate = gate.to(torch.float32)
    if gate.stride(-1) != 1:
        gate = gate.contiguous()
    if sel is None or gate.shape != sel.shape:
        raise BsaShapeError(ERR_SHAPE, "gate must have the shape of sel")
    if gate.dim() == 3:
        a.gate, a.gate_sb, a.gate_sh, a.gate_sn = gate.data_ptr(), gate.stride(0), 0, gate.stride(1)
    else:
        a.gate, a.gate_sb, a.gate_sn = gate.data_ptr(), gate.stride(0), gate.stride(2)
        a.gate_sh = gate.stride(1) if gate.shape[1] > 1 else 0
    return gate


def _base_args(q, k, v, bs, mask_mode, causal, scale, sel, gate, q_blk0=None):
    """q_blk0 (query-block sharding): q holds the query rows starting at block
    q_blk0 of the sequence whose keys k, v hold; sel/gate rows cover q's blocks."""
    _need_cuda(q, k, v, sel, gate)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise BsaShapeError(ERR_SHAPE, "q, k, v must be (B, H, L, D)")
    if not (q.dtype == k.dtype == v.dtype):
        raise BsaError(ERR_DTYPE, "q, k, v must share a dtype")
    B, Hq, Lq, D = q.shape
    Hkv, L = k.shape[1], k.shape[2]
    if q_blk0 is None and Lq != L:
        raise BsaShapeError(ERR_SHAPE, "q and k lengths differ; pass q_blk0 for a query shard")
    nblk = (L + bs - 1) // bs
    nq = (Lq + bs - 1) // bs
    a = AttnArgs()
    a.dtype = _dtype(q)
    a.B, a.Hq, a.Hkv, a.L, a.D, a.bs, a.nblk = B, Hq, Hkv, L, D, bs, nblk
    if q_blk0 is not None:
        a.q_blk0, a.Lq = int(q_blk0), Lq
    a.nq = nq
    a.mask_mode = mask_mode
    a.causal = 1 if causal else 0
    a.scale = float(D ** -0.5 if scale is None else scale)
    keep = []
    s, a.kk = _sel_fields(a, sel, B, Hkv, nq)
    keep.append(s)
    if gate is not None:
        keep.append(_gate_fields(a, gate, s))
    a.status = status_tensor(q.device).data_ptr()
    return a, keep


def attn_fwd(q, k, v, sel, gate=None, *, bs, causal, mask_mode=MASK_SLOT, scale=None,
             out=None, out_gate=None, want_lse=True, q_blk0=None, rope=None):
    """Block-sparse attention forward (bsa_attn_fwd).  Returns (o, lse or None).
    `out` may be a strided (B,Hq,L,D) view (e.g. a transpose of (B,L,Hq,D)).
    q_blk0: q is the query shard starting at that block (k, v: the whole sequence).
    rope=(cos, sin): rotate q inside the kernel (k must be rotated already)."""
    q, k, v = _prep(q), _prep(k), _prep(v)
    a, keep = _base_args(q, k, v, bs, mask_mode, causal, scale, sel, gate, q_blk0)
    keep_rope = _set_rope(a, q, rope) if rope is not None else None
    a.q, a.k, a.v = _view4(q), _view4(k), _view4(v)
    o = torch.empty_like(q, memory_format=torch.contiguous_format) if out is None else out
    a.o = _view4(o)
    if out_gate is not None:
        out_gate = _prep(out_gate)
        a.out_gate = _view4(out_gate)
    lse = None
    if want_lse:
        lse = torch.empty(a.B, a.Hq, a.nq * a.bs, dtype=torch.float32, device=q.device)
        a.lse = lse.data_ptr()
    _check(lib().bsa_attn_fwd(ctypes.byref(a), _stream()))
    return o, lse


def attn_bwd(q, k, v, o, do, sel, lse, gate=None, *, bs, causal, mask_mode=MASK_SLOT,
             scale=None, want_dgate=False, q_blk0=None):
    """Block-sparse attention backward (bsa_attn_bwd).  Returns (dq, dk, dv, dgate or None);
    dgate is per query head, (B, Hq, nq, kk) fp32.  With q_blk0 (a query shard) dk, dv
    are this shard's contributions over the whole sequence."""
    q, k, v, o, do = _prep(q), _prep(k), _prep(v), _prep(o), _prep(do)
    a, keep = _base_args(q, k, v, bs, mask_mode, causal, scale, sel, gate, q_blk0)
    a.q, a.k, a.v, a.o, a.dout = _view4(q), _view4(k), _view4(v), _view4(o), _view4(do)
    cf = torch.contiguous_format
    dq = torch.empty_like(q, memory_format=cf)
    dk = torch.empty_like(k, memory_format=cf)
    dv = torch.empty_like(v, memory_format=cf)
    a.dq, a.dk, a.dv = _view4(dq), _view4(dk), _view4(dv)
    a.lse = lse.data_ptr()
    dgate = None
    if want_dgate:
        dgate = torch.empty(a.B, a.Hq, a.nq, a.kk, dtype=torch.float32, device=q.device)
        a.dgate = dgate.data_ptr()
    L = lib()
    nbytes = L.bsa_attn_bwd_workspace(ctypes.byref(a))
    if nbytes == 0:   # validation failed: the call reports why
        _check(L.bsa_attn_bwd(ctypes.byref(a), None, 0, _stream()))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    _check(L.bsa_attn_bwd(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), nbytes, _stream()))
    return dq, dk, dv, dgate


def _rope_tables(x, rope):
    """(cos, sin) of (L, rot) or (B, L, rot) -> contiguous (B|1, L, rot) in x's dtype."""
    cos, sin = rope
    if cos.dim() == 2:
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    return cos.to(x.dtype).contiguous(), sin.to(x.dtype).contiguous()


def _set_rope(a, x, rope):
    cos, sin = _rope_tables(x, rope)
    a.rope_cos, a.rope_sin = cos.data_ptr(), sin.data_ptr()
    a.rope_sb = cos.stride(0) if cos.shape[0] > 1 else 0
    a.rope_sl = cos.stride(1)
    a.rope_rot = cos.shape[-1]
    return cos, sin


def pool(x, bs, *, grp=1, mean=True, vmin=False, vmax=False, rope=None):
    """Block pooling (bsa_pool) of a (B,H,L,D) tensor -> fp32 (B,H/grp,nblk,D) tensors.
    rope=(cos, sin): pool the partially rotated rows (bsa_rope's arithmetic) instead."""
    _need_cuda(x)
    if not _tma_ok(x):
        x = x.contiguous()
    B, H, L, D = x.shape
    nblk = (L + bs - 1) // bs
    a = PoolArgs()
    a.dtype = _dtype(x)
    a.B, a.H, a.L, a.D, a.bs, a.nblk, a.grp = B, H, L, D, bs, nblk, grp
    a.x = _view4(x)
    keep = _set_rope(a, x, rope) if rope is not None else None
    outs = []
    for flag, name in ((mean, "mean"), (vmin, "vmin"), (vmax, "vmax")):
        if flag:
            t = torch.empty(B, H // grp, nblk, D, dtype=torch.float32, device=x.device)
            setattr(a, name, t.data_ptr())
            outs.append(t)
    a.status = status_tensor(x.device).data_ptr()
    _check(lib().bsa_pool(ctypes.byref(a), _stream()))
    return outs


def select(a_sum, b1, b2=None, *, kind=SCORE_DOT, layout=SEL_SSA, causal=True, topk=8,
           sink=False, want_score=False, want_gate=False, q_blk0=None):
    """Fused scoring + top-k (bsa_select).  a_sum, b1, b2: fp32 (..., nblk, dim); leading
    dims are flattened into G groups.  Returns (sel int32 (..., nq, W), score, gate).
    q_blk0: a_sum holds the nq query blocks starting there (a query shard)."""
    _need_cuda(a_sum, b1, b2)
    lead = a_sum.shape[:-2]
    nq, dim = a_sum.shape[-2:]
    nblk = b1.shape[-2]
    if q_blk0 is None and nq != nblk:
        raise BsaShapeError(ERR_SHAPE, "select: query and key block counts differ; pass q_blk0")
    A = a_sum.reshape(-1, nq, dim).float().contiguous()
    B1 = b1.reshape(-1, nblk, dim).float().contiguous()
    B2 = b2.reshape(-1, nblk, dim).float().contiguous() if b2 is not None else None
    s = SelectArgs()
    s.G, s.nblk, s.dim = A.shape[0], nblk, dim
    if q_blk0 is not None:
        s.q_blk0, s.nq = int(q_blk0), nq
    s.score_kind, s.layout, s.causal, s.topk, s.sink = kind, layout, 1 if causal else 0, topk, \
        1 if sink else 0
    s.a, s.b1 = A.data_ptr(), B1.data_ptr()
    s.b2 = B2.data_ptr() if B2 is not None else None
    L = lib()
    W = L.bsa_select_width(ctypes.byref(s))
    sel = torch.empty(*lead, nq, W, dtype=torch.int32, device=a_sum.device)
    score = gate = None
    if want_score:
        score = torch.empty(*lead, nq, W, dtype=torch.float32, device=a_sum.device)
        s.score_out = score.data_ptr()
    if want_gate:
        gate = torch.empty(*lead, nq, W, dtype=torch.float32, device=a_sum.device)
        s.gate_out = gate.data_ptr()
    s.sel = sel.data_ptr()
    s.status = status_tensor(a_sum.device).data_ptr()
    _check(L.bsa_select(ctypes.byref(s), _stream()))
    return sel, score, gate


def select_lsh(a_sum, b_sum, planes, *, hash_kind=HASH_SIGN, cap=16, causal=True, topk=16,
               scale=1.0, want_score=False, want_gate=False):
    """LSH candidate selection (bsa_select_lsh).  a_sum, b_sum: fp32 (..., nblk, dim) raw
    block summaries (normalised inside); planes: (dim, n_rounds, n_planes).  Returns
    (sel int32 (..., nblk, W), score, gate) in the SSA layout (own block first)."""
    _need_cuda(a_sum, b_sum, planes)
    lead = a_sum.shape[:-2]
    nblk, dim = a_sum.shape[-2:]
    A = a_sum.reshape(-1, nblk, dim).float().contiguous()
    Bk = b_sum.reshape(-1, nblk, dim).float().contiguous()
    R = planes.float().contiguous()
    if R.dim() != 3 or R.shape[0] != dim:
        raise BsaShapeError(ERR_SHAPE, "select_lsh: planes must be (dim, n_rounds, n_planes)")
    s = LshArgs()
    s.G, s.nblk, s.dim = A.shape[0], nblk, dim
    s.hash_kind, s.n_rounds, s.n_planes, s.cap = hash_kind, R.shape[1], R.shape[2], cap
    s.causal, s.topk, s.scale = 1 if causal else 0, topk, float(scale)
    s.a, s.b, s.planes = A.data_ptr(), Bk.data_ptr(), R.data_ptr()
    L = lib()
    W = L.bsa_select_lsh_width(ctypes.byref(s))
    nws = L.bsa_select_lsh_workspace(ctypes.byref(s))
    if nws == 0:
        _check(L.bsa_select_lsh(ctypes.byref(s), None, 0, _stream()))
    ws = torch.empty(nws, dtype=torch.uint8, device=a_sum.device)
    sel = torch.empty(*lead, nblk, W, dtype=torch.int32, device=a_sum.device)
    score = gate = None
    if want_score:
        score = torch.empty(*lead, nblk, W, dtype=torch.float32, device=a_sum.device)
        s.score_out = score.data_ptr()
    if want_gate:
        gate = torch.empty(*lead, nblk, W, dtype=torch.float32, device=a_sum.device)
        s.gate_out = gate.data_ptr()
    s.sel = sel.data_ptr()
    s.status = status_tensor(a_sum.device).data_ptr()
    _check(L.bsa_select_lsh(ctypes.byref(s), ctypes.c_void_p(ws.data_ptr()), nws, _stream()))
    return sel, score, gate


def decode(q, k, v, sel, gate=None, *, bs, L=None, mask_mode=MASK_TOKEN, scale=None, out=None):
    """Decode step (bsa_decode): q (B, Hq, T, D) are the tokens at positions L-T .. L-1
    (all in the last block); k, v (B, Hkv, >= L, D) the cache; sel int32 (B, Hkv, kk) or
    (B, kk) block ids of this step; gate optional fp32 like sel.  Returns o (B, Hq, T, D)."""
    _need_cuda(q, k, v, sel, gate)
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    L = k.shape[2] if L is None else int(L)
    if sel.dtype != torch.int32 or sel.stride(-1) != 1:
        sel = sel.to(torch.int32).contiguous()
    a = DecodeArgs()
    a.dtype = _dtype(q)
    a.B, a.Hq, a.Hkv, a.L, a.D, a.bs, a.T, a.kk = B, Hq, Hkv, L, D, bs, T, sel.shape[-1]
    a.mask_mode = mask_mode
    a.scale = float(D ** -0.5 if scale is None else scale)
    if k.stride(-1) != 1:
        k = k.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()
    if q.stride(-1) != 1:
        q = q.contiguous()
    o = torch.empty_like(q, memory_format=torch.contiguous_format) if out is None else out
    a.q, a.k, a.v, a.o = _view4(q), _view4(k), _view4(v), _view4(o)
    if sel.dim() == 2:
        a.sel, a.sel_sb, a.sel_sh = sel.data_ptr(), sel.stride(0), 0
    elif sel.dim() == 3 and sel.shape[1] in (1, Hkv):
        a.sel, a.sel_sb = sel.data_ptr(), sel.stride(0)
        a.sel_sh = sel.stride(1) if sel.shape[1] > 1 else 0
    else:
        raise BsaShapeError(ERR_SHAPE, "decode: sel must be (B, kk) or (B, Hkv, kk)")
    if gate is not None:
        gate = gate.to(torch.float32).contiguous()
        if gate.shape != sel.shape:
            raise BsaShapeError(ERR_SHAPE, "decode: gate must have the shape of sel")
        a.gate, a.gate_sb = gate.data_ptr(), gate.stride(0)
        a.gate_sh = gate.stride(1) if gate.dim() == 3 and gate.shape[1] > 1 else 0
    a.status = status_tensor(q.device).data_ptr()
    L_ = lib()
    nbytes = L_.bsa_decode_workspace(ctypes.byref(a))
    if nbytes == 0:
        _check(L_.bsa_decode(ctypes.byref(a), None, 0, _stream()))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    _check(L_.bsa_decode(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), nbytes, _stream()))
    return o


def select_scores(score, *, topk, sink=True):
    """_finish top-k of a score matrix (bsa_select_scores).  score: (..., nblk, nblk) ->
    int32 (..., nblk, min(topk, nblk) + 1 + sink), ascending."""
    _need_cuda(score)
    lead = score.shape[:-2]
    nblk = score.shape[-1]
    S = score.reshape(-1, nblk, nblk).float()
    if S.stride(-1) != 1:
        S = S.contiguous()
    a = ScoresArgs()
    a.G, a.nblk, a.topk, a.sink = S.shape[0], nblk, topk, 1 if sink else 0
    a.score, a.score_sg, a.score_si = S.data_ptr(), S.stride(0), S.stride(1)
    W = lib().bsa_select_scores_width(ctypes.byref(a))
    sel = torch.empty(*lead, nblk, W, dtype=torch.int32, device=score.device)
    a.sel = sel.data_ptr()
    a.status = status_tensor(score.device).data_ptr()
    _check(lib().bsa_select_scores(ctypes.byref(a), _stream()))
    return sel


def select_qmax(qtok, kmax, kmin, *, topk, sink=True, cand=None):
    """Max-over-tokens Quest selection (bsa_select_qmax).  qtok: (..., nblk, bs, dim)
    fp32; kmax/kmin: (..., nblk, dim); cand: optional int32 (..., nblk, M).
    Returns int32 (..., nblk, min(topk, nblk) + 1 + sink), ascending."""
    _need_cuda(qtok, kmax, kmin, cand)
    lead = qtok.shape[:-3]
    nblk, bs, dim = qtok.shape[-3:]
    Q = qtok.reshape(-1, nblk, bs, dim).float().contiguous()
    KX = kmax.reshape(-1, nblk, dim).float().contiguous()
    KN = kmin.reshape(-1, nblk, dim).float().contiguous()
    a = QmaxArgs()
    a.G, a.nblk, a.bs, a.dim, a.topk, a.sink = Q.shape[0], nblk, bs, dim, topk, 1 if sink else 0
    a.qtok, a.kmax, a.kmin = Q.data_ptr(), KX.data_ptr(), KN.data_ptr()
    C = None
    if cand is not None:
        C = cand.reshape(-1, nblk, cand.shape[-1]).to(torch.int32).contiguous()
        a.cand, a.M = C.data_ptr(), C.shape[-1]
    s = ScoresArgs()
    s.nblk, s.topk, s.sink = nblk, topk, a.sink
    W = lib().bsa_select_scores_width(ctypes.byref(s))
    sel = torch.empty(*lead, nblk, W, dtype=torch.int32, device=qtok.device)
    a.sel = sel.data_ptr()
    a.status = status_tensor(qtok.device).data_ptr()
    _check(lib().bsa_select_qmax(ctypes.byref(a), _stream()))
    return sel


def sel_csr(sel, *, bs, L, causal, mask_mode=MASK_SLOT):
    """CSR transpose of a selection (bsa_sel_csr) -> (row_ptr, col) int32 tensors."""
    _need_cuda(sel)
    c = CsrArgs()
    sel = sel.to(torch.int32).contiguous()
    if sel.dim() == 3:
        c.B, c.Hs = sel.shape[0], 1
        c.sel_sb, c.sel_sh, c.sel_sn = sel.stride(0), 0, sel.stride(1)
    else:
        c.B, c.Hs = sel.shape[0], sel.shape[1]
        c.sel_sb, c.sel_sh, c.sel_sn = sel.stride(0), sel.stride(1), sel.stride(2)
    c.nblk, c.kk = sel.shape[-2], sel.shape[-1]
    c.bs, c.L, c.mask_mode, c.causal = bs, L, mask_mode, 1 if causal else 0
    c.sel = sel.data_ptr()
    nb = c.B * c.Hs * c.nblk
    row_ptr = torch.empty(nb + 1, dtype=torch.int32, device=sel.device)
    col = torch.empty(max(1, nb * c.kk), dtype=torch.int32, device=sel.device)
    c.row_ptr, c.col = row_ptr.data_ptr(), col.data_ptr()
    c.status = status_tensor(sel.device).data_ptr()
    Lb = lib()
    nbytes = Lb.bsa_csr_workspace(ctypes.byref(c))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=sel.device)
    _check(Lb.bsa_sel_csr(ctypes.byref(c), ctypes.c_void_p(ws.data_ptr()), nbytes, _stream()))
    return row_ptr, col


def centroid_route(key_cent, top_c, *, C, cap, q_blk=None, k_blk=None, rk=None):
    """CentroidSSA bucket routing (bsa_centroid_route).  key_cent (B, nblk) and top_c
    (B, nblk, cpq) integer centroid ids; optional refine with fp32 q_blk / k_blk
    (B, nblk, dim) keeping rk candidates.  Returns int32 (B, nblk, 1 + m): the own
    block, then the candidates (-1 = empty)."""
    _need_cuda(key_cent, top_c)
    kc = key_cent.to(torch.int32).contiguous()
    tc = top_c.to(torch.int32).contiguous()
    B, nblk = kc.shape
    a = CentroidArgs()
    a.B, a.nblk, a.C, a.cpq, a.cap = B, nblk, C, tc.shape[-1], cap
    a.key_cent, a.top_c = kc.data_ptr(), tc.data_ptr()
    keep = []
    if q_blk is not None and rk is not None:
        qb = q_blk.float().contiguous()
        kb = k_blk.float().contiguous()
        keep += [qb, kb]
        a.q_blk, a.k_blk, a.dim, a.rk = qb.data_ptr(), kb.data_ptr(), qb.shape[-1], rk
    L = lib()
    W = L.bsa_centroid_width(ctypes.byref(a))
    sel = torch.empty(B, nblk, W, dtype=torch.int32, device=kc.device)
    a.sel = sel.data_ptr()
    _check(L.bsa_centroid_route(ctypes.byref(a), _stream()))
    return sel


def rope(x, cos, sin, *, out=None):
    """Partial rotary embedding with transformers' rounding (bsa_rope).
    x: (B,H,L,D); cos/sin: (B,L,rot) or (L,rot) in x's dtype."""
    _need_cuda(x, cos, sin)
    if cos.dim() == 2:
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    cos = cos.to(x.dtype).contiguous()
    sin = sin.to(x.dtype).contiguous()
    if x.stride(-1) != 1:
        x = x.contiguous()
    B, H, L, D = x.shape
    a = RopeArgs()
    a.dtype = _dtype(x)
    a.B, a.H, a.L, a.D, a.rot = B, H, L, D, cos.shape[-1]
    a.x = _view4(x)
    y = torch.empty_like(x, memory_format=torch.contiguous_format) if out is None else out
    a.y = _view4(y)
    a.cos, a.sin = cos.data_ptr(), sin.data_ptr()
    a.cs_sb = cos.stride(0) if cos.shape[0] > 1 else 0
    a.cs_sl = cos.stride(1)
    _check(lib().bsa_rope(ctypes.byref(a), _stream()))
    return y
