"""Drop-in for the reference's `triton_kernel` module (src/triton_kernel.py) on
sm_100a: same entry points and argument meaning, backed by libbsa_b200.so.

  bsattn_forward(q, k, v, sel, gate_bias=None, causal=False) -> o      (:184-207)
  bsattn_backward(q, k, v, sel, o, do, gate_bias=None, causal=False)   (:210-234)
      (+ keyword lse= from bsattn_forward_lse: skips the recomputing forward)
  BSAttnFunction.apply(q, k, v, sel, gate_bias, causal)                (:237-254)
  bsattn(q, k, v, sel, gate_bias=None, causal=False)                   (:257-259)

Layouts as in the reference: q, k, v (B, H, L, dh); sel (B, nblk, kk) int with
sel[:, :, 0] the own block, shared over heads; gate (B, nblk, kk) fp32.  As an
extension sel/gate may also be (B, H, nblk, kk) per head.  Block size is
L // nblk (L must be a multiple of nblk, as the reference asserts).  Inputs
need not be contiguous: strided views are read in place by TMA.

Masking (causal): slot 0 is triangular, slot j>0 is dropped when its block id
is >= the query block; non-causal: nothing is masked.  The backward returns no
gradient for gate_bias, like the reference; `bsattn(..., gate_grad=True)`
returns it (the gather path's semantics, src/ssa_model.py:71-74).
"""
import torch

import _bsa

__all__ = ["bsattn_forward", "bsattn_backward", "BSAttnFunction", "bsattn", "bsattn_forward_lse"]


def _geometry(q, sel):
    L = q.shape[2]
    nblk = sel.shape[-2]
    if L % nblk:
        raise ValueError("L (%d) must be a multiple of nblk (%d)" % (L, nblk))
    return L // nblk


def bsattn_forward(q, k, v, sel, gate_bias=None, causal=False):
    """O = block-sparse attention of q over the selected K/V blocks."""
    bs = _geometry(q, sel)
    o, _ = _bsa.attn_fwd(q, k, v, sel, gate_bias, bs=bs, causal=causal, want_lse=False)
    return o


def _forward_lse(q, k, v, sel, gate_bias, causal):
    bs = _geometry(q, sel)
    return _bsa.attn_fwd(q, k, v, sel, gate_bias, bs=bs, causal=causal, want_lse=True)


def bsattn_backward(q, k, v, sel, o, do, gate_bias=None, causal=False, *, lse=None):
    """(dQ, dK, dV) of the block-sparse attention.

    Without `lse` the row log-sum-exp is recomputed by a forward pass, as the
    reference recomputes it (src/triton_kernel.py:106-129), and `o` is not read
    (the reference ignores it too; the recomputed output keeps rowsum(dO * O)
    consistent with the recomputed lse).  With `lse` (an extension: the fp32
    (B, H, L) tensor that `bsattn_forward_lse` returns beside `o`) the backward
    uses the given `o` and `lse` and runs no forward."""
    bs = _geometry(q, sel)
    if lse is None:
        o, lse = _forward_lse(q, k, v, sel, gate_bias, causal)
    dq, dk, dv, _ = _bsa.attn_bwd(q, k, v, o, do, sel, lse, gate_bias, bs=bs, causal=causal)
    return dq, dk, dv


def bsattn_forward_lse(q, k, v, sel, gate_bias=None, causal=False):
    """(o, lse): the forward output and its fp32 row log-sum-exp (log2 domain,
    scale folded in), for callers that run bsattn_backward(..., lse=lse) later."""
    return _forward_lse(q, k, v, sel, gate_bias, causal)


class BSAttnFunction(torch.autograd.Function):
    """Autograd wrapper; gradients for q, k, v (and gate_bias when gate_grad)."""

    @staticmethod
    def forward(ctx, q, k, v, sel, gate_bias, causal, gate_grad=False, mask_mode=_bsa.MASK_SLOT):
        bs = _geometry(q, sel)
        o, lse = _bsa.attn_fwd(q, k, v, sel, gate_bias, bs=bs, causal=causal, mask_mode=mask_mode,
                               want_lse=True)
        ctx.save_for_backward(q, k, v, o, sel, lse,
                              gate_bias if gate_bias is not None else torch.empty(0, device=q.device))
        ctx.has_gate = gate_bias is not None
        ctx.causal = causal
        ctx.mask_mode = mask_mode
        ctx.gate_grad = bool(gate_grad) and gate_bias is not None
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, sel, lse, gate = ctx.saved_tensors
        gate = gate if ctx.has_gate else None
        bs = _geometry(q, sel)
        dq, dk, dv, dg = _bsa.attn_bwd(q, k, v, o, do, sel, lse, gate, bs=bs, causal=ctx.causal,
                                       mask_mode=ctx.mask_mode, want_dgate=ctx.gate_grad)
        dgate = None
        if ctx.gate_grad:
            # per-query-head sums -> the gate's own layout
            if gate.dim() == 3:
                dgate = dg.sum(1)
            else:
                dgate = dg.view(dg.shape[0], gate.shape[1], -1, *dg.shape[2:]).sum(2)
            dgate = dgate.to(gate.dtype)
        return dq, dk, dv, None, dgate, None, None, None


def bsattn(q, k, v, sel, gate_bias=None, causal=False, gate_grad=False, mask_mode=_bsa.MASK_SLOT):
    """Autograd-aware block-sparse attention. Use this for training.  mask_mode
    MASK_TOKEN (an extension) also drops repeated block ids within a row."""
    return BSAttnFunction.apply(q, k, v, sel, gate_bias, causal, gate_grad, mask_mode)
