"""Drop-in for the reference's GQA block-sparse core (src/qwen_blocksparse.py)
on sm_100a.

  blocksparse_forward(q, k, v, *, selector, topk, bs, causal=True, scale=None, q_chunk=4)
  SelectMax(topk, bs, sink=True).select(q, k)     Quest min/max bound (:102-121)
  SelectAll(bs).select(q, k)                       all blocks (:155-165)
  qwen_attention(...)                              the Qwen-style variant: partial RoPE,
                                                   selection, GQA attention and the sigmoid
                                                   output gate in one call (src/patch_qwen.py:41-55)

q: (B, Hq, L, d), k/v: (B, Hkv, L, d), Hq % Hkv == 0; query head h reads KV head
h // (Hq/Hkv).  The selected-block attention masks keys after the query position,
keys past L and repeated block ids, as the reference's gather path does
(:67-72); q_chunk is accepted for signature parity and has no effect (there is
no materialised gather to bound).
"""
import torch

import _bsa
from selection import select_quest

__all__ = ["blocksparse_forward", "SelectMax", "SelectAll", "qwen_attention", "rope_cos_sin"]


class SelectMax:
    """Training-free, RoPE-tolerant Quest-style selector (device kernels)."""

    def __init__(self, topk, bs, sink=True):
        self.topk, self.bs, self.sink = topk, bs, sink

    @torch.no_grad()
    def select(self, q, k):
        return select_quest(q, k, bs=self.bs, topk=self.topk, sink=self.sink).long()


class SelectAll:
    """All blocks; blocksparse_forward runs it without materialising the index."""

    def __init__(self, bs):
        self.bs = bs

    @torch.no_grad()
    def select(self, q, k):
        B, Hq, L, d = q.shape
        nblk = (L + self.bs - 1) // self.bs
        return torch.arange(nblk, device=q.device).view(1, 1, 1, nblk).expand(
            B, k.shape[1], nblk, nblk).contiguous()


def _attend(q, k, v, sel, bs, causal, scale):
    o, _ = _bsa.attn_fwd(q, k, v, sel, None, bs=bs, causal=causal, mask_mode=_bsa.MASK_TOKEN,
                         scale=scale, want_lse=False)
    return o


def blocksparse_forward(q, k, v, *, selector, topk, bs, causal=True, scale=None, q_chunk=4):
    B, Hq, L, d = q.shape
    if Hq % k.shape[1]:
        raise ValueError("Hq must be a multiple of Hkv")
    scale = d ** -0.5 if scale is None else scale
    nblk = (L + bs - 1) // bs
    if (selector is None and topk >= nblk) or isinstance(selector, SelectAll):
        # all blocks: dense attention (causal as requested on the fast path, :37-41;
        # the gather path with SelectAll is always causal, :72)
        return _attend(q, k, v, None, bs, causal if selector is None else True, scale)
    idx = selector.select(q, k)
    if idx.dim() != 4 or idx.shape[0] != B or idx.shape[2] != nblk:
        raise ValueError("selector must return (B, Hkv, nblk, kk)")
    return _attend(q, k, v, idx.to(torch.int32), bs, True, scale)


def rope_cos_sin(L, rot, theta, dtype, device):
    """Default rotary tables for text positions 0..L-1 (fp32 math, cast to dtype), as
    transformers builds them for Qwen3.5-MoE with partial_rotary_factor = rot / head_dim."""
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.int64, device=device).float() / rot))
    f = torch.outer(torch.arange(L, dtype=torch.float32, device=device), inv)
    emb = torch.cat((f, f), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def qwen_attention(q, k, v, cos, sin, gate, *, selector, topk, bs, scale=None):
    """Qwen-style attention core after the q/k norms (src/patch_qwen.py:44-55).

    q: (B, Hq, L, D) pre-RoPE; k: (B, Hkv, L, D) pre-RoPE; v: (B, Hkv, L, D);
    cos/sin: (L, rot) or (B, L, rot); gate: (B, L, Hq*D) output gate.
    Returns (B, L, Hq*D) = attention(rope(q), rope(k), v) * sigmoid(gate), written
    directly in that layout by the attention epilogue."""
    B, Hq, L, D = q.shape
    qr = _bsa.rope(q, cos, sin)
    kr = _bsa.rope(k, cos, sin)
    out = torch.empty(B, L, Hq, D, dtype=q.dtype, device=q.device)
    og = gate.reshape(B, L, Hq, D).transpose(1, 2)
    nblk = (L + bs - 1) // bs
    scale = D ** -0.5 if scale is None else scale
    if (selector is None and topk >= nblk) or isinstance(selector, SelectAll):
        sel = None
    else:
        sel = selector.select(qr, kr).to(torch.int32)
    _bsa.attn_fwd(qr, kr, v, sel, None, bs=bs, causal=True, mask_mode=_bsa.MASK_TOKEN, scale=scale,
                  out=out.transpose(1, 2), out_gate=og, want_lse=False)
    return out.view(B, L, Hq * D)
