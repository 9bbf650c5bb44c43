"""Drop-in for the reference's GQA block-sparse core (src/qwen_blocksparse.py)
on sm_100a.

  blocksparse_forward(q, k, v, *, selector, topk, bs, causal=True, scale=None, q_chunk=4)
  SelectMax(topk, bs, sink=True).select(q, k)     Quest min/max bound (:102-121)
  SelectAll(bs).select(q, k)                       all blocks (:155-165)
  SelectOracle(topk, bs, sink=True, mass=None)     top-k of a given block mass (:124-137)
  SelectRandom(topk, bs, sink=True, seed=0)        uniform random scores (:140-152)
  SelectLastTok(topk, bs, sink=True)               Quest bound of each block's last token (:250-267)
  SelectMaxQMax(topk, bs, sink=True)               Quest bound maxed over the block's tokens (:221-247)
  SelectTwoStage(topk, bs, sink=True, over=4)      block-mean Quest candidates, max-over-token
                                                   re-score (:270-299)
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

__all__ = ["blocksparse_forward", "SelectMax", "SelectAll", "SelectOracle", "SelectRandom",
           "SelectLastTok", "SelectMaxQMax", "SelectTwoStage", "qwen_attention", "rope_cos_sin"]


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


class SelectOracle:
    """Top-k key blocks by a supplied per-block attention mass (B, Hkv, nblk, nblk)."""

    def __init__(self, topk, bs, sink=True, mass=None):
        self.topk, self.bs, self.sink, self.mass = topk, bs, sink, mass

    @torch.no_grad()
    def select_from_mass(self, mass):
        return _bsa.select_scores(mass, topk=self.topk, sink=self.sink).long()

    @torch.no_grad()
    def select(self, q, k):
        if self.mass is None:
            raise ValueError("SelectOracle needs mass set (per-layer teacher)")
        return self.select_from_mass(self.mass)


class SelectRandom:
    """Random causal blocks (lower-bound baseline): the same uniform draws as the
    reference's generator on the same device, then the device top-k."""

    def __init__(self, topk, bs, sink=True, seed=0):
        self.topk, self.bs, self.sink, self.seed = topk, bs, sink, seed

    @torch.no_grad()
    def select(self, q, k):
        B, Hq, L, d = q.shape
        nblk = (L + self.bs - 1) // self.bs
        g = torch.Generator(device=q.device).manual_seed(self.seed)
        score = torch.rand(B, k.shape[1], nblk, nblk, generator=g, device=q.device)
        return _bsa.select_scores(score, topk=self.topk, sink=self.sink).long()


def _token_summaries(q, k, bs):
    """Group-mean query tokens (B, Hkv, nblk, bs, d) with zero padding rows, and the
    key blocks' min / max (B, Hkv, nblk, d), all fp32."""
    B, Hq, L, d = q.shape
    Hkv = k.shape[1]
    nblk = (L + bs - 1) // bs
    (qt,) = _bsa.pool(q, 1, grp=Hq // Hkv)                       # (B, Hkv, L, d)
    if nblk * bs != L:
        qt = torch.nn.functional.pad(qt, (0, 0, 0, nblk * bs - L))
    kmin, kmax = _bsa.pool(k, bs, mean=False, vmin=True, vmax=True)
    return qt.view(B, Hkv, nblk, bs, d), kmin, kmax


class SelectLastTok:
    """SelectMax scored by each query block's last token (group mean) instead of the
    block mean; a padded last block scores with its (zero) padding row, as the
    reference does."""

    def __init__(self, topk, bs, sink=True):
        self.topk, self.bs, self.sink = topk, bs, sink

    @torch.no_grad()
    def select(self, q, k):
        qt, kmin, kmax = _token_summaries(q, k, self.bs)
        qlast = qt[:, :, :, -1, :].contiguous()
        sel, _, _ = _bsa.select(qlast, kmax, kmin, kind=_bsa.SCORE_QUEST, layout=_bsa.SEL_FINISH,
                                topk=self.topk, sink=self.sink)
        return sel.long()


class SelectMaxQMax:
    """Quest bound maxed over the query block's tokens (group-mean per token)."""

    def __init__(self, topk, bs, sink=True):
        self.topk, self.bs, self.sink = topk, bs, sink

    @torch.no_grad()
    def select(self, q, k):
        qt, kmin, kmax = _token_summaries(q, k, self.bs)
        return _bsa.select_qmax(qt, kmax, kmin, topk=self.topk, sink=self.sink).long()


class SelectTwoStage:
    """Stage 1: block-mean Quest picks over*topk candidates (causal); stage 2: the
    max-over-token Quest bound re-scores them and keeps top-k."""

    def __init__(self, topk, bs, sink=True, over=4):
        self.topk, self.bs, self.sink, self.over = topk, bs, sink, over

    @torch.no_grad()
    def select(self, q, k):
        B, Hq, L, d = q.shape
        nblk = (L + self.bs - 1) // self.bs
        qt, kmin, kmax = _token_summaries(q, k, self.bs)
        (qp,) = _bsa.pool(q, self.bs, grp=Hq // k.shape[1])
        M = min(self.over * self.topk, nblk)
        cand, _, _ = _bsa.select(qp, kmax, kmin, kind=_bsa.SCORE_QUEST, layout=_bsa.SEL_RAW, topk=M)
        return _bsa.select_qmax(qt, kmax, kmin, topk=self.topk, sink=self.sink, cand=cand).long()


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
    directly in that layout by the attention epilogue.

    With SelectMax (or all blocks) and head dim 256 the rotation of q is folded
    into the kernels: the selection pools rope(q) inside its pooling kernel and
    the attention rotates its q tile in shared memory after loading it, so the
    rotated q (the largest tensor here) is never written; k, shared by the query
    heads of its group, is rotated once by bsa_rope."""
    B, Hq, L, D = q.shape
    kr = _bsa.rope(k, cos, sin)
    nblk = (L + bs - 1) // bs
    fold = D == 256 and bs == 128 and q.dtype != torch.float32 and \
        (isinstance(selector, (SelectMax, SelectAll)) or (selector is None and topk >= nblk))
    qr = q if fold else _bsa.rope(q, cos, sin)
    out = torch.empty(B, L, Hq, D, dtype=q.dtype, device=q.device)
    og = gate.reshape(B, L, Hq, D).transpose(1, 2)
    nblk = (L + bs - 1) // bs
    scale = D ** -0.5 if scale is None else scale
    if (selector is None and topk >= nblk) or isinstance(selector, SelectAll):
        sel = None
    elif fold:
        sel = select_quest(q, kr, bs=bs, topk=selector.topk, sink=selector.sink, rope=(cos, sin))
    else:
        sel = selector.select(qr, kr).to(torch.int32)
    _bsa.attn_fwd(qr, kr, v, sel, None, bs=bs, causal=True, mask_mode=_bsa.MASK_TOKEN, scale=scale,
                  out=out.transpose(1, 2), out_gate=og, want_lse=False,
                  rope=(cos, sin) if fold else None)
    return out.view(B, L, Hq * D)
