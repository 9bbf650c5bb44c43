"""Drop-in for the reference's BlockSparseSSA module (src/ssa_model.py:93-201)
on sm_100a.

BlockSparseSSA(d, h, block=64, topk=8, sel_dim=32, gate=False, causal=False,
               use_triton=False).forward(x, needle_pos=None)
LSHBucketSSA(d, h, block=32, topk=4, sel_dim=32, n_rounds=4, n_buckets=8, cap=8,
             gate=False, causal=False, scale=None, ...).forward(x, needle_pos=None)
                                                        (src/ssa_model.py:336-513)
CentroidSSA(d, h, block=64, topk=8, sel_dim=32, n_centroids=16, cpq=2, cap=4,
            gate=False, refine_topk=None).forward(x, needle_pos=None)
                                                        (src/ssa_model.py:204-333)

Same parameters (qkv, o, sel_q, sel_k MLP selectors) and outputs.  Selection
runs on device: the selector features are block-pooled (mean for queries,
mean and max for keys) and scored max(sq.sk_mean, sq.sk_max) by the fused
scoring/top-k kernel, which keeps the own block first and the top-k content
blocks after it (ties to the lower block id).  Attention runs on the fused
block-sparse kernels for both settings of use_triton:
  use_triton=True   the gate gets no gradient (reference Triton path, :185-192)
  use_triton=False  the gate is differentiated (reference gather path, :194,
                    :71-74), so the selector MLPs learn through it.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

import _bsa
from triton_kernel import bsattn

__all__ = ["BlockSparseSSA", "LSHBucketSSA", "CentroidSSA", "centroid_select"]


def _mlp_sel(d, sel_dim):
    return nn.Sequential(nn.Linear(d, sel_dim), nn.GELU(), nn.Linear(sel_dim, sel_dim))


class BlockSparseSSA(nn.Module):
    """Content-dependent block-sparse attention with device-side selection."""

    def __init__(self, d, h, block=64, topk=8, sel_dim=32, gate=False, causal=False,
                 use_triton=False):
        super().__init__()
        self.h, self.dh = h, d // h
        self.block, self.topk = block, topk
        self.qkv = nn.Linear(d, 3 * d)
        self.o = nn.Linear(d, d)
        self.sel_q = _mlp_sel(d, sel_dim)
        self.sel_k = _mlp_sel(d, sel_dim)
        self.sel_dim = sel_dim
        self.gate = gate
        self.causal = causal
        self.use_triton = use_triton
        self.distill = False
        self.last_hit = None
        self.last_block_logits = None
        self.distill_logits = None
        self.distill_target = None

    def forward(self, x, needle_pos=None):
        B, L, D = x.shape
        Bs = self.block
        pad = (Bs - L % Bs) % Bs
        if pad:
            x = F.pad(x, (0, 0, 0, pad))
        Lp = L + pad
        nblk = Lp // Bs
        H, dh = self.h, self.dh
        q, k, v = self.qkv(x).chunk(3, -1)
        q = q.view(B, Lp, H, dh).transpose(1, 2)
        k = k.view(B, Lp, H, dh).transpose(1, 2)
        v = v.view(B, Lp, H, dh).transpose(1, 2)

        sqf, skf = self.sel_q(x), self.sel_k(x)                 # (B, Lp, s)
        # exact device selection from block-pooled selector features
        with torch.no_grad():
            (sqp,) = _bsa.pool(sqf.detach().float().unsqueeze(1), Bs)
            skm, skx = _bsa.pool(skf.detach().float().unsqueeze(1), Bs, mean=True, vmax=True)
            sel, _, _ = _bsa.select(sqp, skm, skx, kind=_bsa.SCORE_MAXDOT2, layout=_bsa.SEL_SSA,
                                    causal=self.causal, topk=self.topk)
        sel = sel[:, 0]                                         # (B, nblk, kk) int32

        # differentiable pooled features for the gate and the logged logits
        sq = sqf.view(B, nblk, Bs, self.sel_dim).mean(2)
        skv = skf.view(B, nblk, Bs, self.sel_dim)
        sk_mean, sk_max = skv.mean(2), skv.max(2).values
        self.last_block_logits = torch.maximum(sq[:, -1:] @ sk_mean.transpose(-1, -2),
                                               sq[:, -1:] @ sk_max.transpose(-1, -2))[:, 0]
        if self.distill:
            raw = torch.maximum(sq @ sk_mean.transpose(-1, -2), sq @ sk_max.transpose(-1, -2))
            att = (q @ k.transpose(-1, -2)) * dh ** -0.5
            cm = torch.triu(torch.ones(Lp, Lp, dtype=torch.bool, device=x.device), 1)
            att = att.masked_fill(cm, float("-inf")).softmax(-1)
            am = att.view(B, H, nblk, Bs, nblk, Bs).sum(-1).mean(3)
            self.distill_target = am.mean(1).detach()
            ar = torch.arange(nblk, device=x.device)
            self.distill_logits = raw.masked_fill((ar.view(nblk, 1) < ar.view(1, nblk)).unsqueeze(0), -1e9)

        gate_bias = None
        if self.gate:
            idx = sel.long()
            kk = idx.shape[-1]
            flat = idx.view(B, nblk * kk, 1).expand(-1, -1, self.sel_dim)
            gm = torch.gather(sk_mean, 1, flat).view(B, nblk, kk, self.sel_dim)
            gx = torch.gather(sk_max, 1, flat).view(B, nblk, kk, self.sel_dim)
            raw_sel = torch.maximum((sq.unsqueeze(2) * gm).sum(-1), (sq.unsqueeze(2) * gx).sum(-1))
            gate_bias = F.logsigmoid(raw_sel.float())
            if self.use_triton:
                gate_bias = gate_bias.detach()
        out = bsattn(q, k, v, sel, gate_bias, causal=self.causal,
                     gate_grad=(self.gate and not self.use_triton))
        out = out.reshape(B, H, Lp, dh).transpose(1, 2).reshape(B, Lp, D)[:, :L]
        if needle_pos is not None:
            chosen_last = sel[:, nblk - 1, :].long()
            self.last_hit = (chosen_last == (needle_pos // Bs).unsqueeze(-1)).any(-1).float().mean().item()
        return self.o(out)


class LSHBucketSSA(nn.Module):
    """LSH-bucketed selection + block-sparse attention (reference
    src/ssa_model.py:336-513).  Same parameters (qkv, o, sel_q, sel_k, R).

    Inference branch (dense_select False, the default): the selector features are
    block-pooled on device (mean for queries; max(mean, max) for keys), then
    bsa_select_lsh normalises them, hashes them by the argmax over R's n_buckets
    projections per round, keeps the first `cap` key blocks of every bucket, and
    re-scores the candidates by scale * cosine (top-k, own block first).  Missing
    picks repeat the own block and are dropped by the attention's masks (causal:
    content blocks must precede the query block; non-causal: repeated ids are
    skipped), which is the reference's -inf mask on invalid slots (:480-482).
    dense_select True: all-pairs cosine top-k (:404-414) with the fused
    scoring/top-k kernel.  The learned-hash loss of the training branch
    (learn_hash, :415-435) is not built; last_hash_loss stays None.
    """

    def __init__(self, d, h, block=32, topk=4, sel_dim=32, n_rounds=4, n_buckets=8, cap=8,
                 gate=False, causal=False, scale=None, learn_hash=False, hash_tau=1.0,
                 hash_detach_reps=False):
        super().__init__()
        self.h, self.dh = h, d // h
        self.block, self.topk = block, topk
        self.qkv = nn.Linear(d, 3 * d)
        self.o = nn.Linear(d, d)
        self.sel_q = _mlp_sel(d, sel_dim)
        self.sel_k = _mlp_sel(d, sel_dim)
        self.sel_dim = sel_dim
        self.scale = float(sel_dim ** 0.5) if scale is None else float(scale)
        self.n_rounds, self.n_buckets, self.cap = n_rounds, n_buckets, cap
        self.gate, self.causal = gate, causal
        self.dense_select = False
        self.learn_hash, self.hash_tau = learn_hash, hash_tau
        self.hash_detach_reps = hash_detach_reps
        R0 = torch.randn(sel_dim, n_rounds, n_buckets)
        if learn_hash:
            self.R = nn.Parameter(R0)
        else:
            self.register_buffer("R", R0)
        self.last_hit = None
        self.last_block_logits = None
        self.last_hash_loss = None

    def forward(self, x, needle_pos=None):
        B, L, D = x.shape
        Bs = self.block
        pad = (Bs - L % Bs) % Bs
        if pad:
            x = F.pad(x, (0, 0, 0, pad))
        Lp = L + pad
        nblk = Lp // Bs
        H, dh = self.h, self.dh
        q, k, v = self.qkv(x).chunk(3, -1)
        q = q.view(B, Lp, H, dh).transpose(1, 2)
        k = k.view(B, Lp, H, dh).transpose(1, 2)
        v = v.view(B, Lp, H, dh).transpose(1, 2)

        sqf, skf = self.sel_q(x), self.sel_k(x)
        with torch.no_grad():
            (sqp,) = _bsa.pool(sqf.detach().float().unsqueeze(1), Bs)
            skm, skx = _bsa.pool(skf.detach().float().unsqueeze(1), Bs, mean=True, vmax=True)
            skp = torch.maximum(skm, skx)
            if self.dense_select:
                qn, kn = F.normalize(sqp, dim=-1), F.normalize(skp, dim=-1)
                sel, _, _ = _bsa.select(qn, kn, kind=_bsa.SCORE_DOT, layout=_bsa.SEL_SSA,
                                        causal=self.causal, topk=self.topk)
            else:
                sel, _, _ = _bsa.select_lsh(sqp, skp, self.R.detach(), hash_kind=_bsa.HASH_ARGMAX,
                                            cap=min(self.cap, nblk), causal=self.causal,
                                            topk=self.topk, scale=self.scale)
        sel = sel[:, 0]                                         # (B, nblk, kk) int32

        # differentiable normalised reps for the gate and the logged logits
        sq = F.normalize(sqf.view(B, nblk, Bs, self.sel_dim).mean(2), dim=-1)
        skv = skf.view(B, nblk, Bs, self.sel_dim)
        sk = F.normalize(torch.maximum(skv.mean(2), skv.max(2).values), dim=-1)
        self.last_block_logits = self.scale * torch.bmm(sk, sq[:, nblk - 1:nblk].transpose(-1, -2)).squeeze(-1)

        gate_bias = None
        if self.gate:
            idx = sel.long()
            kk = idx.shape[-1]
            flat = idx.view(B, nblk * kk, 1).expand(-1, -1, self.sel_dim)
            gk = torch.gather(sk, 1, flat).view(B, nblk, kk, self.sel_dim)
            gate_bias = F.logsigmoid(self.scale * (sq.unsqueeze(2) * gk).sum(-1).float())
        mode = _bsa.MASK_SLOT if self.causal else _bsa.MASK_TOKEN
        out = bsattn(q, k, v, sel, gate_bias, causal=self.causal, gate_grad=self.gate,
                     mask_mode=mode)
        out = out.reshape(B, H, Lp, dh).transpose(1, 2).reshape(B, Lp, D)[:, :L]
        if needle_pos is not None:
            chosen_last = sel[:, nblk - 1, :].long()
            self.last_hit = (chosen_last == (needle_pos // Bs).unsqueeze(-1)).any(-1).float().mean().item()
        return self.o(out)


@torch.no_grad()
def centroid_select(sq, sk, cent, *, cpq, cap, refine=None):
    """CentroidSSA's routing (src/ssa_model.py:254-299): key block j -> bucket
    argmax_c sk_j . cent_c (the first `cap` blocks of each bucket by index); query
    block i reads the buckets of its top-`cpq` centroids by sq_i . cent_c, its own
    block dropped from them; optional refine = (q_blk, k_blk, rk): keep the rk
    candidates with the largest q_blk_i . k_blk_j.  sq, sk: (B, nblk, s);
    cent: (C, s).  Returns (sel (B, nblk, 1 + m) int64 with the own block first and
    -1 for empty slots, key_cent (B, nblk), qc (B, nblk, C)).  The centroid scores,
    argmax and top-cpq are O(nblk * C) tensor ops; the buckets, the gather and the
    refine step run in one device kernel (bsa_centroid_route); no nblk x nblk
    tensor exists."""
    C = cent.shape[0]
    nblk = sq.shape[1]
    cpq, cap = min(cpq, C), min(cap, nblk)
    kc = sk @ cent.t()
    qc = sq @ cent.t()
    key_cent = kc.argmax(-1)                                            # (B, nblk)
    top_c = qc.topk(cpq, dim=-1).indices                                # (B, nblk, cpq)
    kw = {}
    if refine is not None:
        q_blk, k_blk, rk = refine
        if rk < cpq * cap:
            kw = dict(q_blk=q_blk, k_blk=k_blk, rk=rk)
    sel = _bsa.centroid_route(key_cent, top_c, C=C, cap=cap, **kw)
    return sel.long(), key_cent, qc


class CentroidSSA(nn.Module):
    """Centroid-routed selection + block-sparse attention (reference
    src/ssa_model.py:204-333); same parameters (qkv, o, sel_q, sel_k, cent).

    The routing tensors are O(nblk * C) (centroid_select); empty slots repeat the
    own block, which the attention skips as a repeated id (TOKEN masks, not
    causal: the reference's CentroidSSA attends without a causal mask and with
    -inf on empty slots, :318-320)."""

    def __init__(self, d, h, block=64, topk=8, sel_dim=32, n_centroids=16, cpq=2, cap=4,
                 gate=False, refine_topk=None):
        super().__init__()
        self.h, self.dh = h, d // h
        self.block, self.topk = block, topk
        self.cpq, self.cap = cpq, cap
        self.qkv = nn.Linear(d, 3 * d)
        self.o = nn.Linear(d, d)
        self.sel_q = _mlp_sel(d, sel_dim)
        self.sel_k = _mlp_sel(d, sel_dim)
        self.sel_dim = sel_dim
        self.cent = nn.Parameter(torch.randn(n_centroids, sel_dim) * (sel_dim ** -0.5))
        self.refine_topk = refine_topk
        self.gate = gate
        self.last_hit = None
        self.last_block_logits = None
        self.align_q = None
        self.align_k = None

    def forward(self, x, needle_pos=None):
        B, L, D = x.shape
        Bs = self.block
        pad = (Bs - L % Bs) % Bs
        if pad:
            x = F.pad(x, (0, 0, 0, pad))
        Lp = L + pad
        nblk = Lp // Bs
        H, dh = self.h, self.dh
        q, k, v = self.qkv(x).chunk(3, -1)
        q = q.view(B, Lp, H, dh).transpose(1, 2)
        k = k.view(B, Lp, H, dh).transpose(1, 2)
        v = v.view(B, Lp, H, dh).transpose(1, 2)
        sq = self.sel_q(x).view(B, nblk, Bs, self.sel_dim).mean(2)
        skv = self.sel_k(x).view(B, nblk, Bs, self.sel_dim)
        sk = torch.maximum(skv.mean(2), skv.max(2).values)
        refine = None
        if self.refine_topk is not None:
            q_blk = q.detach().reshape(B, H, nblk, Bs, dh).mean(3).mean(1)
            k_blk = k.detach().reshape(B, H, nblk, Bs, dh).mean(3).mean(1)
            refine = (q_blk, k_blk, self.refine_topk)
        sel_raw, key_cent, qc_ng = centroid_select(sq.detach(), sk.detach(), self.cent.detach(),
                                                   cpq=self.cpq, cap=self.cap, refine=refine)
        qc = sq @ self.cent.t()
        self.last_block_logits = qc[:, nblk - 1, :].gather(1, key_cent)
        valid = sel_raw >= 0
        own = torch.arange(nblk, device=x.device).view(1, nblk, 1)
        sel = torch.where(valid, sel_raw, own).to(torch.int32)
        gate_bias = None
        if self.gate:
            sel_cent = key_cent.gather(1, sel.long().reshape(B, -1)).reshape(B, nblk, -1)
            gate_bias = F.logsigmoid(torch.gather(qc, 2, sel_cent).float()).masked_fill(~valid, 0.0)
        out = bsattn(q, k, v, sel, gate_bias, causal=False, gate_grad=self.gate,
                     mask_mode=_bsa.MASK_TOKEN)
        out = out.reshape(B, H, Lp, dh).transpose(1, 2).reshape(B, Lp, D)[:, :L]
        if needle_pos is not None:
            chosen_last = sel_raw[:, nblk - 1, :]
            self.last_hit = (chosen_last == (needle_pos // Bs).unsqueeze(-1)).any(-1).float().mean().item()
            self.align_q = qc[:, nblk - 1, :]
            self.align_k_all = sk @ self.cent.t()
        return self.o(out)
