"""Block-sparse decode over a K/V cache (no counterpart in the reference, which
has no decode path; this is the next consumer of its selection).

    cache = DecodeCache(B, Hkv, max_len, D, bs=128, dtype=torch.bfloat16, device="cuda")
    cache.append(k_new, v_new)                      # (B, Hkv, T, D) each
    sel = cache.select_quest(q_new, topk=32)        # Quest bound, _finish layout
    o = decode_attention(q_new, cache, sel)         # (B, Hq, T, D)

The new tokens (positions L-T .. L-1) must lie in the cache's last block.
Selection is the reference's SelectMax rule (src/qwen_blocksparse.py:108-121)
applied to the current block: the query summary is the mean of the new tokens'
queries over the GQA group (for T = bs at a block boundary exactly the prefill
summary of that block), the key summaries are per-block min/max of the
cache (kept incrementally: an append re-pools only the blocks it touches),
then causal top-k + own block (+ sink) sorted ascending (:87-99).  Attention
masks are the TOKEN rules (key position <= query position, repeated ids
once), as in blocksparse_forward.
"""
import torch

import _bsa

__all__ = ["DecodeCache", "decode_attention"]


class DecodeCache:
    """K/V cache (B, Hkv, max_len, D) with per-block min / max key summaries."""

    def __init__(self, B, Hkv, max_len, D, *, bs, dtype=torch.bfloat16, device="cuda"):
        self.bs = bs
        self.k = torch.zeros(B, Hkv, max_len, D, dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)
        nblk = (max_len + bs - 1) // bs
        self.kmin = torch.zeros(B, Hkv, nblk, D, dtype=torch.float32, device=device)
        self.kmax = torch.zeros_like(self.kmin)
        self.L = 0

    def append(self, k_new, v_new):
        T = k_new.shape[2]
        L0, L1 = self.L, self.L + T
        if L1 > self.k.shape[2]:
            raise ValueError("cache full")
        self.k[:, :, L0:L1] = k_new
        self.v[:, :, L0:L1] = v_new
        self.L = L1
        b0, b1 = L0 // self.bs, (L1 - 1) // self.bs + 1
        # re-pool the touched blocks; rows past L count as zeros, as in the prefill pooling
        mn, mx = _bsa.pool(self.k[:, :, b0 * self.bs:min(b1 * self.bs, L1)], self.bs, mean=False,
                           vmin=True, vmax=True)
        self.kmin[:, :, b0:b1] = mn
        self.kmax[:, :, b0:b1] = mx

    def select_quest(self, q_new, *, topk, sink=True):
        """(B, Hkv, W) block ids for the current block: Quest bound of the new tokens'
        group-mean query against every block up to the current one."""
        Hq, Hkv = q_new.shape[1], self.k.shape[1]
        qb = (self.L - 1) // self.bs
        # group-and-row mean (rows past T count as zeros: a positive scale of the
        # summary, which leaves the Quest ranking unchanged)
        (qp,) = _bsa.pool(q_new, self.bs, grp=Hq // Hkv)
        # at least topk key blocks, so the row is topk + 1 (+ sink) wide from the start
        # (blocks after the current one are causally masked; missing picks -> own)
        nb = min(self.kmin.shape[2], max(qb + 1, topk))
        sel, _, _ = _bsa.select(qp.contiguous(), self.kmax[:, :, :nb].contiguous(),
                                self.kmin[:, :, :nb].contiguous(), kind=_bsa.SCORE_QUEST,
                                layout=_bsa.SEL_FINISH, topk=topk, sink=sink, q_blk0=qb)
        return sel[:, :, 0]


def decode_attention(q_new, cache, sel, gate=None, *, scale=None, mask_mode=_bsa.MASK_TOKEN):
    """o (B, Hq, T, D) of the T newest tokens attending to their selected cache blocks."""
    return _bsa.decode(q_new, cache.k, cache.v, sel, gate, bs=cache.bs, L=cache.L,
                       mask_mode=mask_mode, scale=scale)
