"""Decode (bsa_decode, decode.py): the T newest tokens against their selected
cache blocks.  Checked against the float64 oracle's attention rows L-T .. L-1
(TOKEN and SLOT masks, gate, GQA, repeated ids, a partial last block), against
the forward kernel run on the last query block, and the cache's incremental
Quest selection against the prefill SelectMax row."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _case(B, Hq, Hkv, L, D, dev, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, L, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, L, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, L, D, generator=g).to(dtype)
    return q, k, v, g


def _cmp(got, ref, what):
    got, ref = got.float().cpu(), ref.float().cpu()
    excess = ((got - ref).abs() - (2e-2 + 1e-2 * ref.abs())).max().item()
    assert excess <= 0, "%s: %g" % (what, (got - ref).abs().max().item())


@pytest.mark.parametrize("mode,T,bs,D,Hq,Hkv,L", [
    (1, 1, 128, 256, 16, 2, 1000),
    (1, 3, 128, 128, 8, 2, 899),
    (0, 2, 64, 64, 4, 4, 704),
    (0, 1, 32, 64, 2, 1, 513),
])
def test_decode_vs_oracle(cuda, mode, T, bs, D, Hq, Hkv, L):
    import _bsa
    B, kk = 2, 9
    q, k, v, g = _case(B, Hq, Hkv, L, D, cuda, T + bs + D)
    nblk = (L + bs - 1) // bs
    qb = (L - 1) // bs
    sel = torch.randint(0, qb + 1, (B, Hkv, kk), generator=g, dtype=torch.int32)
    sel[..., 0] = qb
    sel[..., 3] = sel[..., 2]            # a repeated id
    gate = torch.randn(B, Hkv, kk, generator=g) * 0.5
    o = _bsa.decode(q[:, :, L - T:].to(cuda), k.to(cuda), v.to(cuda), sel.to(cuda), gate.to(cuda),
                    bs=bs, mask_mode=mode)
    full = torch.arange(nblk).view(1, 1, nblk, 1).expand(B, Hkv, nblk, kk).clone()
    full[:, :, qb] = sel.long()
    gfull = torch.zeros(B, Hkv, nblk, kk)
    gfull[:, :, qb] = gate
    ref = O.attention(q, k, v, full, gfull, bs=bs, causal=True, mask_mode=mode)
    _cmp(o, ref[:, :, L - T:], "decode")


def test_decode_matches_forward_on_last_block(cuda):
    import _bsa
    B, Hq, Hkv, L, D, bs, T = 1, 8, 2, 1500, 128, 128, 4
    q, k, v, g = _case(B, Hq, Hkv, L, D, cuda, 5)
    qb = (L - 1) // bs
    sel = torch.randint(0, qb + 1, (B, Hkv, 1, 12), generator=g, dtype=torch.int32)
    sel[..., 0] = qb
    dq, dk, dv = (t.to(cuda) for t in (q, k, v))
    o_f, _ = _bsa.attn_fwd(dq[:, :, qb * bs:], dk, dv, sel.to(cuda), bs=bs, causal=True,
                           mask_mode=_bsa.MASK_TOKEN, q_blk0=qb, want_lse=False)
    o_d = _bsa.decode(dq[:, :, L - T:], dk, dv, sel[:, :, 0].to(cuda), bs=bs)
    r0 = L - T - qb * bs
    _cmp(o_d, o_f[:, :, r0:r0 + T], "decode vs forward")


def test_decode_cache_selection_matches_prefill_selectmax(cuda):
    import decode
    import qwen_blocksparse as qb_mod
    B, Hq, Hkv, D, bs, topk = 1, 8, 2, 128, 64, 6
    nb = 12
    L = nb * bs
    q, k, v, _ = _case(B, Hq, Hkv, L, D, cuda, 9)
    cache = decode.DecodeCache(B, Hkv, L, D, bs=bs, device=cuda)
    pre = qb_mod.SelectMax(topk, bs).select(q.to(cuda), k.to(cuda))     # (B, Hkv, nblk, W)
    for blk in range(nb):
        rows = slice(blk * bs, (blk + 1) * bs)
        # append a block in two pieces, select once it is complete
        cache.append(k[:, :, rows][:, :, :17].to(cuda), v[:, :, rows][:, :, :17].to(cuda))
        cache.append(k[:, :, rows][:, :, 17:].to(cuda), v[:, :, rows][:, :, 17:].to(cuda))
        sel = cache.select_quest(q[:, :, rows].to(cuda), topk=topk)
        assert torch.equal(sel, pre[:, :, blk]), blk
    o = decode.decode_attention(q[:, :, L - 1:].to(cuda), cache, sel)
    assert o.shape == (B, Hq, 1, D) and torch.isfinite(o.float()).all()
