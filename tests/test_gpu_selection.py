"""GPU parity of pooling, fused scoring + top-k, CSR transpose and RoPE (all
bit-exact against the C oracle / the reference's goldens), and of the Qwen
GQA core (within tolerance)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("grp", [1, 4])
def test_pool_bit_exact(cuda, dtype, grp):
    import _bsa
    gen = torch.Generator().manual_seed(grp)
    x = torch.randn(2, 8, 1000, 64, generator=gen).to(dtype)   # L not a multiple of bs
    outs = _bsa.pool(x.to(cuda), 64, grp=grp, mean=True, vmin=grp == 1, vmax=grp == 1)
    mean, mn, mx = O.pool(x.float(), 64, grp=grp)
    assert np.array_equal(outs[0].cpu().numpy(), mean)
    if grp == 1:
        assert np.array_equal(outs[1].cpu().numpy(), mn)
        assert np.array_equal(outs[2].cpu().numpy(), mx)


@pytest.mark.parametrize("kind,layout,causal,topk,sink,nblk,dim", [
    (O.SCORE_DOT, O.SEL_SSA, True, 16, False, 300, 64),
    (O.SCORE_DOT, O.SEL_SSA, False, 8, False, 130, 64),
    (O.SCORE_MAXDOT2, O.SEL_SSA, True, 8, False, 200, 32),
    (O.SCORE_QUEST, O.SEL_FINISH, True, 32, True, 257, 256),
    (O.SCORE_QUEST, O.SEL_FINISH, True, 3, False, 70, 64),
    (O.SCORE_DOT, O.SEL_SSA, True, 0, False, 10, 64),
    (O.SCORE_DOT, O.SEL_SSA, True, 5, False, 1, 64),
])
def test_select_bit_exact(cuda, kind, layout, causal, topk, sink, nblk, dim):
    import _bsa
    gen = torch.Generator().manual_seed(nblk + topk)
    G = 3
    a = torch.randn(G, nblk, dim, generator=gen)
    b1 = torch.randn(G, nblk, dim, generator=gen)
    b2 = torch.randn(G, nblk, dim, generator=gen) if kind != O.SCORE_DOT else None
    if kind == O.SCORE_QUEST:
        b1, b2 = torch.maximum(b1, b2), torch.minimum(b1, b2)
    ssa = layout == O.SEL_SSA
    sel, sc, gt = _bsa.select(a.to(cuda), b1.to(cuda), b2.to(cuda) if b2 is not None else None,
                              kind=kind, layout=layout, causal=causal, topk=topk, sink=sink,
                              want_score=ssa, want_gate=ssa)
    rsel, rsc, rgt = O.select(a, b1, b2, kind=kind, layout=layout, causal=causal, topk=topk,
                              sink=sink, want_score=ssa, want_gate=ssa)
    assert np.array_equal(sel.cpu().numpy(), rsel)
    if ssa:
        assert np.array_equal(sc.cpu().numpy(), rsc)
        assert np.allclose(gt.cpu().numpy(), rgt, atol=1e-6, rtol=1e-6)


def test_select_ties_go_to_lower_block(cuda):
    import _bsa
    nblk, dim = 100, 8
    ones = torch.ones(1, nblk, dim, device=cuda)      # every score equal
    sel, _, _ = _bsa.select(ones, ones, topk=4, causal=True)
    s = sel.cpu()[0]
    for i in range(nblk):
        assert s[i].tolist() == [i] + list(range(min(i, 4))) + [i] * max(0, 4 - i)


def test_meanpool_selection_config1_full_size(cuda):
    """BASELINE config 1 selection: B1 H4 N4096 D64 block 64, top-8 incl. the diagonal."""
    import selection
    gen = torch.Generator().manual_seed(0)
    q, k = (torch.randn(1, 4, 4096, 64, generator=gen) for _ in range(2))
    sel, _, _ = selection.select_meanpool(q.to(cuda), k.to(cuda), bs=64, topk=7)
    qp, _, _ = O.pool(q, 64)
    kp, _, _ = O.pool(k, 64)
    rsel, _, _ = O.select(qp, kp, topk=7)
    assert sel.shape == (1, 4, 64, 8)
    assert np.array_equal(sel.cpu().numpy(), rsel)


@pytest.mark.parametrize("mode,causal", [(O.MASK_SLOT, True), (O.MASK_SLOT, False),
                                         (O.MASK_TOKEN, True)])
def test_csr_bit_exact(cuda, mode, causal):
    import _bsa
    gen = torch.Generator().manual_seed(1)
    B, H, nblk, kk = 2, 3, 150, 9
    sel = torch.randint(0, nblk, (B, H, nblk, kk), generator=gen, dtype=torch.int32)
    sel[..., 0] = torch.arange(nblk, dtype=torch.int32)
    rp, col = _bsa.sel_csr(sel.to(cuda), bs=64, L=nblk * 64, causal=causal, mask_mode=mode)
    rrp, rcol = O.csr(sel, mask_mode=mode, causal=causal)
    assert np.array_equal(rp.cpu().numpy(), rrp)
    assert np.array_equal(col.cpu().numpy()[:rrp[-1]], rcol)


def test_rope_bit_exact_vs_transformers(cuda):
    import _bsa
    g = golden("rope.npz")
    cos = torch.from_numpy(g["cos"]).to(cuda, torch.bfloat16)
    sin = torch.from_numpy(g["sin"]).to(cuda, torch.bfloat16)
    for x, ref in (("q", "qe"), ("k", "ke")):
        t = torch.from_numpy(g[x]).to(cuda, torch.bfloat16)
        y = _bsa.rope(t, cos, sin)
        assert torch.equal(y.float().cpu(), torch.from_numpy(g[ref]))
        t2 = t.clone()
        _bsa.rope(t2, cos, sin, out=t2)                    # in place
        assert torch.equal(t2, y)


def test_qwen_selectmax_golden(cuda):
    import qwen_blocksparse as qb
    g = golden("qwen_selectmax.npz")
    B, Hq, Hkv, L, d, bs, topk = [int(x) for x in g["meta"]]
    q, k, v = (torch.from_numpy(g[n]).to(cuda) for n in "qkv")
    S = qb.SelectMax(topk, bs, sink=True)
    assert np.array_equal(S.select(q, k).cpu().numpy(), g["idx"])
    out = qb.blocksparse_forward(q, k, v, selector=S, topk=topk, bs=bs)
    assert (out.cpu() - torch.from_numpy(g["o"])).abs().max().item() <= 1e-5


@pytest.mark.parametrize("name", ["qwen_selectall.npz", "qwen_fastpath.npz"])
def test_qwen_allblocks_golden(cuda, name):
    import qwen_blocksparse as qb
    g = golden(name)
    bs = int(g["meta"][5])
    q, k, v = (torch.from_numpy(g[n]).to(cuda) for n in "qkv")
    sel = qb.SelectAll(bs) if name == "qwen_selectall.npz" else None
    out = qb.blocksparse_forward(q, k, v, selector=sel, topk=10 ** 6, bs=bs)
    assert (out.cpu() - torch.from_numpy(g["o"])).abs().max().item() <= 1e-5


def test_qwen_variant_bf16_vs_oracle(cuda):
    """RoPE + Quest selection + GQA attention + sigmoid gate, D=256, bs=128, padded L."""
    import qwen_blocksparse as qb
    gen = torch.Generator().manual_seed(21)
    B, Hq, Hkv, L, D, bs, topk, rot = 1, 8, 2, 2048 + 77, 256, 128, 4, 64
    q, k, v = (torch.randn(B, h, L, D, generator=gen).to(torch.bfloat16) for h in (Hq, Hkv, Hkv))
    gate = torch.randn(B, L, Hq * D, generator=gen).to(torch.bfloat16)
    cos, sin = O.rope_cos_sin(L, rot, 1e7, torch.bfloat16)
    out = qb.qwen_attention(q.to(cuda), k.to(cuda), v.to(cuda), cos.to(cuda), sin.to(cuda),
                            gate.to(cuda), selector=qb.SelectMax(topk, bs), topk=topk, bs=bs)
    qr, kr = O.rope(q, cos, sin), O.rope(k, cos, sin)
    qp, _, _ = O.pool(qr.float(), bs, grp=Hq // Hkv)
    _, kmin, kmax = O.pool(kr.float(), bs)
    sel, _, _ = O.select(qp, kmax, kmin, kind=O.SCORE_QUEST, layout=O.SEL_FINISH, topk=topk, sink=True)
    ref = O.attention(qr, kr, v, torch.from_numpy(sel), bs=bs, causal=True, mask_mode=O.MASK_TOKEN)
    ref = ref.transpose(1, 2).reshape(B, L, Hq * D) * torch.sigmoid(gate.double())
    diff = (out.double().cpu() - ref).abs()
    assert (diff <= 2e-2 + 1e-2 * ref.abs()).all(), diff.max().item()
