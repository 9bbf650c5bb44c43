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


@pytest.mark.parametrize("name", ["lsh_causal.npz", "lsh_noncausal.npz"])
def test_lsh_golden(cuda, name):
    """bsa_select_lsh on the reference LSHBucketSSA's own summaries and planes gives
    its selection exactly (invalid slots -> own block)."""
    import _bsa
    g = golden(name)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
    sel, _, _ = _bsa.select_lsh(dev(g["a"]), dev(g["b"]), dev(g["planes"]),
                                hash_kind=_bsa.HASH_ARGMAX, cap=int(g["cap"]),
                                causal=bool(g["causal"]), topk=int(g["topk"]),
                                scale=float(g["scale"]))
    own = np.arange(g["sel"].shape[1]).reshape(1, -1, 1)
    exp = np.where(g["valid"].astype(bool), g["sel"], own)
    assert np.array_equal(sel.cpu().numpy(), exp)


@pytest.mark.parametrize("hash_kind,causal,cap,topk,planes,rounds,nblk", [
    (1, True, 16, 16, 4, 4, 700),
    (1, False, 8, 12, 3, 2, 257),
    (0, True, 5, 16, 8, 3, 300),
    (0, True, 64, 32, 6, 4, 1000),
    (1, True, 16, 64, 4, 4, 100),
])
def test_lsh_bit_exact_vs_oracle(cuda, hash_kind, causal, cap, topk, planes, rounds, nblk):
    import _bsa
    gen = torch.Generator().manual_seed(nblk + cap)
    G, dim = 3, 64
    a = torch.randn(G, nblk, dim, generator=gen)
    b = a + 0.7 * torch.randn(G, nblk, dim, generator=gen)
    R = torch.randn(dim, rounds, planes, generator=gen)
    sel, sc, gt = _bsa.select_lsh(a.to(cuda), b.to(cuda), R.to(cuda), hash_kind=hash_kind, cap=cap,
                                  causal=causal, topk=topk, scale=2.0, want_score=True,
                                  want_gate=True)
    osel, osc, ogt = O.select_lsh(a, b, R, hash_kind=hash_kind, cap=cap, causal=causal, topk=topk,
                                  scale=2.0, want_score=True, want_gate=True)
    assert np.array_equal(sel.cpu().numpy(), osel)
    assert np.array_equal(sc.cpu().numpy(), osc)
    assert np.allclose(gt.cpu().numpy(), ogt, atol=1e-6)


def test_lsh_config5_full_size(cuda):
    """BASELINE configuration 5 selection (B1 H8 N131072 D64 block 64, 4 sign planes x 4
    rounds, cap 16, top-16): bit-exact against the oracle on the pooled summaries."""
    import _bsa
    import selection
    gen = torch.Generator(device=cuda).manual_seed(5)
    q, k = (torch.randn(1, 8, 131072, 64, device=cuda, generator=gen).to(torch.bfloat16)
            for _ in range(2))
    sel, _, _ = selection.select_lsh(q, k, bs=64, topk=16, n_rounds=4, n_planes=4, cap=16, seed=0)
    assert sel.shape == (1, 8, 2048, 17)
    (qp,) = _bsa.pool(q, 64)
    (kp,) = _bsa.pool(k, 64)
    R = selection.lsh_planes(64, 4, 4, 0)
    osel, _, _ = O.select_lsh(qp.cpu(), kp.cpu(), R, hash_kind=O.HASH_SIGN, cap=16, causal=True,
                              topk=16)
    assert np.array_equal(sel.cpu().numpy(), osel)


def test_lsh_module_matches_oracle_attention(cuda, monkeypatch):
    """ssa_model.LSHBucketSSA: its selection equals the oracle's on the same pooled
    features, and its attention (invalid picks masked: causal by position,
    non-causal as repeated ids) equals the oracle attention over that selection."""
    import _bsa
    import ssa_model
    real = ssa_model.bsattn
    for causal in (True, False):
        torch.manual_seed(7)
        m = ssa_model.LSHBucketSSA(128, 2, block=32, topk=4, n_rounds=3, n_buckets=6, cap=4,
                                   gate=True, causal=causal).to(cuda)
        x = torch.randn(2, 1000, 128, device=cuda)
        seen = {}

        def spy(q, k, v, sel, gate, causal=False, gate_grad=False, mask_mode=0):
            out = real(q, k, v, sel, gate, causal=causal, gate_grad=gate_grad, mask_mode=mask_mode)
            seen.update(q=q, k=k, v=v, sel=sel, gate=gate, mode=mask_mode, out=out)
            return out

        monkeypatch.setattr(ssa_model, "bsattn", spy)
        out = m(x)
        out.float().sum().backward()
        assert torch.isfinite(out).all()
        assert m.sel_q[0].weight.grad is not None and torch.isfinite(m.sel_q[0].weight.grad).all()
        xp = torch.nn.functional.pad(x, (0, 0, 0, 24))
        (sqp,) = _bsa.pool(m.sel_q(xp).detach().float().unsqueeze(1), 32)
        skm, skx = _bsa.pool(m.sel_k(xp).detach().float().unsqueeze(1), 32, mean=True, vmax=True)
        osel, _, _ = O.select_lsh(sqp.cpu()[:, 0], torch.maximum(skm, skx).cpu()[:, 0], m.R.cpu(),
                                  hash_kind=O.HASH_ARGMAX, cap=4, causal=causal, topk=4,
                                  scale=m.scale)
        assert np.array_equal(seen["sel"].cpu().numpy(), osel)
        ref = O.attention(seen["q"].detach().float().cpu(), seen["k"].detach().float().cpu(),
                          seen["v"].detach().float().cpu(), seen["sel"].cpu().long(),
                          seen["gate"].detach().float().cpu(), bs=32, causal=causal,
                          mask_mode=seen["mode"])
        err = (seen["out"].detach().float().cpu() - ref).abs().max().item()
        assert err < 1e-4, err


def test_scores_topk_and_qmax_bit_exact(cuda):
    """bsa_select_scores, bsa_select_qmax (all causal / candidate lists) and the RAW
    layout of bsa_select against the oracle on the same inputs."""
    import _bsa
    gen = torch.Generator().manual_seed(21)
    G, nblk, bs, dim, topk = 3, 70, 32, 48, 7
    score = torch.rand(G, nblk, nblk, generator=gen)
    score[0, 5, :] = 0.5                                   # a fully tied row
    score[1, 9, 3] = float("nan")
    assert np.array_equal(_bsa.select_scores(score.to(cuda), topk=topk).cpu().numpy(),
                          O.select_scores(score, topk=topk))
    qt = torch.randn(G, nblk, bs, dim, generator=gen)
    kmax = torch.randn(G, nblk, dim, generator=gen).abs()
    kmin = -torch.randn(G, nblk, dim, generator=gen).abs()
    assert np.array_equal(_bsa.select_qmax(qt.to(cuda), kmax.to(cuda), kmin.to(cuda), topk=topk,
                                           sink=False).cpu().numpy(),
                          O.select_qmax(qt, kmax, kmin, topk=topk, sink=False))
    qp = qt.mean(2)
    raw, _, _ = _bsa.select(qp.to(cuda), kmax.to(cuda), kmin.to(cuda), kind=_bsa.SCORE_QUEST,
                            layout=_bsa.SEL_RAW, topk=20)
    oraw, _, _ = O.select(qp, kmax, kmin, kind=O.SCORE_QUEST, layout=O.SEL_RAW, topk=20)
    assert np.array_equal(raw.cpu().numpy(), oraw)
    assert np.array_equal(_bsa.select_qmax(qt.to(cuda), kmax.to(cuda), kmin.to(cuda), topk=topk,
                                           cand=raw).cpu().numpy(),
                          O.select_qmax(qt, kmax, kmin, topk=topk, cand=oraw))


def test_other_selectors_golden(cuda):
    """The device SelectOracle / SelectLastTok / SelectMaxQMax / SelectTwoStage on the
    reference's own inputs give the reference's selections (tie rows aside, see the
    oracle test); SelectRandom equals the _finish top-k of its own draws."""
    import qwen_blocksparse as qb
    g = golden("selectors.npz")
    bs, topk = int(g["bs"]), int(g["topk"])
    q, k = torch.from_numpy(g["q"]).to(cuda), torch.from_numpy(g["k"]).to(cuda)
    sel = qb.SelectOracle(topk, bs).select_from_mass(torch.from_numpy(g["mass"]).to(cuda))
    assert np.array_equal(sel.cpu().numpy(), g["oracle"])
    last = g["q"].reshape(1, 2, 2, -1, g["q"].shape[-1]).mean(2)
    lt = qb.SelectLastTok(topk, bs).select(q, k).cpu().numpy()
    nblk = lt.shape[2]
    tied = np.zeros(lt.shape[:3], bool)
    if g["q"].shape[2] % bs:
        tied[:, :, nblk - 1] = True
    assert np.array_equal(lt[~tied], g["lasttok"][~tied])
    assert np.array_equal(qb.SelectMaxQMax(topk, bs).select(q, k).cpu().numpy(), g["qmax"])
    assert np.array_equal(qb.SelectTwoStage(topk, bs, over=2).select(q, k).cpu().numpy(), g["twostage"])
    r = qb.SelectRandom(topk, bs, seed=3).select(q, k)
    gen = torch.Generator(device=cuda).manual_seed(3)
    draws = torch.rand(1, 2, nblk, nblk, generator=gen, device=cuda)
    assert np.array_equal(r.cpu().numpy(), O.select_scores(draws.cpu(), topk=topk))


@pytest.mark.parametrize("layout,causal,topk,dim,nblk", [(O.SEL_SSA, True, 16, 64, 700),
                                                         (O.SEL_SSA, False, 8, 64, 600),
                                                         (O.SEL_SSA, True, 32, 32, 1100),
                                                         (O.SEL_FINISH, True, 12, 64, 700),
                                                         (O.SEL_RAW, True, 16, 32, 520),
                                                         (O.SEL_SSA, True, 1, 64, 2000)])
def test_select_tensor_core_path_exact_with_ties(cuda, monkeypatch, layout, causal, topk, dim, nblk):
    """The tcgen05 tf32 scoring path (default for DOT scores at nblk >= 512) must give
    the exact fp32 selection: checked against the oracle and against the SIMT kernel
    (BSA_SELECT_SIMT=1), on data with many exactly tied scores (repeated key
    summaries) and a group of huge-norm summaries, at every key-split width."""
    import _bsa
    gen = torch.Generator().manual_seed(topk + dim + nblk)
    G = 5
    a = torch.randn(G, nblk, dim, generator=gen)
    b = torch.randn(G, nblk, dim, generator=gen)
    b[1] = b[1, :1]                       # group 1: every key summary identical (all ties)
    b[2, ::3] = b[2, 5]                   # group 2: a third of the keys identical
    a[3] *= 1e4                           # group 3: large scores, small relative gaps
    b[3] = b[3] * 1e-3 + 1.0
    args = dict(kind=_bsa.SCORE_DOT, layout=layout, causal=causal, topk=topk, want_score=layout == 0,
                want_gate=layout == 0)
    o_sel, o_sc, o_gt = O.select(a, b, kind=O.SCORE_DOT, layout=layout, causal=causal, topk=topk,
                                 want_score=layout == 0, want_gate=layout == 0)
    monkeypatch.setenv("BSA_SELECT_SIMT", "1")
    s_simt, _, _ = _bsa.select(a.to(cuda), b.to(cuda), **args)
    monkeypatch.delenv("BSA_SELECT_SIMT")
    monkeypatch.setenv("BSA_SELECT_TC5", "1")
    assert np.array_equal(s_simt.cpu().numpy(), o_sel)
    for split in ("", "1", "2", "8"):
        if split:
            monkeypatch.setenv("BSA_SELECT_SPLIT", split)
        s_tc, sc_tc, gt_tc = _bsa.select(a.to(cuda), b.to(cuda), **args)
        _bsa.check_status(cuda)
        assert np.array_equal(s_tc.cpu().numpy(), o_sel), "split %s" % split
        if layout == 0:
            assert np.array_equal(sc_tc.cpu().numpy(), o_sc)
            assert np.allclose(gt_tc.cpu().numpy(), o_gt, atol=1e-6, rtol=1e-6)


def test_select_tensor_core_path_query_range(cuda, monkeypatch):
    """The tcgen05 selection on a query-block range (the sharded layout) equals the
    rows of the whole-sequence selection."""
    import _bsa
    monkeypatch.setenv("BSA_SELECT_TC5", "1")
    gen = torch.Generator().manual_seed(77)
    nblk, dim = 3000, 64
    a = torch.randn(2, nblk, dim, generator=gen).to(cuda)
    b = torch.randn(2, nblk, dim, generator=gen).to(cuda)
    full, _, _ = _bsa.select(a, b, topk=16)
    for q0, nq in ((0, 1000), (1000, 1000), (2000, 1000), (1234, 777)):
        part, _, _ = _bsa.select(a[:, q0:q0 + nq].contiguous(), b, topk=16, q_blk0=q0)
        assert torch.equal(part, full[:, q0:q0 + nq])


def test_centroid_module_matches_oracle_attention(cuda, monkeypatch):
    """ssa_model.CentroidSSA: its attention over the centroid-routed selection (empty
    slots skipped, no causal mask, gate) equals the oracle attention, and gradients
    reach the selector MLPs and the centroids."""
    import ssa_model
    real = ssa_model.bsattn
    for refine in (None, 3):
        torch.manual_seed(5)
        m = ssa_model.CentroidSSA(128, 2, block=32, n_centroids=6, cpq=2, cap=3, gate=True,
                                  refine_topk=refine).to(cuda)
        x = torch.randn(2, 1000, 128, device=cuda)
        seen = {}

        def spy(q, k, v, sel, gate, causal=False, gate_grad=False, mask_mode=0):
            out = real(q, k, v, sel, gate, causal=causal, gate_grad=gate_grad, mask_mode=mask_mode)
            seen.update(q=q, k=k, v=v, sel=sel, gate=gate, mode=mask_mode, causal=causal, out=out)
            return out

        monkeypatch.setattr(ssa_model, "bsattn", spy)
        out = m(x)
        out.float().sum().backward()
        assert torch.isfinite(out).all()
        assert m.cent.grad is not None and torch.isfinite(m.cent.grad).all()
        ref = O.attention(seen["q"].detach().float().cpu(), seen["k"].detach().float().cpu(),
                          seen["v"].detach().float().cpu(), seen["sel"].cpu().long(),
                          seen["gate"].detach().float().cpu(), bs=32, causal=seen["causal"],
                          mask_mode=seen["mode"])
        err = (seen["out"].detach().float().cpu() - ref).abs().max().item()
        assert err < 1e-4, err


@pytest.mark.parametrize("grp,D,rot", [(8, 256, 64), (1, 256, 64), (2, 64, 32)])
def test_rope_aware_pooling_equals_pooling_rotated(cuda, grp, D, rot):
    """bsa_pool with rope=(cos, sin) pools exactly the values bsa_rope writes."""
    import _bsa
    gen = torch.Generator().manual_seed(grp + D)
    B, Hkv, L, bs = 1, 2, 1000, 128
    x = torch.randn(B, Hkv * grp, L, D, generator=gen).to(torch.bfloat16).to(cuda)
    cos, sin = O.rope_cos_sin(L, rot, 1e7, torch.bfloat16)
    cos, sin = cos.to(cuda), sin.to(cuda)
    xr = _bsa.rope(x, cos, sin)
    a = _bsa.pool(x, bs, grp=grp, rope=(cos, sin))
    r = _bsa.pool(xr, bs, grp=grp)
    assert torch.equal(a[0], r[0])
    if grp == 1:
        a2 = _bsa.pool(x, bs, mean=False, vmin=True, vmax=True, rope=(cos, sin))
        r2 = _bsa.pool(xr, bs, mean=False, vmin=True, vmax=True)
        assert torch.equal(a2[0], r2[0]) and torch.equal(a2[1], r2[1])


def test_rope_inside_attention_equals_rotated_input(cuda):
    """bsa_attn_fwd with the rotation of q folded in (block 128, D 256) gives the
    same output, bit for bit, as the forward on bsa_rope(q); the Qwen drop-in
    (which folds it) matches the unfolded composition."""
    import _bsa
    import qwen_blocksparse as qb
    gen = torch.Generator().manual_seed(5)
    B, Hq, Hkv, L, D, bs, rot = 1, 8, 2, 2048 + 77, 256, 128, 64
    q = torch.randn(B, Hq, L, D, generator=gen).to(torch.bfloat16).to(cuda)
    k, v = (torch.randn(B, Hkv, L, D, generator=gen).to(torch.bfloat16).to(cuda) for _ in range(2))
    cos, sin = (t.to(cuda) for t in O.rope_cos_sin(L, rot, 1e7, torch.bfloat16))
    kr = _bsa.rope(k, cos, sin)
    qr = _bsa.rope(q, cos, sin)
    sel = qb.SelectMax(4, bs).select(qr, kr).to(torch.int32)
    kw = dict(bs=bs, causal=True, mask_mode=_bsa.MASK_TOKEN, want_lse=False)
    o1, _ = _bsa.attn_fwd(qr, kr, v, sel, **kw)
    o2, _ = _bsa.attn_fwd(q, kr, v, sel, rope=(cos, sin), **kw)
    assert torch.equal(o1, o2)
    o3, _ = _bsa.attn_fwd(q, kr, v, None, rope=(cos, sin), **kw)    # all blocks
    o4, _ = _bsa.attn_fwd(qr, kr, v, None, **kw)
    assert torch.equal(o3, o4)
    import selection
    assert torch.equal(selection.select_quest(q, kr, bs=bs, topk=4, rope=(cos, sin)), sel)


@pytest.mark.parametrize("B,nblk,C,cpq,cap,refine", [(2, 300, 8, 2, 6, None), (1, 1000, 16, 3, 8, 5),
                                                     (2, 77, 4, 4, 30, 9), (1, 2048, 32, 2, 64, None)])
def test_centroid_routing_kernel_vs_oracle(cuda, B, nblk, C, cpq, cap, refine):
    """The device routing (bsa_centroid_route, with the module's argmax / top-cpq)
    equals the oracle's tensor-op restatement, with and without the refine step;
    and on the reference's own goldens."""
    import ssa_model
    gen = torch.Generator().manual_seed(nblk + C)
    s = 16
    sq, sk = torch.randn(B, nblk, s, generator=gen), torch.randn(B, nblk, s, generator=gen)
    cent = torch.randn(C, s, generator=gen)
    rf = None
    if refine:
        qb, kb = torch.randn(B, nblk, 24, generator=gen), torch.randn(B, nblk, 24, generator=gen)
        rf = (qb, kb, refine)
    ref, rkc, _ = O.centroid_select(sq, sk, cent, cpq=cpq, cap=cap, refine=rf)
    rfd = tuple(t.to(cuda) for t in rf[:2]) + (refine,) if rf else None
    got, kc, _ = ssa_model.centroid_select(sq.to(cuda), sk.to(cuda), cent.to(cuda), cpq=cpq, cap=cap,
                                           refine=rfd)
    assert torch.equal(kc.cpu(), rkc)
    assert torch.equal(got.cpu(), ref)


@pytest.mark.parametrize("name", ["centroid_plain.npz", "centroid_refine.npz"])
def test_centroid_routing_kernel_golden(cuda, name):
    import ssa_model
    g = golden(name)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
    rk = int(g["refine"])
    refine = (t(g["q_blk"]), t(g["k_blk"]), rk) if rk > 0 else None
    sel, _, _ = ssa_model.centroid_select(t(g["sq"]), t(g["sk"]), t(g["cent"]), cpq=int(g["cpq"]),
                                          cap=int(g["cap"]), refine=refine)
    sel = sel.cpu().numpy()
    valid = g["valid"].astype(bool)
    assert np.array_equal(sel[valid], g["sel"][valid])
    assert (sel[~valid] == -1).all()
