"""Pins the CPU oracle to the reference's own outputs (tests/golden/, made by
tests/golden/make_golden.py from the reference code).  CPU only."""
import numpy as np
import torch
import torch.nn.functional as F

from conftest import golden
from oracle import oracle as O


def _t(a):
    return torch.from_numpy(np.asarray(a))


def _close(a, b, tol):
    err = (torch.as_tensor(a).double() - torch.as_tensor(b).double()).abs().max().item()
    assert err <= tol, err


def _ssa_sel_check(ours, ref):
    """Valid slots must match exactly; slots the reference filled with a masked pick
    (causal, block id >= own) are the own block in ours."""
    B, nblk, kk = ref.shape
    own = np.arange(nblk).reshape(1, nblk)
    assert (ours[..., 0] == own).all() and (ref[..., 0] == own).all()
    valid = ref[..., 1:] < own[..., None]
    assert (ours[..., 1:][valid] == ref[..., 1:][valid]).all()
    fill = np.broadcast_to(own[..., None], ours[..., 1:].shape)
    assert (ours[..., 1:][~valid] == fill[~valid]).all()


def test_ssa_selection_matches_reference():
    for name in ("ssa_gather_causal_gate.npz", "ssa_gather_causal.npz"):
        g = golden(name)
        B, H, L, dh, bs, topk, causal, gate = g["meta"]
        sel, score, _ = O.select(g["fa"], g["fb"], kind=O.SCORE_DOT, layout=O.SEL_SSA,
                                 causal=bool(causal), topk=int(topk), want_score=True)
        _ssa_sel_check(sel, g["sel"])
        raw = g["fa"].astype(np.float64) @ np.swapaxes(g["fb"], -1, -2).astype(np.float64)
        assert np.array_equal(score.astype(np.float64), np.take_along_axis(raw, sel.astype(np.int64), -1))


def test_ssa_noncausal_selection_matches_reference():
    g = golden("ssa_gather_noncausal_gate.npz")
    topk = int(g["meta"][5])
    sel, _, _ = O.select(g["fa"], g["fb"], kind=O.SCORE_DOT, layout=O.SEL_SSA, causal=False, topk=topk)
    assert np.array_equal(sel, g["sel"])


def _gate_from(g, sel):
    raw = torch.from_numpy(g["fa"]) @ torch.from_numpy(g["fb"]).transpose(-1, -2)
    return F.logsigmoid(torch.gather(raw, -1, torch.from_numpy(sel).long()))


def test_ssa_gather_attention_and_grads():
    for name in ("ssa_gather_causal_gate.npz", "ssa_gather_causal.npz", "ssa_gather_noncausal_gate.npz"):
        g = golden(name)
        B, H, L, dh, bs, topk, causal, gate = [int(x) for x in g["meta"]]
        sel = _t(g["sel"])
        gt = _gate_from(g, g["sel"]) if gate else None
        o = O.attention(_t(g["q"]), _t(g["k"]), _t(g["v"]), sel, gt, bs=bs, causal=bool(causal))
        _close(o, g["o"], 1e-5)
        dq, dk, dv, _ = O.attention_grads(_t(g["q"]), _t(g["k"]), _t(g["v"]), sel, _t(g["do"]), gt,
                                          bs=bs, causal=bool(causal))
        for got, ref in ((dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"])):
            _close(got, ref, 1e-5)


def test_triton_kernel_semantics():
    for name in ("triton_interp_causal.npz", "triton_interp_noncausal.npz"):
        g = golden(name)
        B, H, L, dh, bs, kk, causal = [int(x) for x in g["meta"]]
        args = (_t(g["q"]), _t(g["k"]), _t(g["v"]), _t(g["sel"]))
        o = O.attention(*args, _t(g["gate"]), bs=bs, causal=bool(causal))
        _close(o, g["o"], 2e-5)
        dq, dk, dv, _ = O.attention_grads(*args, _t(g["do"]), _t(g["gate"]), bs=bs, causal=bool(causal))
        for got, ref in ((dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"])):
            _close(got, ref, 5e-5)


def test_qwen_selectmax_indices_and_output():
    g = golden("qwen_selectmax.npz")
    B, Hq, Hkv, L, d, bs, topk = [int(x) for x in g["meta"]]
    qp, _, _ = O.pool(g["q"], bs, grp=Hq // Hkv)
    _, kmin, kmax = O.pool(g["k"], bs)
    sel, _, _ = O.select(qp, kmax, kmin, kind=O.SCORE_QUEST, layout=O.SEL_FINISH, topk=topk, sink=True)
    assert np.array_equal(sel, g["idx"])
    o = O.attention(_t(g["q"]), _t(g["k"]), _t(g["v"]), _t(sel), bs=bs, causal=True, mask_mode=O.MASK_TOKEN)
    _close(o, g["o"], 1e-5)


def test_qwen_allblocks_equals_reference():
    for name in ("qwen_selectall.npz", "qwen_fastpath.npz"):
        g = golden(name)
        bs = int(g["meta"][5])
        o = O.attention(_t(g["q"]), _t(g["k"]), _t(g["v"]), None, bs=bs, causal=True, mask_mode=O.MASK_TOKEN)
        _close(o, g["o"], 1e-5)


def test_rope_matches_transformers():
    g = golden("rope.npz")
    B, Hq, Hkv, L, D, rot = [int(x) for x in g["meta"]]
    cos, sin = O.rope_cos_sin(L, rot, float(g["theta"][0]), torch.bfloat16)
    assert torch.equal(cos.float(), _t(g["cos"])[0]) and torch.equal(sin.float(), _t(g["sin"])[0])
    assert torch.equal(O.rope(_t(g["q"]).to(torch.bfloat16), cos, sin).float(), _t(g["qe"]))
    assert torch.equal(O.rope(_t(g["k"]).to(torch.bfloat16), cos, sin).float(), _t(g["ke"]))


def test_csr_oracle_is_a_transpose():
    rng = np.random.default_rng(0)
    B, H, nblk, kk = 2, 3, 17, 5
    sel = rng.integers(0, nblk, (B, H, nblk, kk)).astype(np.int32)
    sel[..., 0] = np.arange(nblk)
    for mode, causal in ((O.MASK_SLOT, True), (O.MASK_SLOT, False), (O.MASK_TOKEN, True)):
        rp, col = O.csr(sel, mask_mode=mode, causal=causal)
        seen = []
        for b in range(B):
            for h in range(H):
                for q in range(nblk):
                    row = sel[b, h, q]
                    for s in range(kk):
                        kb = row[s]
                        if mode == O.MASK_SLOT:
                            act = (not causal) or s == 0 or kb < q
                        else:
                            act = kb not in row[:s] and (not causal or kb <= q)
                        if act:
                            seen.append(((b * H + h) * nblk + kb, q * kk + s))
        seen.sort()
        exp_rp = np.zeros(B * H * nblk + 1, np.int64)
        for bin_, _ in seen:
            exp_rp[bin_ + 1] += 1
        assert np.array_equal(rp, np.cumsum(exp_rp))
        assert np.array_equal(col, np.array([e for _, e in seen], np.int32))


def _lsh_expected(g):
    """The reference's LSH selection with its invalid slots (-inf mask) replaced by
    the own block, which is how the build marks a missing pick."""
    own = np.arange(g["sel"].shape[1]).reshape(1, -1, 1)
    return np.where(g["valid"].astype(bool), g["sel"], own)


def test_lsh_selection_matches_reference():
    """LSHBucketSSA's inference selection (argmax hashing, index-ordered bucket caps,
    cross-round dedup incl. the block-0 quirk, cosine re-score, top-k)."""
    for name in ("lsh_causal.npz", "lsh_noncausal.npz"):
        g = golden(name)
        sel, score, gate = O.select_lsh(g["a"], g["b"], g["planes"], hash_kind=O.HASH_ARGMAX,
                                        cap=int(g["cap"]), causal=bool(g["causal"]),
                                        topk=int(g["topk"]), scale=float(g["scale"]),
                                        want_score=True, want_gate=True)
        assert np.array_equal(sel, _lsh_expected(g)), name
        # own score = scale * cosine of the normalised summaries
        qa = g["a"] / np.maximum(np.linalg.norm(g["a"], axis=-1, keepdims=True), 1e-12)
        kb = g["b"] / np.maximum(np.linalg.norm(g["b"], axis=-1, keepdims=True), 1e-12)
        own = float(g["scale"]) * (qa * kb).sum(-1)
        assert np.allclose(score[..., 0], own, atol=1e-5)
        assert np.allclose(gate, np.log(1 / (1 + np.exp(-score.astype(np.float64)))), atol=1e-5)


def test_lsh_sign_hash_structure():
    """Sign hashing: every pick shares a bucket with its
    query block in some round, precedes it (causal), appears once, and is ranked by
    descending score; a cap of nblk with one round and zero planes' worth of buckets
    degenerates to the dense causal top-k."""
    rng = np.random.default_rng(3)
    G, nblk, dim, rounds, planes, cap, topk = 3, 200, 64, 4, 4, 16, 16
    a = rng.standard_normal((G, nblk, dim)).astype(np.float32)
    b = (a + 0.5 * rng.standard_normal((G, nblk, dim))).astype(np.float32)
    R = rng.standard_normal((dim, rounds, planes)).astype(np.float32)
    sel, score, _ = O.select_lsh(a, b, R, hash_kind=O.HASH_SIGN, cap=cap, causal=True, topk=topk,
                                 want_score=True)
    qn = a / np.linalg.norm(a, axis=-1, keepdims=True)
    kn = b / np.linalg.norm(b, axis=-1, keepdims=True)
    qcode = ((np.einsum("gnd,drc->gnrc", qn, R) > 0) * (1 << np.arange(planes))).sum(-1)
    kcode = ((np.einsum("gnd,drc->gnrc", kn, R) > 0) * (1 << np.arange(planes))).sum(-1)
    for g in range(G):
        for i in range(nblk):
            picks = [j for j in sel[g, i, 1:] if j != i]
            assert len(picks) == len(set(picks))
            for j in picks:
                assert j < i and (qcode[g, i] == kcode[g, j]).any()
            sc = score[g, i, 1:1 + len(picks)]
            assert (np.diff(sc) <= 0).all()
    # one round whose single plane is zero: every block lands in bucket 0, the cap
    # covers all blocks -> dense causal top-k by cosine (ties to the lower block)
    Z = np.zeros((dim, 1, 1), np.float32)
    sel1, _, _ = O.select_lsh(a, b, Z, hash_kind=O.HASH_SIGN, cap=nblk, causal=True, topk=8)
    dense, _, _ = O.select(qn, kn, kind=O.SCORE_DOT, layout=O.SEL_SSA, causal=True, topk=8)
    assert np.array_equal(sel1, dense)


def _selector_summaries(g):
    q, k, bs = g["q"], g["k"], int(g["bs"])
    B, Hq, L, d = q.shape
    Hkv = k.shape[1]
    nblk = (L + bs - 1) // bs
    qt, _, _ = O.pool(q, 1, grp=Hq // Hkv)
    qt = np.concatenate([qt, np.zeros((B, Hkv, nblk * bs - L, d), np.float32)], 2)
    qt = qt.reshape(B, Hkv, nblk, bs, d)
    _, kmin, kmax = O.pool(k, bs)
    qp, _, _ = O.pool(q, bs, grp=Hq // Hkv)
    return qt, kmin, kmax, qp


def test_other_selectors_match_reference():
    """SelectOracle, SelectRandom, SelectLastTok, SelectMaxQMax, SelectTwoStage
    (src/qwen_blocksparse.py:124-299) restated on the oracle's exact summaries.
    The reference breaks score ties in torch.topk's order; the restatement takes
    the lower block id, which only shows on rows whose scores all tie (the padded
    last block's zero last token under SelectLastTok)."""
    g = golden("selectors.npz")
    topk = int(g["topk"])
    assert np.array_equal(O.select_scores(g["mass"], topk=topk), g["oracle"])
    assert np.array_equal(O.select_scores(g["rnd"], topk=topk), g["random"])
    qt, kmin, kmax, qp = _selector_summaries(g)
    last = np.ascontiguousarray(qt[:, :, :, -1])
    sel, _, _ = O.select(last, kmax, kmin, kind=O.SCORE_QUEST, layout=O.SEL_FINISH, topk=topk,
                         sink=True)
    tied = ~last.any(-1)                                    # all-zero query token
    assert np.array_equal(sel[~tied], g["lasttok"][~tied])
    assert (sel[tied][:, :topk] <= np.arange(topk)).all()  # ties -> lowest block ids
    assert np.array_equal(O.select_qmax(qt, kmax, kmin, topk=topk), g["qmax"])
    M = min(2 * topk, qt.shape[2])
    cand, _, _ = O.select(qp, kmax, kmin, kind=O.SCORE_QUEST, layout=O.SEL_RAW, topk=M)
    assert np.array_equal(O.select_qmax(qt, kmax, kmin, topk=topk, cand=cand), g["twostage"])


def test_centroid_routing_matches_reference():
    """The oracle's centroid routing (tensor ops, no nblk^2 tensor) reproduces
    CentroidSSA's selection (src/ssa_model.py:254-299), with and without the refine
    step."""
    for name in ("centroid_plain.npz", "centroid_refine.npz"):
        g = golden(name)
        rk = int(g["refine"])
        refine = (_t(g["q_blk"]), _t(g["k_blk"]), rk) if rk > 0 else None
        sel, _, _ = O.centroid_select(_t(g["sq"]), _t(g["sk"]), _t(g["cent"]),
                                      cpq=int(g["cpq"]), cap=int(g["cap"]), refine=refine)
        sel = sel.numpy()
        valid = g["valid"].astype(bool)
        assert sel.shape == g["sel"].shape, name
        assert np.array_equal(sel[valid], g["sel"][valid]), name
        assert (sel[~valid] == -1).all(), name
