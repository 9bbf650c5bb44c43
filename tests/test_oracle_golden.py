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
