"""Generates the golden fixtures in tests/golden/ by running the REFERENCE's own
code (apoc/fused-block-sparse-attention, src/) on seeded inputs on the CPU.

Run from the repo root, in a container where the reference is mounted:
    python tests/golden/make_golden.py --ref /path/to/reference

Fixtures (npz, fp32 / int32):
  ssa_gather_*.npz    BlockSparseSSA gather path (src/ssa_model.py:121-201, _gather_and_attend
                      :57-90): selection from a supplied raw score matrix, output and
                      autograd gradients w.r.t. q, k, v.  The raw scores are exact
                      products of small-integer features plus a j/1024 tie breaker, so
                      the ranking is identical in any summation order.
  triton_interp_*.npz the reference Triton kernel (src/triton_kernel.py) run by the Triton
                      CPU interpreter (TRITON_INTERPRET=1): forward + backward with gate,
                      causal and non-causal (duplicates in sel).
  qwen_*.npz          qwen_blocksparse.blocksparse_forward with SelectMax / SelectAll / the
                      all-blocks fast path (src/qwen_blocksparse.py:29-121), GQA, padded L.
  lsh_*.npz           LSHBucketSSA's inference selection (src/ssa_model.py:438-470): the raw
                      block summaries it hashes (mean of sel_q, max(mean, max) of sel_k),
                      its planes R, and the selection it attends with, decoded from the
                      gathered keys (key rows carry their block id) and the -inf mask it
                      hands to _sdpa (invalid picks).
  centroid_*.npz      CentroidSSA's routing (src/ssa_model.py:254-299): its selector summaries,
                      centroids, the head-averaged block means its refine step scores with,
                      and the selection it attends with (read back like lsh_*.npz).
  selectors.npz       SelectOracle (random mass), SelectRandom (its CPU draws), SelectLastTok,
                      SelectMaxQMax and SelectTwoStage (src/qwen_blocksparse.py:124-299) on
                      one seeded GQA input with a padded last block.
  module_*.npz        whole modules through their reference (CPU gather / SDPA) path:
                      BlockSparseSSA (causal + gate with a padded L, non-causal),
                      LSHBucketSSA (causal, gate) and CentroidSSA (plain routing and
                      the refine step) with seeded weights: the input, the upstream
                      gradient, every parameter, the output and the gradients of
                      sum(out * dout) w.r.t. the input and every parameter, plus the
                      selection the module attended with (BlockSparseSSA).
  rope.npz            transformers' apply_rotary_pos_emb (qwen3_5_moe) on bf16 inputs, and
                      the cos/sin of Qwen3_5MoeTextRotaryEmbedding for text positions.
"""
import argparse
import os
import sys

import numpy as np
import torch

OUT = os.path.dirname(os.path.abspath(__file__))


def save(name, **arrs):
    path = os.path.join(OUT, name)
    out = {}
    for k, v in arrs.items():
        if isinstance(v, torch.Tensor):
            v = v.detach().cpu()
            v = v.float().numpy() if v.is_floating_point() else v.to(torch.int32).numpy()
        out[k] = np.asarray(v)
    np.savez_compressed(path, **out)
    print("wrote", path, sum(a.nbytes for a in out.values()), "bytes")


def ssa_gather_case(name, B, H, L, dh, bs, topk, causal, gate, seed):
    import ssa_model
    torch.manual_seed(seed)
    d = H * dh
    nblk = L // bs
    m = ssa_model.BlockSparseSSA(d, H, block=bs, topk=topk, causal=causal, gate=gate)
    m.eval()
    qkv = torch.randn(B, L, 3 * d, requires_grad=True)
    fa = torch.randint(-4, 5, (B, nblk, 16)).float()
    fb = torch.randint(-4, 5, (B, nblk, 16)).float()
    fa[..., 0] = 1.0
    fb[..., 0] = torch.arange(nblk).float() / 1024.0
    raw = fa @ fb.transpose(-1, -2)
    del m.qkv
    m.qkv = lambda x: qkv
    del m.o
    m.o = lambda x: x
    m._scores = lambda x, B_, nblk_, Bs_: raw
    captured = {}
    orig = ssa_model._gather_and_attend

    def spy(q, k, v, sel, *a, **kw):
        captured["sel"] = sel.clone()
        return orig(q, k, v, sel, *a, **kw)

    ssa_model._gather_and_attend = spy
    try:
        out = m(torch.zeros(B, L, d))                   # (B, L, d)
    finally:
        ssa_model._gather_and_attend = orig
    do = torch.randn_like(out)
    (out * do).sum().backward()
    g = qkv.grad.view(B, L, 3, H, dh)
    qkv_v = qkv.detach().view(B, L, 3, H, dh)
    to_bhld = lambda t: t.permute(0, 2, 1, 3).contiguous()
    save(name, q=to_bhld(qkv_v[:, :, 0]), k=to_bhld(qkv_v[:, :, 1]), v=to_bhld(qkv_v[:, :, 2]),
         fa=fa, fb=fb, sel=captured["sel"], o=to_bhld(out.detach().view(B, L, H, dh)),
         do=to_bhld(do.view(B, L, H, dh)), dq=to_bhld(g[:, :, 0]), dk=to_bhld(g[:, :, 1]),
         dv=to_bhld(g[:, :, 2]),
         meta=np.array([B, H, L, dh, bs, topk, int(causal), int(gate)], np.int32))


def triton_interp_case(name, B, H, L, dh, bs, kk, causal, seed):
    os.environ["TRITON_INTERPRET"] = "1"
    import triton_kernel
    torch.manual_seed(seed)
    nblk = L // bs
    q, k, v, do = (torch.randn(B, H, L, dh) for _ in range(4))
    own = torch.arange(nblk).view(1, nblk, 1).expand(B, nblk, 1)
    rnd = torch.randint(0, nblk, (B, nblk, kk - 1))
    sel = torch.cat([own, rnd], -1).to(torch.int32)
    gate = torch.randn(B, nblk, kk) * 0.5
    o = triton_kernel.bsattn_forward(q, k, v, sel, gate, causal=causal)
    dq, dk, dv = triton_kernel.bsattn_backward(q, k, v, sel, o, do, gate, causal=causal)
    save(name, q=q, k=k, v=v, do=do, sel=sel, gate=gate, o=o, dq=dq, dk=dk, dv=dv,
         meta=np.array([B, H, L, dh, bs, kk, int(causal)], np.int32))


def qwen_case(name, B, Hq, Hkv, L, d, bs, topk, seed, selector):
    import qwen_blocksparse as qb
    torch.manual_seed(seed)
    q = torch.randn(B, Hq, L, d)
    k = torch.randn(B, Hkv, L, d)
    v = torch.randn(B, Hkv, L, d)
    if selector == "max":
        S = qb.SelectMax(topk, bs, sink=True)
        idx = S.select(q, k)
        out = qb.blocksparse_forward(q, k, v, selector=S, topk=topk, bs=bs, causal=True, q_chunk=3)
    elif selector == "all":
        S = qb.SelectAll(bs)
        idx = S.select(q, k)
        out = qb.blocksparse_forward(q, k, v, selector=S, topk=0, bs=bs, causal=True, q_chunk=3)
    else:  # all-blocks fast path (SDPA)
        idx = torch.zeros(1, dtype=torch.int32)
        out = qb.blocksparse_forward(q, k, v, selector=None, topk=10 ** 6, bs=bs, causal=True)
    save(name, q=q, k=k, v=v, idx=idx, o=out, meta=np.array([B, Hq, Hkv, L, d, bs, topk], np.int32))


def rope_case(name):
    import transformers.models.qwen3_5_moe.modeling_qwen3_5_moe as M
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    torch.manual_seed(7)
    B, Hq, Hkv, L, D, rot, theta = 1, 4, 2, 96, 256, 64, 1e7
    cfg = Qwen3_5MoeTextConfig(head_dim=D, hidden_size=512, num_attention_heads=Hq,
                               num_key_value_heads=Hkv,
                               rope_parameters={"rope_type": "default", "rope_theta": theta,
                                                "partial_rotary_factor": rot / D,
                                                "mrope_section": [11, 11, 10]})
    emb = M.Qwen3_5MoeTextRotaryEmbedding(cfg)
    x = torch.zeros(B, L, 8, dtype=torch.bfloat16)
    cos, sin = emb(x, torch.arange(L).view(1, L))      # (B, L, rot) bf16
    q = torch.randn(B, Hq, L, D).to(torch.bfloat16)
    k = torch.randn(B, Hkv, L, D).to(torch.bfloat16)
    qe, ke = M.apply_rotary_pos_emb(q, k, cos, sin)
    save(name, q=q.float(), k=k.float(), cos=cos.float(), sin=sin.float(), qe=qe.float(),
         ke=ke.float(), meta=np.array([B, Hq, Hkv, L, D, rot], np.int32), theta=np.array([theta]))


def lsh_case(name, B, L, d, h, bs, topk, n_rounds, n_buckets, cap, causal, seed):
    import ssa_model
    torch.manual_seed(seed)
    nblk = L // bs
    m = ssa_model.LSHBucketSSA(d, h, block=bs, topk=topk, n_rounds=n_rounds, n_buckets=n_buckets,
                               cap=cap, causal=causal)
    m.eval()
    x = torch.randn(B, L, d)
    dh = d // h
    # keys carry their block id in dim 0, so the gathered keys reveal the selection
    kid = (torch.arange(L) // bs).float().view(1, L, 1, 1).expand(B, L, h, dh).clone()
    qkv = torch.cat([torch.zeros(B, L, d), kid.reshape(B, L, d), torch.zeros(B, L, d)], -1)
    del m.qkv
    m.qkv = lambda x_: qkv
    cap_ = {}

    def spy(q, k, v, mask):
        cap_["k"], cap_["mask"] = k.detach().clone(), mask.detach().clone()
        return torch.zeros_like(q)

    orig = ssa_model._sdpa
    ssa_model._sdpa = spy
    try:
        with torch.no_grad():
            m(x)
    finally:
        ssa_model._sdpa = orig
    kk = cap_["k"].shape[1] // bs
    ksel = cap_["k"].view(B, h, nblk, kk, bs, dh)[:, 0, :, :, 0, 0].round().to(torch.int32)
    # last query row of each block: under the causal triangle it still sees the whole
    # own block, so a slot is invalid exactly when its additive mask is -inf there
    mlast = cap_["mask"].reshape(B, h, nblk, -1, kk * bs)[:, 0, :, -1, :]
    valid = torch.isfinite(mlast.reshape(B, nblk, kk, bs)[..., 0])
    with torch.no_grad():
        s = m.sel_dim
        a_raw = m.sel_q(x).view(B, nblk, bs, s).mean(2)
        skv = m.sel_k(x).view(B, nblk, bs, s)
        b_raw = torch.maximum(skv.mean(2), skv.max(2).values)
    save(name, a=a_raw, b=b_raw, planes=m.R, scale=torch.tensor(m.scale), sel=ksel,
         valid=valid.to(torch.int32), cap=torch.tensor(cap), topk=torch.tensor(topk),
         causal=torch.tensor(int(causal)))


def centroid_case(name, B, L, d, h, bs, C, cpq, cap, refine, seed):
    import ssa_model
    torch.manual_seed(seed)
    nblk = L // bs
    m = ssa_model.CentroidSSA(d, h, block=bs, n_centroids=C, cpq=cpq, cap=cap, refine_topk=refine)
    m.eval()
    x = torch.randn(B, L, d)
    dh = d // h
    qkv_real = m.qkv(x).detach()
    kid = (torch.arange(L) // bs).float().view(1, L, 1, 1).expand(B, L, h, dh).clone()
    q_real, k_real, _ = qkv_real.chunk(3, -1)
    # keys carry their block id; the refine step scores with the real q/k, so feed those
    # through a second projection call order: the module calls qkv once
    qkv = torch.cat([q_real, kid.reshape(B, L, d), torch.zeros(B, L, d)], -1)
    del m.qkv
    m.qkv = lambda x_: qkv
    cap_ = {}

    def spy(q, k, v, mask):
        cap_["k"], cap_["mask"] = k.detach().clone(), mask.detach().clone()
        return torch.zeros_like(q)

    orig = ssa_model._sdpa
    ssa_model._sdpa = spy
    try:
        with torch.no_grad():
            m(x)
    finally:
        ssa_model._sdpa = orig
    kk = cap_["k"].shape[1] // bs
    ksel = cap_["k"].view(B, h, nblk, kk, bs, dh)[:, 0, :, :, 0, 0].round().to(torch.int32)
    mlast = cap_["mask"].reshape(B, h, nblk, -1, kk * bs)[:, 0, :, -1, :]
    valid = torch.isfinite(mlast.reshape(B, nblk, kk, bs)[..., 0])
    with torch.no_grad():
        s = m.sel_dim
        sq = m.sel_q(x).view(B, nblk, bs, s).mean(2)
        skv = m.sel_k(x).view(B, nblk, bs, s)
        sk = torch.maximum(skv.mean(2), skv.max(2).values)
        kid_blk = kid.reshape(B, L, h, dh).transpose(1, 2).reshape(B, h, nblk, bs, dh).mean(3).mean(1)
        q_blk = q_real.view(B, L, h, dh).transpose(1, 2).reshape(B, h, nblk, bs, dh).mean(3).mean(1)
    save(name, sq=sq, sk=sk, cent=m.cent, q_blk=q_blk, k_blk=kid_blk, sel=ksel,
         valid=valid.to(torch.int32), cpq=torch.tensor(cpq), cap=torch.tensor(cap),
         refine=torch.tensor(refine if refine is not None else -1))


def module_case(name, cls, kwargs, B, L, seed):
    import json

    import ssa_model
    torch.manual_seed(seed)
    m = getattr(ssa_model, cls)(**kwargs)
    d = kwargs["d"]
    x = torch.randn(B, L, d, requires_grad=True)
    cap_ = {}
    orig = ssa_model._gather_and_attend

    def spy(q, k, v, sel, *a, **kw):
        cap_["sel"] = sel.clone()
        return orig(q, k, v, sel, *a, **kw)

    ssa_model._gather_and_attend = spy
    try:
        out = m(x)
    finally:
        ssa_model._gather_and_attend = orig
    dout = torch.randn_like(out)
    (out * dout).sum().backward()
    arrs = dict(x=x, dout=dout, out=out, dx=x.grad, cls=np.array(cls),
                kwargs=np.array(json.dumps(kwargs)), meta=np.array([B, L, d, seed], np.int32))
    for n, prm in m.named_parameters():
        arrs["p:" + n] = prm
        arrs["g:" + n] = prm.grad if prm.grad is not None else torch.zeros_like(prm)
    for n, buf in m.named_buffers():
        arrs["b:" + n] = buf
    if "sel" in cap_:
        arrs["sel"] = cap_["sel"]
    save(name, **arrs)


def selectors_case(name, B, Hq, Hkv, L, d, bs, topk, seed):
    import qwen_blocksparse as qb
    torch.manual_seed(seed)
    q = torch.randn(B, Hq, L, d)
    k = torch.randn(B, Hkv, L, d)
    nblk = (L + bs - 1) // bs
    mass = torch.rand(B, Hkv, nblk, nblk)
    g = torch.Generator().manual_seed(3)
    rnd = torch.rand(B, Hkv, nblk, nblk, generator=g)
    out = dict(q=q, k=k, mass=mass, rnd=rnd, bs=torch.tensor(bs), topk=torch.tensor(topk))
    out["oracle"] = qb.SelectOracle(topk, bs).select_from_mass(mass)
    out["random"] = qb.SelectRandom(topk, bs, seed=3).select(q, k)
    out["lasttok"] = qb.SelectLastTok(topk, bs).select(q, k)
    out["qmax"] = qb.SelectMaxQMax(topk, bs).select(q, k)
    out["twostage"] = qb.SelectTwoStage(topk, bs, over=2).select(q, k)
    save(name, **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BSA_REFERENCE", ""))
    ap.add_argument("--only", default="", help="generate only fixtures whose name starts with this")
    a = ap.parse_args()
    src = os.path.join(a.ref, "src")
    if not os.path.isdir(src):
        sys.exit("reference src/ not found; pass --ref")
    sys.path.insert(0, src)
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    cases = [
        ("ssa_gather_causal_gate.npz", ssa_gather_case, (1, 2, 512, 64, 64, 3, True, True, 1)),
        ("ssa_gather_causal.npz", ssa_gather_case, (2, 1, 256, 64, 32, 4, True, False, 2)),
        ("ssa_gather_noncausal_gate.npz", ssa_gather_case, (1, 2, 256, 64, 64, 2, False, True, 3)),
        ("triton_interp_causal.npz", triton_interp_case, (1, 2, 256, 64, 64, 4, True, 4)),
        ("triton_interp_noncausal.npz", triton_interp_case, (1, 2, 256, 64, 64, 4, False, 5)),
        ("qwen_selectmax.npz", qwen_case, (1, 4, 2, 448, 64, 64, 3, 6, "max")),
        ("qwen_selectall.npz", qwen_case, (1, 4, 2, 200, 64, 32, 0, 8, "all")),
        ("qwen_fastpath.npz", qwen_case, (1, 4, 2, 256, 64, 64, 0, 9, "fast")),
        ("lsh_causal.npz", lsh_case, (2, 2048, 64, 2, 16, 6, 4, 8, 8, True, 10)),
        ("lsh_noncausal.npz", lsh_case, (1, 1024, 64, 2, 16, 4, 3, 6, 5, False, 11)),
        ("selectors.npz", selectors_case, (1, 4, 2, 600, 16, 32, 3, 12)),
        ("centroid_plain.npz", centroid_case, (2, 2048, 64, 2, 32, 8, 2, 6, None, 13)),
        ("centroid_refine.npz", centroid_case, (1, 2048, 64, 2, 32, 8, 3, 8, 5, 14)),
        ("module_ssa_causal_gate.npz", module_case,
         ("BlockSparseSSA", dict(d=64, h=2, block=64, topk=4, causal=True, gate=True), 2, 1000, 15)),
        ("module_ssa_noncausal.npz", module_case,
         ("BlockSparseSSA", dict(d=128, h=4, block=32, topk=3, causal=False, gate=False), 1, 512, 16)),
        ("module_lsh_causal_gate.npz", module_case,
         ("LSHBucketSSA", dict(d=64, h=2, block=32, topk=4, n_rounds=3, n_buckets=6, cap=4,
                               causal=True, gate=True), 1, 1024, 17)),
        ("module_centroid.npz", module_case,
         ("CentroidSSA", dict(d=64, h=2, block=32, n_centroids=6, cpq=2, cap=3, gate=True), 1, 1024,
          18)),
        ("module_centroid_refine.npz", module_case,
         ("CentroidSSA", dict(d=64, h=2, block=32, n_centroids=6, cpq=2, cap=3, refine_topk=3),
          1, 1024, 19)),
    ]
    for name, fn, args in cases:
        if name.startswith(a.only):
            fn(name, *args)
    if "rope.npz".startswith(a.only):
        rope_case("rope.npz")

if __name__ == "__main__":
    main()
