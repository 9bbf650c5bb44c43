"""GPU parity of the attention kernels (through the C ABI) against the float64
oracle and the reference's golden outputs.

Tolerances: bf16/f16 — |got - ref| <= 2e-2 + 1e-2 * |ref| elementwise (the
north-star bound, allclose form); fp32 — max-abs 1e-5 (gradients 2e-5, the golden's own fp32 noise)."""
import pytest
import torch
import torch.nn.functional as F

from conftest import golden
from oracle import oracle as O

pytestmark = pytest.mark.gpu

BF16_ABS, BF16_REL, F32_ABS = 2e-2, 1e-2, 1e-5


def _cmp(got, ref, dtype, what, abs_tol=None):
    """fp32: max-abs <= tol.  bf16/f16: |got - ref| <= atol + rtol * |ref| elementwise
    with atol 2e-2, rtol 1e-2 (the allclose form of the north-star bound)."""
    got = got.detach().double().cpu()
    ref = torch.as_tensor(ref).double().cpu()
    diff = (got - ref).abs()
    err = diff.max().item()
    if dtype == torch.float32:
        tol = F32_ABS if abs_tol is None else abs_tol
        assert err <= tol, "%s: max-abs %.3g > %.3g" % (what, err, tol)
    else:
        atol = BF16_ABS if abs_tol is None else abs_tol
        excess = (diff - (atol + BF16_REL * ref.abs())).max().item()
        assert excess <= 0, "%s: max-abs %.3g exceeds atol+rtol*|ref| by %.3g" % (what, err, excess)


def _dev(g, names, dtype, dev):
    return [torch.from_numpy(g[n]).to(dev, dtype) for n in names]


@pytest.mark.parametrize("name", ["triton_interp_causal.npz", "triton_interp_noncausal.npz"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_bsattn_matches_reference_triton_kernel(cuda, name, dtype):
    import triton_kernel as tk
    g = golden(name)
    B, H, L, dh, bs, kk, causal = [int(x) for x in g["meta"]]
    q, k, v, do = _dev(g, ["q", "k", "v", "do"], dtype, cuda)
    sel = torch.from_numpy(g["sel"]).to(cuda)
    gate = torch.from_numpy(g["gate"]).to(cuda)
    o = tk.bsattn_forward(q, k, v, sel, gate, causal=bool(causal))
    dq, dk, dv = tk.bsattn_backward(q, k, v, sel, o, do, gate, causal=bool(causal))
    torch.cuda.synchronize()
    if dtype == torch.float32:
        refs = (g["o"], g["dq"], g["dk"], g["dv"])
    else:   # low precision: the oracle on the same rounded inputs
        c = [t.cpu() for t in (q, k, v, sel, do, gate)]
        ro = O.attention(c[0], c[1], c[2], c[3], c[5], bs=bs, causal=bool(causal))
        rq, rk, rv, _ = O.attention_grads(c[0], c[1], c[2], c[3], c[4], c[5], bs=bs, causal=bool(causal))
        refs = (ro, rq, rk, rv)
    for got, ref, w in zip((o, dq, dk, dv), refs, "o dq dk dv".split()):
        tol = (1e-5 if w == "o" else 2e-5) if dtype == torch.float32 else None
        _cmp(got, ref, dtype, w, abs_tol=tol)


@pytest.mark.parametrize("name", ["ssa_gather_causal_gate.npz", "ssa_gather_causal.npz",
                                  "ssa_gather_noncausal_gate.npz"])
def test_bsattn_matches_reference_gather_path_fp32(cuda, name):
    import triton_kernel as tk
    g = golden(name)
    B, H, L, dh, bs, topk, causal, gate = [int(x) for x in g["meta"]]
    q, k, v, do = _dev(g, ["q", "k", "v", "do"], torch.float32, cuda)
    sel = torch.from_numpy(g["sel"]).to(cuda)
    gt = None
    if gate:
        raw = torch.from_numpy(g["fa"]) @ torch.from_numpy(g["fb"]).transpose(-1, -2)
        gt = F.logsigmoid(torch.gather(raw, -1, sel.cpu().long())).to(cuda)
    for t in (q, k, v):
        t.requires_grad_(True)
    o = tk.bsattn(q, k, v, sel, gt, causal=bool(causal))
    (o * do).sum().backward()
    _cmp(o, g["o"], torch.float32, "o")
    _cmp(q.grad, g["dq"], torch.float32, "dq", 2e-5)
    _cmp(k.grad, g["dk"], torch.float32, "dk", 2e-5)
    _cmp(v.grad, g["dv"], torch.float32, "dv", 2e-5)


def _random_case(B, H, L, D, bs, kk, dtype, dev, seed, shared=False):
    gen = torch.Generator().manual_seed(seed)
    nblk = L // bs
    q, k, v, do = (torch.randn(B, H, L, D, generator=gen) for _ in range(4))
    shape = (B, nblk, kk) if shared else (B, H, nblk, kk)
    sel = torch.randint(0, nblk, shape, generator=gen)
    sel[..., 0] = torch.arange(nblk).view(*([1] * (len(shape) - 2)), nblk)
    gate = torch.randn(shape, generator=gen) * 0.3
    return [t.to(dev, dtype) for t in (q, k, v, do)] + [sel.to(dev, torch.int32), gate.to(dev)]


@pytest.mark.parametrize("bs,D", [(16, 64), (32, 64), (64, 64), (128, 64), (64, 128)])
@pytest.mark.parametrize("shared", [False, True])
def test_bf16_shapes_vs_oracle(cuda, bs, D, shared):
    import triton_kernel as tk
    B, H, L, kk = 2, 2, 1024, 5
    q, k, v, do, sel, gate = _random_case(B, H, L, D, bs, kk, torch.bfloat16, cuda, bs + D, shared)
    for t in (q, k, v):
        t.requires_grad_(True)
    o = tk.bsattn(q, k, v, sel, gate, causal=True)
    (o.float() * do.float()).sum().backward()
    qc, kc, vc, dc = (t.detach().cpu() for t in (q, k, v, do))
    ro = O.attention(qc, kc, vc, sel.cpu(), gate.cpu(), bs=bs, causal=True)
    rq, rk, rv, _ = O.attention_grads(qc, kc, vc, sel.cpu(), dc, gate.cpu(), bs=bs, causal=True)
    _cmp(o, ro, torch.bfloat16, "o")
    _cmp(q.grad, rq, torch.bfloat16, "dq")
    _cmp(k.grad, rk, torch.bfloat16, "dk")
    _cmp(v.grad, rv, torch.bfloat16, "dv")


@pytest.mark.parametrize("mode,causal", [(0, True), (1, True), (1, False)])
def test_gate_gradient_vs_oracle(cuda, mode, causal):
    """dgate per slot; under TOKEN masks a repeated block id gets no gradient."""
    import triton_kernel as tk
    B, H, L, D, bs, kk = 1, 2, 512, 64, 64, 4
    q, k, v, do, sel, gate = _random_case(B, H, L, D, bs, kk, torch.float32, cuda, 11, shared=True)
    if mode == 1:
        sel[:, 5:, 2] = sel[:, 5:, 1]    # repeated ids
    gate.requires_grad_(True)
    o = tk.bsattn(q, k, v, sel, gate, causal=causal, gate_grad=True, mask_mode=mode)
    (o * do).sum().backward()
    _, _, _, rg = O.attention_grads(q.cpu(), k.cpu(), v.cpu(), sel.cpu(), do.cpu(), gate.detach().cpu(),
                                    bs=bs, causal=causal, mask_mode=mode, want_dgate=True)
    _cmp(gate.grad, rg, torch.float32, "dgate", 1e-4)


def test_backward_is_deterministic_with_hub_blocks(cuda):
    """Every query block selects blocks 0 and 1, so those bins span many dK/dV chunks."""
    import triton_kernel as tk
    B, H, L, D, bs, kk = 1, 2, 8192, 64, 64, 6
    q, k, v, do, sel, gate = _random_case(B, H, L, D, bs, kk, torch.bfloat16, cuda, 5)
    sel[..., 1] = 0
    sel[..., 2] = 1
    r1 = tk.bsattn_backward(q, k, v, sel, None, do, gate, causal=True)
    r2 = tk.bsattn_backward(q, k, v, sel, None, do, gate, causal=True)
    for a, b in zip(r1, r2):
        assert torch.equal(a, b)
    qc, kc, vc, dc = (t.cpu() for t in (q, k, v, do))
    rq, rk, rv, _ = O.attention_grads(qc, kc, vc, sel.cpu(), dc, gate.cpu(), bs=bs, causal=True)
    _cmp(r1[0], rq, torch.bfloat16, "dq")
    _cmp(r1[1], rk, torch.bfloat16, "dk")
    _cmp(r1[2], rv, torch.bfloat16, "dv")


def test_backward_with_saved_lse_equals_recompute(cuda):
    """bsattn_backward(..., lse=) with the (o, lse) of bsattn_forward_lse gives the
    same gradients, bit for bit, as the recomputing form."""
    import triton_kernel as tk
    q, k, v, do, sel, gate = _random_case(1, 2, 2048, 64, 64, 7, torch.bfloat16, cuda, 12)
    o, lse = tk.bsattn_forward_lse(q, k, v, sel, gate, causal=True)
    a = tk.bsattn_backward(q, k, v, sel, o, do, gate, causal=True, lse=lse)
    b = tk.bsattn_backward(q, k, v, sel, None, do, gate, causal=True)
    assert torch.equal(o, tk.bsattn_forward(q, k, v, sel, gate, causal=True))
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_strided_inputs_read_in_place(cuda):
    """q/k/v as transposed views of a (B, L, 3, H, D) projection (no copies)."""
    import triton_kernel as tk
    B, H, L, D, bs, kk = 1, 4, 1024, 64, 64, 4
    gen = torch.Generator().manual_seed(3)
    qkv = torch.randn(B, L, 3, H, D, generator=gen).to(cuda, torch.bfloat16)
    q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
    sel = _random_case(B, H, L, D, bs, kk, torch.bfloat16, cuda, 4, shared=True)[4]
    o = tk.bsattn_forward(q, k, v, sel, None, causal=True)
    ro = O.attention(q.cpu(), k.cpu(), v.cpu(), sel.cpu(), bs=bs, causal=True)
    _cmp(o, ro, torch.bfloat16, "o")


def test_bad_index_sets_status_word(cuda):
    import _bsa
    import triton_kernel as tk
    B, H, L, D, bs, kk = 1, 1, 256, 64, 64, 3
    q, k, v, do, sel, gate = _random_case(B, H, L, D, bs, kk, torch.bfloat16, cuda, 9, shared=True)
    _bsa.check_status(cuda)
    sel[0, 2, 1] = 99
    tk.bsattn_forward(q, k, v, sel, None, causal=True)
    with pytest.raises(_bsa.BsaError) as e:
        _bsa.check_status(cuda)
    assert e.value.status == _bsa.ERR_INDEX


def test_module_drop_in_runs_and_trains(cuda):
    import ssa_model
    torch.manual_seed(0)
    m = ssa_model.BlockSparseSSA(256, 4, block=64, topk=4, causal=True, gate=True).to(cuda)
    x = torch.randn(2, 1000, 256, device=cuda)
    y = m(x, needle_pos=torch.tensor([5, 700], device=cuda))
    y.sum().backward()
    assert y.shape == x.shape and torch.isfinite(y).all()
    assert m.sel_q[0].weight.grad is not None and m.sel_q[0].weight.grad.abs().sum() > 0


@pytest.mark.parametrize("B,H,L,kk,causal,mode,bs", [(1, 2, 4096, 17, True, 0, 64),
                                                     (2, 2, 1984, 5, False, 0, 64),
                                                     (1, 4, 2048 + 64, 9, True, 1, 64),
                                                     (1, 2, 8192, 17, True, 0, 128),
                                                     (2, 2, 3968, 6, False, 0, 128),
                                                     (1, 4, 4096 + 128, 9, True, 1, 128),
                                                     (1, 2, 8192 - 37, 9, True, 0, 128),
                                                     (1, 2, 4096 - 5, 9, True, 1, 64)])
def test_tcgen05_forward_matches_mma_sync_path(cuda, monkeypatch, B, H, L, kk, causal, mode, bs):
    """The block-64 and block-128 D-64 forwards run on tcgen05 (TMEM accumulators);
    the mma.sync kernel (selected with BSA_FWD_LEGACY) must agree, and both match
    the oracle."""
    import _bsa
    gen = torch.Generator().manual_seed(L + kk)
    q, k, v = (torch.randn(B, H, L, 64, generator=gen).to(torch.bfloat16) for _ in range(3))
    nblk = (L + bs - 1) // bs                     # ragged L: a partial last block
    sel = torch.randint(0, nblk, (B, H, nblk, kk), generator=gen)
    sel[..., 0] = torch.arange(nblk)
    gate = (torch.randn(B, H, nblk, kk, generator=gen) * 0.3) if mode == 0 else None
    args = [t.to(cuda) for t in (q, k, v)] + [sel.to(cuda, torch.int32),
                                              gate.to(cuda) if gate is not None else None]
    o5, l5 = _bsa.attn_fwd(*args, bs=bs, causal=causal, mask_mode=mode)
    monkeypatch.setenv("BSA_FWD_LEGACY", "1")
    o1, l1 = _bsa.attn_fwd(*args, bs=bs, causal=causal, mask_mode=mode)
    ref = O.attention(q, k, v, sel, gate, bs=bs, causal=causal, mask_mode=mode)
    _cmp(o5, ref, torch.bfloat16, "o tcgen05")
    _cmp(o1, ref, torch.bfloat16, "o mma.sync")
    assert (l5 - l1).abs().max().item() < 1e-4


@pytest.mark.parametrize("Hq,Hkv,shared,hub,L,mode", [(2, 2, False, False, 4096, 0),
                                                   (4, 4, True, True, 4096, 0),
                                                   (4, 2, False, False, 4096, 0),
                                                   (2, 2, False, False, 4096 - 37, 0),
                                                   (2, 1, True, True, 3072 + 64, 1)])
def test_tcgen05_backward_matches_mma_sync_path(cuda, monkeypatch, Hq, Hkv, shared, hub, L, mode):
    """Block 64 / D 64 backward: dK/dV and dQ (+ dgate) run on tcgen05 by default;
    the persistent tcgen05 dQ kernel (BSA_DQ_F5=0 BSA_DQ_TC05=1) and the mma.sync
    kernels (BSA_BWD_LEGACY) must agree closely, and all match the oracle (incl.
    GQA, hub blocks, a ragged last block and TOKEN masks with repeated ids)."""
    import _bsa
    B, D, bs, kk = 1, 64, 64, 9
    gen = torch.Generator().manual_seed(Hq * 10 + Hkv + hub + L)
    nblk = (L + bs - 1) // bs
    q, do = (torch.randn(B, Hq, L, D, generator=gen).to(torch.bfloat16) for _ in range(2))
    k, v = (torch.randn(B, Hkv, L, D, generator=gen).to(torch.bfloat16) for _ in range(2))
    shape = (B, nblk, kk) if shared else (B, Hkv, nblk, kk)
    sel = torch.randint(0, nblk, shape, generator=gen)
    sel[..., 0] = torch.arange(nblk).view(*([1] * (len(shape) - 2)), nblk)
    if hub:
        sel[..., 1] = 0
        sel[..., 2] = 3
    if mode == 1:
        sel[..., 5] = sel[..., 4]     # repeated ids: no attention, no gate gradient
    gate = torch.randn(shape, generator=gen) * 0.3
    dev = [t.to(cuda) for t in (q, k, v, do)]
    sd, gd = sel.to(cuda, torch.int32), gate.to(cuda)
    o, lse = _bsa.attn_fwd(dev[0], dev[1], dev[2], sd, gd, bs=bs, causal=True, mask_mode=mode)

    def run():
        return _bsa.attn_bwd(dev[0], dev[1], dev[2], o, dev[3], sd, lse, gd, bs=bs, causal=True,
                             want_dgate=True, mask_mode=mode)
    rf = run()
    monkeypatch.setenv("BSA_DQ_F5", "0")
    monkeypatch.setenv("BSA_DQ_TC05", "1")
    r5 = run()
    monkeypatch.setenv("BSA_BWD_LEGACY", "1")
    r1 = run()
    for r in (rf, r5):
        assert torch.allclose(r[3], r1[3], atol=2e-2, rtol=2e-2), (r[3] - r1[3]).abs().max().item()
    rq, rk, rv, rg = O.attention_grads(q, k, v, sel, do, gate, bs=bs, causal=True, mask_mode=mode,
                                       want_dgate=True)
    for i, (ref, name) in enumerate(((rq, "dq"), (rk, "dk"), (rv, "dv"))):
        _cmp(rf[i], ref, torch.bfloat16, name + " tcgen05")
        _cmp(r5[i], ref, torch.bfloat16, name + " tcgen05 persistent")
        _cmp(r1[i], ref, torch.bfloat16, name + " mma.sync")
    dg = rf[3].cpu()                      # per query head -> the gate's own shape
    dg = dg.sum(1) if shared else dg.view(B, Hkv, Hq // Hkv, nblk, kk).sum(2)
    # dgate sums 64 x 64 dS terms whose row offset rowsum(dO * O) uses the bf16-rounded
    # output: the bound scales with the gradient's own magnitude
    _cmp(dg, rg, torch.bfloat16, "dgate tcgen05", abs_tol=0.05 * float(torch.as_tensor(rg).abs().max()))


@pytest.mark.parametrize("L,with_gate", [(2048 - 50, True), (3072, False)])
def test_tcgen05_forward_d256_qwen_layout(cuda, monkeypatch, L, with_gate):
    """Block 128 / D 256 (the Qwen configuration) on the tcgen05 kernel: GQA, TOKEN
    masks with repeated ids, a ragged last block and the sigmoid output gate, against
    the mma.sync kernel and the oracle."""
    import _bsa
    B, Hq, Hkv, D, bs, kk = 1, 4, 2, 256, 128, 7
    gen = torch.Generator().manual_seed(L)
    q = torch.randn(B, Hq, L, D, generator=gen).to(torch.bfloat16)
    k, v = (torch.randn(B, Hkv, L, D, generator=gen).to(torch.bfloat16) for _ in range(2))
    nblk = (L + bs - 1) // bs
    sel = torch.randint(0, nblk, (B, Hkv, nblk, kk), generator=gen)
    sel[..., 0] = torch.arange(nblk)
    sel[..., 3] = sel[..., 2]
    og = torch.randn(B, Hq, L, D, generator=gen).to(torch.bfloat16) if with_gate else None
    args = [t.to(cuda) for t in (q, k, v)] + [sel.to(cuda, torch.int32), None]
    kw = dict(bs=bs, causal=True, mask_mode=_bsa.MASK_TOKEN,
              out_gate=og.to(cuda) if og is not None else None)
    o5, l5 = _bsa.attn_fwd(*args, **kw)
    monkeypatch.setenv("BSA_FWD_LEGACY", "1")
    o1, l1 = _bsa.attn_fwd(*args, **kw)
    ref = O.attention(q, k, v, sel, None, bs=bs, causal=True, mask_mode=1, out_gate=og)
    _cmp(o5, ref, torch.bfloat16, "o tcgen05")
    _cmp(o1, ref, torch.bfloat16, "o mma.sync")
    assert (l5 - l1).abs().max().item() < 1e-4


def test_tcgen05_forward_d256_identity_selection(cuda, monkeypatch):
    """All-blocks mode (sel = NULL: every causal block) on the block-128 / D-256
    tcgen05 kernel equals the mma.sync kernel and the oracle (dense causal)."""
    import _bsa
    B, Hq, Hkv, D, bs, L = 1, 4, 2, 256, 128, 1500
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(B, Hq, L, D, generator=gen).to(torch.bfloat16)
    k, v = (torch.randn(B, Hkv, L, D, generator=gen).to(torch.bfloat16) for _ in range(2))
    nblk = (L + bs - 1) // bs
    args = [t.to(cuda) for t in (q, k, v)] + [None, None]
    o5, _ = _bsa.attn_fwd(*args, bs=bs, causal=True, mask_mode=_bsa.MASK_TOKEN)
    monkeypatch.setenv("BSA_FWD_LEGACY", "1")
    o1, _ = _bsa.attn_fwd(*args, bs=bs, causal=True, mask_mode=_bsa.MASK_TOKEN)
    ident = torch.arange(nblk).view(1, 1, 1, nblk).expand(B, Hkv, nblk, nblk)
    ref = O.attention(q, k, v, ident, None, bs=bs, causal=True, mask_mode=1)
    _cmp(o5, ref, torch.bfloat16, "o tcgen05")
    _cmp(o1, ref, torch.bfloat16, "o mma.sync")


@pytest.mark.parametrize("Hq,Hkv,shared,hub,L,mode", [(2, 2, False, False, 4096, 0),
                                                   (4, 4, True, True, 4096, 0),
                                                   (4, 2, False, False, 4096 - 37, 0),
                                                   (2, 1, True, True, 3072 + 64, 1)])
def test_stored_ds_dq_matches_recomputing_dq(cuda, monkeypatch, Hq, Hkv, shared, hub, L, mode):
    """Without a gate gradient the block-64 backward takes dQ from the dS tiles the
    dK/dV kernel stores (bsa_attn_dq_ds.cu); the recomputing dQ kernel
    (BSA_DQ_DS=0) must agree closely, dK/dV bit for bit, and both match the oracle
    (GQA, hub blocks, a ragged last block, TOKEN masks with repeated ids)."""
    import _bsa
    B, D, bs, kk = 1, 64, 64, 9
    gen = torch.Generator().manual_seed(Hq * 7 + Hkv + hub + L)
    nblk = (L + bs - 1) // bs
    q, do = (torch.randn(B, Hq, L, D, generator=gen).to(torch.bfloat16) for _ in range(2))
    k, v = (torch.randn(B, Hkv, L, D, generator=gen).to(torch.bfloat16) for _ in range(2))
    shape = (B, nblk, kk) if shared else (B, Hkv, nblk, kk)
    sel = torch.randint(0, nblk, shape, generator=gen)
    sel[..., 0] = torch.arange(nblk).view(*([1] * (len(shape) - 2)), nblk)
    if hub:
        sel[..., 1] = 0
        sel[..., 2] = 3
    if mode == 1:
        sel[..., 5] = sel[..., 4]
    gate = torch.randn(shape, generator=gen) * 0.3
    dev = [t.to(cuda) for t in (q, k, v, do)]
    sd, gd = sel.to(cuda, torch.int32), gate.to(cuda)
    o, lse = _bsa.attn_fwd(dev[0], dev[1], dev[2], sd, gd, bs=bs, causal=True, mask_mode=mode)

    def run():
        return _bsa.attn_bwd(dev[0], dev[1], dev[2], o, dev[3], sd, lse, gd, bs=bs, causal=True,
                             mask_mode=mode)
    r_ds = run()
    r_ds2 = run()
    monkeypatch.setenv("BSA_DQ_DS", "0")
    r_re = run()
    _bsa.check_status(cuda)
    for x, y in zip(r_ds[:3], r_ds2[:3]):
        assert torch.equal(x, y)                          # deterministic
    assert torch.equal(r_ds[1], r_re[1]) and torch.equal(r_ds[2], r_re[2])
    assert (r_ds[0].float() - r_re[0].float()).abs().max().item() < 2e-2
    rq, rk, rv, _ = O.attention_grads(q, k, v, sel, do, gate, bs=bs, causal=True, mask_mode=mode)
    _cmp(r_ds[0], rq, torch.bfloat16, "dq (stored dS)")
    _cmp(r_ds[1], rk, torch.bfloat16, "dk")
    _cmp(r_ds[2], rv, torch.bfloat16, "dv")
