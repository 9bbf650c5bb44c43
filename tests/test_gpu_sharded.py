"""Query-range support of the kernels (q_blk0: a shard of the query blocks
against the whole key sequence), which the query-block sharding across GPUs
runs on every rank.  Emulated on one GPU: each shard's selection rows, O, lse
and dQ rows must equal the rows of the unsharded call, and the dK/dV partials
of all shards must sum to the unsharded dK/dV.  A two-process NCCL run of
sharded.ShardedBlockSparse (2 or 4 ranks, when the box has that many GPUs) is
checked the same way and against the fp64 oracle."""
import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "fused-block-sparse-attention_b200")


def _case(B, H, L, D, dtype, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    return [torch.randn(B, H, L, D, device=dev, generator=g).to(dtype) for _ in range(4)]


@pytest.mark.parametrize("bs,D,world,dtype,tc_dq", [
    (64, 64, 4, torch.bfloat16, False),   # tcgen05 forward / dK-dV
    (64, 64, 2, torch.bfloat16, True),    # + tcgen05 dQ
    (32, 64, 4, torch.bfloat16, False),   # mma.sync kernels
    (32, 32, 2, torch.float32, False),    # fp32 SIMT kernels
])
def test_query_range_matches_unsharded(cuda, monkeypatch, bs, D, world, dtype, tc_dq):
    import _bsa
    if tc_dq:
        monkeypatch.setenv("BSA_DQ_TC05", "1")
    B, H, L, topk = 1, 2, 2048 if dtype != torch.float32 else 512, 6
    q, k, v, do = _case(B, H, L, D, dtype, cuda, bs + world)
    (qp,) = _bsa.pool(q, bs)
    (kp,) = _bsa.pool(k, bs)
    sel, _, _ = _bsa.select(qp, kp, topk=topk)
    o, lse = _bsa.attn_fwd(q, k, v, sel, bs=bs, causal=True)
    dq, dk, dv, _ = _bsa.attn_bwd(q, k, v, o, do, sel, lse, bs=bs, causal=True)
    nblk = L // bs
    nq = nblk // world
    dk_sum = torch.zeros_like(dk, dtype=torch.float32)
    dv_sum = torch.zeros_like(dv, dtype=torch.float32)
    for r in range(world):
        a = r * nq
        rows = slice(a * bs, (a + nq) * bs)
        qs, dos = q[:, :, rows], do[:, :, rows]
        s_r, _, _ = _bsa.select(qp[:, :, a:a + nq], kp, topk=topk, q_blk0=a)
        assert torch.equal(s_r, sel[:, :, a:a + nq])
        o_r, lse_r = _bsa.attn_fwd(qs, k, v, s_r, bs=bs, causal=True, q_blk0=a)
        assert torch.equal(o_r, o[:, :, rows])
        assert torch.equal(lse_r, lse[:, :, rows])
        dq_r, dk_r, dv_r, _ = _bsa.attn_bwd(qs, k, v, o_r, dos, s_r, lse_r, bs=bs, causal=True,
                                            q_blk0=a)
        assert torch.equal(dq_r, dq[:, :, rows])
        dk_sum += dk_r.float()
        dv_sum += dv_r.float()
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    assert (dk_sum - dk.float()).abs().max().item() < tol
    assert (dv_sum - dv.float()).abs().max().item() < tol


def test_query_range_validation(cuda):
    import _bsa
    q, k, v, _ = _case(1, 1, 512, 64, torch.bfloat16, cuda, 1)
    sel = torch.zeros(1, 1, 4, 2, dtype=torch.int32, device=cuda)
    with pytest.raises(_bsa.BsaShapeError):   # range past L
        _bsa.attn_fwd(q[:, :, :256], k, v, sel, bs=64, causal=True, q_blk0=6)
    with pytest.raises(_bsa.BsaShapeError):   # lengths differ without a range
        _bsa.attn_fwd(q[:, :, :256], k, v, sel, bs=64, causal=True)


def _nccl_worker(rank, world, port, L, out_q):
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import sharded
        dev = torch.device("cuda", rank)
        q, k, v, do = _case(1, 2, L, 64, torch.bfloat16, dev, 77)
        Ls = L // world
        sl = slice(rank * Ls, (rank + 1) * Ls)
        m = sharded.ShardedBlockSparse(bs=64, topk=8, causal=True)
        qs, ks, vs, dos = (t[:, :, sl].contiguous() for t in (q, k, v, do))
        o, ctx = m.forward(qs, ks, vs)
        dq, dk, dv = m.backward(qs, o, dos, ctx)
        kv_group = dist.new_group(list(range(world)))
        o2 = m.forward_pipelined(qs, ks, vs, kv_group=kv_group)   # per-head pipelined forward
        torch.cuda.synchronize()
        assert torch.equal(o, o2)
        out_q.put((rank, ctx[2].cpu().numpy(), o.float().cpu().numpy(), dq.float().cpu().numpy(),
                   dk.float().cpu().numpy(), dv.float().cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_nccl_matches_oracle(cuda, world):
    """world NCCL ranks of sharded.ShardedBlockSparse (query-block shards, K/V and
    summary all-gathers, selection-row exchange, dK/dV reduce-scatter) against the
    unsharded GPU path (bitwise for selection, O and dQ) and against the fp64
    oracle restatement of the reference's gather path (selection exact, values
    within the bf16 tolerance of the other attention tests)."""
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    import torch.multiprocessing as mp
    import _bsa
    from oracle import oracle as O
    L = 4096
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, 29655 + world, L, out_q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, *vals = out_q.get(timeout=300)
        res[r] = vals
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    q, k, v, do = _case(1, 2, L, 64, torch.bfloat16, cuda, 77)
    (qp,) = _bsa.pool(q, 64)
    (kp,) = _bsa.pool(k, 64)
    sel, _, _ = _bsa.select(qp, kp, topk=8)
    o, lse = _bsa.attn_fwd(q, k, v, sel, bs=64, causal=True)
    dq, dk, dv, _ = _bsa.attn_bwd(q, k, v, o, do, sel, lse, bs=64, causal=True)
    Ls, nq = L // world, L // world // 64
    for r in range(world):
        s_r, o_r, dq_r, dk_r, dv_r = res[r]
        rows = slice(r * Ls, (r + 1) * Ls)
        assert np.array_equal(s_r, sel[:, :, r * nq:(r + 1) * nq].cpu().numpy())
        assert np.array_equal(o_r, o[:, :, rows].float().cpu().numpy())
        assert np.array_equal(dq_r, dq[:, :, rows].float().cpu().numpy())
        assert np.abs(dk_r - dk[:, :, rows].float().cpu().numpy()).max() < 3e-2
        assert np.abs(dv_r - dv[:, :, rows].float().cpu().numpy()).max() < 3e-2

    # the gathered shards against the oracle
    qc, kc, vc, dc = (t.float().cpu() for t in (q, k, v, do))
    rqp, _, _ = O.pool(qc, 64)
    rkp, _, _ = O.pool(kc, 64)
    rsel, _, _ = O.select(rqp, rkp, topk=8)
    got_sel = np.concatenate([res[r][0] for r in range(world)], axis=2)
    assert np.array_equal(got_sel, rsel)
    rs = torch.from_numpy(rsel)
    ro = O.attention(qc, kc, vc, rs, None, bs=64, causal=True)
    rq, rk, rv, _ = O.attention_grads(qc, kc, vc, rs, dc, None, bs=64, causal=True)
    for i, ref, name in ((1, ro, "o"), (2, rq, "dq"), (3, rk, "dk"), (4, rv, "dv")):
        got = torch.from_numpy(np.concatenate([res[r][i] for r in range(world)], axis=2)).double()
        ref = ref.double()
        bad = ((got - ref).abs() > 2e-2 + 1e-2 * ref.abs()).sum().item()
        assert bad == 0, "%s: %d elements outside 2e-2 + 1e-2|ref|" % (name, bad)
