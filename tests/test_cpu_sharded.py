"""Query-block sharding (sharded.ShardedBlockSparse) on gloo ranks on the CPU.

Two (and four) processes each hold one shard of Q, K, V, dO.  The partitioning,
the all-gathers of K, V and the pooled key summaries, and the reduce-scatter of
dK/dV are the product code; the four compute steps are checker implementations
built on the oracle (this file's OracleOps), since the CUDA kernels need a GPU.
Every rank's selection rows must equal the single-process oracle selection
bit for bit, and its O, dQ and dK/dV shards must match the single-process
oracle attention and gradients."""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "fused-block-sparse-attention_b200")

B, H, D, BS, TOPK = 1, 2, 32, 32, 5


def _paths():
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)


def _problem(L):
    g = torch.Generator().manual_seed(L)
    return [torch.randn(B, H, L, D, generator=g, dtype=torch.float64) for _ in range(4)]


class OracleOps:
    """The same four calls as sharded.CudaOps, computed by the oracle on full-length
    tensors whose rows outside this rank's query range are zero (rows are
    independent, so the local rows are exact)."""

    @staticmethod
    def pool(x, bs):
        from oracle import oracle as O
        return torch.from_numpy(O.pool(x, bs)[0])

    @staticmethod
    def select(qp, kp, *, topk, causal, q_blk0):
        from oracle import oracle as O
        nq, nblk = qp.shape[-2], kp.shape[-2]
        a = torch.zeros(kp.shape, dtype=torch.float32)
        a[..., q_blk0:q_blk0 + nq, :] = qp
        sel, _, _ = O.select(a, kp, kind=O.SCORE_DOT, layout=O.SEL_SSA, causal=causal, topk=topk)
        return torch.from_numpy(sel[..., q_blk0:q_blk0 + nq, :].copy())

    @staticmethod
    def _full(q, sel, L, q_blk0, bs):
        qf = torch.zeros(q.shape[0], q.shape[1], L, q.shape[3], dtype=q.dtype)
        r0 = q_blk0 * bs
        qf[:, :, r0:r0 + q.shape[2]] = q
        nblk = L // bs
        own = torch.arange(nblk).view(1, 1, nblk, 1).expand(sel.shape[0], sel.shape[1], nblk,
                                                             sel.shape[3]).clone()
        own[:, :, q_blk0:q_blk0 + sel.shape[2]] = sel.long()
        return qf, own, r0

    @staticmethod
    def attn_fwd(q, k, v, sel, *, bs, causal, q_blk0):
        from oracle import oracle as O
        L = k.shape[2]
        qf, sf, r0 = OracleOps._full(q, sel, L, q_blk0, bs)
        o = O.attention(qf, k, v, sf, bs=bs, causal=causal)
        return o[:, :, r0:r0 + q.shape[2]].contiguous(), None

    @staticmethod
    def attn_bwd(q, k, v, o, do, sel, lse, *, bs, causal, q_blk0):
        from oracle import oracle as O
        L = k.shape[2]
        qf, sf, r0 = OracleOps._full(q, sel, L, q_blk0, bs)
        dof = torch.zeros_like(qf)
        dof[:, :, r0:r0 + q.shape[2]] = do
        dq, dk, dv, _ = O.attention_grads(qf, k, v, sf, dof, bs=bs, causal=causal)
        return dq[:, :, r0:r0 + q.shape[2]].contiguous(), dk, dv


def _worker(rank, world, port, L, out_q):
    _paths()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sharded
        q, k, v, do = _problem(L)
        Ls = L // world
        sl = slice(rank * Ls, (rank + 1) * Ls)
        m = sharded.ShardedBlockSparse(bs=BS, topk=TOPK, causal=True, ops=OracleOps())
        qs, ks, vs, dos = (t[:, :, sl].contiguous() for t in (q, k, v, do))
        o, ctx = m.forward(qs, ks, vs)
        dq, dk, dv = m.backward(qs, o, dos, ctx)
        out_q.put((rank, ctx[2].numpy(), o.numpy(), dq.numpy(), dk.numpy(), dv.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,L,port", [(2, 512, 29631), (4, 1024, 29633), (8, 1024, 29637)])
def test_query_block_sharding_matches_single_process(world, L, port):
    _paths()
    from oracle import oracle as O
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, L, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, *vals = out_q.get(timeout=300)
        res[r] = vals
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v, do = _problem(L)
    qp, kp = O.pool(q, BS)[0], O.pool(k, BS)[0]
    sel, _, _ = O.select(qp, kp, kind=O.SCORE_DOT, layout=O.SEL_SSA, causal=True, topk=TOPK)
    sel_t = torch.from_numpy(sel).long()
    o = O.attention(q, k, v, sel_t, bs=BS, causal=True)
    dq, dk, dv, _ = O.attention_grads(q, k, v, sel_t, do, bs=BS, causal=True)
    Ls, nq = L // world, L // world // BS
    for r in range(world):
        s_r, o_r, dq_r, dk_r, dv_r = res[r]
        rows = slice(r * Ls, (r + 1) * Ls)
        assert np.array_equal(s_r, sel[:, :, r * nq:(r + 1) * nq])
        assert np.allclose(o_r, o[:, :, rows].numpy(), atol=1e-10)
        assert np.allclose(dq_r, dq[:, :, rows].numpy(), atol=1e-10)
        # dK/dV partials are summed in fp32 by the reduce-scatter
        assert np.allclose(dk_r, dk[:, :, rows].numpy(), atol=1e-5)
        assert np.allclose(dv_r, dv[:, :, rows].numpy(), atol=1e-5)


def test_block_ranges():
    _paths()
    import sharded
    assert sharded.block_ranges(8, 4) == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        sharded.block_ranges(10, 4)
