"""Query-block sharding of selection + block-sparse attention across GPUs, one
process per GPU (torch.distributed; NCCL over NVLink on the GPU box).

Rank r owns the contiguous query blocks [a_r, b_r) of the sequence: their Q and
dO rows, their selection rows, O and dQ.  K and V arrive sharded the same way
(each rank holds the rows of its own blocks, as a sequence-parallel model
produces them).

  forward   1. all-gather K and V into local HBM (sequence-major buffers, so the
               gathered tensor is a strided (B, H, L, D) view with no copy);
            2. pool this rank's K blocks (mean, fp32) and all-gather the pooled
               summaries (nblk x D per head, small);
            3. select: this rank's pooled queries against every key block,
               causal top-k with the own block first (bsa_select with a query
               range);
            4. attention over the local query blocks (bsa_attn_fwd with q_blk0).
  backward  dQ stays local; dK/dV are this rank's contributions over the whole
            sequence, summed across ranks and returned to their owners by one
            reduce_scatter (fp32 accumulation).

No kernel reads another GPU's memory: every collective lands in local HBM
before a kernel touches it.  The reference has no multi-GPU path; this is the
sharding its long-context configurations call for.

The compute steps go through an `ops` object (default: the CUDA kernels of
_bsa), so the partitioning and collective logic can be exercised by gloo ranks
on the CPU with checker implementations of the same four calls.
"""
import torch
import torch.distributed as dist

import _bsa

__all__ = ["block_ranges", "CudaOps", "ShardedBlockSparse"]


def block_ranges(nblk, world):
    """Contiguous, equal query-block ranges [(a_r, b_r)] (nblk % world == 0)."""
    if nblk % world:
        raise ValueError("nblk (%d) must be a multiple of the world size (%d)" % (nblk, world))
    n = nblk // world
    return [(r * n, (r + 1) * n) for r in range(world)]


class CudaOps:
    """The device kernels behind each step (libbsa_b200.so)."""

    @staticmethod
    def pool(x, bs):
        return _bsa.pool(x, bs)[0]

    @staticmethod
    def select(qp, kp, *, topk, causal, q_blk0):
        sel, _, _ = _bsa.select(qp, kp, kind=_bsa.SCORE_DOT, layout=_bsa.SEL_SSA, causal=causal,
                                topk=topk, q_blk0=q_blk0)
        return sel

    @staticmethod
    def attn_fwd(q, k, v, sel, *, bs, causal, q_blk0):
        return _bsa.attn_fwd(q, k, v, sel, None, bs=bs, causal=causal, q_blk0=q_blk0)

    @staticmethod
    def attn_bwd(q, k, v, o, do, sel, lse, *, bs, causal, q_blk0):
        dq, dk, dv, _ = _bsa.attn_bwd(q, k, v, o, do, sel, lse, None, bs=bs, causal=causal,
                                      q_blk0=q_blk0)
        return dq, dk, dv


def _gather_rows(x, group):
    """x: (n, ...) this rank's rows -> (world * n, ...) in rank order, in a new
    contiguous buffer (one all_gather_into_tensor)."""
    world = dist.get_world_size(group)
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _reduce_scatter_rows(x, group):
    """x: (world * n, ...) per-rank partial sums -> this rank's (n, ...) slice of
    the sum over ranks (one reduce_scatter_tensor)."""
    world = dist.get_world_size(group)
    out = torch.empty((x.shape[0] // world,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    return out


def _seq_major(x):
    """(B, H, n, D) -> contiguous (n, B, H, D)."""
    return x.permute(2, 0, 1, 3).contiguous()


def _bhld(x):
    """(L, B, H, D) buffer -> its (B, H, L, D) strided view."""
    return x.permute(1, 2, 0, 3)


class ShardedBlockSparse:
    """Selection + attention over query-block shards.  All tensors are this
    rank's shard (B, H, Ls, D), Ls = L / world, a multiple of bs."""

    def __init__(self, *, bs, topk, causal=True, group=None, ops=None):
        self.bs, self.topk, self.causal = bs, topk, causal
        self.group = group
        self.ops = ops if ops is not None else CudaOps()

    def _geometry(self, q):
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        Ls = q.shape[2]
        if Ls % self.bs:
            raise ValueError("shard length (%d) must be a multiple of the block size" % Ls)
        nblk = world * Ls // self.bs
        a, _ = block_ranges(nblk, world)[rank]
        return world, rank, nblk, a

    def gather_kv(self, k, v):
        """All-gathers the K, V shards -> (B, H, L, D) strided views of local buffers."""
        return _bhld(_gather_rows(_seq_major(k), self.group)), \
            _bhld(_gather_rows(_seq_major(v), self.group))

    def select(self, q, k):
        """This rank's selection rows (B, H, nq, 1 + min(topk, nblk-1)), int32."""
        world, rank, nblk, a = self._geometry(q)
        qp = self.ops.pool(q, self.bs)                        # (B, H, nq, D) fp32
        kp_local = self.ops.pool(k, self.bs)
        kp = _bhld(_gather_rows(_seq_major(kp_local), self.group)).contiguous()
        return self.ops.select(qp, kp, topk=self.topk, causal=self.causal, q_blk0=a)

    def forward(self, q, k, v):
        """Returns (o, ctx): o is this rank's (B, H, Ls, D) output; ctx carries what
        backward needs (the gathered K/V, the selection and the row lse)."""
        _, _, _, a = self._geometry(q)
        # K/V first: every rank reaches this collective at once, before the
        # position-dependent (causal, unbalanced) selection work
        kf, vf = self.gather_kv(k, v)
        sel = self.select(q, k)
        o, lse = self.ops.attn_fwd(q, kf, vf, sel, bs=self.bs, causal=self.causal, q_blk0=a)
        return o, (kf, vf, sel, lse)

    def backward(self, q, o, do, ctx):
        """Returns this rank's (dq, dk, dv) shards; dk/dv are summed over ranks."""
        kf, vf, sel, lse = ctx
        _, _, _, a = self._geometry(q)
        dq, dk, dv = self.ops.attn_bwd(q, kf, vf, o, do, sel, lse, bs=self.bs, causal=self.causal,
                                       q_blk0=a)
        dk_s = _reduce_scatter_rows(_seq_major(dk.float()), self.group)
        dv_s = _reduce_scatter_rows(_seq_major(dv.float()), self.group)
        return dq, _bhld(dk_s).to(dk.dtype).contiguous(), _bhld(dv_s).to(dv.dtype).contiguous()
