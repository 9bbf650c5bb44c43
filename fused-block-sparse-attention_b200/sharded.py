"""Query-block sharding of selection + block-sparse attention across GPUs, one
process per GPU (torch.distributed; NCCL over NVLink on the GPU box).

Rank r owns the contiguous query blocks [a_r, b_r) of the sequence: their Q and
dO rows, their selection rows, O and dQ.  K and V arrive sharded the same way
(each rank holds the rows of its own blocks, as a sequence-parallel model
produces them).

  forward   1. all-gather K and V into local HBM (one collective per (batch,
               head) slice, so the gathered (B, H, L, D) tensor is contiguous and
               neither side needs a layout copy);
            2. pool this rank's Q and K blocks (mean, fp32) and all-gather both
               pooled summaries (nblk x D per head, small);
            3. select: causal selection costs grow with the query position, so
               the selection rows are split by equal causal area instead
               (select_ranges: rank r scores query blocks [s_r, e_r) against
               every earlier key block, one tcgen05 selection call with a query
               range), and the rows are returned to their owners by one
               all-gather of the int32 selection (a few bytes per row);
            4. attention over the local query blocks (bsa_attn_fwd with q_blk0);
               with kk blocks per query block the attention itself is balanced.
  backward  dQ stays local; dK/dV are this rank's contributions over the whole
            sequence, summed across ranks and returned to their owners by one
            reduce_scatter (dK and dV copied rank-major into one fp32 buffer,
            the copy doing the conversion, then a single NCCL call instead of
            one per (batch, head) slice).  The per-rank partials come out of the backward in
            the input dtype (bf16): each is rounded once (relative 2^-9) before
            the fp32 sum, so the summed dK/dV carry at most that rounding of
            each rank's share, the same order as the single-GPU result's own
            final rounding to bf16.

A process group is optional: without an initialised torch.distributed (one
GPU) every collective is the identity and the ranges cover the whole sequence.

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

__all__ = ["block_ranges", "select_ranges", "CudaOps", "ShardedBlockSparse"]


def block_ranges(nblk, world):
    """Contiguous, equal query-block ranges [(a_r, b_r)] (nblk % world == 0)."""
    if nblk % world:
        raise ValueError("nblk (%d) must be a multiple of the world size (%d)" % (nblk, world))
    n = nblk // world
    return [(r * n, (r + 1) * n) for r in range(world)]


def select_ranges(nblk, world, causal=True, align=128):
    """Query-block ranges [(s_r, e_r)] for the selection step.  Causal row i scores
    i key blocks, so the ranges split the triangle sum_{i<e} (i + 1) into equal
    areas (boundaries rounded to multiples of `align` blocks, the selection
    kernel's query tile, when that keeps every range non-empty); non-causal rows
    cost the same and the ranges are the contiguous block_ranges."""
    if not causal or world == 1:
        return block_ranges(nblk, world)
    total = nblk * (nblk + 1) / 2.0
    cuts = [0]
    for r in range(1, world):
        # e with e (e + 1) / 2 = r / world * total
        e = int(round(((1 + 8.0 * total * r / world) ** 0.5 - 1) / 2))
        if align > 1 and nblk >= 16 * align * world:
            e = int(round(e / align)) * align
        cuts.append(min(max(e, cuts[-1] + 1), nblk - (world - r)))
    cuts.append(nblk)
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def _world(group):
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


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
    def attn_fwd(q, k, v, sel, *, bs, causal, q_blk0, out=None, want_lse=True):
        return _bsa.attn_fwd(q, k, v, sel, None, bs=bs, causal=causal, q_blk0=q_blk0, out=out,
                             want_lse=want_lse)

    @staticmethod
    def attn_bwd(q, k, v, o, do, sel, lse, *, bs, causal, q_blk0):
        dq, dk, dv, _ = _bsa.attn_bwd(q, k, v, o, do, sel, lse, None, bs=bs, causal=causal,
                                      q_blk0=q_blk0)
        return dq, dk, dv


def _gather_seq(x, group, async_op=False):
    """x: (B, H, n, ...) this rank's rows along dim 2 -> (B, H, world * n, ...) in rank
    order, contiguous: one all_gather_into_tensor per (b, h) slice, each slice
    contiguous on both sides, so no layout copy is needed on either end.  With
    async_op, returns (out, works): the caller waits on the works before use."""
    world, _ = _world(group)
    if world == 1:
        return (x, []) if async_op else x
    x = x.contiguous()
    B, H, n = x.shape[:3]
    out = torch.empty((B, H, world * n) + tuple(x.shape[3:]), dtype=x.dtype, device=x.device)
    works = []
    for b in range(B):
        for h in range(H):
            w = dist.all_gather_into_tensor(out[b, h], x[b, h], group=group, async_op=async_op)
            if async_op:
                works.append(w)
    return (out, works) if async_op else out


def _gather_small(x, group):
    """Same result as _gather_seq for small tensors (pooled summaries, selection
    rows): one all_gather_into_tensor into a rank-major buffer, then one copy
    into (B, H, world * n, ...) instead of one collective per (batch, head)."""
    world, _ = _world(group)
    if world == 1:
        return x
    x = x.contiguous()
    B, H, n = x.shape[:3]
    rest = tuple(x.shape[3:])
    buf = torch.empty((world * B, H, n) + rest, dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(buf, x, group=group)
    perm = (1, 2, 0, 3) + tuple(range(4, 4 + len(rest)))
    return buf.view((world, B, H, n) + rest).permute(perm).reshape((B, H, world * n) + rest)


def _reduce_scatter_pair(x, y, group):
    """x, y: (B, H, world * n, ...) per-rank partial sums of the same shape -> this
    rank's (B, H, n, ...) slices of their fp32 sums over ranks.  Both are copied
    (and converted) into one rank-major fp32 buffer (world, 2, B, H, n, ...), so a
    single reduce_scatter_tensor returns (2, B, H, n, ...)."""
    world, _ = _world(group)
    if world == 1:
        return x.float(), y.float()
    B, H, L = x.shape[:3]
    n, rest = L // world, tuple(x.shape[3:])
    buf = torch.empty((world, 2, B, H, n) + rest, dtype=torch.float32, device=x.device)
    perm = (2, 0, 1, 3) + tuple(range(4, 4 + len(rest)))
    for i, t in enumerate((x, y)):
        buf[:, i].copy_(t.reshape((B, H, world, n) + rest).permute(perm))
    out = torch.empty((2, B, H, n) + rest, dtype=torch.float32, device=x.device)
    dist.reduce_scatter_tensor(out, buf.view((world * 2, B, H, n) + rest), group=group)
    return out[0], out[1]


def _reduce_scatter_seq(x, group):
    """x: (B, H, world * n, ...) per-rank partial sums -> this rank's (B, H, n, ...)
    slice of the sum over ranks (one reduce_scatter_tensor per (b, h) slice)."""
    world, _ = _world(group)
    if world == 1:
        return x
    x = x.contiguous()
    B, H, L = x.shape[:3]
    out = torch.empty((B, H, L // world) + tuple(x.shape[3:]), dtype=x.dtype, device=x.device)
    for b in range(B):
        for h in range(H):
            dist.reduce_scatter_tensor(out[b, h], x[b, h], group=group)
    return out


class ShardedBlockSparse:
    """Selection + attention over query-block shards.  All tensors are this
    rank's shard (B, H, Ls, D), Ls = L / world, a multiple of bs."""

    def __init__(self, *, bs, topk, causal=True, group=None, ops=None):
        self.bs, self.topk, self.causal = bs, topk, causal
        self.group = group
        self.ops = ops if ops is not None else CudaOps()

    def _geometry(self, q):
        world, rank = _world(self.group)
        Ls = q.shape[2]
        if Ls % self.bs:
            raise ValueError("shard length (%d) must be a multiple of the block size" % Ls)
        nblk = world * Ls // self.bs
        a, _ = block_ranges(nblk, world)[rank]
        return world, rank, nblk, a

    def gather_kv(self, k, v):
        """All-gathers the K, V shards -> (B, H, L, D) contiguous local buffers."""
        return _gather_seq(k, self.group), _gather_seq(v, self.group)

    def select(self, q, k):
        """This rank's selection rows (B, H, nq, 1 + min(topk, nblk-1)), int32,
        computed over the equal-area ranges of select_ranges and exchanged."""
        return self._select(q, k, None)

    def select_and_gather(self, q, k, v):
        """(K, V gathered, this rank's selection rows).  The K/V all-gathers are
        started after the small pooled-summary gathers and run while this rank
        computes its selection rows (the collectives of one communicator run in
        order, so the summaries must go first); the selection-row exchange
        follows once K/V have arrived."""
        if _world(self.group)[0] == 1:
            return k, v, self._select(q, k, None)
        box = {}

        def start():
            box["k"], wk = _gather_seq(k, self.group, async_op=True)
            box["v"], wv = _gather_seq(v, self.group, async_op=True)
            box["works"] = wk + wv

        sel = self._select(q, k, start)
        for w in box["works"]:
            w.wait()
        return box["k"], box["v"], sel

    def _select(self, q, k, before_exchange):
        world, rank, nblk, a = self._geometry(q)
        nq = q.shape[2] // self.bs
        qp_local = self.ops.pool(q, self.bs)                  # (B, H, nq, D) fp32
        kp = _gather_small(self.ops.pool(k, self.bs), self.group)
        if world == 1 or not self.causal:
            qp = None
        else:
            qp = _gather_small(qp_local, self.group)
        if before_exchange is not None:
            before_exchange()                                 # start the K/V gathers
        if qp is None:
            return self.ops.select(qp_local, kp, topk=self.topk, causal=self.causal, q_blk0=a)
        ranges = select_ranges(nblk, world, self.causal)
        s0, s1 = ranges[rank]
        mine = self.ops.select(qp[:, :, s0:s1].contiguous(), kp, topk=self.topk,
                               causal=self.causal, q_blk0=s0)     # (B, H, s1 - s0, W)
        width = max(e - b for b, e in ranges)
        pad = torch.zeros(mine.shape[0], mine.shape[1], width, mine.shape[3], dtype=mine.dtype,
                          device=mine.device)
        pad[:, :, :s1 - s0] = mine
        every = _gather_small(pad, self.group)                # (B, H, world * width, W)
        rows = torch.cat([every[:, :, r * width:r * width + (e - b)]
                          for r, (b, e) in enumerate(ranges)], dim=2)
        return rows[:, :, a:a + nq].contiguous()

    def forward(self, q, k, v):
        """Returns (o, ctx): o is this rank's (B, H, Ls, D) output; ctx carries what
        backward needs (the gathered K/V, the selection and the row lse)."""
        _, _, _, a = self._geometry(q)
        # K/V first: every rank reaches this collective at once, before the
        # position-dependent (causal, unbalanced) selection work
        kf, vf, sel = self.select_and_gather(q, k, v)
        o, lse = self.ops.attn_fwd(q, kf, vf, sel, bs=self.bs, causal=self.causal, q_blk0=a)
        return o, (kf, vf, sel, lse)

    def forward_pipelined(self, q, k, v, kv_group=None):
        """Forward only, for long sequences where moving K and V dominates: the K/V
        all-gathers run per head on `kv_group` (a second communicator over the
        same ranks, so they proceed while the selection's own collectives run on
        this module's group), the selection is computed meanwhile, and the
        attention of head h starts as soon as head h's K and V have arrived, so
        it overlaps the transfer of the later heads.  Returns this rank's o."""
        world, rank, nblk, a = self._geometry(q)
        if world == 1:
            sel = self.select(q, k)
            return self.ops.attn_fwd(q, k, v, sel, bs=self.bs, causal=self.causal, q_blk0=a,
                                     want_lse=False)[0]
        kvg = kv_group if kv_group is not None else self.group
        k, v = k.contiguous(), v.contiguous()
        B, H, n = k.shape[:3]
        kf = torch.empty((B, H, world * n) + tuple(k.shape[3:]), dtype=k.dtype, device=k.device)
        vf = torch.empty_like(kf)
        works = [[] for _ in range(H)]
        for h in range(H):
            for b in range(B):
                works[h].append(dist.all_gather_into_tensor(kf[b, h], k[b, h], group=kvg,
                                                            async_op=True))
                works[h].append(dist.all_gather_into_tensor(vf[b, h], v[b, h], group=kvg,
                                                            async_op=True))
        sel = self._select(q, k, None)
        o = torch.empty_like(q, memory_format=torch.contiguous_format)
        for h in range(H):
            for w in works[h]:
                w.wait()
            self.ops.attn_fwd(q[:, h:h + 1], kf[:, h:h + 1], vf[:, h:h + 1], sel[:, h:h + 1],
                              bs=self.bs, causal=self.causal, q_blk0=a, out=o[:, h:h + 1],
                              want_lse=False)
        return o

    def backward(self, q, o, do, ctx):
        """Returns this rank's (dq, dk, dv) shards; dk/dv are summed over ranks."""
        kf, vf, sel, lse = ctx
        _, _, _, a = self._geometry(q)
        dq, dk, dv = self.ops.attn_bwd(q, kf, vf, o, do, sel, lse, bs=self.bs, causal=self.causal,
                                       q_blk0=a)
        if _world(self.group)[0] == 1:
            return dq, dk, dv
        dk_s, dv_s = _reduce_scatter_pair(dk, dv, self.group)
        return dq, dk_s.to(dk.dtype), dv_s.to(dv.dtype)
