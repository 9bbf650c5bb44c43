"""Device block selection built on the pooling and fused top-k kernels.

  select_meanpool   mean-pooled q.k per head, own block + top-k content blocks
                    (the selection of the BASELINE configurations 1-3; ranking
                    and fill rules of src/ssa_model.py:151-162)
  select_quest      Quest min/max bound per KV head with _finish semantics
                    (src/qwen_blocksparse.py:87-121)
  select_lsh        LSH bucketing of the mean-pooled, L2-normalised block vectors
                    (sign of n_planes seeded Gaussian hyperplanes per round, the
                    BASELINE configuration 5; or the reference's argmax rule of
                    LSHBucketSSA, src/ssa_model.py:438-470), candidates re-scored
                    by the exact cosine

All functions run on the current CUDA stream; indices are int32.
"""
import torch

import _bsa


def select_meanpool(q, k, *, bs, topk, causal=True, want_gate=False, want_score=False):
    """q, k: (B, H, L, D).  Returns (sel, gate, score): sel int32
    (B, H, nblk, 1 + min(topk, nblk-1)) with sel[..., 0] = own block, then content
    blocks by descending pooled q.k (ties to the lower block id); optional fp32
    logsigmoid(score) gate and raw scores of the same shape."""
    if k.shape[1] != q.shape[1]:
        raise ValueError("select_meanpool: q and k need the same head count")
    (qp,) = _bsa.pool(q, bs)
    (kp,) = _bsa.pool(k, bs)
    sel, score, gate = _bsa.select(qp, kp, kind=_bsa.SCORE_DOT, layout=_bsa.SEL_SSA, causal=causal,
                                   topk=topk, want_gate=want_gate, want_score=want_score)
    return sel, gate, score


def select_quest(q, k, *, bs, topk, sink=True, rope=None):
    """q (B, Hq, L, D), k (B, Hkv, L, D) -> int32 (B, Hkv, nblk, min(topk,nblk)+1+sink),
    sorted ascending: top-k by sum_d max(q_d*kmax_d, q_d*kmin_d) with q mean-pooled over
    the query group and the block, causal, missing picks -> own, plus own and sink.
    rope=(cos, sin): q is pooled after its partial rotary embedding (computed inside
    the pooling kernel, the values of bsa_rope), so the rotated q is never stored."""
    grp = q.shape[1] // k.shape[1]
    (qp,) = _bsa.pool(q, bs, grp=grp, rope=rope)
    kmin, kmax = _bsa.pool(k, bs, mean=False, vmin=True, vmax=True)
    sel, _, _ = _bsa.select(qp, kmax, kmin, kind=_bsa.SCORE_QUEST, layout=_bsa.SEL_FINISH,
                            topk=topk, sink=sink)
    return sel


def lsh_planes(dim, n_rounds=4, n_planes=4, seed=0):
    """Seeded N(0,1) hyperplanes (dim, n_rounds, n_planes), fp32, on the CPU."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(dim, n_rounds, n_planes, generator=g)


def select_lsh(q, k, *, bs, topk, n_rounds=4, n_planes=4, cap=16, seed=0, planes=None,
               hash_kind="sign", causal=True, scale=1.0, want_gate=False, want_score=False):
    """q, k: (B, H, L, D).  Mean-pools both per block, L2-normalises, hashes each block
    once per round (sign bits of n_planes hyperplanes -> 2**n_planes buckets, or the
    argmax over n_planes projections), keeps the first `cap` key blocks of every
    bucket, and picks per query block the top-k by scale * cosine among the blocks
    sharing one of its buckets.  Returns (sel, gate, score): sel int32
    (B, H, nblk, 1 + min(topk, nblk-1, n_rounds*cap)), own block first."""
    if k.shape[1] != q.shape[1]:
        raise ValueError("select_lsh: q and k need the same head count")
    if planes is None:
        planes = lsh_planes(q.shape[-1], n_rounds, n_planes, seed)
    planes = planes.to(q.device, torch.float32)
    kind = _bsa.HASH_SIGN if hash_kind == "sign" else _bsa.HASH_ARGMAX
    (qp,) = _bsa.pool(q, bs)
    (kp,) = _bsa.pool(k, bs)
    sel, score, gate = _bsa.select_lsh(qp, kp, planes, hash_kind=kind, cap=cap, causal=causal,
                                       topk=topk, scale=scale, want_gate=want_gate,
                                       want_score=want_score)
    return sel, gate, score
