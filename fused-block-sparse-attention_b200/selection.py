"""Device block selection built on the pooling and fused top-k kernels.

  select_meanpool   mean-pooled q.k per head, own block + top-k content blocks
                    (the selection of the BASELINE configurations 1-3; ranking
                    and fill rules of src/ssa_model.py:151-162)
  select_quest      Quest min/max bound per KV head with _finish semantics
                    (src/qwen_blocksparse.py:87-121)

All functions run on the current CUDA stream; indices are int32.
"""
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


def select_quest(q, k, *, bs, topk, sink=True):
    """q (B, Hq, L, D), k (B, Hkv, L, D) -> int32 (B, Hkv, nblk, min(topk,nblk)+1+sink),
    sorted ascending: top-k by sum_d max(q_d*kmax_d, q_d*kmin_d) with q mean-pooled over
    the query group and the block, causal, missing picks -> own, plus own and sink."""
    grp = q.shape[1] // k.shape[1]
    (qp,) = _bsa.pool(q, bs, grp=grp)
    kmin, kmax = _bsa.pool(k, bs, mean=False, vmin=True, vmax=True)
    sel, _, _ = _bsa.select(qp, kmax, kmin, kind=_bsa.SCORE_QUEST, layout=_bsa.SEL_FINISH,
                            topk=topk, sink=sink)
    return sel
