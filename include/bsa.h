/*
 * bsa.h — C ABI of the B200-native fused block-sparse attention library
 * (libbsa_b200.so).  Plain pointers, sizes and strides only; no torch types.
 *
 * The reference (apoc/fused-block-sparse-attention, Python + Triton) has no C
 * interface: its boundary is the Python functions listed beside each entry
 * point.  Each entry point here replaces the device work behind one of them,
 * and the Python modules in fused-block-sparse-attention_b200/ bind these
 * symbols through ctypes with the reference's call signatures.
 *
 * Conventions
 *  - All device pointers are on the current CUDA device; all work is enqueued
 *    on `stream` (a cudaStream_t, 0 = legacy default stream); no entry point
 *    synchronises the host.
 *  - Tensors of shape (B, H, L, D) are described by a bsa_view: a base pointer
 *    plus element strides of the B, H and L axes; the D axis must be
 *    unit-stride.  bf16/f16 views read through TMA need 16-byte aligned base
 *    pointers and strides that are multiples of 8 elements.
 *  - Every call returns a bsa_status.  On an error nothing is launched and
 *    bsa_last_error() returns a one-line message (thread-local).
 *  - `status` (optional, may be NULL) points at one int32 in device memory.
 *    Kernels OR error bits into it: BSA_DEVERR_INDEX when a selected block id
 *    is outside [0, nblk) (that slot is then treated as masked), and
 *    BSA_DEVERR_TIMEOUT when a bounded wait on a TMA barrier gave up.
 *    The caller clears and reads it.
 */
#ifndef BSA_B200_H
#define BSA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *bsa_stream_t; /* == cudaStream_t */

typedef enum {
  BSA_OK = 0,
  BSA_ERR_SHAPE = 1,       /* inconsistent or out-of-range sizes            */
  BSA_ERR_DTYPE = 2,       /* unsupported element type                      */
  BSA_ERR_STRIDE = 3,      /* stride/alignment not accepted (copy first)    */
  BSA_ERR_UNSUPPORTED = 4, /* valid, but no kernel instance for this shape  */
  BSA_ERR_INDEX = 5,       /* reported by bsa_status_decode for INDEX bits  */
  BSA_ERR_LAUNCH = 6,      /* CUDA launch / driver error                    */
  BSA_ERR_TIMEOUT = 7,     /* reported by bsa_status_decode for TIMEOUT     */
  BSA_ERR_WORKSPACE = 8,   /* workspace pointer NULL or too small           */
  BSA_ERR_ARG = 9          /* NULL required pointer / bad enum value        */
} bsa_status;

#define BSA_DEVERR_INDEX 1
#define BSA_DEVERR_TIMEOUT 2

typedef enum { BSA_BF16 = 0, BSA_F16 = 1, BSA_F32 = 2 } bsa_dtype;

/* How selected slots are masked.
 *  BSA_MASK_SLOT  — triton_kernel.py semantics (reference src/triton_kernel.py:57-61):
 *                   causal: slot 0 gets the triu mask (key row > query row),
 *                   slot j>0 is dropped when its block id >= the query block;
 *                   non-causal: nothing is masked, duplicates count twice.
 *  BSA_MASK_TOKEN — qwen gather semantics (reference src/qwen_blocksparse.py:67-72):
 *                   a key is valid iff its position <= the query position
 *                   (only when causal != 0), < L, and its slot is the first
 *                   occurrence of that block id in the row. */
typedef enum { BSA_MASK_SLOT = 0, BSA_MASK_TOKEN = 1 } bsa_mask_mode;

typedef struct {
  void *ptr;
  int64_t sb, sh, sl; /* element strides of the B, H and L axes */
} bsa_view;

/* One struct for the forward and backward attention calls.
 * q: (B,Hq,L,D); k, v: (B,Hkv,L,D); Hq % Hkv == 0, query head h reads KV head
 * h / (Hq/Hkv).  L <= nblk*bs; rows past L read as zero (padding).
 * sel: int32 (B, Hs, nblk, kk) block ids addressed as
 *      sel[b*sel_sb + (h/(Hq/Hkv))*sel_sh + qblk*sel_sn + slot]; sel_sh = 0
 *      shares one selection over all heads (the reference layout (B,nblk,kk)).
 *      sel == NULL means the identity selection (kk == nblk, slot j -> block j).
 * gate: optional fp32 additive bias per selected block, addressed like sel.
 * lse: fp32 (B, Hq, nblk*bs), row log2-sum-exp written by the forward and
 *      read by the backward (internal format: log2 domain, scale folded in).
 * out_gate: optional (same dtype as q) sigmoid output gate, o *= sigmoid(g),
 *      addressed like o (reference src/patch_qwen.py:55). */
typedef struct {
  int32_t dtype;
  int32_t B, Hq, Hkv, L, D;
  int32_t bs, nblk, kk;
  int32_t mask_mode, causal;
  float scale;
  bsa_view q, k, v, o;
  bsa_view dout, dq, dk, dv; /* backward only */
  bsa_view out_gate;         /* forward only, ptr NULL = none */
  const int32_t *sel;
  int64_t sel_sb, sel_sh, sel_sn;
  const float *gate;
  int64_t gate_sb, gate_sh, gate_sn;
  float *lse;
  float *dgate; /* backward, optional: fp32 (B,Hq,nblk,kk) per-head d(loss)/d(gate) */
  int32_t *status;
  /* Query-block range (a shard of the query side; 0, 0 = all queries): q, o,
   * dout, dq, out_gate hold Lq rows that start at row q_blk0*bs of the sequence,
   * i.e. the query blocks [q_blk0, q_blk0 + ceil(Lq/bs)); sel, gate, dgate, lse
   * hold the rows of those blocks only; k, v, dk, dv cover the whole sequence
   * (L rows, nblk blocks).  Masks use the global block indices.  Lq must be a
   * multiple of bs unless the range ends at L.  No reference counterpart: used by
   * the query-block sharding across GPUs. */
  int32_t q_blk0, Lq;
  /* Forward only, optional (rope_cos NULL = none): the partial rotary embedding
   * of q is applied inside the attention kernel, after q is loaded and before
   * the first product, with the arithmetic of bsa_rope (transformers'
   * apply_rotary_pos_emb, each product and sum rounded to the dtype).  cos/sin:
   * (B, L, rope_rot) in q's dtype with element strides rope_sb (0 = shared over
   * the batch) and rope_sl, indexed by the token position.  Supported by the
   * block-128 tcgen05 kernel at D 256, rope_rot a multiple of 16, at most 64 (the
   * Qwen configuration: 64 of 256 dims).  k must already be rotated. */
  const void *rope_cos, *rope_sin;
  int64_t rope_sb, rope_sl;
  int32_t rope_rot;
} bsa_attn_args;

/* Forward: o = softmax(q k^T * scale + gate + mask) v over the selected blocks.
 * Replaces triton_kernel.bsattn_forward (reference src/triton_kernel.py:184-207,
 * kernel :20-74) and the gather core of qwen_blocksparse.blocksparse_forward
 * (src/qwen_blocksparse.py:57-84), including GQA (:39,:74-81) and the sigmoid
 * output gate of patch_qwen (src/patch_qwen.py:55). */
bsa_status bsa_attn_fwd(const bsa_attn_args *a, bsa_stream_t stream);

/* Backward: dq, dk, dv (and optional dgate) from dout, o and the forward's lse.
 * Replaces triton_kernel.bsattn_backward (reference src/triton_kernel.py:210-234,
 * kernel :77-181).  dk/dv are produced per key block over a CSR transpose of
 * sel (no float atomics; bitwise deterministic).  Needs a device workspace of
 * bsa_attn_bwd_workspace(a) bytes, 256-byte aligned.  For block 64 / head dim
 * 64 in bf16/f16 without dgate the workspace also holds every 64x64 dS tile of
 * the active entries (B*Hq*nq*kk*8 KB, 4.6 GB at 262k tokens x 8 heads, kk 17;
 * at most 24 GB, beyond which the recomputing dQ path is used): the dK/dV
 * kernel writes them and the dQ kernel reads them back. */
size_t bsa_attn_bwd_workspace(const bsa_attn_args *a);
bsa_status bsa_attn_bwd(const bsa_attn_args *a, void *workspace, size_t workspace_bytes,
                        bsa_stream_t stream);

/* Block pooling: per (b, output head, block) mean / min / max over the bs rows
 * of the block (rows past L count as zeros, as after F.pad).  With grp > 1 the
 * mean first averages grp consecutive input heads per row (output head
 * hk = input head / grp), as qwen SelectMax does (src/qwen_blocksparse.py:113);
 * min/max need grp == 1 (src/qwen_blocksparse.py:115-116).  Summation order is
 * sequential (heads, then rows) in fp32, so results are bitwise reproducible.
 * Outputs are contiguous fp32 (B, H/grp, nblk, D); any of them may be NULL.
 * Replaces the pooling of BlockSparseSSA._scores (src/ssa_model.py:113-117). */
typedef struct {
  int32_t dtype;
  int32_t B, H, L, D, bs, nblk, grp;
  bsa_view x;
  float *mean, *vmin, *vmax;
  int32_t *status;
  /* Optional (rope_cos NULL = none): pool the rows of x after the partial rotary
   * embedding of bsa_rope (same rounding), without writing the rotated tensor:
   * cos/sin (B, L, rope_rot) in x's dtype, strides rope_sb (0 = shared), rope_sl;
   * rope_rot a multiple of 16. */
  const void *rope_cos, *rope_sin;
  int64_t rope_sb, rope_sl;
  int32_t rope_rot;
} bsa_pool_args;
bsa_status bsa_pool(const bsa_pool_args *a, bsa_stream_t stream);

/* Block-pair scoring fused with a streaming top-k; the nblk x nblk score matrix
 * is never stored.  G independent groups (e.g. b*H + h), each with nblk query
 * summaries a[g,i,:] and key summaries b1/b2[g,j,:] (fp32, contiguous, dim wide).
 *  score_kind DOT:     s = sum_d a_d*b1_d                 (mean-pooled q.k)
 *             MAXDOT2: s = max(sum a*b1, sum a*b2)        (src/ssa_model.py:118-119)
 *             QUEST:   s = sum_d a_d*(a_d>=0 ? b1_d : b2_d), b1=kmax, b2=kmin
 *                                                         (src/qwen_blocksparse.py:117-120)
 *  each sum is one fp32 fma chain over d = 0..dim-1 starting from 0.
 *  Ranking: higher score first, ties to the lower block id.
 *  layout SSA:    row i = [i, top-T content blocks by rank], T = min(topk, nblk-1);
 *                 candidates j != i (and j < i when causal); missing picks are
 *                 filled with i (src/ssa_model.py:151-162).
 *  layout FINISH: top-T over j <= i with T = min(topk, nblk), missing picks -> i,
 *                 then append i (and block 0 when sink), sorted ascending
 *                 (src/qwen_blocksparse.py:87-99).
 *  layout RAW:    the top-T over j <= i, T = min(topk, nblk), in rank order,
 *                 -1 where fewer exist (stage 1 of SelectTwoStage,
 *                 src/qwen_blocksparse.py:285-286).
 *  score_out / gate_out (optional, SSA only): the score of each selected block
 *  and logsigmoid(score) (src/ssa_model.py:189-191).  topk <= 32. */
typedef enum { BSA_SCORE_DOT = 0, BSA_SCORE_MAXDOT2 = 1, BSA_SCORE_QUEST = 2 } bsa_score_kind;
typedef enum { BSA_SEL_SSA = 0, BSA_SEL_FINISH = 1, BSA_SEL_RAW = 2 } bsa_sel_layout;
typedef struct {
  int32_t G, nblk, dim;
  int32_t score_kind, layout, causal, topk, sink;
  const float *a, *b1, *b2;
  int32_t *sel;      /* (G, nblk, width) */
  float *score_out;  /* optional (G, nblk, width) */
  float *gate_out;   /* optional (G, nblk, width) */
  int32_t *status;
  /* query-block range (0, 0 = all): a holds the summaries of the query blocks
   * [q_blk0, q_blk0 + nq) only and sel/score/gate their nq rows; b1/b2 keep all
   * nblk key blocks; masks and the own block use global indices.  No reference
   * counterpart: used by the query-block sharding across GPUs. */
  int32_t q_blk0, nq;
} bsa_select_args;
int32_t bsa_select_width(const bsa_select_args *a);
bsa_status bsa_select(const bsa_select_args *a, bsa_stream_t stream);

/* LSH candidate selection in the SSA layout (row i = [i, picks...]).
 * Replaces the inference branch of LSHBucketSSA (reference
 * src/ssa_model.py:438-470).  Per group g: query summaries a[g,i,:] and key
 * summaries b[g,j,:] (fp32, contiguous, dim wide) are L2-normalised
 * (y = x / max(|x|, 1e-12), src/ssa_model.py:397-399) and hashed once per round:
 *   ARGMAX: bucket = argmax_c <y, planes[:, r, c]>, n_planes buckets (:438-439);
 *   SIGN:   bucket = bits [<y, planes[:, r, c]> > 0], 2^n_planes buckets.
 * Each (round, bucket) keeps its first `cap` key blocks by index (:441-450).
 * Candidates of query block i = the key blocks in its bucket of every round,
 * deduplicated, excluding i (and j > i when causal) (:451-462); like the
 * reference, which dedups ids clamped at 0, block 0 is also dropped when an
 * earlier round's list had an empty slot (:452-457); score =
 * scale * <yq_i, yk_j>; the top min(topk, max(1, nblk-1), n_rounds*cap) by
 * (score desc, block asc) follow i in the row; missing picks are filled with i
 * (their score_out is 0, as the reference's gscore, :472-476).  planes:
 * (dim, n_rounds, n_planes) fp32.  Dots are fp32 fma chains over d from 0. */
typedef enum { BSA_HASH_ARGMAX = 0, BSA_HASH_SIGN = 1 } bsa_hash_kind;
typedef struct {
  int32_t G, nblk, dim;
  int32_t hash_kind, n_rounds, n_planes, cap, causal, topk;
  float scale;
  const float *a, *b, *planes;
  int32_t *sel;      /* (G, nblk, width) */
  float *score_out;  /* optional (G, nblk, width) */
  float *gate_out;   /* optional (G, nblk, width): logsigmoid(score_out) */
  int32_t *status;
} bsa_lsh_args;
int32_t bsa_select_lsh_width(const bsa_lsh_args *a);
size_t bsa_select_lsh_workspace(const bsa_lsh_args *a);
bsa_status bsa_select_lsh(const bsa_lsh_args *a, void *workspace, size_t workspace_bytes,
                          bsa_stream_t stream);

/* Decode: the T newest tokens (positions L-T .. L-1, all in the last block
 * (L-1)/bs) attend to the selected blocks of a K/V cache.  No reference
 * counterpart (the reference has no decode path); the arithmetic is
 * bsa_attn_fwd's restricted to those rows: logit = scale * q.k + gate[slot],
 * causal by position, SLOT or TOKEN masks as in bsa_attn_args (slot 0 = the own
 * block in SLOT mode).  q, o: (B, Hq, T, D); k, v: (B, Hkv, >= L, D) with rows
 * [0, L) valid; sel: int32 (B, Hs, kk) block ids for this step (sel_sh = 0 shares
 * one row over the KV heads), gate: optional fp32 addressed like sel.  Split-K
 * over the selected blocks with a fp32 workspace of bsa_decode_workspace bytes.
 * Limits: (Hq/Hkv)*T <= 32, D and bs divide 256, bs <= 128. */
typedef struct {
  int32_t dtype, B, Hq, Hkv, L, D, bs, T, kk, mask_mode;
  float scale;
  bsa_view q, k, v, o;
  const int32_t *sel;
  int64_t sel_sb, sel_sh;
  const float *gate;
  int64_t gate_sb, gate_sh;
  int32_t *status;
} bsa_decode_args;
size_t bsa_decode_workspace(const bsa_decode_args *a);
bsa_status bsa_decode(const bsa_decode_args *a, void *workspace, size_t workspace_bytes,
                      bsa_stream_t stream);

/* Top-k of a caller-supplied score matrix with _finish semantics (reference
 * src/qwen_blocksparse.py:87-99): per row i of score (G, nblk, nblk) (element
 * strides score_sg, score_si, unit column stride) the top min(topk, nblk) over
 * j <= i by (score desc, block asc), non-finite or missing picks -> i, then i
 * and (sink) block 0 appended, ascending.  Backs SelectOracle (a per-block
 * attention mass, :124-137) and SelectRandom (uniform draws, :140-152). */
typedef struct {
  int32_t G, nblk, topk, sink;
  const float *score;
  int64_t score_sg, score_si;
  int32_t *sel; /* (G, nblk, bsa_select_scores_width) */
  int32_t *status;
} bsa_scores_args;
int32_t bsa_select_scores_width(const bsa_scores_args *a);
bsa_status bsa_select_scores(const bsa_scores_args *a, bsa_stream_t stream);

/* Per-token Quest bound, max over the query block's tokens, with _finish
 * semantics: score(i, j) = max_t sum_d q[i,t,d] * (q >= 0 ? kmax[j,d] : kmin[j,d])
 * over the bs token rows of query block i (padding rows included as zeros, as
 * the reference pads), candidates j <= i — all of them (SelectMaxQMax,
 * src/qwen_blocksparse.py:221-247) or the M per-row candidates in cand, -1 or
 * j > i ignored (SelectTwoStage's re-score, :270-299).  qtok: fp32
 * (G, nblk, bs, dim) group-mean query tokens; kmax/kmin: fp32 (G, nblk, dim).
 * Each token score is one fp32 fma chain over d from 0. */
typedef struct {
  int32_t G, nblk, bs, dim, topk, sink, M;
  const float *qtok, *kmax, *kmin;
  const int32_t *cand; /* optional (G, nblk, M) */
  int32_t *sel;        /* (G, nblk, bsa_select_scores_width) */
  int32_t *status;
} bsa_qmax_args;
bsa_status bsa_select_qmax(const bsa_qmax_args *a, bsa_stream_t stream);

/* CSR transpose of a selection: for every (b, sel head, key block) the list of
 * entries e = qblk*kk + slot whose slot is active under the mask rules of
 * bsa_attn_args, in ascending e.  row_ptr: int32 (B*Hs*nblk + 1);
 * col: int32, capacity B*Hs*nblk*kk.  Used internally by bsa_attn_bwd and
 * exported for testing.  Has no single reference counterpart: it replaces the
 * atomic scatter of src/triton_kernel.py:178-179. */
typedef struct {
  int32_t B, Hs, nblk, kk, bs, L;
  int32_t mask_mode, causal;
  const int32_t *sel;
  int64_t sel_sb, sel_sh, sel_sn;
  int32_t *row_ptr, *col;
  int32_t *status;
  /* query-block range (0, 0 = all nblk): sel holds rows for the query blocks
   * [q_blk0, q_blk0 + nq) and entries are e = (qblk - q_blk0)*kk + slot */
  int32_t q_blk0, nq;
} bsa_csr_args;
size_t bsa_csr_workspace(const bsa_csr_args *a);
bsa_status bsa_sel_csr(const bsa_csr_args *a, void *workspace, size_t workspace_bytes,
                       bsa_stream_t stream);

/* The same CSR transpose for callers that cannot allocate device memory (a
 * locked or exhausted memory pool, a host runtime that owns every device
 * allocation, a loop that must not enter the allocator).  No counterpart in the
 * reference.  Its scratch is a fixed 16 MiB device array inside the library
 * (held by every GPU that loads it until exit); selections needing more are
 * rejected with BSA_ERR_UNSUPPORTED.  The first call on a device resolves the
 * array's address and should precede any stream capture; the address is kept
 * for the life of the process, so it does not survive cudaDeviceReset (do not
 * call this entry point after resetting a device in the same process).  Calls
 * share the array, so calls that overlap on the GPU race.  Allocates nothing. */
bsa_status bsa_sel_csr_noalloc(const bsa_csr_args *a, bsa_stream_t stream);

/* CentroidSSA's bucket routing (reference src/ssa_model.py:263-299): bucket c
 * holds the first cap key blocks j (by index) with key_cent[b,j] == c; query
 * block i reads the buckets of top_c[b,i,0..cpq) (cpq-major, cap-minor), its own
 * block replaced by -1; with q_blk (refine, rk < cpq*cap) only the rk candidates
 * of largest q_blk[b,i].k_blk[b,j] (fp32 fma chains over dim) are kept, best
 * first, -1 for missing picks.  sel: int32 (B, nblk, bsa_centroid_width(a)) with
 * the own block in column 0.  key_cent / top_c come from the module's
 * differentiable centroid scores (argmax / top-cpq), which stay in torch. */
typedef struct {
  int32_t B, nblk, C, cpq, cap, dim, rk;
  const int32_t *key_cent; /* (B, nblk) */
  const int32_t *top_c;    /* (B, nblk, cpq) */
  const float *q_blk, *k_blk; /* (B, nblk, dim), optional (refine) */
  int32_t *sel;
} bsa_centroid_args;
int32_t bsa_centroid_width(const bsa_centroid_args *a);
bsa_status bsa_centroid_route(const bsa_centroid_args *a, bsa_stream_t stream);

/* Partial rotary embedding with the arithmetic of transformers'
 * apply_rotary_pos_emb (qwen3_5_moe, v5.5.0): on the first `rot` dims,
 * y = x*cos + rotate_half(x)*sin with each product and the sum rounded to the
 * tensor dtype; dims >= rot are copied.  cos/sin: (B, L, rot) in x's dtype with
 * element strides cs_sb, cs_sl.  y may alias x.  Used by the Qwen variant
 * (reference src/patch_qwen.py:47-48). */
typedef struct {
  int32_t dtype;
  int32_t B, H, L, D, rot;
  bsa_view x, y;
  const void *cos, *sin;
  int64_t cs_sb, cs_sl;
} bsa_rope_args;
bsa_status bsa_rope(const bsa_rope_args *a, bsa_stream_t stream);

/* Turns a device status word (already copied to the host) into a bsa_status. */
bsa_status bsa_status_decode(int32_t device_word);

/* Thread-local message of the last failing call ("" if none). */
const char *bsa_last_error(void);

/* Library version (major*10000 + minor*100 + patch). */
int32_t bsa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* BSA_B200_H */
