"""Attention oracles for the draft and verify paths (numpy, test infrastructure only).

Layouts follow the reference's packed "THD" convention: queries ``[sum Q, Hq, D]``
and keys/values ``[sum K, Hkv, D]`` with per-request row ranges given by the
query/key length lists. Query head ``h`` reads KV head ``h // (Hq // Hkv)``,
which is what SDPA ``enable_gqa=True`` and ``repeat_interleave`` do
(dspark_qwen/model.py:58-59).

All arithmetic runs in ``compute_dtype`` (float64 by default, so the oracle is
at least as exact as the reference's float32 SDPA).
"""
import numpy as np


def _attend(q, k, v, visible, scale, compute_dtype):
    """One request: q [nq,Hq,D], k/v [nk,Hkv,D], visible [nq,nk] bool or None."""
    nq, hq, d = q.shape
    nk, hkv, _ = k.shape
    groups = hq // hkv
    qf = q.astype(compute_dtype, copy=False).reshape(nq, hkv, groups, d).transpose(1, 2, 0, 3)
    kf = k.astype(compute_dtype, copy=False).transpose(1, 2, 0)          # [Hkv, D, nk]
    vf = v.astype(compute_dtype, copy=False).transpose(1, 0, 2)          # [Hkv, nk, D]
    scores = np.matmul(qf.reshape(hkv, groups * nq, d), kf) * compute_dtype(scale)
    scores = scores.reshape(hkv, groups, nq, nk)
    if visible is not None:
        scores = np.where(visible[None, None], scores, -np.inf)
    scores = scores - scores.max(axis=-1, keepdims=True)
    p = np.exp(scores)
    p /= p.sum(axis=-1, keepdims=True)
    out = np.matmul(p.reshape(hkv, groups * nq, nk), vf).reshape(hkv, groups, nq, d)
    return out.transpose(2, 0, 1, 3).reshape(nq, hq, d)


def _bottom_right(nq, nk):
    """Query r of nq sees key j of nk iff j <= nk - nq + r (bottom-right aligned)."""
    return np.arange(nk)[None, :] <= np.arange(nk - nq, nk)[:, None]


def noncausal_varlen(q, k, v, query_lengths, key_lengths, scale, compute_dtype=np.float64):
    """Every query row of a request sees all of that request's keys.

    Restates ``test_only_noncausal_varlen`` (dspark_qwen/packed_draft.py:35-47):
    per-request SDPA with ``attn_mask=None, is_causal=False, enable_gqa=True``.
    """
    rows, qo, ko = [], 0, 0
    for nq, nk in zip(query_lengths, key_lengths):
        rows.append(_attend(q[qo:qo + nq], k[ko:ko + nk], v[ko:ko + nk], None, scale, compute_dtype))
        qo += nq
        ko += nk
    return np.concatenate(rows) if rows else np.zeros((0,) + q.shape[1:], compute_dtype)


def bottom_right_varlen(q, k, v, query_lengths, key_lengths, scale, compute_dtype=np.float64):
    """Bottom-right causal varlen attention; rows past sum(key_lengths) never read.

    Restates ``test_only_dense_varlen`` (dspark_qwen/varlen_target.py:98-112) and
    ``test_only_persistent_sdpa`` (dspark_qwen/persistent_qwen_target.py:30-42):
    query r of a request with nq queries and nk keys sees key j iff j <= nk-nq+r.
    A capacity tail after the last request is excluded by construction.
    """
    rows, qo, ko = [], 0, 0
    for nq, nk in zip(query_lengths, key_lengths):
        if not 0 < nq <= nk:
            raise ValueError('bottom-right causal attention needs 0 < q <= k per request')
        rows.append(_attend(q[qo:qo + nq], k[ko:ko + nk], v[ko:ko + nk],
                            _bottom_right(nq, nk), scale, compute_dtype))
        qo += nq
        ko += nk
    return np.concatenate(rows) if rows else np.zeros((0,) + q.shape[1:], compute_dtype)


def two_segment_attention(q, query_lengths, segments, scale, causal, compute_dtype=np.float64):
    """Keys of request i are the concatenation of two row ranges of two tensors.

    ``segments[i] = ((kA, vA, a_start, a_len), (kB, vB, b_start, b_len))``. This is
    the gather that ``PersistentTargetKV.prepare_attention``
    (dspark_qwen/persistent_target_kv.py:441-460) materialises (resident prefix,
    then scratch rows) and that ``PackedDraft.backbone`` builds with
    concat + index_select (dspark_qwen/packed_draft.py:215-226), followed by the
    bottom-right (``causal=True``) or non-causal attention of that gathered K/V.
    """
    rows, qo = [], 0
    for nq, ((ka, va, a0, na), (kb, vb, b0, nb)) in zip(query_lengths, segments):
        kk = np.concatenate([ka[a0:a0 + na], kb[b0:b0 + nb]])
        vv = np.concatenate([va[a0:a0 + na], vb[b0:b0 + nb]])
        nk = na + nb
        visible = _bottom_right(nq, nk) if causal else None
        rows.append(_attend(q[qo:qo + nq], kk, vv, visible, scale, compute_dtype))
        qo += nq
    return np.concatenate(rows)


def block_mask(anchors, block_size, context_length):
    """Training-layout draft mask, True = visible.

    Restates ``block_mask`` (dspark_qwen/model.py:12-19): query row of block b sees
    context key j iff j < anchors[b], and every row of its own block (bidirectional
    inside the block); other blocks are invisible. Shape ``[n*bs, ctx + n*bs]``.
    """
    anchors = np.asarray(anchors, dtype=np.int64)
    n = anchors.size
    q_block = np.arange(n * block_size) // block_size
    ctx = np.arange(context_length)
    visible_context = ctx[None, :] < anchors[q_block][:, None]
    visible_block = q_block[:, None] == q_block[None, :]
    return np.concatenate((visible_context, visible_block), axis=-1)


def training_layout_attention(q, k, v, context_lengths, anchors, block_size, scale,
                              compute_dtype=np.float64):
    """Packed training-layout draft attention over several sequences.

    Sequence s contributes ``len(anchors[s]) * block_size`` query rows and
    ``context_lengths[s] + len(anchors[s]) * block_size`` key rows laid out as
    [context ; blocks], exactly the K/V that ``DraftAttention.forward`` builds with
    ``project_kv(cat(context, z))`` (dspark_qwen/model.py:47-61). Each sequence is
    attended with ``block_mask`` (model.py:12-19); sequences never see each other,
    which is the document-isolation rule of the vendored NeMo packing mask.
    """
    rows, qo, ko = [], 0, 0
    for ctx, anc in zip(context_lengths, anchors):
        nq = len(anc) * block_size
        nk = ctx + nq
        visible = block_mask(anc, block_size, ctx)
        rows.append(_attend(q[qo:qo + nq], k[ko:ko + nk], v[ko:ko + nk], visible, scale, compute_dtype))
        qo += nq
        ko += nk
    return np.concatenate(rows)
