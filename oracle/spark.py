"""SparK baseline oracle in numpy (test infrastructure).

Restates the reference's per-token channel pruning and its decode-time
recovery:

* rotatek/baselines/spark.py:15-58            per_token_channel_prune: score
  k^2 * ||Q||_2 (norm over the query window, per channel), keep the top
  D_keep channels of each token, K_compact = the kept values in channel order,
  keep_mask, pruned_mean = mean of the token's pruned values
* integrations/.../kv_pruning_utils.py:63-90  ChannelPruner.update_spark: the
  queries are the last QUERY_WINDOW (32) query tokens, averaged over each GQA
  group before scoring
* integrations/.../llava_next/llama_visionzip.py:226-242  recovery (fill with
  pruned_mean, write the kept values into the kept channels), concatenation
  [prompt | recovered | text] and the dense decode

``pack_indices`` is the layout this build's SparK decode reads: each token's
kept channels in ascending order (what the boolean-index assignment of
llama_visionzip.py:230 walks).  Pinned against fixtures written by the
reference's own ``update_spark`` and its Triton dense decode
(tests/golden/make_golden.py, spark_* fixtures).
"""
from __future__ import annotations

import numpy as np

from oracle import decode as odec

QUERY_WINDOW = 32


def per_token_channel_prune(queries, keys, ratio: float):
    """(K_compact, keep_mask, pruned_mean) of spark.py:15-58 in float32.

    queries [B, H, Q, D] (already grouped to the KV heads), keys [B, H, S, D].
    Ties between equal scores are broken towards the lower channel (a stable
    descending sort); the reference's unstable argsort may order them either
    way, so fixtures use inputs without ties."""
    q = np.asarray(queries, dtype=np.float32)
    k = np.asarray(keys, dtype=np.float32)
    d = k.shape[-1]
    keep = d - int(d * ratio)
    q_norm = np.sqrt((q.astype(np.float64) ** 2).sum(axis=-2)).astype(np.float32)[..., None, :]
    scores = (k * k) * q_norm
    order = np.argsort(-scores, axis=-1, kind="stable")
    keep_idx = np.sort(order[..., :keep], axis=-1)
    compact = np.take_along_axis(k, keep_idx, axis=-1)
    mask = np.zeros(k.shape, dtype=bool)
    np.put_along_axis(mask, keep_idx, True, axis=-1)
    pruned = np.take_along_axis(k, order[..., keep:], axis=-1)
    mean = pruned.astype(np.float64).mean(axis=-1, keepdims=True)
    return compact, mask, mean


def update_spark_queries(query_states, num_kv_groups: int):
    """The scoring queries of update_spark: the last QUERY_WINDOW query tokens,
    mean over each KV head's group (kv_pruning_utils.py:78-82)."""
    q = np.asarray(query_states, dtype=np.float64)
    b, hq, s, d = q.shape
    w = min(QUERY_WINDOW, s)
    return q[:, :, -w:].reshape(b, hq // num_kv_groups, num_kv_groups, w, d).mean(axis=2)


def pack_indices(keep_mask) -> np.ndarray:
    """keep_mask [..., D] bool -> kept channels [..., D_keep] ascending (uint8)."""
    m = np.asarray(keep_mask, dtype=bool)
    keep = int(m.sum(axis=-1).max()) if m.size else 0
    if m.size and not np.all(m.sum(axis=-1) == keep):
        raise ValueError("every token must keep the same number of channels")
    order = np.argsort(~m, axis=-1, kind="stable")[..., :keep]
    return order.astype(np.uint8)


def recover(k_compact, keep_idx, pruned_mean) -> np.ndarray:
    """Full-width visual Keys: pruned_mean everywhere, the kept values in
    their channels (llama_visionzip.py:228-230); float64."""
    kc = np.asarray(k_compact, dtype=np.float64)
    idx = np.asarray(keep_idx, dtype=np.int64)
    mean = np.asarray(pruned_mean, dtype=np.float64)
    out = np.broadcast_to(mean, kc.shape[:-1] + (128,)).copy()
    np.put_along_axis(out, idx, kc, axis=-1)
    return out


def spark_decode(q_full, k_full, v_full, mask_full, k_compact, keep_idx, pruned_mean, v_sparse,
                 num_kv_groups: int) -> np.ndarray:
    """The dense decode over [k_full ; recovered] / [v_full ; v_sparse] with
    mask_full over the prompt/text span (float64, [B, 1, H_q, D]): the
    RotateK oracle with R = I and no delta_mu is exactly that decode."""
    rec = recover(k_compact, keep_idx, pruned_mean)
    b, h = rec.shape[:2]
    eye = np.broadcast_to(np.eye(128), (b, h, 128, 128))
    return odec.rotatek_decode(q_full, eye, None, k_full, v_full, mask_full, rec, v_sparse, num_kv_groups)
