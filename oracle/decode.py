"""Decode attention oracle in numpy float64 (test infrastructure).

Restates the arithmetic of the reference's `paper` kernels:

* rotatek/kernels/fused_decode.py:131-148   q~ = q . R_partial,  bias = q . delta_mu
* fused_decode.py:158-183                   visual logits = (q~ . k~) * s + bias * s
* fused_decode.py:243-273                   prompt/text logits = (q . k) * s, masked to
                                             -inf where mask_full == 0 (254-258)
* fused_decode.py:151, 238                  running max starts at -1e30
* fused_decode.py:275-296                   merge, out = acc / (l + 1e-6), cast to q's dtype
* full_channel_flash_decoding.py:34-155     dense split-K decode, same normalisation

with s = 1/sqrt(D) (fused_decode.py:340).  The online softmax of the kernels
equals the closed form below because every partial is rescaled to the final
running max before the division; the -1e30 floor only matters when no token
is attended (then out = 0 / (0 + 1e-6) = 0).
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np


def _f64(x) -> Optional[np.ndarray]:
    if x is None:
        return None
    if hasattr(x, "detach"):
        x = x.detach().cpu().float().numpy()
    return np.asarray(x, dtype=np.float64)


def _softmax_merge(logits: np.ndarray, values: np.ndarray) -> np.ndarray:
    """logits [B, H, S] (may hold -inf), values [B, H, S, D] -> [B, H, D]."""
    if logits.shape[-1] == 0:
        return np.zeros(values.shape[:2] + values.shape[-1:], dtype=np.float64)
    m = np.maximum(np.max(logits, axis=-1, keepdims=True), -1e30)
    p = np.exp(logits - m)
    l = p.sum(axis=-1, keepdims=True)
    acc = np.einsum("bhs,bhsd->bhd", p, values)
    return acc / (l + 1e-6)


def rotatek_decode(q_full, R_partial, delta_mu, k_full, v_full, mask_full, k_sparse,
                   v_sparse, num_kv_groups: int) -> np.ndarray:
    """Float64 reference of ``rotatek_decode_fused_triton``; returns [B, 1, H_q, D]."""
    q = _f64(q_full)
    R = _f64(R_partial)
    dm = _f64(delta_mu)
    kf, vf = _f64(k_full), _f64(v_full)
    ks, vs = _f64(k_sparse), _f64(v_sparse)
    mask = _f64(mask_full)
    bsz, heads, head_dim = q.shape
    kv_of = np.arange(heads) // num_kv_groups
    scale = 1.0 / math.sqrt(head_dim)

    q_rot = np.einsum("bhd,bhdk->bhk", q, R[:, kv_of])
    bias = np.einsum("bhd,bhd->bh", q, dm[:, kv_of]) if dm is not None else np.zeros((bsz, heads))
    logit_v = np.einsum("bhk,bhsk->bhs", q_rot, ks[:, kv_of]) * scale + (bias * scale)[..., None]
    logit_f = np.einsum("bhd,bhsd->bhs", q, kf[:, kv_of]) * scale
    logit_f = np.where(mask[:, None, :] != 0, logit_f, -np.inf)

    logits = np.concatenate([logit_f, logit_v], axis=-1)
    values = np.concatenate([vf[:, kv_of], vs[:, kv_of]], axis=-2)
    return _softmax_merge(logits, values)[:, None]


def full_channel_decode(q, k, v, num_kv_groups: int = 1) -> np.ndarray:
    """Float64 reference of ``full_channel_decode_triton``; returns [B, 1, H_q, D]."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    heads, head_dim = q.shape[1], q.shape[2]
    kv_of = np.arange(heads) // num_kv_groups
    logits = np.einsum("bhd,bhsd->bhs", q, k[:, kv_of]) / math.sqrt(head_dim)
    return _softmax_merge(logits, v[:, kv_of])[:, None]
