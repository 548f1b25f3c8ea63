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
    """logits [G, S] (may hold -inf), values [S, D] -> [G, D]."""
    if logits.shape[-1] == 0:
        return np.zeros((logits.shape[0], values.shape[-1]), dtype=np.float64)
    m = np.maximum(np.max(logits, axis=-1, keepdims=True), -1e30)
    p = np.exp(logits - m)
    l = p.sum(axis=-1, keepdims=True)
    return (p @ values) / (l + 1e-6)


def rotatek_decode(q_full, R_partial, delta_mu, k_full, v_full, mask_full, k_sparse,
                   v_sparse, num_kv_groups: int) -> np.ndarray:
    """Float64 reference of ``rotatek_decode_fused_triton``; returns [B, 1, H_q, D].

    Works one (batch, KV head) at a time, so full-size decode steps fit in memory."""
    q = _f64(q_full)
    bsz, heads, head_dim = q.shape
    hkv = heads // num_kv_groups
    g = num_kv_groups
    scale = 1.0 / math.sqrt(head_dim)
    mask = None if mask_full is None else _f64(mask_full)
    out = np.zeros((bsz, 1, heads, head_dim), dtype=np.float64)
    for b in range(bsz):
        for h in range(hkv):
            qg = q[b, h * g:(h + 1) * g]                                  # [G, D]
            R = _f64(R_partial[b, h])
            q_rot = qg @ R
            bias = qg @ _f64(delta_mu[b, h]) if delta_mu is not None else np.zeros(g)
            logit_v = (q_rot @ _f64(k_sparse[b, h]).T) * scale + (bias * scale)[:, None]
            logit_f = (qg @ _f64(k_full[b, h]).T) * scale
            if mask is not None:
                logit_f = np.where(mask[b][None, :] != 0, logit_f, -np.inf)
            logits = np.concatenate([logit_f, logit_v], axis=-1)
            values = np.concatenate([_f64(v_full[b, h]), _f64(v_sparse[b, h])], axis=0)
            out[b, 0, h * g:(h + 1) * g] = _softmax_merge(logits, values)
    return out


def full_channel_decode(q, k, v, num_kv_groups: int = 1) -> np.ndarray:
    """Float64 reference of ``full_channel_decode_triton``; returns [B, 1, H_q, D]."""
    q = _f64(q)
    bsz, heads, head_dim = q.shape
    g = num_kv_groups
    out = np.zeros((bsz, 1, heads, head_dim), dtype=np.float64)
    for b in range(bsz):
        for h in range(heads // g):
            qg = q[b, h * g:(h + 1) * g]
            logits = (qg @ _f64(k[b, h]).T) / math.sqrt(head_dim)
            out[b, 0, h * g:(h + 1) * g] = _softmax_merge(logits, _f64(v[b, h]))
    return out
