"""Key-projection oracle in numpy (test infrastructure).

Restates the prefill Key path of the attention adapters and the sums the
covariance pass takes over its visual span:

  llava_next/llama_visionzip.py:144     key_states = k_proj(hidden_states)
                                        (nn.Linear: X W^T + b, one rounding to the
                                        storage dtype; float64 accumulation here)
  llama_visionzip.py:147                .view(B, S, H_kv, D).transpose(1, 2)
  llama_visionzip.py:152-153            apply_rotary_pos_emb (transformers 4.49,
                                        modeling_llama): k * cos + rotate_half(k) * sin,
                                        rotate_half(k) = cat(-k[D/2:], k[:D/2]);
                                        each product and the sum rounded to the
                                        storage dtype, as torch's bf16 / fp16 ops do
  qwen/qwen2_5vl_visionzip.py:932-942   same, after the multimodal sections of
                                        cos / sin are merged (a [B, S, D] table)
  kv_pruning_utils.py:112-115           the raw sums behind mean and covariance of
                                        the visual Keys: sum_s k k^T, sum_s k

Pinned against tests/golden/kproj_bf16.npz, made by running torch's nn.Linear and
transformers' apply_rotary_pos_emb on CPU (tests/golden/make_golden.py).
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

from oracle.bf16 import round_to


def rotate_half(x: np.ndarray) -> np.ndarray:
    """transformers modeling_llama.rotate_half: cat(-x2, x1) over the last axis."""
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def key_projection(hidden: np.ndarray, w_k: np.ndarray, bias: Optional[np.ndarray], cos: np.ndarray,
                   sin: np.ndarray, storage: str, head_dim: int = 128) -> np.ndarray:
    """Post-RoPE Keys [B, H_kv, S, D] from hidden [B, S, hidden], w_k [H_kv D, hidden],
    bias [H_kv D] or None, cos / sin [B | 1, S, D] (values already in `storage`)."""
    x = np.asarray(hidden, dtype=np.float64)
    w = np.asarray(w_k, dtype=np.float64)
    k = x @ w.T
    if bias is not None:
        k = k + np.asarray(bias, dtype=np.float64)
    k = round_to(k, storage).astype(np.float64)
    b, s, _ = x.shape
    h = w.shape[0] // head_dim
    k = k.reshape(b, s, h, head_dim).transpose(0, 2, 1, 3)          # [B, H, S, D]
    c = np.asarray(cos, dtype=np.float64)[:, None]                  # [B | 1, 1, S, D]
    sn = np.asarray(sin, dtype=np.float64)[:, None]
    kc = round_to(k * c, storage).astype(np.float64)
    rs = round_to(rotate_half(k) * sn, storage).astype(np.float64)
    return round_to(kc + rs, storage)


ULP = {"bfloat16": 2.0 ** -7, "float16": 2.0 ** -10}


def key_mismatch(ours, ref, storage: str) -> Tuple[float, float]:
    """How far two post-RoPE Key tensors are apart: (fraction of elements that
    differ, largest |difference| in ulps of the element's RoPE pair magnitude
    sqrt(k_d^2 + k_{d+D/2}^2)).  Two correct implementations differ only where
    the projection's accumulation order moves a value across a rounding
    boundary (one ulp of k), which RoPE can turn into a few ulps of a small
    output (cancellation), never more than a few ulps of the pair."""
    a = np.asarray(ours, np.float64)
    r = np.asarray(ref, np.float64)
    half = r.shape[-1] // 2
    pair = np.sqrt(r[..., :half] ** 2 + r[..., half:] ** 2)
    mag = np.concatenate([pair, pair], axis=-1)
    d = np.abs(a - r)
    worst = d / np.maximum(mag * ULP[storage], np.finfo(np.float32).tiny)
    return float((d > 0).mean()), float(worst.max()) if worst.size else 0.0


def visual_sums(keys: np.ndarray, vis_start: int, vis_len: int) -> Tuple[np.ndarray, np.ndarray]:
    """(sum_s k k^T [B, H, D, D], sum_s k [B, H, D]) over tokens [vis_start, vis_start + vis_len), float64."""
    v = np.asarray(keys[:, :, vis_start:vis_start + vis_len], dtype=np.float64)
    return np.einsum("bhsi,bhsj->bhij", v, v), v.sum(axis=2)
