"""Preallocated span-split KV cache for RotateK decode.

The reference's split-mode cache (integrations/lmms_eval/models/model_utils/
cache_utils.py:48-55) appends each decode step's Keys and Values with
``torch.cat`` -- a copy of the whole Value cache per layer per step -- and the
adapters then build ``k_full = cat(prompt, text)`` and ``v_full = cat(V[:s_p],
V[s_p + s_v:])`` for every call (llama_visionzip.py:203-214): O(cache) copies
per step that cost more than the decode itself once the kernel is fast.

``SpanKVCache`` allocates each layer once, with room for ``max_new_tokens``
text tokens, in an order that keeps both decode spans contiguous:

    keys_full  [B, H_kv, S_p + T_max, D]          prompt | text (grows)
    values     [B, H_kv, S_p + T_max + S_v, D]    prompt | text (grows) | visual
    keys_rot   [B, H_kv, S_v, D_keep]             rotated, truncated visual Keys

so ``decode_args`` hands ``rotatek_decode`` plain views (no mask: every stored
token is valid) and ``update`` writes the new tokens in place.  The attention
result does not depend on where a token sits in memory (softmax sums over all
of them), so the order differs from the reference's [prompt | visual | text]
without changing any output.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch


@dataclass
class _Layer:
    keys_full: torch.Tensor      # [B, H, S_p + T_max, D]
    values: torch.Tensor         # [B, H, S_p + T_max + S_v, D]
    keys_rot: torch.Tensor       # [B, H, S_v, D_keep]
    rotation: torch.Tensor       # R_partial [B, H, D, D_keep]
    delta_mu: Optional[torch.Tensor]
    s_prompt: int
    s_vision: int
    s_text: int
    t_max: int


class SpanKVCache:
    """Split KV cache with in-place decode appends (RotateK layers)."""

    def __init__(self, max_new_tokens: int):
        if max_new_tokens < 0:
            raise ValueError("max_new_tokens must be >= 0")
        self.max_new_tokens = max_new_tokens
        self.layers: List[_Layer] = []
        self._seen_tokens = 0

    def __len__(self):
        return len(self.layers)

    def store_pruned(self, key_states_pruned, key_states_prompt, key_states_text, value_states,
                     rotation, delta_mu, layer_idx: int) -> None:
        """Prefill-time write of one layer (the split-mode store of
        cache_utils.py:93-113 plus the RotateK state of kv_pruning_utils.py:155-156).
        ``value_states`` is [B, H, S_p + S_v + S_t, D] in prefill order."""
        if layer_idx != len(self.layers):
            raise ValueError(f"layers must be stored in order (expected {len(self.layers)}, got {layer_idx})")
        b, h, s_p, d = key_states_prompt.shape
        s_v, s_t = key_states_pruned.shape[2], key_states_text.shape[2]
        if value_states.shape[2] != s_p + s_v + s_t:
            raise ValueError("value_states must cover prompt + visual + text tokens")
        t_max = s_t + self.max_new_tokens
        dev, dt = key_states_prompt.device, key_states_prompt.dtype
        kf = torch.empty(b, h, s_p + t_max, d, dtype=dt, device=dev)
        kf[:, :, :s_p].copy_(key_states_prompt)
        kf[:, :, s_p:s_p + s_t].copy_(key_states_text)
        v = torch.empty(b, h, s_p + t_max + s_v, d, dtype=value_states.dtype, device=dev)
        v[:, :, :s_p].copy_(value_states[:, :, :s_p])
        v[:, :, s_p:s_p + s_t].copy_(value_states[:, :, s_p + s_v:])
        v[:, :, s_p + t_max:].copy_(value_states[:, :, s_p:s_p + s_v])
        # The text slots not written yet are read by static_decode_args' full-capacity
        # views and only masked out of the logits: the P.V product still multiplies
        # their Values by a zero weight, so they must hold finite numbers (0 * NaN
        # is NaN).  Zero them once here.
        kf[:, :, s_p + s_t:].zero_()
        v[:, :, s_p + s_t:s_p + t_max].zero_()
        if layer_idx == 0:
            self._seen_tokens += s_p + s_v + s_t
        self.layers.append(_Layer(kf, v, key_states_pruned.contiguous(), rotation, delta_mu, s_p, s_v, s_t, t_max))

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int) -> None:
        """Decode-time append of n new tokens ([B, H, n, D]) to the text span, in place."""
        L = self.layers[layer_idx]
        n = key_states.shape[2]
        if L.s_text + n > L.t_max:
            raise ValueError(f"text span full: {L.s_text} + {n} tokens > capacity {L.t_max}")
        pos = L.s_prompt + L.s_text
        L.keys_full[:, :, pos:pos + n].copy_(key_states)
        L.values[:, :, pos:pos + n].copy_(value_states)
        L.s_text += n
        if layer_idx == 0:
            self._seen_tokens += n

    def decode_args(self, layer_idx: int) -> dict:
        """Keyword arguments of ``rotatek_decode`` for this layer (views; q_full and
        num_kv_groups are the caller's)."""
        L = self.layers[layer_idx]
        s_f = L.s_prompt + L.s_text
        return dict(R_partial=L.rotation, delta_mu=L.delta_mu, k_full=L.keys_full[:, :, :s_f],
                    v_full=L.values[:, :, :s_f], mask_full=None, k_sparse=L.keys_rot,
                    v_sparse=L.values[:, :, L.s_prompt + L.t_max:])

    # ---- static-shape decode (CUDA-graph capture): the append position and the
    # validity mask live on the device, the views cover the whole capacity
    def write_at(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
                 index: torch.Tensor) -> None:
        """Write n new tokens ([B, H, n, D]) at text slots ``index`` (device int64
        [n], absolute positions in keys_full / values); host counters untouched."""
        L = self.layers[layer_idx]
        L.keys_full.index_copy_(2, index, key_states)
        L.values.index_copy_(2, index, value_states)

    def capacity_mask(self, layer_idx: int = 0) -> torch.Tensor:
        """A [B, S_p + T_max] uint8 mask, 1 on the prompt and the text stored so far."""
        L = self.layers[layer_idx]
        m = torch.zeros(L.keys_full.shape[0], L.s_prompt + L.t_max, dtype=torch.uint8,
                        device=L.keys_full.device)
        m[:, :L.s_prompt + L.s_text] = 1
        return m

    def static_decode_args(self, layer_idx: int, mask: torch.Tensor) -> dict:
        """``decode_args`` over the whole text capacity, unwritten slots masked."""
        L = self.layers[layer_idx]
        cap = L.s_prompt + L.t_max
        return dict(R_partial=L.rotation, delta_mu=L.delta_mu, k_full=L.keys_full[:, :, :cap],
                    v_full=L.values[:, :, :cap], mask_full=mask, k_sparse=L.keys_rot,
                    v_sparse=L.values[:, :, cap:])

    def get_seq_length(self, layer_idx: int = 0) -> int:
        if len(self.layers) <= layer_idx:
            return 0
        L = self.layers[layer_idx]
        return L.s_prompt + L.s_vision + L.s_text


__all__ = ["SpanKVCache"]
