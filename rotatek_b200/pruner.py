"""``update_rotatek`` on the B200 builder, for ``ChannelPruner``
(integrations/lmms_eval/models/model_utils/kv_pruning_utils.py:38-169).

``ChannelPruner.update_rotatek`` is the one pruner method on the RotateK hot
path; ThinK and SparK (update_think / update_spark) are other methods and stay
with the reference.  This module provides a pruner with the reference's
constructor, span split and ``update_rotatek`` contract:

    kept, kv_prompt, kv_text, keep_mask, value_states = pruner.update_rotatek(
        key_states, query_states, value_states, attention_mask, num_key_value_groups)

and leaves ``current_rotatek_R_partial`` / ``current_rotatek_delta_mu`` on the
pruner, as kv_pruning_utils.py:155-156 does.  To switch an existing checkout,
assign ``ChannelPruner.update_rotatek = rotatek_b200.pruner.update_rotatek``.
"""
from __future__ import annotations

from rotatek_b200.rotation import QUERY_WINDOW, build_rotation, keep_count


def split_spans(pruner, key_states):
    """(prompt Keys, visual Keys, text Keys) views of [B, H_kv, S, D]
    (kv_pruning_utils.py:26-35)."""
    total = key_states.shape[-2]
    prompt = max(0, min(pruner.prompt_seqlen, total))
    query = max(0, min(pruner.query_seqlen, max(total - prompt, 0)))
    vision_end = total - query if query > 0 else total
    kv_prompt = key_states[:, :, :prompt, :]
    keys_vision = key_states[:, :, prompt:vision_end, :]
    kv_text = key_states[:, :, -query:, :] if query > 0 else key_states[:, :, :0, :]
    return kv_prompt, keys_vision, kv_text


def update_rotatek(self, key_states, query_states, value_states, attention_mask,
                   num_key_value_groups):
    """RotateK for one layer at prefill: rotate the visual Keys into the top
    eigenbasis of their (query-weighted) covariance and keep D_keep channels.
    Same inputs, outputs and side attributes as the reference method."""
    del attention_mask
    assert key_states.shape[-2] == query_states.shape[-2]
    head_dim = key_states.shape[-1]
    kv_prompt, keys_vision, kv_text = split_spans(self, key_states)
    keep = keep_count(head_dim, self.ratio)
    window = min(QUERY_WINDOW, query_states.shape[2])
    queries_recent = query_states[..., query_states.shape[2] - window:, :]
    kept, R, delta_mu, keep_mask = build_rotation(keys_vision, queries_recent, keep,
                                                  num_key_value_groups)
    self.current_rotatek_R_partial = R
    self.current_rotatek_delta_mu = delta_mu
    return kept, kv_prompt, kv_text, keep_mask, value_states


class ChannelPruner:
    """Pruner with the reference's constructor (kv_pruning_utils.py:38-42)
    carrying the B200 ``update_rotatek``."""

    def __init__(self, ratio, prompt_seqlen, query_seqlen):
        self.ratio = ratio
        self.prompt_seqlen = prompt_seqlen
        self.query_seqlen = query_seqlen

    update_rotatek = update_rotatek


def init_channel_pruner(module):
    """Attach a fresh pruner to attention module ``module`` (kv_pruning_utils.py:163-169)."""
    module.channel_pruner = ChannelPruner(ratio=module.config.channel_ratio,
                                          prompt_seqlen=module.config.prompt_seqlen,
                                          query_seqlen=module.config.query_seqlen)
