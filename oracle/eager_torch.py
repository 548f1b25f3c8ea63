"""The reference's eager PyTorch path on CPU, used as the timed CPU baseline
(test infrastructure).

The reference has no eager decode for RotateK (its decode is Triton only), so
``rotatek_decode_eager`` restates rotatek/kernels/fused_decode.py:131-296 with
batched torch ops in fp32 -- one einsum per span, one softmax over both spans,
one weighted sum.  ``update_rotatek_eager`` follows
kv_pruning_utils.py:105-160 with torch ops (the `eigh` solver; the default
power-iteration solver asserts CUDA, rotation.py:87).
"""
from __future__ import annotations

import math

import torch


def rotatek_decode_eager(q_full, R_partial, delta_mu, k_full, v_full, mask_full, k_sparse,
                         v_sparse, num_kv_groups: int) -> torch.Tensor:
    q = q_full.float()
    bsz, heads, head_dim = q.shape
    hkv = R_partial.shape[1]
    g = num_kv_groups
    scale = 1.0 / math.sqrt(head_dim)
    qg = q.view(bsz, hkv, g, head_dim)
    q_rot = torch.einsum("bhgd,bhdk->bhgk", qg, R_partial.float())
    logit_v = torch.einsum("bhgk,bhsk->bhgs", q_rot, k_sparse.float())
    if delta_mu is not None:
        logit_v = logit_v + torch.einsum("bhgd,bhd->bhg", qg, delta_mu.float())[..., None]
    logit_v = logit_v * scale
    logit_f = torch.einsum("bhgd,bhsd->bhgs", qg, k_full.float()) * scale
    logit_f = logit_f.masked_fill(mask_full[:, None, None, :] == 0, float("-inf"))
    logits = torch.cat([logit_f, logit_v], dim=-1)
    m = logits.amax(dim=-1, keepdim=True).clamp(min=-1e30)
    p = torch.exp(logits - m)
    l = p.sum(dim=-1, keepdim=True)
    sf = k_full.shape[-2]
    acc = torch.einsum("bhgs,bhsd->bhgd", p[..., :sf], v_full.float()) + \
        torch.einsum("bhgs,bhsd->bhgd", p[..., sf:], v_sparse.float())
    out = acc / (l + 1e-6)
    return out.reshape(bsz, 1, heads, head_dim).to(q_full.dtype)


def update_rotatek_eager(keys_vision, queries_recent, keep: int, num_kv_groups: int,
                         query_aware: bool = True):
    """(kept, R_partial, delta_mu, keep_mask) for visual Keys [B, H_kv, S_v, D]."""
    bsz, hkv, _, d = keys_vision.shape
    mean = keys_vision.float().mean(dim=-2, keepdim=True)
    kc = keys_vision - mean.to(keys_vision.dtype)
    cov = torch.einsum("bhsd,bhse->bhde", kc, kc).float()
    cov = 0.5 * (cov + cov.transpose(-1, -2))
    if query_aware:
        w = queries_recent.shape[2]
        qr = queries_recent
        if qr.shape[1] != hkv:
            qr = qr.view(bsz, hkv, num_kv_groups, w, d).mean(dim=2)
        qn = qr.float().norm(dim=-2, p=2)
        qn = qn.clamp(min=1e-3 * qn.median(dim=-1, keepdim=True).values)
        cov = cov * (qn.unsqueeze(-1) * qn.unsqueeze(-2))
        cov = 0.5 * (cov + cov.transpose(-1, -2))
        ridge = 1e-4 * cov.diagonal(dim1=-2, dim2=-1).abs().mean(dim=-1, keepdim=True).clamp(min=1e-6)
        cov = cov + ridge.unsqueeze(-1) * torch.eye(d, dtype=cov.dtype)
    _, vecs = torch.linalg.eigh(cov)
    R = vecs.flip(dims=[-1])[..., :keep].to(keys_vision.dtype)
    kept = torch.matmul(keys_vision, R)
    r32 = R.float()
    dm = (mean - torch.matmul(torch.matmul(mean, r32), r32.transpose(-2, -1))).squeeze(-2)
    mask = torch.zeros(bsz, hkv, d, dtype=torch.bool)
    mask[..., :keep] = True
    return kept, R, dm.to(keys_vision.dtype), mask
