"""Seeded synthetic inputs for the RotateK hot path.

The reference measures its kernels on synthetic tensors (scripts/paper/kernel/
kernel_profile.py:49-70 draws everything N(0,1)); its model runs use real Keys.
This module stands in for both with the low-rank-plus-noise Key generator the
benchmark configurations name:

    K = Z . A + 0.1 * N(0, 1),   Z ~ N(0, 1) [.., S, rank],
    A ~ N(0, 1) [rank, D] with column (channel) scales log-uniform in [0.1, 10]

one independent ``A`` per (batch, KV head).  Values, decode queries and the
prefill query window are N(0, 1).  Every draw comes from an explicit
``torch.Generator`` so a (seed, shape) pair always gives the same tensors on
the same device type.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

QUERY_WINDOW = 32  # kv_pruning_utils.py:23 -- recent queries used for weighting


def _gen(seed: int, device) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def lowrank_keys(batch: int, heads: int, seq: int, head_dim: int = 128, rank: int = 32,
                 noise: float = 0.1, seed: int = 0, device="cpu",
                 dtype=torch.float32) -> torch.Tensor:
    """Keys [batch, heads, seq, head_dim] = Z.A + noise.N(0,1), drawn in fp32 then cast."""
    g = _gen(seed, device)
    z = torch.randn(batch, heads, seq, rank, generator=g, device=device)
    a = torch.randn(batch, heads, rank, head_dim, generator=g, device=device)
    u = torch.rand(batch, heads, 1, head_dim, generator=g, device=device)
    col_scale = torch.exp(math.log(0.1) + u * (math.log(10.0) - math.log(0.1)))
    a = a * col_scale
    k = torch.matmul(z, a)
    k.add_(noise * torch.randn(batch, heads, seq, head_dim, generator=g, device=device))
    return k.to(dtype)


def normal(shape, seed: int, device="cpu", dtype=torch.float32) -> torch.Tensor:
    g = _gen(seed, device)
    return torch.randn(*shape, generator=g, device=device).to(dtype)


@dataclass
class PrefillInputs:
    """One attention layer at prefill: full Keys/Values/queries over the spans."""
    keys: torch.Tensor       # [B, H_kv, S_p + S_v + S_t, D]
    values: torch.Tensor     # [B, H_kv, S, D]
    queries: torch.Tensor    # [B, H_q, S, D] (only the last QUERY_WINDOW rows matter)
    prompt_len: int
    vision_len: int
    text_len: int


def make_prefill(batch: int, q_heads: int, kv_heads: int, prompt_len: int, vision_len: int,
                 text_len: int, head_dim: int = 128, seed: int = 0, device="cpu",
                 dtype=torch.float32, full_queries: bool = False) -> PrefillInputs:
    """Prefill tensors for one layer.  Keys of every span come from the low-rank
    generator (the visual span is what the rotation is built on).  When
    ``full_queries`` is False only the last QUERY_WINDOW query rows are drawn and
    the rest are zero -- the pruner reads only that window."""
    seq = prompt_len + vision_len + text_len
    keys = lowrank_keys(batch, kv_heads, seq, head_dim, seed=seed, device=device, dtype=dtype)
    values = normal((batch, kv_heads, seq, head_dim), seed + 1, device, dtype)
    if full_queries:
        queries = normal((batch, q_heads, seq, head_dim), seed + 2, device, dtype)
    else:
        w = min(QUERY_WINDOW, seq)
        queries = torch.zeros(batch, q_heads, seq, head_dim, device=device, dtype=dtype)
        queries[:, :, seq - w:] = normal((batch, q_heads, w, head_dim), seed + 2, device, dtype)
    return PrefillInputs(keys, values, queries, prompt_len, vision_len, text_len)


@dataclass
class DecodeInputs:
    """Arguments of ``rotatek_decode`` (fused_decode.py:303-313) for one layer."""
    q_full: torch.Tensor      # [B, H_q, D]
    R_partial: torch.Tensor   # [B, H_kv, D, D_keep]
    delta_mu: Optional[torch.Tensor]  # [B, H_kv, D]
    k_full: torch.Tensor      # [B, H_kv, S_f, D]
    v_full: torch.Tensor      # [B, H_kv, S_f, D]
    mask_full: torch.Tensor   # [B, S_f] uint8
    k_sparse: torch.Tensor    # [B, H_kv, S_v, D_keep]
    v_sparse: torch.Tensor    # [B, H_kv, S_v, D]
    num_kv_groups: int

    def as_kwargs(self) -> dict:
        return dict(q_full=self.q_full, R_partial=self.R_partial, delta_mu=self.delta_mu,
                    k_full=self.k_full, v_full=self.v_full, mask_full=self.mask_full,
                    k_sparse=self.k_sparse, v_sparse=self.v_sparse,
                    num_kv_groups=self.num_kv_groups)

    def nbytes(self) -> int:
        """Algorithmic bytes of one decode step: every input read once, output written once."""
        ts = [self.q_full, self.R_partial, self.k_full, self.v_full, self.k_sparse, self.v_sparse]
        if self.delta_mu is not None:
            ts.append(self.delta_mu)
        n = sum(t.numel() * t.element_size() for t in ts)
        return n + self.q_full.numel() * self.q_full.element_size()


def orthonormal_basis(batch: int, heads: int, head_dim: int, keep: int, seed: int,
                      device="cpu") -> torch.Tensor:
    """Random orthonormal [B, H, D, keep] (QR of a Gaussian), fp32."""
    g = _gen(seed, device)
    m = torch.randn(batch, heads, head_dim, keep, generator=g, device=device)
    qmat, _ = torch.linalg.qr(m)
    return qmat


def make_decode(batch: int, q_heads: int, kv_heads: int, vision_len: int, full_len: int,
                head_dim: int = 128, keep: int = 32, seed: int = 0, device="cpu",
                dtype=torch.float32, with_bias: bool = True,
                basis: Optional[torch.Tensor] = None) -> DecodeInputs:
    """Decode-step inputs with the shapes of the adapters' call
    (llama_visionzip.py:203-214).  Visual Keys come from the low-rank generator
    and are rotated by an orthonormal basis (a random one unless ``basis`` is
    given), so ``k_sparse = K_vis . R`` holds realistic magnitudes; ``delta_mu``
    is the mean correction of that basis, as kv_pruning_utils.py:152-156 forms it."""
    groups = q_heads // kv_heads
    k_vis = lowrank_keys(batch, kv_heads, vision_len, head_dim, seed=seed, device=device)
    if basis is None:
        basis = orthonormal_basis(batch, kv_heads, head_dim, keep, seed + 7, device)
    r_cast = basis.to(dtype)
    r32 = r_cast.float()
    k_sparse = torch.matmul(k_vis.to(dtype), r_cast) if dtype != torch.float32 else torch.matmul(k_vis, r32)
    delta_mu = None
    if with_bias:
        mu = k_vis.mean(dim=-2, keepdim=True)
        delta_mu = (mu - torch.matmul(torch.matmul(mu, r32), r32.transpose(-2, -1))).squeeze(-2).to(dtype)
    k_full = lowrank_keys(batch, kv_heads, full_len, head_dim, seed=seed + 3, device=device, dtype=dtype)
    v_full = normal((batch, kv_heads, full_len, head_dim), seed + 4, device, dtype)
    v_sparse = normal((batch, kv_heads, vision_len, head_dim), seed + 5, device, dtype)
    q_full = normal((batch, q_heads, head_dim), seed + 6, device, dtype)
    mask_full = torch.ones(batch, full_len, dtype=torch.uint8, device=device)
    return DecodeInputs(q_full, r_cast.contiguous(), delta_mu, k_full, v_full, mask_full,
                        k_sparse.contiguous(), v_sparse, groups)


@dataclass
class SparkInputs:
    """Arguments of ``spark_decode`` for one layer: SparK's per-token channel
    pruning (rotatek/baselines/spark.py:15-58) of low-rank visual Keys."""
    q_full: torch.Tensor        # [B, H_q, D]
    k_full: torch.Tensor        # [B, H_kv, S_f, D]
    v_full: torch.Tensor        # [B, H_kv, S_f, D]
    mask_full: torch.Tensor     # [B, S_f] uint8
    k_kept: torch.Tensor        # [B, H_kv, S_v, D_keep] kept values, channel order
    keep_mask: torch.Tensor     # [B, H_kv, S_v, D] bool
    pruned_mean: torch.Tensor   # [B, H_kv, S_v, 1]
    v_sparse: torch.Tensor      # [B, H_kv, S_v, D]
    num_kv_groups: int

    def recovered(self) -> torch.Tensor:
        """Full-width visual Keys as the adapters rebuild them
        (llama_visionzip.py:228-230)."""
        b, h, s, _ = self.k_kept.shape
        rec = self.pruned_mean.expand(b, h, s, self.keep_mask.shape[-1]).contiguous()
        rec[self.keep_mask] = self.k_kept.reshape(-1)
        return rec


def spark_prune(queries: torch.Tensor, keys: torch.Tensor, keep: int):
    """(K_compact, keep_mask, pruned_mean) of spark.py:15-58 for queries
    [B, H, Q, D] (grouped to the KV heads) and keys [B, H, S, D], in the keys'
    dtype: score k^2 * ||Q||_2, keep the top `keep` channels per token (ties
    broken by torch.topk), kept values in channel order, mean of the rest."""
    q_norm = torch.norm(queries, dim=-2, p=2).unsqueeze(-2)
    scores = torch.pow(keys, 2) * q_norm
    top = torch.topk(scores, keep, dim=-1).indices.sort(dim=-1).values
    k_kept = torch.gather(keys, -1, top)
    mask = torch.zeros_like(keys, dtype=torch.bool)
    mask.scatter_(-1, top, True)
    pruned_mean = (keys.float().sum(-1, keepdim=True) - k_kept.float().sum(-1, keepdim=True)) / (
        keys.shape[-1] - keep)
    return k_kept.contiguous(), mask, pruned_mean.to(keys.dtype)


def make_spark(batch: int, q_heads: int, kv_heads: int, vision_len: int, full_len: int, keep: int = 32,
               head_dim: int = 128, seed: int = 0, device="cpu", dtype=torch.float32) -> SparkInputs:
    """SparK decode-step inputs: low-rank visual Keys pruned per token against a
    N(0,1) query window (grouped by the mean over each KV head's queries, as
    ChannelPruner.update_spark does), N(0,1) Values and decode queries."""
    groups = q_heads // kv_heads
    k_vis = lowrank_keys(batch, kv_heads, vision_len, head_dim, seed=seed, device=device, dtype=dtype)
    window = normal((batch, q_heads, QUERY_WINDOW, head_dim), seed + 1, device, dtype)
    grouped = window.view(batch, kv_heads, groups, QUERY_WINDOW, head_dim).mean(2)
    k_kept, mask, mean = spark_prune(grouped, k_vis, keep)
    k_full = lowrank_keys(batch, kv_heads, full_len, head_dim, seed=seed + 3, device=device, dtype=dtype)
    v_full = normal((batch, kv_heads, full_len, head_dim), seed + 4, device, dtype)
    v_sparse = normal((batch, kv_heads, vision_len, head_dim), seed + 5, device, dtype)
    q_full = normal((batch, q_heads, head_dim), seed + 6, device, dtype)
    mask_full = torch.ones(batch, full_len, dtype=torch.uint8, device=device)
    return SparkInputs(q_full, k_full, v_full, mask_full, k_kept, mask, mean, v_sparse, groups)
