"""Rotation-builder oracle in numpy (test infrastructure).

Restates ``ChannelPruner.update_rotatek`` with the exact-eigh solver
(integrations/lmms_eval/models/model_utils/kv_pruning_utils.py:92-160):

  26-35    span split: prompt = [:p], visual = [p : S - t], text = [-t:]
  108      keep = D - min(D, max(0, int(D * ratio)))
  112      mu = mean over the visual tokens, in fp32
  113      K_c = K - mu.to(K.dtype)           (rounded to K's dtype)
  114-115  C = K_c^T K_c, output in K's dtype, then fp32; C = (C + C^T) / 2
  117-140  query weighting (window 32, GQA group mean in the query dtype, L2 over
           the window in fp32, floor at 1e-3 * lower median, C *= q q^T,
           symmetrise, ridge 1e-4 * max(mean|diag|, 1e-6))
  145-150  eigh, eigenvalues ascending -> flip -> first `keep` columns -> K's dtype
  152      kept = K_vis . R  (uncentered Keys)
  153-156  delta_mu = mu - (mu R) R^T with R = fp32(R in K's dtype) -> K's dtype
  158-159  keep_mask[..., :keep] = True

``storage`` names the dtype the reference would hold the Keys in
('float32' | 'bfloat16' | 'float16'); every rounding step above is applied
with ``oracle.bf16.round_to``.  Accumulations run in float64, so the oracle is
at least as accurate as the reference at every step it does not round.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

from oracle.bf16 import round_to

QUERY_WINDOW = 32


def keep_count(head_dim: int, ratio: float) -> int:
    """kv_pruning_utils.py:108."""
    return head_dim - min(head_dim, max(0, int(head_dim * ratio)))


def split_spans(keys: np.ndarray, prompt_seqlen: int, query_seqlen: int):
    """kv_pruning_utils.py:26-35 -- (prompt, visual, text) views of [B, H, S, D]."""
    total = keys.shape[-2]
    p = max(0, min(prompt_seqlen, total))
    t = max(0, min(query_seqlen, max(total - p, 0)))
    vision_end = total - t if t > 0 else total
    prompt = keys[:, :, :p]
    vision = keys[:, :, p:vision_end]
    text = keys[:, :, total - t:] if t > 0 else keys[:, :, :0]
    return prompt, vision, text


def query_weights(queries: np.ndarray, num_kv_heads: int, storage: str) -> np.ndarray:
    """kv_pruning_utils.py:121-132 -- per-(b, kv head) channel weights q_norm [B, H_kv, D]."""
    window = min(QUERY_WINDOW, queries.shape[2])
    recent = np.asarray(queries[:, :, queries.shape[2] - window:], dtype=np.float64)
    bsz, hq, _, d = recent.shape
    if hq != num_kv_heads:
        g = hq // num_kv_heads
        recent = round_to(recent.reshape(bsz, num_kv_heads, g, window, d).mean(axis=2), storage)
        recent = np.asarray(recent, dtype=np.float64)
    q_norm = np.sqrt((recent ** 2).sum(axis=-2))
    med = np.sort(q_norm, axis=-1)[..., (d - 1) // 2]          # torch.median: lower median
    return np.maximum(q_norm, 1e-3 * med[..., None])


def weight_covariance(cov: np.ndarray, q_norm: np.ndarray) -> np.ndarray:
    """kv_pruning_utils.py:133-140 -- C * q q^T, symmetrise, diagonal ridge."""
    d = cov.shape[-1]
    cov = cov * (q_norm[..., :, None] * q_norm[..., None, :])
    cov = 0.5 * (cov + np.swapaxes(cov, -1, -2))
    ridge = 1e-4 * np.maximum(np.abs(np.diagonal(cov, axis1=-2, axis2=-1)).mean(axis=-1), 1e-6)
    return cov + ridge[..., None, None] * np.eye(d)


def covariance(vision: np.ndarray, storage: str, round_cov: bool = True):
    """kv_pruning_utils.py:112-115 -- (mu [B,H,D], symmetric C [B,H,D,D]).

    With ``round_cov`` False the centred Keys and the covariance stay in
    float64 (only the mean is rounded to ``storage`` before centring) -- the
    arithmetic of a build that accumulates the covariance in fp32."""
    k = np.asarray(vision, dtype=np.float64)
    mu = np.asarray(round_to(k.mean(axis=-2), "float32"), dtype=np.float64)
    kc = k - np.asarray(round_to(mu, storage), dtype=np.float64)[..., None, :]
    if round_cov:
        kc = np.asarray(round_to(kc, storage), dtype=np.float64)
    cov = np.einsum("bhsd,bhse->bhde", kc, kc)
    if round_cov:
        cov = np.asarray(round_to(cov, storage), dtype=np.float64)
    cov = 0.5 * (cov + np.swapaxes(cov, -1, -2))
    return mu, cov


@dataclass
class RotationResult:
    kept: np.ndarray        # [B, H_kv, S_v, keep]  in storage precision
    R_partial: np.ndarray   # [B, H_kv, D, keep]    in storage precision
    delta_mu: np.ndarray    # [B, H_kv, D]          in storage precision
    keep_mask: np.ndarray   # [B, H_kv, D] bool
    cov: np.ndarray         # [B, H_kv, D, D] the matrix that was eigendecomposed
    eigvals: np.ndarray     # [B, H_kv, D] descending
    mean: np.ndarray        # [B, H_kv, D] fp32 visual mean


def build_rotation(keys_vision, queries: Optional[np.ndarray], keep: int, num_kv_groups: int,
                   query_aware: bool = True, storage: str = "float32",
                   round_cov: bool = True) -> RotationResult:
    """The rotation build for one layer from the visual Keys [B, H_kv, S_v, D]
    (``round_cov``: see ``covariance``)."""
    kv = np.asarray(keys_vision, dtype=np.float64)
    bsz, hkv, _, d = kv.shape
    mu, cov = covariance(kv, storage, round_cov)
    if query_aware:
        cov = weight_covariance(cov, query_weights(queries, hkv, storage))
    cov32 = np.asarray(round_to(cov, "float32"), dtype=np.float64)
    w, vecs = np.linalg.eigh(cov32)
    w = w[..., ::-1]
    vecs = vecs[..., ::-1]
    R = np.asarray(round_to(vecs[..., :keep], storage), dtype=np.float64)
    kept = round_to(np.einsum("bhsd,bhdk->bhsk", kv, R), storage)
    mu_proj = np.einsum("bhk,bhdk->bhd", np.einsum("bhd,bhdk->bhk", mu, R), R)
    delta_mu = round_to(mu - mu_proj, storage)
    mask = np.zeros((bsz, hkv, d), dtype=bool)
    mask[..., :keep] = True
    return RotationResult(kept, R.astype(np.float32), delta_mu, mask, cov, w, mu.astype(np.float32))


def projector(R: np.ndarray) -> np.ndarray:
    """P = R (R^T R)^-1 R^T -- the orthogonal projector onto span(R), float64."""
    R = np.asarray(R, dtype=np.float64)
    gram = np.swapaxes(R, -1, -2) @ R
    return R @ np.linalg.solve(gram, np.swapaxes(R, -1, -2))


def projector_distance(R_a, R_b) -> np.ndarray:
    """||P_a - P_b||_F per (b, h): 0 for equal subspaces, sqrt(2k) at most.
    Invariant to column signs and to any rotation inside the kept subspace."""
    diff = projector(R_a) - projector(R_b)
    return np.sqrt((diff ** 2).sum(axis=(-1, -2)))


def subspace_iteration(cov: np.ndarray, v0: np.ndarray, num_iters: int) -> np.ndarray:
    """The reference's optional solver, ``power_iteration_gpu``
    (rotatek/rotation.py:68-91): from a start V0 [..., D, k], ``num_iters``
    times V <- cov V, then V <- V L^-T with L the Cholesky factor of V^T V (so
    V^T V = I).  float64 here; the reference runs it in cov's dtype from
    torch.randn(generator=manual_seed(seed)) on the device."""
    v = np.asarray(v0, dtype=np.float64)
    c = np.asarray(cov, dtype=np.float64)
    for _ in range(num_iters):
        v = c @ v
        gram = np.swapaxes(v, -1, -2) @ v
        L = np.linalg.cholesky(gram)
        # V L^-T: solve L X^T = V^T
        v = np.swapaxes(np.linalg.solve(L, np.swapaxes(v, -1, -2)), -1, -2)
    return v
