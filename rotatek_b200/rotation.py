"""RotateK rotation builder on B200 -- the counterpart of ``rotatek.rotation``
plus the fused prefill build that ``ChannelPruner.update_rotatek`` performs.

``power_iteration_gpu`` keeps the reference's signature (rotatek/rotation.py:
68-91) and the ``_ROTATEK_QUERY_AWARE_ACTIVE`` flag (rotation.py:18), but
returns the *converged* top-k eigenvectors (descending eigenvalue) from a
batched 128x128 eigensolver (Householder tridiagonalisation, Sturm
multisection, inverse iteration) instead of five unconverged subspace
iterations from a random start; ``num_iters`` and ``seed`` are accepted and
unused.  The subspace is the one the iteration approaches, and decode depends
only on that subspace (logits equal q . (P k + (I - P) mu), P = R R^T).

``build_rotation`` runs the whole build of kv_pruning_utils.py:105-160 for one
layer in three kernels: tcgen05 covariance of the visual Keys, the eigensolver
with the centring / query weighting / top-k / delta_mu fused in, and the rotation
K_vis . R.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import torch

from rotatek_b200 import _lib

# Same switch as the reference (rotation.py:18, kv_pruning_utils.py:21).
_ROTATEK_QUERY_AWARE_ACTIVE = bool(int(os.environ.get("ROTATEK_QUERY_AWARE", "1")))

QUERY_WINDOW = 32  # kv_pruning_utils.py:23

_build_ws = {}


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _workspace(device: torch.device, need: int) -> torch.Tensor:
    """A per-device scratch buffer of at least ``need`` bytes, reused across calls
    on the current stream.  Its first 256 bytes are the device-status word,
    zeroed here once (the kernels only ever set bits in it)."""
    idx = device.index
    ws = _build_ws.get(idx)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        ws[:256].zero_()
        _build_ws[idx] = ws
    return ws


def read_build_status(device=None) -> int:
    """Read and clear the device-status word of this device's builder workspace
    (0: every bounded wait of the builder kernels completed)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    ws = _build_ws.get(dev.index)
    if ws is None:
        return 0
    lib = _lib.load()
    st = ctypes.c_uint32(0)
    _lib.check(lib.rtk_read_status(ctypes.c_void_p(ws.data_ptr()), _stream(dev), ctypes.byref(st)))
    return st.value


def _eigh(mats: torch.Tensor, k: int, vecs: torch.Tensor, vals: Optional[torch.Tensor]) -> None:
    lib = _lib.load()
    ws = _workspace(mats.device, lib.rtk_eigh_topk_workspace_size(mats.shape[0]))
    D = _lib.describe
    _lib.check(lib.rtk_eigh_topk(D(mats), k, D(vecs), D(vals), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                 _stream(mats.device)))


def power_iteration_gpu(cov: torch.Tensor, k: int, num_iters: int = 5, seed: int = 0) -> torch.Tensor:
    """Top-k eigenvectors of ``cov`` ([..., D, D]) as columns, [..., D, k], in
    descending eigenvalue order, each column's largest component positive.

    Drop-in for rotatek.rotation.power_iteration_gpu; ``num_iters`` and ``seed``
    are ignored (the result is converged, not an iterate)."""
    del num_iters, seed
    assert cov.is_cuda
    d = cov.shape[-1]
    lead = cov.shape[:-2]
    mats = cov.reshape(-1, d, d).to(torch.float32).contiguous()
    vecs = torch.empty(mats.shape[0], d, k, dtype=torch.float32, device=cov.device)
    _eigh(mats, k, vecs, None)
    return vecs.reshape(*lead, d, k).to(cov.dtype)


def eigh_topk(cov: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(eigenvalues [..., D] descending, top-k eigenvectors [..., D, k]) of fp32 ``cov``."""
    _lib.require_cuda(cov)
    d = cov.shape[-1]
    lead = cov.shape[:-2]
    mats = cov.reshape(-1, d, d).to(torch.float32).contiguous()
    vecs = torch.empty(mats.shape[0], d, k, dtype=torch.float32, device=cov.device)
    vals = torch.empty(mats.shape[0], d, dtype=torch.float32, device=cov.device)
    _eigh(mats, k, vecs, vals)
    return vals.reshape(*lead, d), vecs.reshape(*lead, d, k)


def key_covariance(keys: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(sum_s k k^T [B, H, 128, 128] fp32, sum_s k [B, H, 128] fp32) of keys [B, H, S, 128]."""
    if keys.dim() != 4:
        raise ValueError("keys must be [B, H, S, D]")
    _lib.require_cuda(keys)
    b, h, _, d = keys.shape
    cov = torch.empty(b, h, d, d, dtype=torch.float32, device=keys.device)
    ksum = torch.empty(b, h, d, dtype=torch.float32, device=keys.device)
    D = _lib.describe
    _lib.check(_lib.load().rtk_key_covariance(D(keys), D(cov), D(ksum), _stream(keys.device)))
    return cov, ksum


def rotate_keys(keys: torch.Tensor, R: torch.Tensor) -> torch.Tensor:
    """kept = keys . R ([B, H, S, 128] x [B, H, 128, keep] -> [B, H, S, keep], in
    the Keys' dtype): the rotation pass of ``build_rotation`` on its own."""
    if keys.dim() != 4 or R.dim() != 4:
        raise ValueError("keys must be [B, H, S, D] and R [B, H, D, keep]")
    _lib.require_cuda(keys, R)
    b, h, s, _ = keys.shape
    kept = torch.empty(b, h, s, R.shape[-1], dtype=keys.dtype, device=keys.device)
    lib = _lib.load()
    ws = _workspace(keys.device, 256)
    D = _lib.describe
    _lib.check(lib.rtk_rotate_keys(D(keys), D(R), D(kept), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                   _stream(keys.device)))
    return kept


def keep_count(head_dim: int, channel_ratio: float) -> int:
    """Channels kept for a pruning ratio (kv_pruning_utils.py:108)."""
    return head_dim - min(head_dim, max(0, int(head_dim * channel_ratio)))


def build_rotation(keys_vision: torch.Tensor, queries_recent: Optional[torch.Tensor], keep: int,
                   num_kv_groups: int, query_aware: Optional[bool] = None,
                   return_eigvals: bool = False):
    """The RotateK prefill build of one layer.

    keys_vision     [B, H_kv, S_v, D]   visual-span Keys (any strides)
    queries_recent  [B, H_q, W, D]      the last W (<= 32) queries, or None
    keep            channels kept (``keep_count(D, channel_ratio)``)

    Returns (kept [B, H_kv, S_v, keep], R_partial [B, H_kv, D, keep],
    delta_mu [B, H_kv, D], keep_mask [B, H_kv, D] bool) -- the values
    ``update_rotatek`` returns / stores (kv_pruning_utils.py:152-160), all but
    the mask in the Keys' dtype; with ``return_eigvals`` also the eigenvalues
    [B, H_kv, D] (fp32, descending) of the solved matrix."""
    if keys_vision.dim() != 4:
        raise ValueError("keys_vision must be [B, H_kv, S_v, D]")
    if query_aware is None:
        query_aware = _ROTATEK_QUERY_AWARE_ACTIVE
    q = queries_recent if query_aware else None
    _lib.require_cuda(keys_vision, q)
    b, h, s, d = keys_vision.shape
    dev = keys_vision.device
    dt = keys_vision.dtype
    kept = torch.empty(b, h, s, keep, dtype=dt, device=dev)
    R = torch.empty(b, h, d, keep, dtype=dt, device=dev)
    dm = torch.empty(b, h, d, dtype=dt, device=dev)
    ev = torch.empty(b, h, d, dtype=torch.float32, device=dev) if return_eigvals else None
    lib = _lib.load()
    ws = _workspace(dev, lib.rtk_build_rotation_workspace_size(b, h, d))
    D = _lib.describe
    _lib.check(lib.rtk_build_rotation(D(keys_vision), D(q), num_kv_groups, keep, D(kept), D(R), D(dm),
                                      D(ev), ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(dev)))
    mask = torch.zeros(b, h, d, dtype=torch.bool, device=dev)
    mask[..., :keep] = True
    if return_eigvals:
        return kept, R, dm, mask, ev
    return kept, R, dm, mask


def _check_projection_args(hidden_states: torch.Tensor, w_k: torch.Tensor) -> None:
    """The shape checks the output allocation depends on (the library checks the rest)."""
    if hidden_states.dim() != 3:
        raise ValueError("hidden_states must be [B, S, hidden]")
    if w_k.dim() != 2 or w_k.shape[0] % 128 != 0 or w_k.shape[0] == 0 or w_k.shape[1] != hidden_states.shape[2]:
        raise ValueError("w_k must be [H_kv * 128, hidden] in the hidden states' dtype")


def _cos_sin_3d(cos: torch.Tensor, sin: torch.Tensor):
    """cos / sin as [B | 1, S, D] views (HF hands them over as [B, S, D]; a
    [S, D] table broadcasts over the batch)."""
    if cos.dim() == 2:
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    if cos.dim() != 3 or sin.shape != cos.shape:
        raise ValueError("cos / sin must be [B, S, D] (or [S, D]) tensors of the same shape")
    return cos, sin


def key_projection(hidden_states: torch.Tensor, w_k: torch.Tensor, bias: Optional[torch.Tensor],
                   cos: torch.Tensor, sin: torch.Tensor, vis_start: int, vis_len: int):
    """Post-RoPE Keys straight from the hidden states (projection, bias and
    RoPE in one tensor-core kernel), then the covariance sums of their visual
    span from the Keys just written.

    Equals ``apply_rotary_pos_emb(k_proj(hidden_states).view(B, S, H_kv, D)
    .transpose(1, 2), cos, sin)`` -- llama_visionzip.py:144-153 -- (rounded as
    torch rounds those ops; up to the projection's accumulation order) and
    ``key_covariance`` of its tokens [vis_start, vis_start + vis_len).

    hidden_states [B, S, hidden]; w_k [H_kv * 128, hidden] (``k_proj.weight``);
    bias [H_kv * 128] or None; cos / sin [B | 1, S, 128] in the same dtype
    (bf16 / fp16).  Returns (keys [B, H_kv, S, 128], cov [B, H_kv, 128, 128]
    fp32, ksum [B, H_kv, 128] fp32)."""
    _check_projection_args(hidden_states, w_k)
    cos, sin = _cos_sin_3d(cos, sin)
    _lib.require_cuda(hidden_states, w_k, bias, cos, sin)
    b, s, _ = hidden_states.shape
    h = w_k.shape[0] // 128
    dev = hidden_states.device
    keys = torch.empty(b, h, s, 128, dtype=hidden_states.dtype, device=dev)
    cov = torch.empty(b, h, 128, 128, dtype=torch.float32, device=dev)
    ksum = torch.empty(b, h, 128, dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws = _workspace(dev, lib.rtk_key_projection_workspace_size(b, h, s, vis_start, vis_len, dev.index))
    D = _lib.describe
    _lib.check(lib.rtk_key_projection(D(hidden_states), D(w_k), D(bias), D(cos), D(sin), vis_start, vis_len,
                                      D(keys), D(cov), D(ksum), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                      _stream(dev)))
    return keys, cov, ksum


def build_rotation_projected(hidden_states: torch.Tensor, w_k: torch.Tensor, bias: Optional[torch.Tensor],
                             cos: torch.Tensor, sin: torch.Tensor, vis_start: int, vis_len: int,
                             queries_recent: Optional[torch.Tensor], keep: int, num_kv_groups: int,
                             query_aware: Optional[bool] = None):
    """``key_projection`` + ``build_rotation`` on the visual span in one call
    (the covariance sums are taken once, by the projection step): from one
    layer's hidden states to the Keys of every token and the RotateK state of
    the visual span.

    Returns (keys [B, H_kv, S, 128], kept [B, H_kv, vis_len, keep], R_partial,
    delta_mu, keep_mask) -- ``build_rotation``'s outputs for
    ``keys[:, :, vis_start:vis_start + vis_len]`` preceded by the Keys."""
    _check_projection_args(hidden_states, w_k)
    if query_aware is None:
        query_aware = _ROTATEK_QUERY_AWARE_ACTIVE
    q = queries_recent if query_aware else None
    cos, sin = _cos_sin_3d(cos, sin)
    _lib.require_cuda(hidden_states, w_k, bias, cos, sin, q)
    b, s, _ = hidden_states.shape
    h, d = w_k.shape[0] // 128, 128
    dev = hidden_states.device
    dt = hidden_states.dtype
    keys = torch.empty(b, h, s, d, dtype=dt, device=dev)
    kept = torch.empty(b, h, vis_len, keep, dtype=dt, device=dev)
    R = torch.empty(b, h, d, keep, dtype=dt, device=dev)
    dm = torch.empty(b, h, d, dtype=dt, device=dev)
    lib = _lib.load()
    ws = _workspace(dev, lib.rtk_build_rotation_projected_workspace_size(b, h, s, vis_start, vis_len, dev.index))
    D = _lib.describe
    _lib.check(lib.rtk_build_rotation_projected(
        D(hidden_states), D(w_k), D(bias), D(cos), D(sin), vis_start, vis_len, D(q), num_kv_groups, keep,
        D(keys), D(kept), D(R), D(dm), None, ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(dev)))
    mask = torch.zeros(b, h, d, dtype=torch.bool, device=dev)
    mask[..., :keep] = True
    return keys, kept, R, dm, mask


__all__ = ["_ROTATEK_QUERY_AWARE_ACTIVE", "power_iteration_gpu", "eigh_topk", "key_covariance",
           "keep_count", "build_rotation", "rotate_keys", "read_build_status", "key_projection",
           "build_rotation_projected"]
