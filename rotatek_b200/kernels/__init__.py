"""Decode entry points with the reference's signatures.

Mirrors ``rotatek.kernels`` (rotatek/kernels/__init__.py:15-26): the model
adapters call ``rotatek_decode`` (RotateK) and ``full_channel_decode``
(Full / ThinK / SparK) by keyword and get the same return conventions and
ValueErrors.  There is one backend -- the sm_100a kernels of
librotatek_b200.so -- so ``ROTATEK_KERNEL`` is kept only as an exported name
(it reports "b200"); setting it to the reference's 'paper' or 'gqa' selects
the same kernels.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from rotatek_b200 import _lib

ROTATEK_KERNEL = "b200"

_ws_size_cache = {}


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dtype_code(t: torch.Tensor) -> int:
    return _lib._DTYPES.get(t.dtype, -1)


def rotatek_decode(
    q_full: torch.Tensor,                # [B, H_q, D]
    R_partial: torch.Tensor,             # [B, H_kv, D, D_keep]
    delta_mu: Optional[torch.Tensor],    # [B, H_kv, D] or None
    k_full: torch.Tensor,                # [B, H_kv, S_full, D]
    v_full: torch.Tensor,                # [B, H_kv, S_full, D]
    mask_full: Optional[torch.Tensor],   # [B, S_full] uint8
    k_sparse: torch.Tensor,              # [B, H_kv, S_sparse, D_keep]
    v_sparse: torch.Tensor,              # [B, H_kv, S_sparse, D]
    num_kv_groups: int,
    *,
    out: Optional[torch.Tensor] = None,  # [B, 1, H_q, D] to write into (any strides, channel stride 1)
) -> Tuple[torch.Tensor, None, None]:
    """RotateK decode of one query token; returns (out [B, 1, H_q, D], None, None).

    Same contract as ``rotatek_decode_fused_triton``
    (rotatek/kernels/fused_decode.py:303-420): visual logits use the rotated
    query q.R and the q.delta_mu bias, prompt/text logits the full query, both
    spans share one softmax, tokens with mask_full == 0 are skipped, and the
    output is acc / (l + 1e-6) in q's dtype.  Unlike the reference the output
    is a fresh tensor, never an alias of a cached buffer -- unless the caller
    passes ``out`` (an extension: e.g. a head-major view of a collective's send
    buffer, so that no copy precedes the gather).  Inputs may be strided views
    (e.g. the adapters' ``value_states[:, :, s_p:s_p + s_v]``); nothing is
    copied.
    """
    if q_full.dim() != 3:
        raise ValueError("q_full must be [B, H_q, D]")
    if R_partial.dim() != 4:
        raise ValueError("R_partial must be [B, H_kv, D, D_keep]")
    if mask_full is not None and mask_full.dtype != torch.uint8:
        raise ValueError("mask_full must be uint8")
    bsz, heads, head_dim = q_full.shape
    h_kv = R_partial.shape[1]
    if num_kv_groups <= 0 or heads // num_kv_groups != h_kv:
        raise ValueError(
            f"R_partial H_kv={h_kv} but H_q={heads}, num_kv_groups={num_kv_groups}")
    if heads != h_kv * num_kv_groups:
        # the reference's floor-division check lets this through and then reads
        # past the last KV head (fused_decode.py:124, 335)
        raise ValueError(f"H_q={heads} is not H_kv={h_kv} * num_kv_groups={num_kv_groups}")
    _lib.require_cuda(q_full, R_partial, delta_mu, k_full, v_full, mask_full, k_sparse, v_sparse)
    lib = _lib.load()
    dev = q_full.device
    key = ("rk", _dtype_code(q_full), bsz, heads, h_kv, head_dim, R_partial.shape[-1],
           k_full.shape[-2], k_sparse.shape[-2], dev.index)
    need = _ws_size_cache.get(key)
    if need is None:
        need = (lib.rtk_rotatek_decode_workspace_size(*key[1:-1], dev.index),
                lib.rtk_decode_workspace_counter_bytes(bsz, heads))
        _ws_size_cache[key] = need
    ws = _lib.workspace(dev, *need)
    if out is None:
        out = torch.empty((bsz, 1, heads, head_dim), dtype=q_full.dtype, device=dev)
    elif out.shape != (bsz, 1, heads, head_dim) or out.dtype != q_full.dtype or out.device != dev:
        raise ValueError(f"out must be [B, 1, H_q, D] = {(bsz, 1, heads, head_dim)} in q's dtype on q's device")
    D = _lib.describe
    _lib.check(lib.rtk_rotatek_decode(
        D(q_full), D(R_partial), D(delta_mu), D(k_full), D(v_full), D(mask_full), D(k_sparse),
        D(v_sparse), num_kv_groups, D(out), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
        _stream(dev)))
    return out, None, None


def _as_u8(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t


def quantize_visual_fp8(k_sparse: torch.Tensor, v_sparse: torch.Tensor):
    """fp8 (e4m3) copy of a visual span for ``rotatek_decode_fp8``.

    k_sparse [B, H_kv, S_v, D_keep] (D_keep 16 / 32 / 64) and v_sparse
    [B, H_kv, S_v, 128], bf16 or fp16.  Returns (k8, k_scale, v8, v_scale):
    e4m3 bytes as uint8, k8 [B, H_kv, S_v, D_keep] and v8 the Values
    transposed, [B, H_kv, 128, S_v] (token stride 1; a view of rows padded to
    16 bytes), and fp32 scales [B, H_kv, D_keep] (per rotated channel) /
    [B, H_kv, S_v] (per token), with k ~= k_scale[c] * e4m3(k8[.., t, c]),
    v ~= v_scale[t] * e4m3(v8[.., d, t]), scale = amax / 448."""
    if k_sparse.dim() != 4 or v_sparse.dim() != 4:
        raise ValueError("k_sparse must be [B, H_kv, S, D_keep] and v_sparse [B, H_kv, S, 128]")
    _lib.require_cuda(k_sparse, v_sparse)
    b, h, s, dk = k_sparse.shape
    dev = k_sparse.device
    k8 = torch.empty(b, h, s, dk, dtype=torch.uint8, device=dev)
    if v_sparse.shape[-1] != 128:
        raise ValueError("k_sparse must be [B, H_kv, S, D_keep] and v_sparse [B, H_kv, S, 128]")
    v8 = torch.empty(b, h, 128, (s + 15) // 16 * 16, dtype=torch.uint8, device=dev)[..., :s]
    ksc = torch.empty(b, h, dk, dtype=torch.float32, device=dev)
    vsc = torch.empty(b, h, s, dtype=torch.float32, device=dev)
    D = _lib.describe
    _lib.check(_lib.load().rtk_quantize_visual_fp8(D(k_sparse), D(v_sparse), D(k8), D(ksc), D(v8), D(vsc),
                                                     _stream(dev)))
    return k8, ksc, v8, vsc


def rotatek_decode_fp8(q_full, R_partial, delta_mu, k_full, v_full, mask_full, k8, k_scale, v8, v_scale,
                       num_kv_groups: int):
    """``rotatek_decode`` with the visual span in fp8: the visual Keys are
    k_scale[c] * e4m3(k8[.., t, c]) and the visual Values v_scale[t] *
    e4m3(v8[.., d, t]) (v8 = V transposed, [B, H_kv, 128, S_v]; both from
    ``quantize_visual_fp8``; uint8 or float8_e4m3fn tensors); the prompt/text span
    and the output stay in q's dtype.  Returns (out [B, 1, H_q, D], None, None)."""
    if q_full.dim() != 3:
        raise ValueError("q_full must be [B, H_q, D]")
    if R_partial.dim() != 4:
        raise ValueError("R_partial must be [B, H_kv, D, D_keep]")
    k8, v8 = _as_u8(k8), _as_u8(v8)
    _lib.require_cuda(q_full, R_partial, delta_mu, k_full, v_full, mask_full, k8, k_scale, v8, v_scale)
    bsz, heads, head_dim = q_full.shape
    h_kv = R_partial.shape[1]
    lib = _lib.load()
    dev = q_full.device
    key = ("rk", _dtype_code(q_full), bsz, heads, h_kv, head_dim, R_partial.shape[-1],
           k_full.shape[-2], k8.shape[-2], dev.index)
    need = _ws_size_cache.get(key)
    if need is None:
        need = (lib.rtk_rotatek_decode_workspace_size(*key[1:-1], dev.index),
                lib.rtk_decode_workspace_counter_bytes(bsz, heads))
        _ws_size_cache[key] = need
    ws = _lib.workspace(dev, *need)
    out = torch.empty((bsz, 1, heads, head_dim), dtype=q_full.dtype, device=dev)
    D = _lib.describe
    _lib.check(lib.rtk_rotatek_decode_fp8(
        D(q_full), D(R_partial), D(delta_mu), D(k_full), D(v_full), D(mask_full), D(k8), D(k_scale), D(v8),
        D(v_scale), num_kv_groups, D(out), ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(dev)))
    return out, None, None


def full_channel_decode(
    q: torch.Tensor,                   # [B, H_q, D]
    k: torch.Tensor,                   # [B, H_kv, S, D]
    v: torch.Tensor,                   # [B, H_kv, S, D]
    num_kv_groups: int = 1,
) -> torch.Tensor:
    """Full-channel split-K decode of one query token; returns [B, 1, H_q, D].

    Same contract as ``full_channel_decode_triton``
    (rotatek/kernels/full_channel_flash_decoding.py:162-229) without its
    ``.contiguous()`` copies: strided k / v are read in place.
    """
    if q.dim() != 3:
        raise ValueError("q must be [B, H_q, D]")
    bsz, heads, head_dim = q.shape
    if k.shape[-1] != head_dim or v.shape[-1] != head_dim:
        raise ValueError("k/v head_dim must match q's")
    _lib.require_cuda(q, k, v)
    lib = _lib.load()
    dev = q.device
    key = ("fc", _dtype_code(q), bsz, heads, k.shape[1], head_dim, k.shape[-2], dev.index)
    need = _ws_size_cache.get(key)
    if need is None:
        need = (lib.rtk_full_channel_decode_workspace_size(*key[1:-1], dev.index),
                lib.rtk_decode_workspace_counter_bytes(bsz, heads))
        _ws_size_cache[key] = need
    ws = _lib.workspace(dev, *need)
    out = torch.empty((bsz, 1, heads, head_dim), dtype=q.dtype, device=dev)
    D = _lib.describe
    _lib.check(lib.rtk_full_channel_decode(
        D(q), D(k), D(v), num_kv_groups, D(out), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
        _stream(dev)))
    return out


def think_selection(think_mask: torch.Tensor, keep: int, dtype: torch.dtype) -> torch.Tensor:
    """R_sel [B, H_kv, D, keep] = the identity's columns of each head's kept
    channels in channel order (q . R_sel picks q's kept channels).  No host
    synchronisation: the kept channels come from a stable sort of the mask."""
    b, h, d = think_mask.shape
    order = torch.sort((~think_mask).to(torch.uint8), dim=-1, stable=True).indices[..., :keep]
    R = torch.zeros(b, h, d, keep, dtype=dtype, device=think_mask.device)
    R.scatter_(2, order.unsqueeze(2), 1)
    return R


def think_decode(
    q_full: torch.Tensor,                # [B, H_q, D]
    think_mask: torch.Tensor,            # [B, H_kv, D] bool, True = kept (ChannelPruner.current_think_mask)
    key_pruned: torch.Tensor,            # [B, H_kv, S_vis, D_keep] kept channels, channel order
    k_full: torch.Tensor,                # [B, H_kv, S_full, D]
    v_full: torch.Tensor,                # [B, H_kv, S_full, D]
    mask_full: Optional[torch.Tensor],   # [B, S_full] uint8
    v_sparse: torch.Tensor,              # [B, H_kv, S_vis, D]
    num_kv_groups: int,
    selection: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """The ThinK baseline's decode without recovering full-width Keys.

    The adapters zero-fill the pruned channels of the visual Keys, concatenate
    prompt, visual and text Keys and run ``full_channel_decode``
    (llama_visionzip.py:217-240).  A zero channel adds nothing to q . k, so the
    same logits are q[kept] . k_pruned on the visual span and q . k on the
    prompt/text span -- the RotateK kernel with R = the kept channels'
    selection and no delta_mu.  ``selection`` is ``think_selection(think_mask,
    D_keep, q.dtype)``, built here when not given; the mask is fixed after
    prefill, so a caller can build it once per layer.  Returns [B, 1, H_q, D]."""
    if selection is None:
        selection = think_selection(think_mask, key_pruned.shape[-1], q_full.dtype)
    out, _, _ = rotatek_decode(q_full=q_full, R_partial=selection, delta_mu=None, k_full=k_full, v_full=v_full,
                               mask_full=mask_full, k_sparse=key_pruned, v_sparse=v_sparse,
                               num_kv_groups=num_kv_groups)
    return out


def pack_spark_indices(keep_mask: torch.Tensor, d_keep: int, validate: bool = True) -> torch.Tensor:
    """Kept channels of a SparK keep mask, ascending: keep_mask [B, H_kv, S, 128]
    bool (``ChannelPruner.current_spark_mask``, rotatek/baselines/spark.py:15-58)
    -> keep_idx [B, H_kv, S, d_keep] uint8 for ``spark_decode``.  The mask is
    fixed after prefill, so this runs once per layer.  ``validate`` checks on
    the device that every token keeps exactly d_keep channels and raises
    ValueError otherwise (one host synchronisation)."""
    if keep_mask.dim() != 4:
        raise ValueError("keep_mask must be [B, H_kv, S, D]")
    _lib.require_cuda(keep_mask)
    b, h, s, _ = keep_mask.shape
    dev = keep_mask.device
    mask = keep_mask.view(torch.uint8) if keep_mask.dtype == torch.bool else keep_mask
    idx = torch.empty(b, h, s, d_keep, dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev) if validate else None
    D = _lib.describe
    _lib.check(_lib.load().rtk_spark_pack(D(mask), D(idx),
                                          ctypes.c_void_p(status.data_ptr() if validate else 0), _stream(dev)))
    if validate and int(status.item()) != 0:
        raise ValueError(f"keep_mask: some token does not keep exactly {d_keep} channels")
    return idx


def spark_decode(
    q_full: torch.Tensor,                # [B, H_q, D]
    k_full: torch.Tensor,                # [B, H_kv, S_full, D]
    v_full: torch.Tensor,                # [B, H_kv, S_full, D]
    mask_full: Optional[torch.Tensor],   # [B, S_full] uint8 or None
    k_kept: torch.Tensor,                # [B, H_kv, S_vis, D_keep] kept channels, channel order
    keep_idx: torch.Tensor,              # [B, H_kv, S_vis, D_keep] uint8 (pack_spark_indices)
    pruned_mean: torch.Tensor,           # [B, H_kv, S_vis, 1]
    v_sparse: torch.Tensor,              # [B, H_kv, S_vis, D]
    num_kv_groups: int,
) -> torch.Tensor:
    """The SparK baseline's decode without recovering full-width Keys.

    The adapters fill a [B, H_kv, S_vis, D] buffer with each token's
    ``pruned_mean``, write the kept values into the kept channels, concatenate
    prompt, visual and text Keys and run ``full_channel_decode``
    (llama_visionzip.py:226-242).  This computes that decode in one kernel that
    rebuilds each 32-token block of recovered Keys in shared memory, so the
    visual Keys cost D_keep values + D_keep index bytes + one mean per token in
    HBM instead of 128 values.  ``mask_full`` masks the prompt/text span as in
    ``rotatek_decode``.  Returns [B, 1, H_q, D] in q's dtype."""
    if q_full.dim() != 3:
        raise ValueError("q_full must be [B, H_q, D]")
    if k_kept.dim() != 4:
        raise ValueError("k_kept must be [B, H_kv, S_vis, D_keep]")
    if mask_full is not None and mask_full.dtype != torch.uint8:
        raise ValueError("mask_full must be uint8")
    if pruned_mean.dim() == 3:
        pruned_mean = pruned_mean.unsqueeze(-1)
    _lib.require_cuda(q_full, k_full, v_full, mask_full, k_kept, keep_idx, pruned_mean, v_sparse)
    bsz, heads, head_dim = q_full.shape
    h_kv = k_kept.shape[1]
    lib = _lib.load()
    dev = q_full.device
    key = ("rk", _dtype_code(q_full), bsz, heads, h_kv, head_dim, k_kept.shape[-1],
           k_full.shape[-2], k_kept.shape[-2], dev.index)
    need = _ws_size_cache.get(key)
    if need is None:
        need = (lib.rtk_rotatek_decode_workspace_size(*key[1:-1], dev.index),
                lib.rtk_decode_workspace_counter_bytes(bsz, heads))
        _ws_size_cache[key] = need
    ws = _lib.workspace(dev, *need)
    out = torch.empty((bsz, 1, heads, head_dim), dtype=q_full.dtype, device=dev)
    D = _lib.describe
    _lib.check(lib.rtk_spark_decode(
        D(q_full), D(k_full), D(v_full), D(mask_full), D(k_kept), D(keep_idx), D(pruned_mean), D(v_sparse),
        num_kv_groups, D(out), ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(dev)))
    return out


__all__ = ["ROTATEK_KERNEL", "rotatek_decode", "full_channel_decode", "think_decode", "think_selection",
           "quantize_visual_fp8", "rotatek_decode_fp8", "pack_spark_indices", "spark_decode"]
