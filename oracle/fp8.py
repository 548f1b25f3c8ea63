"""fp8 (e4m3) visual-span oracle in numpy (test infrastructure).

The fp8 storage is this build's extension (the reference keeps the visual span
in the model dtype); its decode is rotatek_decode (fused_decode.py:131-296, see
oracle/decode.py) on the dequantised values, so parity is: the quantisation
bit-exact, the decode within the 16-bit path's tolerance of the float64 decode
of the dequantised span.

  K~ [B, H, S, D_keep]: scale[b, h, c] = amax_t |k~| / 448 (1 if 0), per channel
  V  [B, H, S, 128]:    scale[b, h, t] = amax_d |v|  / 448 (1 if 0), per token
  x8 = e4m3(x / scale): fp32 division, then round to nearest even with 3
       fraction bits, exponent >= -6 (subnormal step 2^-9), saturating at 448.

``round_e4m3`` is pinned against torch's float8_e4m3fn conversion
(tests/test_fp8_cpu.py).
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


def round_e4m3(x) -> np.ndarray:
    """Nearest e4m3 value (ties to even), saturating at +-448; float64 out."""
    x = np.asarray(x, dtype=np.float64)
    a = np.minimum(np.abs(x), E4M3_MAX)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -6)))
    q = np.exp2(e - 3)
    r = np.minimum(np.round(a / q) * q, E4M3_MAX)
    return np.copysign(r, x)


def _scale(amax: np.ndarray) -> np.ndarray:
    amax = np.asarray(amax, dtype=np.float32)
    sc = amax / np.float32(E4M3_MAX)
    return np.where(amax > 0, sc, np.float32(1.0)).astype(np.float32)


def quantize_visual(k_sparse, v_sparse):
    """(k_q, k_scale, v_q, v_scale): e4m3 values (float64) and fp32 scales, as
    the device quantisation produces them from 16-bit inputs (given as float)."""
    k = np.asarray(k_sparse, dtype=np.float32)
    v = np.asarray(v_sparse, dtype=np.float32)
    ksc = _scale(np.abs(k).max(axis=2) if k.shape[2] else np.zeros(k.shape[:2] + k.shape[3:], np.float32))
    vsc = _scale(np.abs(v).max(axis=3))
    kq = round_e4m3(k / ksc[:, :, None, :])
    vq = round_e4m3(v / vsc[..., None])
    return kq, ksc, vq, vsc


def dequantize(kq, ksc, vq, vsc):
    """The visual Keys and Values the fp8 decode attends over (float64)."""
    return (np.asarray(kq, np.float64) * np.asarray(ksc, np.float64)[:, :, None, :],
            np.asarray(vq, np.float64) * np.asarray(vsc, np.float64)[..., None])
