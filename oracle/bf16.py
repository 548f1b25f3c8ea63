"""bfloat16 rounding in numpy (test infrastructure).

bfloat16 keeps the top 16 bits of an IEEE float32.  Rounding is to nearest,
ties to even, on the dropped 16 bits -- the conversion torch performs in
``tensor.to(torch.bfloat16)`` for finite values.  NaN stays NaN.
"""
from __future__ import annotations

import numpy as np


def round_bf16(x) -> np.ndarray:
    """float -> nearest bfloat16 value, returned as float32."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32).reshape(f.shape)
    nan = np.isnan(f)
    if nan.any():
        out = np.where(nan, f, out)
    return out


def truncate_bf16(x) -> np.ndarray:
    """float -> bfloat16 by dropping the low 16 bits (round toward zero), as float32.

    Triton's interpreter (TRITON_INTERPRET=1, triton 3.6) converts fp32 to bf16
    this way when a kernel stores a bf16 output; compiled Triton and CUDA round
    to nearest even.  Used only to compare against fixtures made under the
    interpreter."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    return (f.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32).reshape(f.shape)


def round_to(x, dtype: str) -> np.ndarray:
    """Round float data to the storage dtype named by ``dtype``
    ('float32' | 'bfloat16' | 'float16'), returned as float32."""
    if dtype == "bfloat16":
        return round_bf16(x)
    if dtype == "float16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(x, dtype=np.float32)
