"""The fp8 oracle's e4m3 rounding against torch's float8_e4m3fn conversion (CPU)."""
import numpy as np
import torch

from oracle import fp8 as ofp8


def test_round_e4m3_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(20000) * 40.0,                       # normals across the range
        rng.standard_normal(5000) * 2.0 ** -7,                   # subnormals and the smallest normals
        np.array([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10,
                  1.0625, 1.1875, 17.0, 19.0, 240.0, 232.0]),    # exact ties (to even)
    ]).astype(np.float32)
    x = np.clip(x, -448.0, 448.0)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(ofp8.round_e4m3(x), want)


def test_quantize_roundtrip_error_bound():
    """Per-channel / per-token scaling keeps every element within half an e4m3
    step (2^-4 relative) of its group's range."""
    rng = np.random.default_rng(1)
    k = rng.standard_normal((2, 3, 100, 32)).astype(np.float32) * np.logspace(1, -2, 32, dtype=np.float32)
    v = rng.standard_normal((2, 3, 100, 128)).astype(np.float32)
    kq, ksc, vq, vsc = ofp8.quantize_visual(k, v)
    kd, vd = ofp8.dequantize(kq, ksc, vq, vsc)
    assert np.all(np.abs(kd - k) <= 2.0 ** -4 * np.abs(k) + 2.0 ** -9 * ksc[:, :, None, :] + 1e-30)
    assert np.all(np.abs(vd - v) <= 2.0 ** -4 * np.abs(v) + 2.0 ** -9 * vsc[..., None] + 1e-30)
    assert np.abs(kq).max() <= 448 and np.abs(vq).max() <= 448
