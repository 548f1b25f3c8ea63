"""fp8 (e4m3) visual span on the GPU: quantisation bit-exact against the oracle,
decode against the float64 decode of the dequantised span.

Tolerances (written out per dtype, as for the 16-bit decode): bf16 2e-3
absolute + 2^-8 relative, fp16 1e-3 + 2^-10.  The fp8 path multiplies e4m3
values (exact in f16) with the rotated query split into f16 hi + lo and with
the softmax weights rounded to f16 (11 bits; the Values they weight carry 4),
so it is held to the same bar as the 16-bit path on the values it reads.  How far the
quantisation itself moves the output from the 16-bit decode is measured, not
gated tightly (the synthetic inputs say little about real attention).
"""
import numpy as np
import pytest
import torch

from oracle import decode as odec
from oracle import fp8 as ofp8
from rotatek_b200 import _lib, synthetic as syn
from rotatek_b200.kernels import quantize_visual_fp8, rotatek_decode, rotatek_decode_fp8

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.bfloat16: (2e-3, 2.0 ** -8), torch.float16: (1e-3, 2.0 ** -10)}


def f64(t):
    return t.detach().double().cpu().numpy()


def e4m3_values(t8):
    return t8.view(torch.float8_e4m3fn).float().cpu().numpy().astype(np.float64)


def values_natural(v8):
    """The device's V^T bytes [B, H, 128, S] as e4m3 values [B, H, S, 128]."""
    return e4m3_values(v8).swapaxes(-1, -2)


def check(out, want, dtype):
    atol, rtol = TOL[dtype]
    err = np.abs(out.float().cpu().numpy() - want)
    bound = atol + rtol * np.abs(want)
    assert np.all(err <= bound), f"max err {err.max():.3e} (worst excess {(err - bound).max():.3e})"


@pytest.mark.parametrize("dtype,B,Hq,Hkv,Sv,Sf,keep", [
    (torch.bfloat16, 2, 28, 4, 1000, 70, 32),     # config-2 group size, ragged last visual block
    (torch.float16, 1, 8, 2, 333, 45, 16),
    (torch.bfloat16, 2, 16, 1, 200, 33, 64),      # 16 heads per unit
    (torch.bfloat16, 1, 4, 4, 64, 0, 32),         # no prompt/text span
])
def test_quantize_bit_exact_and_decode(dtype, B, Hq, Hkv, Sv, Sf, keep):
    d = syn.make_decode(B, Hq, Hkv, Sv, Sf, keep=keep, seed=Sv + keep, device=DEV, dtype=dtype)
    k8, ksc, v8, vsc = quantize_visual_fp8(d.k_sparse, d.v_sparse)
    kq, ksc_o, vq, vsc_o = ofp8.quantize_visual(f64(d.k_sparse), f64(d.v_sparse))
    np.testing.assert_array_equal(ksc.cpu().numpy(), ksc_o)
    np.testing.assert_array_equal(vsc.cpu().numpy(), vsc_o)
    np.testing.assert_array_equal(e4m3_values(k8), kq)
    assert v8.shape == (B, Hkv, 128, Sv) and v8.stride(-1) == 1 and v8.stride(-2) % 16 == 0
    np.testing.assert_array_equal(values_natural(v8), vq)
    # the channel rows' padding to 16 tokens is written as zeros
    s16 = (Sv + 15) // 16 * 16
    padded = torch.as_strided(v8, (B, Hkv, 128, s16), v8.stride())
    assert int(padded[..., Sv:].count_nonzero()) == 0

    out, _, _ = rotatek_decode_fp8(d.q_full, d.R_partial, d.delta_mu, d.k_full, d.v_full, d.mask_full,
                                   k8, ksc, v8, vsc, d.num_kv_groups)
    kd, vd = ofp8.dequantize(kq, ksc_o, vq, vsc_o)
    kw = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in d.as_kwargs().items()}
    kw.update(k_sparse=kd, v_sparse=vd)
    check(out, odec.rotatek_decode(**kw), dtype)
    assert _lib.read_status() == 0


def test_masks_no_bias_and_views():
    """Partial prompt/text mask, no delta_mu, strided prompt/text views, fp8
    tensors passed as float8_e4m3fn."""
    dtype = torch.bfloat16
    d = syn.make_decode(2, 8, 2, 300, 90, keep=32, seed=5, device=DEV, dtype=dtype, with_bias=False)
    kbig = torch.zeros(2, 2, 200, 128, dtype=dtype, device=DEV)
    kbig[:, :, 50:140] = d.k_full
    mask = (torch.rand(2, 90, device=DEV) < 0.6).to(torch.uint8)
    k8, ksc, v8, vsc = quantize_visual_fp8(d.k_sparse, d.v_sparse)
    out, _, _ = rotatek_decode_fp8(d.q_full, d.R_partial, None, kbig[:, :, 50:140], d.v_full, mask,
                                   k8.view(torch.float8_e4m3fn), ksc, v8.view(torch.float8_e4m3fn), vsc, 4)
    kq, ksc_o, vq, vsc_o = ofp8.quantize_visual(f64(d.k_sparse), f64(d.v_sparse))
    kd, vd = ofp8.dequantize(kq, ksc_o, vq, vsc_o)
    want = odec.rotatek_decode(d.q_full.cpu(), d.R_partial.cpu(), None, d.k_full.cpu(), d.v_full.cpu(),
                               mask.cpu(), kd, vd, 4)
    check(out, want, dtype)


def test_values_in_wider_rows_and_one_token():
    """V^T rows wider than the span (a view into a larger buffer) decode like the
    quantiser's own rows; a one-token visual span."""
    dtype = torch.bfloat16
    for sv in (1, 150):
        d = syn.make_decode(2, 14, 2, sv, 20, keep=32, seed=40 + sv, device=DEV, dtype=dtype)
        k8, ksc, v8, vsc = quantize_visual_fp8(d.k_sparse, d.v_sparse)
        wide = torch.full((2, 2, 128, 256 + 48), 0x7F, dtype=torch.uint8, device=DEV)  # e4m3 NaN outside the view
        wide[..., 32:32 + sv] = v8
        v8w = wide[..., 32:32 + sv]
        args = (d.q_full, d.R_partial, d.delta_mu, d.k_full, d.v_full, d.mask_full, k8, ksc)
        out, _, _ = rotatek_decode_fp8(*args, v8, vsc, d.num_kv_groups)
        out_w, _, _ = rotatek_decode_fp8(*args, v8w, vsc, d.num_kv_groups)
        assert torch.equal(out, out_w)
        kq, ksc_o, vq, vsc_o = ofp8.quantize_visual(f64(d.k_sparse), f64(d.v_sparse))
        kd, vd = ofp8.dequantize(kq, ksc_o, vq, vsc_o)
        kw = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in d.as_kwargs().items()}
        kw.update(k_sparse=kd, v_sparse=vd)
        check(out, odec.rotatek_decode(**kw), dtype)


def test_fp8_error_against_16bit_decode_at_config2_shape():
    """Config-2 shape (B=32, 28/4 heads, 64 + 15360 + 576 tokens): the decode
    matches the float64 decode of the dequantised span, and the fp8 span moves
    the output by what e4m3's 3 fraction bits imply (measured 5.0 % relative on
    these N(0,1) Values: the rounding error of a Value, up to 2^-4 of it, is
    averaged over the tokens like the Values themselves)."""
    dtype = torch.bfloat16
    d = syn.make_decode(32, 28, 4, 15360, 640, keep=32, seed=9, device=DEV, dtype=dtype)
    ref, _, _ = rotatek_decode(**d.as_kwargs())
    k8, ksc, v8, vsc = quantize_visual_fp8(d.k_sparse, d.v_sparse)
    out, _, _ = rotatek_decode_fp8(d.q_full, d.R_partial, d.delta_mu, d.k_full, d.v_full, d.mask_full,
                                   k8, ksc, v8, vsc, d.num_kv_groups)
    rel = float((out.float() - ref.float()).norm() / ref.float().norm())
    assert rel < 0.1, rel
    # exact path on a few batch rows (the float64 oracle is slow at full size)
    sub = {k: (v[:2].cpu() if torch.is_tensor(v) else v) for k, v in d.as_kwargs().items()}
    kq, ksc_o, vq, vsc_o = ofp8.quantize_visual(f64(d.k_sparse[:2]), f64(d.v_sparse[:2]))
    kd, vd = ofp8.dequantize(kq, ksc_o, vq, vsc_o)
    sub.update(k_sparse=kd, v_sparse=vd)
    check(out[:2], odec.rotatek_decode(**sub), dtype)
    assert _lib.read_status() == 0


def test_fp8_graph_capture():
    d = syn.make_decode(2, 8, 2, 500, 40, keep=32, seed=3, device=DEV, dtype=torch.bfloat16)
    k8, ksc, v8, vsc = quantize_visual_fp8(d.k_sparse, d.v_sparse)
    args = (d.q_full, d.R_partial, d.delta_mu, d.k_full, d.v_full, d.mask_full, k8, ksc, v8, vsc, 4)
    eager, _, _ = rotatek_decode_fp8(*args)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out, _, _ = rotatek_decode_fp8(*args)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_fp8_errors():
    d = syn.make_decode(1, 4, 1, 64, 8, keep=32, seed=1, device=DEV, dtype=torch.bfloat16)
    k8, ksc, v8, vsc = quantize_visual_fp8(d.k_sparse, d.v_sparse)
    with pytest.raises(ValueError, match="k_scale must be"):
        rotatek_decode_fp8(d.q_full, d.R_partial, d.delta_mu, d.k_full, d.v_full, d.mask_full,
                           k8, ksc[..., :16], v8, vsc, 4)
    with pytest.raises(ValueError, match="v_sparse_fp8 must be"):
        rotatek_decode_fp8(d.q_full, d.R_partial, d.delta_mu, d.k_full, d.v_full, d.mask_full,
                           k8, ksc, v8.float(), vsc, 4)
