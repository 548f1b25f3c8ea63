"""SparK baseline decode on the GPU: pack_spark_indices + spark_decode against
the float64 oracle of the adapters' recovery + dense decode, and against the
reference's own outputs (spark_* fixtures).

Tolerances as for the 16-bit decode (tests/test_decode_gpu.py): bf16 2e-3
absolute + 2^-8 relative, fp16 1e-3 + 2^-10.  The recovered Keys are exact
16-bit values (a copy of the kept values and the mean), so the fused decode is
held to the dense decode's bar.
"""
import numpy as np
import pytest
import torch

from oracle import spark as osp
from rotatek_b200 import _lib, synthetic as syn
from rotatek_b200.kernels import full_channel_decode, pack_spark_indices, spark_decode

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.bfloat16: (2e-3, 2.0 ** -8), torch.float16: (1e-3, 2.0 ** -10)}


def f64(t):
    return None if t is None else t.detach().double().cpu().numpy()


def check(out, want, dtype):
    atol, rtol = TOL[dtype]
    err = np.abs(out.float().cpu().numpy() - want)
    bound = atol + rtol * np.abs(want)
    assert np.all(err <= bound), f"max err {err.max():.3e} (worst excess {(err - bound).max():.3e})"


def oracle(d, idx, mask=None):
    return osp.spark_decode(f64(d.q_full), f64(d.k_full), f64(d.v_full), None if mask is None else f64(mask),
                            f64(d.k_kept), idx.cpu().numpy(), f64(d.pruned_mean), f64(d.v_sparse),
                            d.num_kv_groups)


@pytest.mark.parametrize("dtype,B,Hq,Hkv,Sv,Sf,keep", [
    (torch.bfloat16, 2, 28, 4, 1000, 70, 32),     # config-2 group size (G=7), ragged last block
    (torch.float16, 1, 8, 2, 333, 45, 16),
    (torch.bfloat16, 2, 16, 1, 200, 33, 64),      # 16 heads per unit, D_keep 64
    (torch.bfloat16, 1, 4, 4, 64, 0, 32),         # MHA, no prompt/text span
    (torch.float16, 1, 32, 2, 97, 10, 32),        # two head chunks of 16
])
def test_spark_decode_matches_oracle(dtype, B, Hq, Hkv, Sv, Sf, keep):
    d = syn.make_spark(B, Hq, Hkv, Sv, Sf, keep=keep, seed=Sv + keep, device=DEV, dtype=dtype)
    idx = pack_spark_indices(d.keep_mask, keep)
    np.testing.assert_array_equal(idx.cpu().numpy(), osp.pack_indices(d.keep_mask.cpu().numpy()))
    out = spark_decode(d.q_full, d.k_full, d.v_full, d.mask_full, d.k_kept, idx, d.pruned_mean, d.v_sparse,
                       d.num_kv_groups)
    assert out.shape == (B, 1, Hq, 128) and out.dtype == dtype
    check(out, oracle(d, idx, d.mask_full), dtype)
    assert _lib.read_status() == 0


def test_spark_matches_reference_outputs(golden):
    """The reference's update_spark outputs (bf16, D_keep 64, ragged visual
    span) through pack + fused decode give the reference's Triton decode of
    the recovered cache."""
    g = golden("spark_bf16")
    p, v = g["prompt_len"], g["vision_len"]
    t = lambda x: torch.as_tensor(np.asarray(x, dtype=np.float32)).to(DEV).to(torch.bfloat16)
    keys, values = t(g["keys"]), t(g["values"])
    k_full = torch.cat([keys[:, :, :p], keys[:, :, p + v:]], dim=2)
    v_full = torch.cat([values[:, :, :p], values[:, :, p + v:]], dim=2)
    mask = torch.as_tensor(g["keep_mask"]).to(DEV)
    idx = pack_spark_indices(mask, g["k_compact"].shape[-1])
    out = spark_decode(t(g["q_decode"]), k_full, v_full, None, t(g["k_compact"]), idx, t(g["pruned_mean"]),
                       values[:, :, p:p + v], g["num_kv_groups"])
    # the float64 oracle (pinned to these outputs on the CPU) at the usual bar
    want = osp.spark_decode(f64(t(g["q_decode"])), f64(k_full), f64(v_full), None, g["k_compact"],
                            idx.cpu().numpy(), g["pruned_mean"], f64(values[:, :, p:p + v]), g["num_kv_groups"])
    check(out, want, torch.bfloat16)
    # the reference's own numbers: Triton's interpreter stores bf16 by truncation,
    # so they may sit one bf16 ulp below a rounded result, on top of that bar
    ref = g["out_spark"]
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)
    atol, rtol = TOL[torch.bfloat16]
    err = np.abs(out.float().cpu().numpy() - ref)
    assert np.all(err <= atol + rtol * np.abs(ref) + ulp), err.max()


def test_masks_views_and_3d_mean():
    """Partial prompt/text mask, strided prompt/text and visual Value views (the
    adapters' value_states[:, :, s_p:s_p + s_v]), pruned_mean given as [B, H, S]."""
    dtype = torch.bfloat16
    d = syn.make_spark(2, 8, 2, 300, 90, keep=32, seed=5, device=DEV, dtype=dtype)
    vbig = torch.zeros(2, 2, 500, 128, dtype=dtype, device=DEV)
    vbig[:, :, 100:400] = d.v_sparse
    kbig = torch.zeros(2, 2, 200, 128, dtype=dtype, device=DEV)
    kbig[:, :, 50:140] = d.k_full
    mask = (torch.rand(2, 90, device=DEV) < 0.6).to(torch.uint8)
    idx = pack_spark_indices(d.keep_mask, 32)
    out = spark_decode(d.q_full, kbig[:, :, 50:140], d.v_full, mask, d.k_kept, idx, d.pruned_mean[..., 0],
                       vbig[:, :, 100:400], 4)
    check(out, oracle(d, idx, mask), dtype)


def test_equals_dense_decode_of_recovered_keys_at_config2_shape():
    """Config-2 shape (B=32, 28/4 heads, 64 + 15360 + 576 tokens, D_keep 32):
    the fused decode against this library's dense decode of the adapters'
    recovered and concatenated cache; a few batch rows against the oracle."""
    dtype = torch.bfloat16
    d = syn.make_spark(32, 28, 4, 15360, 640, keep=32, seed=9, device=DEV, dtype=dtype)
    idx = pack_spark_indices(d.keep_mask, 32)
    out = spark_decode(d.q_full, d.k_full, d.v_full, None, d.k_kept, idx, d.pruned_mean, d.v_sparse, 7)
    dense = full_channel_decode(d.q_full, torch.cat([d.k_full, d.recovered()], dim=2),
                                torch.cat([d.v_full, d.v_sparse], dim=2), 7)
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(out.float(), dense.float(), atol=atol, rtol=rtol)
    sub = syn.SparkInputs(*(x[:2] if torch.is_tensor(x) else x for x in (
        d.q_full, d.k_full, d.v_full, d.mask_full, d.k_kept, d.keep_mask, d.pruned_mean, d.v_sparse)), 7)
    check(out[:2], oracle(sub, idx[:2]), dtype)
    assert _lib.read_status() == 0


def test_spark_graph_capture():
    d = syn.make_spark(2, 8, 2, 500, 40, keep=32, seed=3, device=DEV, dtype=torch.bfloat16)
    idx = pack_spark_indices(d.keep_mask, 32)
    args = (d.q_full, d.k_full, d.v_full, d.mask_full, d.k_kept, idx, d.pruned_mean, d.v_sparse, 4)
    eager = spark_decode(*args)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = spark_decode(*args)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_spark_errors():
    d = syn.make_spark(1, 4, 1, 64, 8, keep=32, seed=1, device=DEV, dtype=torch.bfloat16)
    idx = pack_spark_indices(d.keep_mask, 32)
    bad = d.keep_mask.clone()
    bad[0, 0, 3, :] = True
    with pytest.raises(ValueError, match="exactly 32"):
        pack_spark_indices(bad, 32)
    with pytest.raises(ValueError, match="keep_idx must be"):
        spark_decode(d.q_full, d.k_full, d.v_full, None, d.k_kept, idx.int(), d.pruned_mean, d.v_sparse, 4)
    with pytest.raises(ValueError, match="pruned_mean must be"):
        spark_decode(d.q_full, d.k_full, d.v_full, None, d.k_kept, idx, d.pruned_mean[:, :, :10], d.v_sparse, 4)
    d32 = syn.make_spark(1, 4, 1, 64, 8, keep=32, seed=1, device=DEV, dtype=torch.float32)
    with pytest.raises(RuntimeError, match="SparK decode needs"):
        spark_decode(d32.q_full, d32.k_full, d32.v_full, None, d32.k_kept, idx, d32.pruned_mean, d32.v_sparse, 4)
