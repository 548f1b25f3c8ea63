"""Pin the timed CPU baseline (oracle/eager_torch.py) to the reference's own outputs.

``rotatek_decode_eager`` and ``update_rotatek_eager`` are what ``bench.py``
times as the reference's CPU path (its `cpu_baseline` and `--impl reference`
legs).  These tests hold them to the fixtures that tests/golden/make_golden.py
made by running the reference's code: the `paper` Triton decode kernels under
TRITON_INTERPRET=1 (rotatek/kernels/fused_decode.py:303-420,
full_channel_flash_decoding.py:162-229) and ChannelPruner.update_rotatek with
ROTATEK_SOLVER=eigh (kv_pruning_utils.py:92-160).  No GPU needed.
"""
import numpy as np
import pytest
import torch

from oracle import rotation as orot
from oracle.bf16 import truncate_bf16
from oracle.eager_torch import rotatek_decode_eager, update_rotatek_eager

TORCH_DTYPE = {"float32": torch.float32, "bfloat16": torch.bfloat16}


def _decode_args(g, dtype):
    """The fixture's decode inputs as CPU tensors holding the stored dtype's values."""
    p, v = g["prompt_len"], g["vision_len"]
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dtype)  # noqa: E731
    keys, values = t(g["keys"]), t(g["values"])
    k_full = torch.cat([keys[:, :, :p], keys[:, :, p + v:]], dim=2)
    v_full = torch.cat([values[:, :, :p], values[:, :, p + v:]], dim=2)
    mask = torch.ones(k_full.shape[0], k_full.shape[2], dtype=torch.uint8)
    return dict(q_full=t(g["q_decode"]), R_partial=t(g["R_partial"]), delta_mu=t(g["delta_mu"]),
                k_full=k_full, v_full=v_full, mask_full=mask, k_sparse=t(g["kept"]),
                v_sparse=values[:, :, p:p + v], num_kv_groups=int(g["num_kv_groups"]))


@pytest.mark.parametrize("case", ["cfg1_fp32", "small_bf16"])
def test_eager_decode_matches_reference_kernel(golden, case):
    """fp32: within 1e-5 + 1e-5 relative of the reference kernel.  bf16: the
    reference kernel loads bf16 and computes in fp32, so the eager port is run
    on the fp32 values of the bf16 inputs; its fp32 output truncated to bf16 (the
    interpreter's store) must give the fixture's bits for >= 99 % of outputs and
    lie within one bf16 ulp everywhere."""
    g = golden(case)
    args = _decode_args(g, TORCH_DTYPE[g["dtype"]])
    if g["dtype"] == "float32":
        out = rotatek_decode_eager(**args).numpy()
        np.testing.assert_allclose(out, g["out_rotatek"], atol=1e-5, rtol=1e-5)
        return
    args32 = {k: (x.float() if torch.is_tensor(x) and x.is_floating_point() else x) for k, x in args.items()}
    out = truncate_bf16(rotatek_decode_eager(**args32).numpy())
    assert np.mean(out == g["out_rotatek"]) >= 0.99
    np.testing.assert_allclose(out, g["out_rotatek"], atol=0, rtol=2.0 ** -7)
    # and the bf16 call itself (fp32 math, round-to-nearest store) within the bf16 bar
    direct = rotatek_decode_eager(**args).float().numpy()
    np.testing.assert_allclose(direct, g["out_rotatek"], atol=2e-3, rtol=2.0 ** -7)


def test_eager_decode_honours_mask(golden):
    """mask_full == 0 drops those prompt/text tokens (fused_decode.py:254-258):
    the eager port against the fixture made with a partial mask and no delta_mu."""
    g = golden("dec_mask_nobias_fp32")
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))  # noqa: E731
    out = rotatek_decode_eager(t(g["q_full"]), t(g["R_partial"]), None, t(g["k_full"]), t(g["v_full"]),
                               torch.from_numpy(g["mask_full"]), t(g["k_sparse"]), t(g["v_sparse"]),
                               int(g["num_kv_groups"])).numpy()
    assert not g["has_bias"] and g["mask_full"].min() == 0
    np.testing.assert_allclose(out, g["out_rotatek"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("case", ["cfg1_fp32", "small_bf16"])
def test_eager_build_matches_update_rotatek(golden, case):
    """The eager build against update_rotatek's own outputs: same keep mask,
    the same subspace (projector distance), delta_mu and kept up to column sign.
    The port runs the reference's torch ops in the same order, so here it gives
    the fixture's bits; the bars leave room only for a BLAS that sums in
    another order (fp32: 1e-5; bf16: one bf16 ulp)."""
    g = golden(case)
    dtype = TORCH_DTYPE[g["dtype"]]
    p, v = g["prompt_len"], g["vision_len"]
    keys = torch.from_numpy(g["keys"]).to(dtype)
    queries = torch.from_numpy(g["queries_window"]).to(dtype)
    keep = orot.keep_count(keys.shape[-1], g["ratio"])
    kept, R, dm, mask = update_rotatek_eager(keys[:, :, p:p + v], queries, keep, int(g["num_kv_groups"]),
                                             query_aware=bool(g["query_aware"]))
    np.testing.assert_array_equal(mask.numpy(), g["keep_mask"])
    R = R.float().numpy()
    dist = orot.projector_distance(R, g["R_partial"])
    fp32 = g["dtype"] == "float32"
    assert dist.max() < (1e-5 if fp32 else 1e-3), dist
    sign = np.sign((R.astype(np.float64) * g["R_partial"]).sum(axis=-2))[:, :, None, :]
    tol = 1e-5 if fp32 else 2.0 ** -7
    np.testing.assert_allclose(dm.float().numpy(), g["delta_mu"], atol=tol)
    scale = np.abs(g["kept"]).max()
    np.testing.assert_allclose(kept.float().numpy(), g["kept"] * sign, atol=tol * scale)
