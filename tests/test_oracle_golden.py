"""Pin the CPU oracle against outputs of the reference's own code.

The fixtures under tests/golden were produced by tests/golden/make_golden.py,
which runs the reference's `paper` Triton kernels (TRITON_INTERPRET=1) and
ChannelPruner.update_rotatek (ROTATEK_SOLVER=eigh).  Nothing here needs a GPU.
"""
import numpy as np
import pytest

from oracle import decode as odec
from oracle import rotation as orot
from oracle.bf16 import round_bf16, truncate_bf16

# The reference kernels compute in fp32 and store the output in q's dtype.
# fp32: the reference itself sits ~1e-5 from the float64 closed form at logits
# of magnitude ~50, so the bar is 1e-5 absolute plus 1e-5 relative.
# bf16: 2e-3 absolute plus 2^-8 relative -- the output is itself rounded to
# bf16 (half an ulp is 2^-9 relative), and small fixtures with peaked softmax
# produce outputs up to ~2.5 where that rounding alone exceeds 2e-3.
TOL = {"float32": (1e-5, 1e-5), "bfloat16": (2e-3, 2.0 ** -8)}


def assert_matches_reference(oracle_out, ref_out, dtype):
    """fp32: within TOL.  bf16: the fixtures come from Triton's interpreter, which
    truncates fp32 -> bf16 on store; the oracle truncated the same way must give
    the same bits (>= 99 %, the rest one ulp away from a rounding boundary)."""
    if dtype == "float32":
        atol, rtol = TOL[dtype]
        np.testing.assert_allclose(oracle_out, ref_out, atol=atol, rtol=rtol)
        return
    t = truncate_bf16(oracle_out)
    same = np.mean(t == ref_out)
    assert same >= 0.99, same
    np.testing.assert_allclose(t, ref_out, atol=0, rtol=2.0 ** -7)


def test_bf16_rounding_matches_torch():
    import torch
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 37.0
    x[:4] = [1.00390625, 1.01171875, -3.0e38, 0.0]      # ties and extremes
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(round_bf16(x), want)


@pytest.mark.parametrize("case", ["cfg1_fp32", "small_bf16"])
def test_decode_oracle_matches_reference_kernel(golden, case):
    g = golden(case)
    p, v = g["prompt_len"], g["vision_len"]
    keys, values = g["keys"], g["values"]
    k_full = np.concatenate([keys[:, :, :p], keys[:, :, p + v:]], axis=2)
    v_full = np.concatenate([values[:, :, :p], values[:, :, p + v:]], axis=2)
    mask = np.ones(k_full.shape[:1] + k_full.shape[2:3], dtype=np.uint8)
    out = odec.rotatek_decode(g["q_decode"], g["R_partial"], g["delta_mu"], k_full, v_full, mask,
                              g["kept"], values[:, :, p:p + v], g["num_kv_groups"])
    assert_matches_reference(out, g["out_rotatek"], g["dtype"])
    dense = odec.full_channel_decode(g["q_decode"], keys, values, g["num_kv_groups"])
    assert_matches_reference(dense, g["out_dense"], g["dtype"])


@pytest.mark.parametrize("case", ["dec_mask_nobias_fp32", "dec_empty_visual_fp32",
                                  "dec_empty_full_fp32", "dec_g7_bf16"])
def test_decode_edge_cases(golden, case):
    g = golden(case)
    out = odec.rotatek_decode(g["q_full"], g["R_partial"], g.get("delta_mu"), g["k_full"],
                              g["v_full"], g["mask_full"], g["k_sparse"], g["v_sparse"],
                              g["num_kv_groups"])
    assert_matches_reference(out, g["out_rotatek"], g["dtype"])


@pytest.mark.parametrize("case", ["dense_g1_fp32", "dense_g4_bf16"])
def test_dense_oracle(golden, case):
    g = golden(case)
    out = odec.full_channel_decode(g["q"], g["k"], g["v"], g["num_kv_groups"])
    assert_matches_reference(out, g["out_dense"], g["dtype"])


@pytest.mark.parametrize("case,inputs", [("cfg1_fp32", "cfg1_fp32"),
                                         ("cfg1_fp32_plain", "cfg1_fp32"),
                                         ("small_bf16", "small_bf16")])
def test_rotation_oracle_matches_update_rotatek(golden, case, inputs):
    g, src = golden(case), golden(inputs)
    p, v = g["prompt_len"], g["vision_len"]
    keys = src["keys"]
    _, vision, _ = orot.split_spans(keys, p, g["text_len"])
    assert vision.shape[2] == v
    keep = orot.keep_count(keys.shape[-1], g["ratio"])
    res = orot.build_rotation(vision, src["queries_window"], keep, g["num_kv_groups"],
                              query_aware=bool(g["query_aware"]), storage=g["dtype"])
    np.testing.assert_array_equal(res.keep_mask, g["keep_mask"])
    # the subspace is what decode depends on: compare projectors (sign/rotation invariant)
    dist = orot.projector_distance(res.R_partial, g["R_partial"])
    bound = 1e-4 if g["dtype"] == "float32" else 3e-2
    assert dist.max() < bound, dist
    # eigenvalues are separated here, so columns match up to sign
    cos = np.abs((res.R_partial.astype(np.float64) * g["R_partial"]).sum(axis=-2))
    assert cos.min() > (1 - 1e-4 if g["dtype"] == "float32" else 0.95), cos.min()
    tol = 2e-4 if g["dtype"] == "float32" else 0.1
    np.testing.assert_allclose(res.delta_mu, g["delta_mu"], atol=tol)
    scale = np.abs(g["kept"]).max()
    np.testing.assert_allclose(res.kept, g["kept"] * np.sign(cos_signs(res.R_partial, g["R_partial"])),
                               atol=tol * scale)


def cos_signs(a, b):
    """Per-column sign aligning b's eigenvectors with a's: [B, H, 1, k]."""
    s = np.sign((np.asarray(a, np.float64) * np.asarray(b, np.float64)).sum(axis=-2))
    return s[:, :, None, :]


def test_solved_matrix_matches_reference_at_tiny_scale(golden):
    """The matrix the reference hands to eigh (captured from update_rotatek) for
    Keys so small that mean|diag| < 1e-2: pins the centring, the query weighting
    and the ridge 1e-4 * max(mean|diag|, 1e-6) (kv_pruning_utils.py:112-140)."""
    g = golden("tiny_solved_fp32")
    p, v = int(g["prompt_len"]), int(g["vision_len"])
    vision = g["keys"][:, :, p:p + v]
    hkv = vision.shape[1]
    _, cov = orot.covariance(vision, "float32")
    mat = orot.weight_covariance(cov, orot.query_weights(g["queries_window"], hkv, "float32"))
    ref = g["solved"].astype(np.float64)
    assert np.abs(np.diagonal(ref, axis1=-2, axis2=-1)).mean(axis=-1).max() < 1e-2
    np.testing.assert_allclose(mat, ref, rtol=0, atol=2e-6 * np.abs(ref).max())


@pytest.mark.parametrize("case", ["kproj_bf16", "kproj_f16_nobias"])
def test_key_projection_oracle_matches_reference_path(golden, case):
    """k_proj + apply_rotary_pos_emb as the adapters run them (nn.Linear and
    transformers on CPU, llama_visionzip.py:144-153) against the oracle's
    float64 restatement with torch's roundings: the same bits except where the
    projection's accumulation order crosses a rounding boundary (<= 0.2 % of
    the elements, each within 2 ulps of its RoPE pair's magnitude)."""
    from oracle import projection as oproj
    g = golden(case)
    st = g["dtype"]
    k = oproj.key_projection(g["hidden"], g["w_k"], g.get("bias"), g["cos"], g["sin"], st)
    assert k.shape == g["keys"].shape
    frac, worst = oproj.key_mismatch(k, g["keys"], st)
    assert frac <= 2e-3 and worst <= 2.0, (frac, worst)
    # the spans cover the sequence; the sums are those of the stored Keys
    cov, ksum = oproj.visual_sums(g["keys"], g["vis_start"], g["vis_len"])
    v = g["keys"][:, :, g["vis_start"]:g["vis_start"] + g["vis_len"]].astype(np.float64)
    np.testing.assert_allclose(ksum, v.sum(axis=2))
    np.testing.assert_allclose(cov[0, 0], v[0, 0].T @ v[0, 0])


def _spark_spans(g):
    p, v = g["prompt_len"], g["vision_len"]
    keys, values = g["keys"], g["values"]
    return (keys[:, :, p:p + v], np.concatenate([keys[:, :, :p], keys[:, :, p + v:]], axis=2),
            np.concatenate([values[:, :, :p], values[:, :, p + v:]], axis=2), values[:, :, p:p + v])


def test_spark_prune_oracle_matches_update_spark(golden):
    """fp32 (no score ties): the same kept channels and values as the reference's
    ChannelPruner.update_spark, the pruned mean within fp32 summation order."""
    from oracle import spark as osp
    g = golden("spark_fp32")
    k_vis = _spark_spans(g)[0]
    q = osp.update_spark_queries(g["queries_window"], g["num_kv_groups"])
    kc, mask, mean = osp.per_token_channel_prune(q, k_vis, g["ratio"])
    np.testing.assert_array_equal(mask, g["keep_mask"])
    np.testing.assert_array_equal(kc, g["k_compact"])
    np.testing.assert_allclose(mean, g["pruned_mean"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("case", ["spark_fp32", "spark_bf16"])
def test_spark_recovery_and_decode_oracle(golden, case):
    """Packing the mask to ascending channels and recovering gives the
    adapters' recovered Keys bit for bit; the decode over them matches the
    reference's dense Triton decode."""
    from oracle import spark as osp
    g = golden(case)
    _, k_full, v_full, v_vis = _spark_spans(g)
    idx = osp.pack_indices(g["keep_mask"])
    assert idx.shape[-1] == 128 - int(128 * g["ratio"])
    np.testing.assert_array_equal(osp.recover(g["k_compact"], idx, g["pruned_mean"]), g["recovered"])
    out = osp.spark_decode(g["q_decode"], k_full, v_full, None, g["k_compact"], idx, g["pruned_mean"], v_vis,
                           g["num_kv_groups"])
    assert_matches_reference(out, g["out_spark"], g["dtype"])


def test_subspace_iteration_restatement():
    """oracle.rotation.subspace_iteration (the reference's power_iteration_gpu,
    rotatek/rotation.py:68-91): orthonormal after every step, and on a spectrum
    with a clear gap after the k-th eigenvalue it reaches LAPACK's subspace."""
    rng = np.random.default_rng(7)
    q, _ = np.linalg.qr(rng.standard_normal((3, 128, 128)))
    lam = np.concatenate([np.linspace(4.0, 2.0, 8), np.linspace(1.0, 0.1, 120)])
    cov = (q * lam) @ np.swapaxes(q, -1, -2)
    v0 = rng.standard_normal((3, 128, 8))
    v1 = orot.subspace_iteration(cov, v0, 1)
    assert np.abs(np.swapaxes(v1, -1, -2) @ v1 - np.eye(8)).max() < 1e-12
    v = orot.subspace_iteration(cov, v0, 60)
    w, vecs = np.linalg.eigh(cov)
    assert orot.projector_distance(v, vecs[..., ::-1][..., :8]).max() < 1e-8
