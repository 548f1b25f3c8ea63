"""Fused Key projection (k_proj + RoPE + visual-span sums) parity on the GPU.

Oracles: the golden fixtures made by running torch's nn.Linear and
transformers' apply_rotary_pos_emb (the adapters' prefill Key path,
llama_visionzip.py:144-153) on CPU, and the float64 restatement in
oracle/projection.py.  Two correct implementations of this path differ only
where the projection's accumulation order moves k across a rounding boundary,
so the Keys must agree bit for bit on >= 99.8 % of the elements and within 2
ulps of each element's RoPE pair magnitude everywhere (oracle.projection.key_mismatch).
The sums must be those of the Keys the kernel wrote: 1e-5 relative (fp32
accumulation) against float64 sums of its own output.
"""
import numpy as np
import pytest
import torch

from oracle import projection as oproj
from rotatek_b200 import rotation as rot

pytestmark = pytest.mark.gpu
DEV = "cuda"
TORCH_DT = {"bfloat16": torch.bfloat16, "float16": torch.float16}


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def rope_tables(batch, seq, dtype, theta=10000.0, per_batch=True, offset=0):
    inv = 1.0 / theta ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128)
    pos = torch.arange(offset, offset + seq, dtype=torch.float32)[:, None] * inv[None]
    ang = torch.cat([pos, pos], dim=-1)
    cos, sin = ang.cos().to(dtype), ang.sin().to(dtype)
    if per_batch:
        return (cos.unsqueeze(0).expand(batch, -1, -1).contiguous().to(DEV),
                sin.unsqueeze(0).expand(batch, -1, -1).contiguous().to(DEV))
    return cos.unsqueeze(0).to(DEV), sin.unsqueeze(0).to(DEV)


def check_sums(keys, cov, ksum, vs, vl):
    want_cov, want_ks = oproj.visual_sums(f64(keys), vs, vl)
    num = np.sqrt(((f64(cov) - want_cov) ** 2).sum(axis=(-1, -2)))
    den = np.sqrt((want_cov ** 2).sum(axis=(-1, -2)))
    if vl == 0:
        assert np.abs(f64(cov)).max() == 0 and np.abs(f64(ksum)).max() == 0
        return
    assert (num / den).max() < 1e-5, (num / den).max()
    np.testing.assert_allclose(f64(ksum), want_ks, rtol=1e-5, atol=1e-4 * np.abs(want_ks).max())


@pytest.mark.parametrize("case", ["kproj_bf16", "kproj_f16_nobias"])
def test_key_projection_matches_reference_path(golden, case):
    g = golden(case)
    dt = TORCH_DT[g["dtype"]]
    t = {k: torch.from_numpy(np.asarray(g[k], np.float32)).to(dt).to(DEV)
         for k in ("hidden", "w_k", "cos", "sin", "bias") if k in g}
    keys, cov, ksum = rot.key_projection(t["hidden"], t["w_k"], t.get("bias"), t["cos"], t["sin"],
                                         g["vis_start"], g["vis_len"])
    frac, worst = oproj.key_mismatch(f64(keys), g["keys"], g["dtype"])
    assert frac <= 2e-3 and worst <= 2.0, (frac, worst)
    check_sums(keys, cov, ksum, g["vis_start"], g["vis_len"])


@pytest.mark.parametrize("dtype,B,S,hidden,H,vs,vl,bias,per_batch", [
    (torch.bfloat16, 2, 1000, 512, 4, 64, 900, True, True),     # 8 units -> 8-CTA clusters
    (torch.bfloat16, 1, 100, 64, 1, 10, 80, False, False),      # shorter than one tile
    (torch.float16, 2, 700, 256, 2, 0, 700, True, False),       # no prompt, no text
    (torch.bfloat16, 1, 300, 128, 2, 0, 0, True, True),         # no visual span: zero sums
    (torch.bfloat16, 2, 300, 64, 40, 20, 250, False, True),     # 40 units of 4 tiles
    (torch.bfloat16, 8, 300, 128, 15, 20, 250, True, True),     # odd H; CTA ranges cross units
    (torch.bfloat16, 1, 4000, 3584, 4, 32, 3900, True, False),  # Qwen2.5-VL-7B K projection width
    (torch.bfloat16, 3, 259, 128, 2, 1, 257, True, True),       # one prompt and one text token
])
def test_key_projection_vs_oracle(dtype, B, S, hidden, H, vs, vl, bias, per_batch):
    gen = torch.Generator(device=DEV).manual_seed(S + hidden)
    x = torch.randn(B, S, hidden, device=DEV, generator=gen).to(dtype)
    w = (torch.randn(H * 128, hidden, device=DEV, generator=gen) * hidden ** -0.5).to(dtype)
    b = (torch.randn(H * 128, device=DEV, generator=gen) * 0.1).to(dtype) if bias else None
    cos, sin = rope_tables(B, S, dtype, per_batch=per_batch, offset=7)
    keys, cov, ksum = rot.key_projection(x, w, b, cos, sin, vs, vl)
    st = "bfloat16" if dtype == torch.bfloat16 else "float16"
    want = oproj.key_projection(f64(x), f64(w), None if b is None else f64(b), f64(cos), f64(sin), st)
    frac, worst = oproj.key_mismatch(f64(keys), want, st)
    assert frac <= 2e-3 and worst <= 2.0, (frac, worst)
    check_sums(keys, cov, ksum, vs, vl)
    assert rot.read_build_status() == 0


def test_key_projection_cos_sin_16_byte_rows():
    """cos / sin rows that are 16- but not 32-byte aligned (a view into wider
    tables) take the 128-bit load path; the result equals the one from
    contiguous copies of the same tables bit for bit."""
    B, S, hidden, H, vs, vl = 2, 600, 256, 2, 40, 500
    gen = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(B, S, hidden, device=DEV, generator=gen).to(torch.bfloat16)
    w = (torch.randn(H * 128, hidden, device=DEV, generator=gen) * hidden ** -0.5).to(torch.bfloat16)
    b = (torch.randn(H * 128, device=DEV, generator=gen) * 0.1).to(torch.bfloat16)
    cos, sin = rope_tables(B, S, torch.bfloat16)
    # rows of 136 elements (272 bytes), the table starting 8 elements in: 16-byte aligned only
    wide_c = torch.zeros(B, S, 136, device=DEV, dtype=torch.bfloat16)
    wide_s = torch.zeros_like(wide_c)
    wide_c[..., 8:] = cos
    wide_s[..., 8:] = sin
    cos_v, sin_v = wide_c[..., 8:], wide_s[..., 8:]
    assert cos_v.data_ptr() % 32 == 16 and cos_v.stride(1) * 2 % 32 == 16
    keys, cov, ksum = rot.key_projection(x, w, b, cos_v, sin_v, vs, vl)
    keys2, cov2, ksum2 = rot.key_projection(x, w, b, cos, sin, vs, vl)
    assert torch.equal(keys, keys2)
    assert torch.equal(cov, cov2) and torch.equal(ksum, ksum2)
    assert rot.read_build_status() == 0


def test_key_projection_matches_torch_on_gpu():
    """Against the adapters' own ops run by torch on the GPU (cuBLAS k_proj,
    transformers-style RoPE in bf16), at a LLaVA-NeXT-7B-like width."""
    B, S, hidden, H = 2, 2100, 4096, 2
    gen = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(B, S, hidden, device=DEV, generator=gen).to(torch.bfloat16)
    w = (torch.randn(H * 128, hidden, device=DEV, generator=gen) * hidden ** -0.5).to(torch.bfloat16)
    cos, sin = rope_tables(B, S, torch.bfloat16)
    keys, _, _ = rot.key_projection(x, w, None, cos, sin, 32, 2000)
    k = torch.nn.functional.linear(x, w).view(B, S, H, 128).transpose(1, 2)
    half = torch.cat([-k[..., 64:], k[..., :64]], dim=-1)
    ref = k * cos[:, None] + half * sin[:, None]
    frac, worst = oproj.key_mismatch(f64(keys), f64(ref), "bfloat16")
    assert frac <= 2e-3 and worst <= 2.0, (frac, worst)


def test_build_rotation_projected_matches_two_step_build():
    """One call from hidden states equals key_projection followed by
    build_rotation on the visual span of those Keys (same sums up to fp32
    summation order, so the same R up to bf16 rounding flips)."""
    B, S, hidden, H, G, vs, vl = 2, 64 + 3000 + 40, 1024, 2, 3, 64, 3000
    gen = torch.Generator(device=DEV).manual_seed(11)
    z = torch.randn(B, S, 24, device=DEV, generator=gen)
    x = (z @ torch.randn(24, hidden, device=DEV, generator=gen) +
         0.1 * torch.randn(B, S, hidden, device=DEV, generator=gen)).to(torch.bfloat16)
    w = (torch.randn(H * 128, hidden, device=DEV, generator=gen) * hidden ** -0.5).to(torch.bfloat16)
    b = (torch.randn(H * 128, device=DEV, generator=gen) * 0.1).to(torch.bfloat16)
    q = torch.randn(B, H * G, 32, 128, device=DEV, generator=gen).to(torch.bfloat16)
    cos, sin = rope_tables(B, S, torch.bfloat16)
    keys, kept, R, dm, mask = rot.build_rotation_projected(x, w, b, cos, sin, vs, vl, q, 32, G)
    keys2, _, _ = rot.key_projection(x, w, b, cos, sin, vs, vl)
    assert torch.equal(keys, keys2)
    kept2, R2, dm2, mask2 = rot.build_rotation(keys[:, :, vs:vs + vl], q, 32, G)
    P, P2 = f64(R) @ f64(R).swapaxes(-1, -2), f64(R2) @ f64(R2).swapaxes(-1, -2)
    assert np.sqrt(((P - P2) ** 2).sum(axis=(-1, -2))).max() < 2e-2
    np.testing.assert_allclose(f64(dm), f64(dm2), atol=2e-2 * np.abs(f64(dm2)).max())
    # kept is the rotation of the visual Keys by the returned R
    want = f64(keys[:, :, vs:vs + vl]) @ f64(R)
    assert np.abs(f64(kept) - want).max() <= 2 ** -7 * np.abs(want).max()
    assert torch.equal(mask, mask2)
    assert rot.read_build_status() == 0


def test_key_projection_graph_capture():
    B, S, hidden, H = 1, 600, 256, 2
    gen = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(B, S, hidden, device=DEV, generator=gen).to(torch.bfloat16)
    w = (torch.randn(H * 128, hidden, device=DEV, generator=gen) * hidden ** -0.5).to(torch.bfloat16)
    cos, sin = rope_tables(B, S, torch.bfloat16)
    eager = rot.key_projection(x, w, None, cos, sin, 16, 500)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        rot.key_projection(x, w, None, cos, sin, 16, 500)   # warm-up outside capture
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = rot.key_projection(x, w, None, cos, sin, 16, 500)
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, out):
        assert torch.equal(a, b)


def test_key_projection_errors():
    x = torch.zeros(1, 10, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(128, 64, device=DEV, dtype=torch.bfloat16)
    cos = torch.zeros(1, 10, 128, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="visual span"):
        rot.key_projection(x, w, None, cos, cos, 5, 6)
    with pytest.raises(ValueError, match="w_k must be"):
        rot.key_projection(x, w[:100], None, cos, cos, 0, 10)
    with pytest.raises(RuntimeError, match="bfloat16 or float16"):
        rot.key_projection(x.float(), w.float(), None, cos.float(), cos.float(), 0, 10)
