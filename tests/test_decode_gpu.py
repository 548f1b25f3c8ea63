"""Decode parity on the GPU: rotatek_b200.kernels vs the float64 oracle.

Tolerances (written out per dtype):
  fp32  1e-5 absolute + 1e-5 relative  (the reference itself sits ~1e-5 from
        the float64 closed form at logits of magnitude ~50)
  bf16  2e-3 absolute + 2^-8 relative  (the output is stored in bf16: half an
        ulp is 2^-9 relative, so outputs above 0.5 need the relative term)
  fp16  1e-3 absolute + 2^-10 relative
"""
import math

import numpy as np
import pytest
import torch

from oracle import decode as odec
from rotatek_b200 import _lib, synthetic as syn
from rotatek_b200.kernels import full_channel_decode, rotatek_decode

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-5), torch.bfloat16: (2e-3, 2.0 ** -8),
       torch.float16: (1e-3, 2.0 ** -10)}
DEV = "cuda"


def _t(x, dtype):
    return torch.as_tensor(np.asarray(x, dtype=np.float32)).to(DEV).to(dtype)


def check(out, want, dtype):
    atol, rtol = TOL[dtype]
    got = out.float().cpu().numpy()
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    assert np.all(err <= bound), f"max err {err.max():.3e} (worst excess {(err - bound).max():.3e})"


def assert_status_clean():
    assert _lib.read_status() == 0


@pytest.mark.parametrize("case", ["cfg1_fp32", "small_bf16"])
def test_golden_prefill_cases(golden, case):
    g = golden(case)
    dtype = {"float32": torch.float32, "bfloat16": torch.bfloat16}[g["dtype"]]
    p, v = g["prompt_len"], g["vision_len"]
    keys, values = _t(g["keys"], dtype), _t(g["values"], dtype)
    k_full = torch.cat([keys[:, :, :p], keys[:, :, p + v:]], dim=2)
    v_full = torch.cat([values[:, :, :p], values[:, :, p + v:]], dim=2)
    mask = torch.ones(k_full.shape[0], k_full.shape[2], dtype=torch.uint8, device=DEV)
    args = dict(q_full=_t(g["q_decode"], dtype), R_partial=_t(g["R_partial"], dtype),
                delta_mu=_t(g["delta_mu"], dtype), k_full=k_full, v_full=v_full, mask_full=mask,
                k_sparse=_t(g["kept"], dtype), v_sparse=values[:, :, p:p + v],
                num_kv_groups=g["num_kv_groups"])
    out, a, b = rotatek_decode(**args)
    assert a is None and b is None and out.shape == (keys.shape[0], 1, args["q_full"].shape[1], 128)
    want = odec.rotatek_decode(**{k: (x.cpu() if torch.is_tensor(x) else x) for k, x in args.items()})
    check(out, want, dtype)
    dense = full_channel_decode(args["q_full"], keys, values, num_kv_groups=g["num_kv_groups"])
    check(dense, odec.full_channel_decode(args["q_full"].cpu(), keys.cpu(), values.cpu(),
                                          g["num_kv_groups"]), dtype)
    assert_status_clean()


@pytest.mark.parametrize("case", ["dec_mask_nobias_fp32", "dec_empty_visual_fp32",
                                  "dec_empty_full_fp32", "dec_g7_bf16"])
def test_golden_decode_edge_cases(golden, case):
    g = golden(case)
    dtype = {"float32": torch.float32, "bfloat16": torch.bfloat16}[g["dtype"]]
    args = dict(q_full=_t(g["q_full"], dtype), R_partial=_t(g["R_partial"], dtype),
                delta_mu=_t(g["delta_mu"], dtype) if g["has_bias"] else None,
                k_full=_t(g["k_full"], dtype), v_full=_t(g["v_full"], dtype),
                mask_full=torch.as_tensor(g["mask_full"]).to(DEV),
                k_sparse=_t(g["k_sparse"], dtype), v_sparse=_t(g["v_sparse"], dtype),
                num_kv_groups=g["num_kv_groups"])
    out, _, _ = rotatek_decode(**args)
    want = odec.rotatek_decode(**{k: (x.cpu() if torch.is_tensor(x) else x) for k, x in args.items()})
    check(out, want, dtype)
    assert_status_clean()


def make(dtype, B, Hq, Hkv, Sv, Sf, keep=32, seed=0, bias=True):
    return syn.make_decode(B, Hq, Hkv, Sv, Sf, keep=keep, seed=seed, device=DEV, dtype=dtype,
                           with_bias=bias)


def run_and_check(d, dtype, mask=None):
    kw = d.as_kwargs()
    if mask is not None:
        kw["mask_full"] = mask
    out, _, _ = rotatek_decode(**kw)
    want = odec.rotatek_decode(**{k: (x.cpu() if torch.is_tensor(x) else x) for k, x in kw.items()})
    check(out, want, dtype)
    return out


# (dtype, B, H_q, H_kv, S_v, S_f, keep): tensor-core path shapes (bf16/fp16, D=128,
# keep in {16,32,64}) across group sizes 1..20, ragged spans, and generic-path shapes
SHAPES = [
    (torch.bfloat16, 2, 28, 4, 1000, 100, 32),     # G=7, the headline group
    (torch.bfloat16, 1, 8, 8, 777, 13, 32),        # G=1 (MHA)
    (torch.bfloat16, 3, 8, 2, 4096, 640, 16),      # G=4, keep 16
    (torch.bfloat16, 2, 16, 2, 130, 65, 64),       # G=8, keep 64
    (torch.bfloat16, 1, 12, 1, 300, 40, 32),       # G=12 -> 16-head tile
    (torch.bfloat16, 1, 40, 2, 200, 70, 32),       # G=20 -> two head chunks
    (torch.float16, 2, 28, 4, 1500, 200, 32),      # fp16
    (torch.bfloat16, 1, 4, 2, 1, 1, 32),           # one token per span
    (torch.bfloat16, 2, 8, 2, 64, 64, 32),         # exact block multiples
    (torch.bfloat16, 1, 8, 2, 300, 50, 48),        # keep 48 -> generic kernel
    (torch.float32, 2, 8, 2, 576, 96, 32),         # fp32 -> generic kernel
]


@pytest.mark.parametrize("dtype,B,Hq,Hkv,Sv,Sf,keep", SHAPES)
def test_decode_shapes(dtype, B, Hq, Hkv, Sv, Sf, keep):
    d = make(dtype, B, Hq, Hkv, Sv, Sf, keep=keep, seed=B * 100 + Hq)
    run_and_check(d, dtype)
    assert_status_clean()


def test_decode_mask_and_no_bias():
    d = make(torch.bfloat16, 2, 28, 4, 700, 333, seed=5, bias=False)
    g = torch.Generator(device=DEV).manual_seed(3)
    mask = (torch.rand(2, 333, generator=g, device=DEV) < 0.4).to(torch.uint8)
    run_and_check(d, torch.bfloat16, mask=mask)
    mask.zero_()                                   # every prompt/text token masked
    run_and_check(d, torch.bfloat16, mask=mask)


def test_decode_empty_spans():
    for sv, sf in [(0, 50), (90, 0), (0, 0)]:
        d = make(torch.bfloat16, 2, 8, 2, sv, sf, seed=sv + sf)
        out = run_and_check(d, torch.bfloat16)
        if sv == 0 and sf == 0:
            assert torch.count_nonzero(out) == 0


def test_decode_strided_views():
    """The adapters pass v_sparse as a slice of the whole V cache and cat'ed k/v_full."""
    B, Hq, Hkv, Sp, Sv, St = 2, 28, 4, 64, 1200, 100
    dtype = torch.bfloat16
    d = make(dtype, B, Hq, Hkv, Sv, Sp + St, seed=9)
    v_cache = syn.normal((B, Hkv, Sp + Sv + St, 128), 11, DEV, dtype)
    kw = d.as_kwargs()
    kw["v_sparse"] = v_cache[:, :, Sp:Sp + Sv]
    kw["v_full"] = torch.cat([v_cache[:, :, :Sp], v_cache[:, :, Sp + Sv:]], dim=2)
    assert not kw["v_sparse"].is_contiguous()
    out, _, _ = rotatek_decode(**kw)
    want = odec.rotatek_decode(**{k: (x.cpu() if torch.is_tensor(x) else x) for k, x in kw.items()})
    check(out, want, dtype)
    # head-major Keys stored [B, S, H, D] and viewed as [B, H, S, D]
    ks = d.k_sparse.transpose(1, 2).contiguous().transpose(1, 2)
    kw["k_sparse"] = ks
    out2, _, _ = rotatek_decode(**kw)
    check(out2, want, dtype)


def bf16_half_ulp(x):
    """Half the bf16 spacing at |x|: the error of rounding x to bf16."""
    a = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    return np.where(a > 0, 2.0 ** (e - 8), 0.0)


def test_decode_config2_full_size():
    """benchmark config 2 at full size: B=32, 28/4 heads, 64+15360+576, keep 32, bf16.

    The north-star bar is max-abs 2e-3 on the bf16 output.  Outputs here reach
    |x| ~ 4, where storing in bf16 alone moves a value by up to 2^-7, so the bar
    is applied beyond that rounding: |out - oracle| <= 2e-3 + half_ulp_bf16(oracle).
    Most outputs must equal the correctly rounded float64 value outright."""
    from oracle.bf16 import round_bf16
    d = make(torch.bfloat16, 32, 28, 4, 15360, 640, seed=2024)
    out, _, _ = rotatek_decode(**d.as_kwargs())
    want = odec.rotatek_decode(**{k: (x.cpu() if torch.is_tensor(x) else x)
                                  for k, x in d.as_kwargs().items()})
    got = out.float().cpu().numpy()
    excess = np.abs(got - want) - bf16_half_ulp(want)
    assert excess.max() <= 2e-3, excess.max()
    assert np.mean(got == round_bf16(want)) >= 0.99
    assert_status_clean()


def test_workspace_reuse_across_shapes():
    """One workspace serves calls whose unit counts grow and shrink: a larger
    B * H_q call must not read an earlier call's partials as ticket counters."""
    seq = [(torch.bfloat16, 2, 8, 2, 300, 40), (torch.float32, 1, 4, 2, 200, 30),
           (torch.bfloat16, 8, 28, 4, 2000, 100), (torch.bfloat16, 1, 8, 8, 900, 10),
           (torch.bfloat16, 16, 28, 4, 3000, 200), (torch.float32, 4, 16, 4, 100, 20),
           (torch.bfloat16, 16, 28, 4, 3000, 200)]
    for n, (dtype, B, Hq, Hkv, Sv, Sf) in enumerate(seq):
        run_and_check(make(dtype, B, Hq, Hkv, Sv, Sf, seed=300 + n), dtype)
    assert_status_clean()


def test_repeat_calls_identical():
    """Ticket counters return to zero: a second call gives the same bits."""
    d = make(torch.bfloat16, 4, 28, 4, 3000, 200, seed=17)
    a, _, _ = rotatek_decode(**d.as_kwargs())
    b, _, _ = rotatek_decode(**d.as_kwargs())
    torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_full_channel_decode_shapes():
    for dtype, B, Hq, Hkv, S in [(torch.bfloat16, 2, 28, 4, 16000), (torch.bfloat16, 1, 8, 8, 99),
                                 (torch.float16, 3, 32, 8, 1000), (torch.float32, 1, 4, 2, 500)]:
        q = syn.normal((B, Hq, 128), 1, DEV, dtype)
        k = syn.lowrank_keys(B, Hkv, S, seed=2, device=DEV, dtype=dtype)
        v = syn.normal((B, Hkv, S, 128), 3, DEV, dtype)
        out = full_channel_decode(q, k, v, num_kv_groups=Hq // Hkv)
        check(out, odec.full_channel_decode(q.cpu(), k.cpu(), v.cpu(), Hq // Hkv), dtype)


def test_cuda_graph_capture_and_replay():
    """graph_bench.py:27-44 captures the decode call; the replayed graph must match eager."""
    d = make(torch.bfloat16, 4, 28, 4, 2000, 100, seed=21)
    kw = d.as_kwargs()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            eager, _, _ = rotatek_decode(**kw)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured, _, _ = rotatek_decode(**kw)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(captured, eager, rtol=0, atol=0)


def test_reference_value_errors():
    d = make(torch.bfloat16, 1, 8, 2, 64, 8, seed=1)
    kw = d.as_kwargs()
    with pytest.raises(ValueError, match=r"q_full must be \[B, H_q, D\]"):
        rotatek_decode(**{**kw, "q_full": kw["q_full"][0]})
    with pytest.raises(ValueError, match="R_partial must be"):
        rotatek_decode(**{**kw, "R_partial": kw["R_partial"][0]})
    with pytest.raises(ValueError, match="mask_full must be uint8"):
        rotatek_decode(**{**kw, "mask_full": kw["mask_full"].bool()})
    with pytest.raises(ValueError, match="R_partial H_kv=2 but H_q=8, num_kv_groups=2"):
        rotatek_decode(**{**kw, "num_kv_groups": 2})
    with pytest.raises(ValueError, match="k_sparse must be"):
        rotatek_decode(**{**kw, "k_sparse": kw["k_sparse"][:, :1]})
    with pytest.raises(ValueError, match=r"q must be \[B, H_q, D\]"):
        full_channel_decode(kw["q_full"][0], kw["k_full"], kw["v_full"], 4)
    with pytest.raises(ValueError, match="head_dim must match"):
        full_channel_decode(kw["q_full"], kw["k_full"][..., :64], kw["v_full"], 4)


@pytest.mark.parametrize("dtype,G", [(torch.bfloat16, 7), (torch.float32, 1)])
def test_think_decode_matches_recovered_dense(dtype, G):
    """ThinK: the fused decode on the kept channels equals the dense decode on
    Keys with the pruned channels zero-filled (llama_visionzip.py:217-240)."""
    from rotatek_b200.kernels import think_decode
    B, Hkv, Sv, Sf, D, keep = 2, 2, 300, 40, 128, 32
    gen = torch.Generator().manual_seed(11)
    k_vis = torch.randn(B, Hkv, Sv, D, generator=gen)
    scores = torch.rand(B, Hkv, D, generator=gen)
    think_mask = torch.zeros(B, Hkv, D, dtype=torch.bool)
    think_mask.scatter_(2, scores.topk(keep, dim=-1).indices, True)
    sel = think_mask.unsqueeze(2).expand(-1, -1, Sv, -1)
    key_pruned = k_vis[sel].view(B, Hkv, Sv, keep)
    recovered = torch.zeros_like(k_vis)
    recovered[sel] = key_pruned.reshape(-1)
    k_full = torch.randn(B, Hkv, Sf, D, generator=gen)
    v_full = torch.randn(B, Hkv, Sf, D, generator=gen)
    v_vis = torch.randn(B, Hkv, Sv, D, generator=gen)
    q = torch.randn(B, Hkv * G, D, generator=gen)
    cu = lambda t: t.to(DEV, dtype)  # noqa: E731
    got = think_decode(cu(q), think_mask.to(DEV), cu(key_pruned), cu(k_full), cu(v_full), None, cu(v_vis), G)
    # float64 restatement of the adapters' path, on the same (rounded) inputs:
    # dense decode over [prompt/text | zero-filled visual Keys]
    rnd = lambda t: np.asarray(t.to(dtype).float().numpy(), dtype=np.float64)  # noqa: E731
    want = odec.full_channel_decode(rnd(q), rnd(torch.cat([k_full, recovered], -2)),
                                    rnd(torch.cat([v_full, v_vis], -2)), G)
    rel = 2.0 ** -8 if dtype == torch.bfloat16 else 1e-5
    tol = (2e-3 if dtype == torch.bfloat16 else 1e-5) + rel * np.abs(want).max()
    np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=0, atol=tol)


def _rows(kw, rows):
    """The decode arguments restricted to batch rows `rows`, on the CPU (batch
    rows are independent units, so the oracle of a subset is a subset of the oracle)."""
    idx = torch.as_tensor(rows, device=DEV)
    out = {}
    for k, x in kw.items():
        out[k] = x.index_select(0, idx).cpu() if torch.is_tensor(x) else x
    return out


@pytest.mark.parametrize("sf", [1025, 3000])
def test_decode_long_masked_full_span(sf):
    """Prompt/text spans longer than the kernel's 1024-byte header mask: the
    mask is read per token from global memory (fused_decode.py:254-258 honours
    it at any length).  ~40 % of the tokens masked, plus a row with none kept."""
    d = make(torch.bfloat16, 3, 28, 4, 2000, sf, seed=40 + sf)
    g = torch.Generator(device=DEV).manual_seed(sf)
    mask = (torch.rand(3, sf, generator=g, device=DEV) < 0.6).to(torch.uint8)
    mask[2].zero_()
    run_and_check(d, torch.bfloat16, mask=mask)
    assert_status_clean()


@pytest.mark.parametrize("sf", [333, 1024, 1500])
def test_decode_strided_mask(sf):
    """mask_full as a strided view (every other column of a wider buffer) and as
    an unaligned slice: the header's register-staged path (S_f <= 1024) and the
    global-memory path (S_f > 1024)."""
    d = make(torch.bfloat16, 2, 28, 4, 900, sf, seed=sf, bias=False)
    g = torch.Generator(device=DEV).manual_seed(7 + sf)
    wide = (torch.rand(2, 2 * sf + 3, generator=g, device=DEV) < 0.55).to(torch.uint8)
    strided = wide[:, 1:1 + 2 * sf:2]
    assert strided.stride(-1) == 2
    run_and_check(d, torch.bfloat16, mask=strided)
    shifted = wide[:, 3:3 + sf]
    assert shifted.data_ptr() % 16 != 0
    run_and_check(d, torch.bfloat16, mask=shifted)
    assert_status_clean()


def test_decode_config5_shape():
    """Benchmark config 5 on one GPU at full size: B=64, 64 query / 8 KV heads
    (G=8), 64 prompt + 31 744 visual + 960 text tokens (S_f = 1024, the header
    mask's limit), keep 32, bf16, with a partial mask.  Four batch rows, spread
    over the batch, are checked against the float64 oracle."""
    d = make(torch.bfloat16, 64, 64, 8, 31744, 1024, seed=72)
    g = torch.Generator(device=DEV).manual_seed(72)
    mask = (torch.rand(64, 1024, generator=g, device=DEV) < 0.9).to(torch.uint8)
    kw = {**d.as_kwargs(), "mask_full": mask}
    out, _, _ = rotatek_decode(**kw)
    rows = [0, 21, 42, 63]
    want = odec.rotatek_decode(**_rows(kw, rows))
    check(out[rows], want, torch.bfloat16)
    assert torch.isfinite(out).all()
    assert_status_clean()


def test_decode_config3_layer_shape():
    """One layer of benchmark config 3 at full size: fp16, 32 query = 32 KV heads
    (G=1, MHA), batch 8, 16 384 visual tokens, and the span-split cache's
    prompt | text capacity (32 + 128 tokens) with the unwritten text slots
    masked, as a CUDA-graph decode step passes them.  Three rows checked."""
    sp, cap = 32, 128
    d = make(torch.float16, 8, 32, 32, 16384, sp + cap, seed=33)
    mask = torch.zeros(8, sp + cap, dtype=torch.uint8, device=DEV)
    mask[:, :sp + 40] = 1            # 40 text tokens written so far
    kw = {**d.as_kwargs(), "mask_full": mask}
    out, _, _ = rotatek_decode(**kw)
    rows = [0, 3, 7]
    want = odec.rotatek_decode(**_rows(kw, rows))
    check(out[rows], want, torch.float16)
    assert_status_clean()


def test_bounded_wait_timeout_is_reported_and_recoverable():
    """The error path of every bounded wait: a wait on an mbarrier that nothing
    arrives on (no copy in flight) gives up after 1 ms, the kernel returns,
    rtk_read_status reports RTK_DEVICE_TIMEOUT once and clears it, and the
    next decode on the same workspace and context matches the oracle."""
    d = make(torch.bfloat16, 2, 28, 4, 700, 90, seed=123)
    run_and_check(d, torch.bfloat16)                 # the device's workspace exists
    assert_status_clean()
    _lib.selftest_wait_timeout(limit_ns=1_000_000)
    assert _lib.read_status() == _lib.RTK_DEVICE_TIMEOUT
    assert _lib.read_status() == 0                   # read clears it
    run_and_check(d, torch.bfloat16)
    assert_status_clean()
    with pytest.raises(ValueError, match="limit_ns"):
        _lib.selftest_wait_timeout(limit_ns=0)


def test_decode_into_a_caller_buffer():
    """out= writes the result into the caller's tensor -- here the head-major
    send buffer of a head-sharded all_gather, viewed as [B, 1, H_q, D] -- and
    returns it; the values are those of a fresh output."""
    d = make(torch.bfloat16, 3, 28, 4, 900, 70, seed=31)
    kw = d.as_kwargs()
    want = odec.rotatek_decode(**{k: (x.cpu() if torch.is_tensor(x) else x) for k, x in kw.items()})
    send = torch.full((28, 3, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    view = send.permute(1, 0, 2).unsqueeze(1)
    out, _, _ = rotatek_decode(**kw, out=view)
    assert out.data_ptr() == send.data_ptr()
    check(out, want, torch.bfloat16)
    check(send.permute(1, 0, 2).unsqueeze(1), want, torch.bfloat16)
    fresh, _, _ = rotatek_decode(**kw)
    torch.testing.assert_close(out, fresh, rtol=0, atol=0)
    with pytest.raises(ValueError, match="out must be"):
        rotatek_decode(**kw, out=torch.empty(3, 1, 28, 64, dtype=torch.bfloat16, device=DEV))


@pytest.mark.parametrize("reserve", [8, 64])
def test_decode_with_sms_left_free(reserve):
    """With SMs left to a concurrent collective the decode runs on fewer CTAs
    (a different split of the same blocks): same results within the tolerance,
    and the workspace sized for all SMs still serves it."""
    d = make(torch.bfloat16, 4, 28, 4, 3000, 200, seed=37)
    try:
        _lib.set_decode_sm_reserve(reserve)
        run_and_check(d, torch.bfloat16)
        full_channel = d.as_kwargs()
        dense = full_channel_decode(full_channel["q_full"], full_channel["k_full"], full_channel["v_full"], 7)
        check(dense, odec.full_channel_decode(full_channel["q_full"].cpu(), full_channel["k_full"].cpu(),
                                              full_channel["v_full"].cpu(), 7), torch.bfloat16)
    finally:
        _lib.set_decode_sm_reserve(0)
    assert_status_clean()
