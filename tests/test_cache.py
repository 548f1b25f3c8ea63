"""SpanKVCache: the preallocated split cache gives rotatek_decode the same token
spans the reference's cache + adapter build with torch.cat
(cache_utils.py:48-55, llama_visionzip.py:203-214), with appends in place."""
import numpy as np
import pytest
import torch

from oracle import decode as odec
from rotatek_b200 import synthetic as syn
from rotatek_b200.cache import SpanKVCache

B, HQ, HKV, SP, SV, ST, D, KEEP = 2, 8, 2, 16, 100, 12, 128, 32


def _prefill(device="cpu", dtype=torch.float32, seed=0):
    g = torch.Generator().manual_seed(seed)
    k_prompt = torch.randn(B, HKV, SP, D, generator=g).to(device, dtype)
    k_text = torch.randn(B, HKV, ST, D, generator=g).to(device, dtype)
    k_rot = torch.randn(B, HKV, SV, KEEP, generator=g).to(device, dtype)
    values = torch.randn(B, HKV, SP + SV + ST, D, generator=g).to(device, dtype)
    R = torch.linalg.qr(torch.randn(B, HKV, D, KEEP, generator=g))[0].to(device, dtype)
    dm = (0.1 * torch.randn(B, HKV, D, generator=g)).to(device, dtype)
    return k_prompt, k_text, k_rot, values, R, dm


def _reference_spans(k_prompt, k_text, values, s_vision):
    s_p = k_prompt.shape[2]
    return (torch.cat([k_prompt, k_text], dim=-2),
            torch.cat([values[:, :, :s_p], values[:, :, s_p + s_vision:]], dim=-2),
            values[:, :, s_p:s_p + s_vision])


def test_views_match_reference_spans_across_appends():
    k_prompt, k_text, k_rot, values, R, dm = _prefill()
    cache = SpanKVCache(max_new_tokens=5)
    cache.store_pruned(k_rot, k_prompt, k_text, values, R, dm, 0)
    g = torch.Generator().manual_seed(1)
    for step in range(5):
        kn, vn = torch.randn(B, HKV, 1, D, generator=g), torch.randn(B, HKV, 1, D, generator=g)
        cache.update(kn, vn, 0)
        k_text = torch.cat([k_text, kn], dim=-2)        # the reference cache's append
        values = torch.cat([values, vn], dim=-2)
        a = cache.decode_args(0)
        kf, vf, vs = _reference_spans(k_prompt, k_text, values, SV)
        assert torch.equal(a["k_full"], kf) and torch.equal(a["v_full"], vf) and torch.equal(a["v_sparse"], vs)
        assert torch.equal(a["k_sparse"], k_rot) and a["mask_full"] is None
        assert cache.get_seq_length(0) == SP + SV + ST + step + 1
    with pytest.raises(ValueError):
        cache.update(kn, vn, 0)


def test_decode_through_cache_matches_oracle():
    k_prompt, k_text, k_rot, values, R, dm = _prefill(seed=3)
    cache = SpanKVCache(max_new_tokens=2)
    cache.store_pruned(k_rot, k_prompt, k_text, values, R, dm, 0)
    kn, vn = torch.randn(B, HKV, 2, D), torch.randn(B, HKV, 2, D)
    cache.update(kn, vn, 0)
    q = torch.randn(B, HQ, D)
    got = odec.rotatek_decode(q_full=q, num_kv_groups=HQ // HKV, **cache.decode_args(0))
    kf, vf, vs = _reference_spans(k_prompt, torch.cat([k_text, kn], -2), torch.cat([values, vn], -2), SV)
    want = odec.rotatek_decode(q, R, dm, kf, vf, torch.ones(B, kf.shape[2], dtype=torch.uint8), k_rot, vs,
                               HQ // HKV)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-12)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gpu_decode_through_cache_is_bit_identical(dtype):
    from rotatek_b200.kernels import rotatek_decode
    k_prompt, k_text, k_rot, values, R, dm = _prefill("cuda", dtype, seed=4)
    cache = SpanKVCache(max_new_tokens=3)
    cache.store_pruned(k_rot, k_prompt, k_text, values, R, dm, 0)
    q = torch.randn(B, HQ, D, device="cuda").to(dtype)
    for _ in range(3):
        kn = torch.randn(B, HKV, 1, D, device="cuda").to(dtype)
        vn = torch.randn(B, HKV, 1, D, device="cuda").to(dtype)
        cache.update(kn, vn, 0)
        k_text = torch.cat([k_text, kn], dim=-2)
        values = torch.cat([values, vn], dim=-2)
        got, _, _ = rotatek_decode(q_full=q, num_kv_groups=HQ // HKV, **cache.decode_args(0))
        kf, vf, vs = _reference_spans(k_prompt, k_text, values, SV)
        want, _, _ = rotatek_decode(q_full=q, R_partial=R, delta_mu=dm, k_full=kf, v_full=vf,
                                    mask_full=torch.ones(B, kf.shape[2], dtype=torch.uint8, device="cuda"),
                                    k_sparse=k_rot, v_sparse=vs, num_kv_groups=HQ // HKV)
        assert torch.equal(got, want)


def test_capacity_slots_zeroed_at_store():
    """Text slots past the stored tokens hold zeros, whatever the allocator
    handed out: the full-capacity decode views read them (masked logits, but
    their Values still enter P.V with weight 0, and 0 * NaN is NaN)."""
    k_prompt, k_text, k_rot, values, R, dm = _prefill()
    cache = SpanKVCache(max_new_tokens=7)
    empty = torch.empty
    torch.empty = lambda *a, **k: empty(*a, **k).fill_(float("nan"))  # uninitialised = NaN
    try:
        cache.store_pruned(k_rot, k_prompt, k_text, values, R, dm, 0)
    finally:
        torch.empty = empty
    L = cache.layers[0]
    cap = L.s_prompt + L.t_max
    assert not torch.isnan(L.keys_full).any() and not torch.isnan(L.values).any()
    assert torch.count_nonzero(L.keys_full[:, :, SP + ST:cap]) == 0
    assert torch.count_nonzero(L.values[:, :, SP + ST:cap]) == 0
    args = cache.static_decode_args(0, cache.capacity_mask(0))
    assert args["k_full"].shape[2] == cap and args["mask_full"].shape == (B, cap)


def test_step_budget_raises_past_capacity():
    """The e2e decoder's host-side step count: the (max_new_tokens + 1)-th step
    raises before it would write past the cache's text capacity."""
    from rotatek_b200.llama_e2e import StepBudget
    budget = StepBudget(3)
    for _ in range(3):
        budget.take()
    with pytest.raises(RuntimeError, match="exceeds max_new_tokens=3"):
        budget.take()
    assert budget.used == 3
