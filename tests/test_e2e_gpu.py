"""End-to-end decode on a small random-init Llama (the LLaVA-NeXT decoder shape
scaled down): prefill with the per-layer RotateK build, greedy decode through
the fused kernel, CUDA-graph replay identical to eager steps, and one layer's
decode attention against the float64 oracle on the cache it built."""
import numpy as np
import pytest
import torch

from oracle import decode as odec
from rotatek_b200.llama_e2e import DecoderConfig, RandomLlamaDecoder

pytestmark = pytest.mark.gpu
CFG = DecoderConfig(layers=2, hidden=256, heads=2, kv_heads=2, head_dim=128, ffn=512, vocab=1000,
                    prompt=16, vision=256, text=8, max_new_tokens=4)


def _model(batch=2):
    m = RandomLlamaDecoder(CFG, "cuda", seed=0)
    logits = m.prefill(m.prompt_embeddings(batch, seed=1))
    m.init_decode(logits.argmax(-1))
    return m


def test_graph_replay_matches_eager():
    m = _model()
    eager = [m.decode_step().clone() for _ in range(3)]
    toks_eager = m.token.clone()
    m = _model()
    first = m.decode_step().clone()              # warm-up: workspaces, cuBLAS handles
    g = m.capture_decode_graph()
    got = [first]
    for _ in range(2):
        got.append(g.replay().clone())
    torch.cuda.synchronize()
    for a, b in zip(eager, got):
        assert torch.equal(a, b)
    assert torch.equal(toks_eager, m.token)
    # the cache holds max_new_tokens = 4 appends: one more replay, then no more
    g.replay()
    with pytest.raises(RuntimeError, match="exceeds max_new_tokens"):
        g.replay()
    with pytest.raises(RuntimeError, match="exceeds max_new_tokens"):
        m.decode_step()
    torch.cuda.synchronize()
    assert int(m.slot) == CFG.prompt + CFG.text + CFG.max_new_tokens
    del g


def test_unwritten_text_slots_cannot_poison_the_output(monkeypatch):
    """The full-capacity decode views cover text slots not written yet; they
    are masked out of the logits, and the cache zeroes them so that the P.V
    product never multiplies a leftover NaN by its zero weight.  NaN put into
    the memory the cache is about to take must not reach the output."""
    from rotatek_b200.cache import SpanKVCache
    from rotatek_b200.kernels import rotatek_decode
    # every tensor the cache takes uninitialised starts as NaN here
    store, empty = SpanKVCache.store_pruned, torch.empty

    def nan_empty(*a, **k):
        return empty(*a, **k).fill_(float("nan"))

    def poisoned_store(self, *a, **k):
        torch.empty = nan_empty
        try:
            return store(self, *a, **k)
        finally:
            torch.empty = empty

    monkeypatch.setattr(SpanKVCache, "store_pruned", poisoned_store)
    m = RandomLlamaDecoder(CFG, "cuda", seed=0)
    logits = m.prefill(m.prompt_embeddings(2, seed=1))
    m.init_decode(logits.argmax(-1))
    L = m.cache.layers[0]
    cap = L.s_prompt + L.t_max
    assert torch.count_nonzero(L.keys_full[:, :, L.s_prompt + L.s_text:cap]) == 0
    assert torch.count_nonzero(L.values[:, :, L.s_prompt + L.s_text:cap]) == 0
    q = torch.randn(2, CFG.heads, CFG.head_dim, device="cuda", dtype=CFG.dtype)
    args = m.cache.static_decode_args(0, m.mask)
    out, _, _ = rotatek_decode(q_full=q, num_kv_groups=1, **args)
    assert torch.isfinite(out).all()
    want = odec.rotatek_decode(q_full=q, num_kv_groups=1, **args)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=0,
                               atol=1e-3 + 2.0 ** -10 * np.abs(want).max())


def test_layer_attention_matches_oracle():
    m = _model(batch=2)
    m.decode_step()                              # one token in the text span
    # layer 0 of the next step, recomputed from the model's own pieces
    c = m.cfg
    x = m.embed[m.token].view(2, 1, c.hidden)
    cos, sin = m.cos.index_select(0, m.pos), m.sin.index_select(0, m.pos)
    L = m.layers[0]
    q, k, v = m._qkv(L, x)
    q, k = m._rope(q, cos, sin), m._rope(k, cos, sin)
    m.mask.index_fill_(1, m.slot, 1)
    m.cache.write_at(k, v, 0, m.slot)
    args = m.cache.static_decode_args(0, m.mask)
    from rotatek_b200.kernels import rotatek_decode
    out, _, _ = rotatek_decode(q_full=q[:, :, 0], num_kv_groups=1, **args)
    want = odec.rotatek_decode(q_full=q[:, :, 0], num_kv_groups=1, **args)
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-3 + 2.0 ** -10 * np.abs(want).max())
    assert int(m.mask.sum()) == 2 * (c.prompt + c.text + 2)


def test_fused_key_projection_prefill_matches_adapter_order():
    """Prefill through build_rotation_projected (fused K projection + RoPE +
    covariance sums) against the adapters' order (QKV GEMM, torch RoPE,
    build_rotation): layer 0 stores the same Keys up to the projection's
    accumulation order and spans the same subspace."""
    from dataclasses import replace
    from oracle import projection as oproj
    outs = []
    for fused in (True, False):
        m = RandomLlamaDecoder(replace(CFG, fused_key_projection=fused), "cuda", seed=0)
        logits = m.prefill(m.prompt_embeddings(2, seed=1))
        outs.append((m.cache.layers[0], logits.float()))
    (a, la), (b, lb) = outs
    n = a.s_prompt + a.s_text                     # prompt | text stored so far
    frac, worst = oproj.key_mismatch(a.keys_full[:, :, :n].float().cpu().numpy(),
                                     b.keys_full[:, :, :n].float().cpu().numpy(), "float16")
    assert frac <= 5e-3 and worst <= 4.0, (frac, worst)
    rel = torch.linalg.vector_norm((a.keys_rot - b.keys_rot).float()) / torch.linalg.vector_norm(b.keys_rot.float())
    assert float(rel) < 1e-2
    Ra, Rb = a.rotation.double(), b.rotation.double()
    dist = torch.linalg.matrix_norm(Ra @ Ra.transpose(-1, -2) - Rb @ Rb.transpose(-1, -2))
    assert float(dist.max()) < 1e-2
    assert float((la - lb).abs().max()) <= 2e-2 * float(lb.abs().max())
