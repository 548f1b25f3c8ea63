"""Generate golden fixtures by running the reference's own code on CPU.

Run in a container that holds the reference checkout (it is not needed
afterwards; the fixtures are committed):

    python tests/golden/make_golden.py --reference <path-to-rotatek-checkout>

What runs:
* ``ChannelPruner.update_rotatek`` from
  integrations/lmms_eval/models/model_utils/kv_pruning_utils.py, loaded by file
  path with ROTATEK_SOLVER=eigh (the default power-iteration solver asserts a
  CUDA tensor, rotatek/rotation.py:87), with and without ROTATEK_QUERY_AWARE;
* the `paper` decode kernels ``rotatek_decode_fused_triton`` and
  ``full_channel_decode_triton`` (rotatek/kernels/fused_decode.py,
  full_channel_flash_decoding.py) under TRITON_INTERPRET=1;
* the adapters' prefill Key path (llava_next/llama_visionzip.py:144-153):
  torch's nn.Linear as k_proj and transformers' LlamaRotaryEmbedding /
  apply_rotary_pos_emb, which the adapter imports (llama_visionzip.py:26-33),
  on CPU (kproj_* fixtures);
* ``ChannelPruner.update_spark`` (the SparK baseline, rotatek/baselines/spark.py)
  and the adapters' SparK decode branch: recovery, concatenation and
  ``full_channel_decode_triton`` (spark_* fixtures).

Inputs come from ``rotatek_b200.synthetic`` with fixed seeds.  Each case is one
``.npz`` holding inputs, reference outputs, and scalar metadata.  bf16 tensors
are stored as float32 arrays of their exact bf16 values.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _load_pruner_module(reference: str, solver: str, query_aware: bool, tag: str):
    os.environ["ROTATEK_SOLVER"] = solver
    os.environ["ROTATEK_QUERY_AWARE"] = "1" if query_aware else "0"
    path = os.path.join(reference, "integrations/lmms_eval/models/model_utils/kv_pruning_utils.py")
    spec = importlib.util.spec_from_file_location(f"_ref_kv_pruning_{tag}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _np(t):
    return t.detach().cpu().float().numpy()


def prefill_case(name, mods, torch, synth, *, batch, q_heads, kv_heads, prompt, vision, text,
                 ratio, dtype, seed, query_aware=True, decode=True, paper=None, dense=None,
                 store_inputs=True):
    pre = synth.make_prefill(batch, q_heads, kv_heads, prompt, vision, text, seed=seed, dtype=dtype)
    groups = q_heads // kv_heads
    pruner = mods[query_aware].ChannelPruner(ratio=ratio, prompt_seqlen=prompt, query_seqlen=text)
    kept, kv_prompt, kv_text, keep_mask, values = pruner.update_rotatek(
        pre.keys, pre.queries, pre.values, None, num_key_value_groups=groups)
    R = pruner.current_rotatek_R_partial
    dm = pruner.current_rotatek_delta_mu
    out = dict(
        keys=_np(pre.keys), values=_np(pre.values),
        queries_window=_np(pre.queries[:, :, -min(32, pre.queries.shape[2]):]),
        kept=_np(kept), R_partial=_np(R), delta_mu=_np(dm), keep_mask=keep_mask.numpy(),
        prompt_len=prompt, vision_len=vision, text_len=text, ratio=ratio,
        num_kv_groups=groups, query_aware=int(query_aware),
        dtype=str(dtype).replace("torch.", ""))
    if not store_inputs:  # same seed and shape as another case: keep only the outputs
        for key in ("keys", "values", "queries_window"):
            out.pop(key)
    if decode:
        q_dec = synth.normal((batch, q_heads, pre.keys.shape[-1]), seed + 11, dtype=dtype)
        s_p, s_v = kv_prompt.shape[-2], kept.shape[-2]
        k_full = torch.cat([kv_prompt, kv_text], dim=-2)
        v_full = torch.cat([values[:, :, :s_p], values[:, :, s_p + s_v:]], dim=-2)
        mask = torch.ones(batch, k_full.shape[-2], dtype=torch.uint8)
        o, _, _ = paper(q_full=q_dec, R_partial=R, delta_mu=dm, k_full=k_full, v_full=v_full,
                        mask_full=mask, k_sparse=kept, v_sparse=values[:, :, s_p:s_p + s_v],
                        num_kv_groups=groups)
        od = dense(q_dec, pre.keys, values, num_kv_groups=groups)
        out.update(q_decode=_np(q_dec), out_rotatek=_np(o), out_dense=_np(od))
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"wrote {name}.npz")


def solved_matrix_case(name, mods, torch, synth, *, batch, q_heads, kv_heads, prompt, vision, text,
                       ratio, scale, seed):
    """The exact matrix the reference hands to torch.linalg.eigh (captured by
    wrapping that function around one update_rotatek call), for Keys scaled
    down so far that mean|diag| < 1e-2, where the ridge's clamp is active."""
    pre = synth.make_prefill(batch, q_heads, kv_heads, prompt, vision, text, seed=seed,
                             dtype=torch.float32)
    keys = pre.keys * scale
    pruner = mods[True].ChannelPruner(ratio=ratio, prompt_seqlen=prompt, query_seqlen=text)
    seen = []
    real_eigh = torch.linalg.eigh

    def capture(mat, *a, **k):
        seen.append(mat.detach().clone())
        return real_eigh(mat, *a, **k)

    torch.linalg.eigh = capture
    try:
        pruner.update_rotatek(keys, pre.queries, pre.values, None, num_key_value_groups=q_heads // kv_heads)
    finally:
        torch.linalg.eigh = real_eigh
    solved = seen[0]
    diag_mean = solved.diagonal(dim1=-2, dim2=-1).abs().mean(dim=-1)
    assert float(diag_mean.max()) < 1e-2, diag_mean
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), keys=_np(keys),
                        queries_window=_np(pre.queries[:, :, -min(32, pre.queries.shape[2]):]),
                        solved=_np(solved), prompt_len=prompt, vision_len=vision, text_len=text,
                        num_kv_groups=q_heads // kv_heads, dtype="float32")
    print(f"wrote {name}.npz")


def decode_case(name, torch, synth, paper, *, batch, q_heads, kv_heads, vision, full, keep,
                dtype, seed, with_bias=True, mask_density=1.0):
    d = synth.make_decode(batch, q_heads, kv_heads, vision, full, keep=keep, seed=seed,
                          dtype=dtype, with_bias=with_bias)
    mask = d.mask_full
    if mask_density < 1.0:
        g = torch.Generator().manual_seed(seed + 99)
        mask = (torch.rand(batch, full, generator=g) < mask_density).to(torch.uint8)
    o, _, _ = paper(q_full=d.q_full, R_partial=d.R_partial, delta_mu=d.delta_mu,
                    k_full=d.k_full, v_full=d.v_full, mask_full=mask, k_sparse=d.k_sparse,
                    v_sparse=d.v_sparse, num_kv_groups=d.num_kv_groups)
    out = dict(q_full=_np(d.q_full), R_partial=_np(d.R_partial), k_full=_np(d.k_full),
               v_full=_np(d.v_full), mask_full=mask.numpy(), k_sparse=_np(d.k_sparse),
               v_sparse=_np(d.v_sparse), out_rotatek=_np(o), num_kv_groups=d.num_kv_groups,
               has_bias=int(with_bias), dtype=str(dtype).replace("torch.", ""))
    if with_bias:
        out["delta_mu"] = _np(d.delta_mu)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"wrote {name}.npz")


def dense_case(name, torch, synth, dense, *, batch, q_heads, kv_heads, seq, dtype, seed):
    q = synth.normal((batch, q_heads, 128), seed, dtype=dtype)
    k = synth.lowrank_keys(batch, kv_heads, seq, seed=seed + 1, dtype=dtype)
    v = synth.normal((batch, kv_heads, seq, 128), seed + 2, dtype=dtype)
    o = dense(q, k, v, num_kv_groups=q_heads // kv_heads)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), q=_np(q), k=_np(k), v=_np(v),
                        out_dense=_np(o), num_kv_groups=q_heads // kv_heads,
                        dtype=str(dtype).replace("torch.", ""))
    print(f"wrote {name}.npz")


def spark_case(name, mods, torch, synth, dense, *, batch, q_heads, kv_heads, prompt, vision, text, ratio,
               dtype, seed):
    """SparK: the reference's ``ChannelPruner.update_spark`` on a prefill, then
    the adapters' decode branch for one query token -- recovery (fill every
    channel with the token's pruned_mean, the kept values into the kept
    channels; llama_visionzip.py:226-230, restated here with the same torch
    operations), concatenation [prompt | recovered | text] and the reference's
    ``full_channel_decode_triton`` over the whole cache."""
    pre = synth.make_prefill(batch, q_heads, kv_heads, prompt, vision, text, seed=seed, dtype=dtype)
    groups = q_heads // kv_heads
    pruner = mods[True].ChannelPruner(ratio=ratio, prompt_seqlen=prompt, query_seqlen=text)
    kc, kv_prompt, kv_text, _, values = pruner.update_spark(
        pre.keys, pre.queries, pre.values, None, num_key_value_groups=groups)
    mask = pruner.current_spark_mask
    mean = pruner.current_spark_pruned_mean
    b, h, s_v = kc.shape[:3]
    rec = mean.expand(b, h, s_v, pre.keys.shape[-1]).contiguous()
    rec[mask] = kc.reshape(-1)
    q_dec = synth.normal((batch, q_heads, pre.keys.shape[-1]), seed + 11, dtype=dtype)
    o = dense(q_dec, torch.cat([kv_prompt, rec, kv_text], dim=-2), values, num_kv_groups=groups)
    out = dict(keys=_np(pre.keys), values=_np(values), queries_window=_np(pre.queries[:, :, -32:]), k_compact=_np(kc),
               keep_mask=mask.numpy(), pruned_mean=_np(mean), recovered=_np(rec), q_decode=_np(q_dec),
               out_spark=_np(o), prompt_len=prompt, vision_len=vision, text_len=text, ratio=ratio,
               num_kv_groups=groups, dtype=str(dtype).replace("torch.", ""))
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"wrote {name}.npz")


def kproj_case(name, torch, *, batch, seq, hidden, kv_heads, vis_start, vis_len, dtype, seed, bias=True):
    """The adapters' prefill Key path (llama_visionzip.py:144-153) on CPU: nn.Linear
    k_proj, view / transpose, transformers' LlamaRotaryEmbedding cos / sin and
    apply_rotary_pos_emb.  (The visual span's sums follow from the stored Keys.)"""
    from transformers.models.llama.configuration_llama import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding, apply_rotary_pos_emb
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, seq, hidden, generator=g).to(dtype)
    lin = torch.nn.Linear(hidden, kv_heads * 128, bias=bias)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(kv_heads * 128, hidden, generator=g) * hidden ** -0.5)
        if bias:
            lin.bias.copy_(torch.randn(kv_heads * 128, generator=g) * 0.1)
    lin = lin.to(dtype)
    cfg = LlamaConfig(hidden_size=kv_heads * 128, num_attention_heads=kv_heads, num_key_value_heads=kv_heads,
                      head_dim=128, max_position_embeddings=4096, rope_theta=10000.0)
    rope = LlamaRotaryEmbedding(cfg)
    pos = torch.arange(seq).unsqueeze(0).expand(batch, seq)
    with torch.no_grad():
        cos, sin = rope(x, pos)
        k = lin(x).view(batch, seq, kv_heads, 128).transpose(1, 2)
        _, k = apply_rotary_pos_emb(k, k, cos, sin)
    out = dict(hidden=_np(x), w_k=_np(lin.weight), cos=_np(cos), sin=_np(sin), keys=_np(k),
               vis_start=vis_start, vis_len=vis_len, dtype=str(dtype).replace("torch.", ""))
    if bias:
        out["bias"] = _np(lin.bias)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"wrote {name}.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--only", default=None, help="write only the fixture of this name")
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, args.reference)
    sys.path.insert(0, REPO)
    import torch
    from rotatek_b200 import synthetic as synth
    from rotatek.kernels.fused_decode import rotatek_decode_fused_triton as paper
    from rotatek.kernels.full_channel_flash_decoding import full_channel_decode_triton as dense

    mods = {True: _load_pruner_module(args.reference, "eigh", True, "qa"),
            False: _load_pruner_module(args.reference, "eigh", False, "plain")}

    def want(name):
        return args.only is None or args.only == name
    bf16 = torch.bfloat16
    # benchmark config 1: fp32, B=2, 8/2 heads, 32 + 576 + 64, ratio 0.75
    if want("cfg1_fp32"):
        prefill_case("cfg1_fp32", mods, torch, synth, batch=2, q_heads=8, kv_heads=2, prompt=32,
                     vision=576, text=64, ratio=0.75, dtype=torch.float32, seed=1,
                     paper=paper, dense=dense)
    # the same shape without query weighting (ROTATEK_QUERY_AWARE=0)
    if want("cfg1_fp32_plain"):
        prefill_case("cfg1_fp32_plain", mods, torch, synth, batch=2, q_heads=8, kv_heads=2,
                     prompt=32, vision=576, text=64, ratio=0.75, dtype=torch.float32, seed=1,
                     query_aware=False, decode=False, store_inputs=False)
    # bf16, ragged visual span (not a multiple of 64), GQA group 2
    if want("small_bf16"):
        prefill_case("small_bf16", mods, torch, synth, batch=1, q_heads=4, kv_heads=2, prompt=8,
                     vision=200, text=24, ratio=0.75, dtype=bf16, seed=2, paper=paper, dense=dense)
    # decode edge cases (fp32): partial mask and no delta_mu, G=3, D_keep=16
    if want("dec_mask_nobias_fp32"):
        decode_case("dec_mask_nobias_fp32", torch, synth, paper, batch=2, q_heads=6, kv_heads=2,
                    vision=70, full=45, keep=16, dtype=torch.float32, seed=3, with_bias=False,
                    mask_density=0.6)
    # empty visual span; empty prompt/text span
    if want("dec_empty_visual_fp32"):
        decode_case("dec_empty_visual_fp32", torch, synth, paper, batch=1, q_heads=4, kv_heads=1,
                    vision=0, full=40, keep=32, dtype=torch.float32, seed=4)
    if want("dec_empty_full_fp32"):
        decode_case("dec_empty_full_fp32", torch, synth, paper, batch=1, q_heads=2, kv_heads=2,
                    vision=100, full=0, keep=32, dtype=torch.float32, seed=5)
    # bf16 decode at G=7 (the headline group size) with a mostly-masked text span
    if want("dec_g7_bf16"):
        decode_case("dec_g7_bf16", torch, synth, paper, batch=1, q_heads=7, kv_heads=1, vision=300,
                    full=90, keep=32, dtype=bf16, seed=6, mask_density=0.5)
    # dense decode, MHA (G=1) and G=4
    if want("dense_g1_fp32"):
        dense_case("dense_g1_fp32", torch, synth, dense, batch=1, q_heads=2, kv_heads=2, seq=150,
                   dtype=torch.float32, seed=7)
    if want("dense_g4_bf16"):
        dense_case("dense_g4_bf16", torch, synth, dense, batch=2, q_heads=8, kv_heads=2, seq=333,
                   dtype=bf16, seed=8)

    # the matrix the reference solves, at a scale where the ridge's clamp matters
    if want("tiny_solved_fp32"):
        solved_matrix_case("tiny_solved_fp32", mods, torch, synth, batch=1, q_heads=4, kv_heads=2,
                           prompt=8, vision=300, text=24, ratio=0.75, scale=1e-5, seed=12)

    # SparK baseline: prune (fp32, benchmark config-1 shape) and bf16 with a
    # ragged visual span and D_keep 64
    if want("spark_fp32"):
        spark_case("spark_fp32", mods, torch, synth, dense, batch=2, q_heads=8, kv_heads=2, prompt=32,
                   vision=576, text=64, ratio=0.75, dtype=torch.float32, seed=15)
    if want("spark_bf16"):
        spark_case("spark_bf16", mods, torch, synth, dense, batch=1, q_heads=4, kv_heads=2, prompt=8,
                   vision=200, text=24, ratio=0.5, dtype=bf16, seed=16)

    # prefill Key path: projection with bias + RoPE, ragged spans (20 | 230 | 50)
    if want("kproj_bf16"):
        kproj_case("kproj_bf16", torch, batch=2, seq=300, hidden=256, kv_heads=2, vis_start=20,
                   vis_len=230, dtype=bf16, seed=13)
    if want("kproj_f16_nobias"):
        kproj_case("kproj_f16_nobias", torch, batch=1, seq=200, hidden=192, kv_heads=3, vis_start=0,
                   vis_len=170, dtype=torch.float16, seed=14, bias=False)


if __name__ == "__main__":
    main()
