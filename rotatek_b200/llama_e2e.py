"""A random-init LLaVA-NeXT-7B-shaped decoder (Vicuna-style Llama) that runs the
RotateK path end to end: prefill with the per-layer rotation build, then
greedy decode through the fused decode kernel.

It stands in for the reference's LLaVA-NeXT attention adapter
(integrations/lmms_eval/models/model_utils/llava_next/llama_visionzip.py): at
prefill each layer's post-RoPE Keys go through ``ChannelPruner.update_rotatek``
(here ``rotation.build_rotation``, kv_pruning_utils.py:92-160) into the
span-split cache, and every decode step calls ``rotatek_decode`` on the
rotated-truncated visual Keys plus the full-width prompt/text Keys
(llama_visionzip.py:197-215).  The vision tower is bypassed: the visual span is
synthetic embeddings.  Weights are random (there is no checkpoint); the shapes
are the model's, so every byte and FLOP of the real model is moved and done.

Prefill computes each layer's Keys with ``build_rotation_projected`` (K
projection and RoPE in one tensor-core kernel, then the visual span's
covariance sums and the rest of the build), Queries and Values with cuBLAS; set
``fused_key_projection=False`` for the adapters' order (fused QKV GEMM, torch
RoPE, ``build_rotation`` on the visual slice).

Decode steps are static-shape -- the append slot, the RoPE position and the
text-span mask live on the device -- so a whole step (32 layers) is one CUDA
graph replay.  Linear layers are cuBLAS GEMMs (torch), prefill attention is
torch's scaled_dot_product_attention; the RotateK build, cache and decode are
this package's kernels.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from rotatek_b200.cache import SpanKVCache
from rotatek_b200.kernels import rotatek_decode
from rotatek_b200.rotation import QUERY_WINDOW, build_rotation, build_rotation_projected, keep_count


@dataclass
class DecoderConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 32
    head_dim: int = 128
    ffn: int = 11008
    vocab: int = 32000
    rope_theta: float = 10000.0
    eps: float = 1e-6
    prompt: int = 32           # tokens before the image
    vision: int = 16384        # visual-span tokens (synthetic embeddings)
    text: int = 32             # question tokens after the image
    channel_ratio: float = 0.75
    max_new_tokens: int = 128
    dtype: torch.dtype = torch.float16
    fused_key_projection: bool = True   # prefill K through key projection + build in one call


class RandomLlamaDecoder:
    def __init__(self, cfg: DecoderConfig, device, seed: int = 0):
        self.cfg = c = cfg
        self.device = torch.device(device)
        g = torch.Generator(device=self.device).manual_seed(seed)

        def w(*shape, scale=0.02):
            return (torch.randn(*shape, generator=g, device=self.device, dtype=torch.float32) * scale).to(c.dtype)

        qkv_out = (c.heads + 2 * c.kv_heads) * c.head_dim
        self.embed = w(c.vocab, c.hidden, scale=1.0)
        self.layers = []
        for _ in range(c.layers):
            self.layers.append(dict(
                ln1=torch.ones(c.hidden, device=self.device, dtype=c.dtype),
                wqkv=w(qkv_out, c.hidden), wo=w(c.hidden, c.heads * c.head_dim),
                ln2=torch.ones(c.hidden, device=self.device, dtype=c.dtype),
                wgu=w(2 * c.ffn, c.hidden), wdown=w(c.hidden, c.ffn)))
        self.norm = torch.ones(c.hidden, device=self.device, dtype=c.dtype)
        self.lm_head = w(c.vocab, c.hidden)
        max_pos = c.prompt + c.vision + c.text + c.max_new_tokens
        inv = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, device=self.device,
                                                     dtype=torch.float32) / c.head_dim))
        ang = torch.arange(max_pos, device=self.device, dtype=torch.float32)[:, None] * inv[None, :]
        ang = torch.cat([ang, ang], dim=-1)
        self.cos, self.sin = ang.cos().to(c.dtype), ang.sin().to(c.dtype)
        self.keep = keep_count(c.head_dim, c.channel_ratio)
        self.cache = None

    # ------------------------------------------------------------------ pieces
    def _rms(self, x, weight):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.eps)).to(x.dtype) * weight

    @staticmethod
    def _rot_half(x):
        h = x.shape[-1] // 2
        return torch.cat([-x[..., h:], x[..., :h]], dim=-1)

    def _rope(self, x, cos, sin):           # x [B, H, S, D], cos/sin [S, D]
        return x * cos + self._rot_half(x) * sin

    def _mlp(self, L, x):
        gu = F.linear(self._rms(x, L["ln2"]), L["wgu"])
        gate, up = gu.chunk(2, dim=-1)
        return F.linear(F.silu(gate) * up, L["wdown"])

    def _qkv(self, L, x):
        c = self.cfg
        b, s, _ = x.shape
        qkv = F.linear(self._rms(x, L["ln1"]), L["wqkv"]).view(b, s, c.heads + 2 * c.kv_heads, c.head_dim)
        q = qkv[:, :, :c.heads].transpose(1, 2)
        k = qkv[:, :, c.heads:c.heads + c.kv_heads].transpose(1, 2)
        v = qkv[:, :, c.heads + c.kv_heads:].transpose(1, 2)
        return q, k, v

    # ------------------------------------------------------------------ prefill
    def prompt_embeddings(self, batch: int, seed: int = 1):
        """[B, S_p + S_v + S_t, hidden]: prompt and question tokens embedded, the
        visual span synthetic (the vision tower is bypassed)."""
        c = self.cfg
        g = torch.Generator(device=self.device).manual_seed(seed)
        toks = torch.randint(0, c.vocab, (batch, c.prompt + c.text), generator=g, device=self.device)
        emb = self.embed[toks]
        vis = torch.randn(batch, c.vision, c.hidden, generator=g, device=self.device, dtype=torch.float32)
        vis = vis.to(c.dtype)
        return torch.cat([emb[:, :c.prompt], vis, emb[:, c.prompt:]], dim=1)

    @torch.no_grad()
    def prefill(self, x: torch.Tensor) -> torch.Tensor:
        """Run the prompt, build every layer's rotation into a fresh cache; returns
        the last position's logits [B, vocab]."""
        c = self.cfg
        s_total = x.shape[1]
        s_p, s_v = c.prompt, c.vision
        cos, sin = self.cos[:s_total], self.sin[:s_total]
        self.cache = SpanKVCache(max_new_tokens=c.max_new_tokens)
        groups = c.heads // c.kv_heads
        b = x.shape[0]
        hq, hk = c.heads * c.head_dim, c.kv_heads * c.head_dim
        for li, L in enumerate(self.layers):
            if c.fused_key_projection:
                # K = RoPE(x W_k^T) for every token from one tensor-core kernel,
                # then the visual span's sums and the rest of the build on those Keys
                xn = self._rms(x, L["ln1"])
                q = F.linear(xn, L["wqkv"][:hq]).view(b, s_total, c.heads, c.head_dim).transpose(1, 2)
                v = F.linear(xn, L["wqkv"][hq + hk:]).view(b, s_total, c.kv_heads, c.head_dim)
                v = v.transpose(1, 2).contiguous()
                q = self._rope(q, cos, sin)
                k, kept, R, dm, _ = build_rotation_projected(xn, L["wqkv"][hq:hq + hk], None, cos, sin, s_p, s_v,
                                                             q[:, :, -QUERY_WINDOW:], self.keep, groups)
                del xn
            else:
                q, k, v = self._qkv(L, x)
                q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
                k = k.contiguous()
                v = v.contiguous()
                # RotateK build of this layer (ChannelPruner.update_rotatek's body)
                kept, R, dm, _ = build_rotation(k[:, :, s_p:s_p + s_v], q[:, :, -QUERY_WINDOW:], self.keep, groups)
            a = F.scaled_dot_product_attention(q, k.repeat_interleave(groups, 1) if groups > 1 else k,
                                               v.repeat_interleave(groups, 1) if groups > 1 else v, is_causal=True)
            x = x + F.linear(a.transpose(1, 2).reshape(b, s_total, -1), L["wo"])
            x = x + self._mlp(L, x)
            self.cache.store_pruned(kept, k[:, :, :s_p], k[:, :, s_p + s_v:], v, R, dm, li)
            del q, k, v, a
        self.seq_len = s_total
        return F.linear(self._rms(x[:, -1:], self.norm), self.lm_head)[:, 0]

    # ------------------------------------------------------------------ decode
    def init_decode(self, first_token: torch.Tensor):
        """Static decode state after prefill: token [B], RoPE position, cache slot
        and the text-span mask, all on the device.  The cache has room for
        ``max_new_tokens`` appends; ``steps`` counts the steps run on the host."""
        c = self.cfg
        self.token = first_token.view(-1).clone()
        self.pos = torch.tensor([self.seq_len], device=self.device, dtype=torch.long)
        self.slot = torch.tensor([c.prompt + c.text], device=self.device, dtype=torch.long)
        self._slot_last = c.prompt + c.text + c.max_new_tokens - 1
        self.mask = self.cache.capacity_mask(0)
        self.steps = StepBudget(c.max_new_tokens)

    def capture_decode_graph(self) -> "DecodeGraph":
        """``decode_step`` captured in a CUDA graph; each ``replay`` is one step and
        counts against the cache's room like an eager step."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            logits = self.decode_step()
        return DecodeGraph(g, logits, self.steps)

    @torch.no_grad()
    def decode_step(self) -> torch.Tensor:
        """One greedy step for the whole batch: consumes self.token, writes the
        next token into it, advances the device position / slot / mask.
        Static shapes only (CUDA-graph capturable).  Returns the logits."""
        c = self.cfg
        if not torch.cuda.is_current_stream_capturing():
            self.steps.take()          # a captured step is counted at each replay
        b = self.token.shape[0]
        x = self.embed[self.token].view(b, 1, c.hidden)
        cos, sin = self.cos.index_select(0, self.pos), self.sin.index_select(0, self.pos)
        # the host count above keeps the slot in range; the clamp keeps a replay
        # that bypassed it from indexing past the text capacity into the Values'
        # visual span (or out of the tensor)
        slot = self.slot.clamp_max(self._slot_last)
        self.mask.index_fill_(1, slot, 1)
        groups = c.heads // c.kv_heads
        for li, L in enumerate(self.layers):
            q, k, v = self._qkv(L, x)
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            self.cache.write_at(k, v, li, slot)
            o, _, _ = rotatek_decode(q_full=q[:, :, 0], num_kv_groups=groups,
                                     **self.cache.static_decode_args(li, self.mask))
            x = x + F.linear(o.view(b, 1, -1), L["wo"])
            x = x + self._mlp(L, x)
        logits = F.linear(self._rms(x, self.norm), self.lm_head)[:, 0]
        self.token.copy_(logits.argmax(-1))
        self.pos.add_(1)
        self.slot.add_(1)
        return logits

    def attention_bytes_per_step(self) -> int:
        """Algorithmic bytes the decode attention moves per step (all layers)."""
        c = self.cfg
        b = self.token.shape[0]
        e = torch.finfo(c.dtype).bits // 8
        cap = c.prompt + c.text + c.max_new_tokens
        per_layer = b * c.kv_heads * (c.vision * (self.keep + c.head_dim) + 2 * cap * c.head_dim) * e
        per_layer += b * c.heads * c.head_dim * e * 2 + b * c.kv_heads * c.head_dim * (self.keep + 1) * e
        return per_layer * c.layers


class StepBudget:
    """Host-side count of the decode steps a cache has room for: ``take`` raises
    once ``limit`` steps have run, before the step writes past the text span."""

    def __init__(self, limit: int):
        self.limit = limit
        self.used = 0

    def take(self) -> None:
        if self.used >= self.limit:
            raise RuntimeError(f"decode step {self.used + 1} exceeds max_new_tokens={self.limit}: "
                               "the cache has no room for another token")
        self.used += 1


class DecodeGraph:
    """A captured decode step.  ``replay`` checks the step budget first."""

    def __init__(self, graph: "torch.cuda.CUDAGraph", logits: torch.Tensor, steps: StepBudget):
        self.graph, self.logits, self.steps = graph, logits, steps

    def replay(self) -> torch.Tensor:
        self.steps.take()
        self.graph.replay()
        return self.logits


__all__ = ["DecoderConfig", "RandomLlamaDecoder", "StepBudget", "DecodeGraph"]
