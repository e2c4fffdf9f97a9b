"""gpt-oss causal LM for packed-sequence training and prefill, built on this package's ops.

Parameters keep the checkpoint layout:
  * attention q/k/v are stored fused as one [Hq*D + 2*Hkv*D, H] bf16 weight (one GEMM);
  * experts keep the MXFP4 bytes (uint8 blocks [E, N, K/32, 16] and scales [E, N, K/32]) as
    buffers, never as trainable parameters, so no bf16 container trick is needed to shard
    them (the reference packs them into bf16 Parameters for FSDP2 and patches torch's foreach
    copy to protect the NaN bit patterns, models/gpt_oss/fsdp2_fix.py:14-30);
  * LoRA factors are fp32 masters in PEFT shapes (A [r, in], B [out, r]; experts
    A [E, r, in], B [E, out, r]).

Routing replay (R3): ``forward_hidden(..., routing_indices=[T, L, K])`` makes layer l use the
recorded expert ids instead of its own top-k (reference: models/gpt_oss/routing_replay.py:31-137,
quantization.py:593-636).  Activation checkpointing is per decoder layer (non-reentrant).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.utils.checkpoint as ckpt

from ...ops import mxfp4
from ...ops.attention import AttentionOutputCache, AttentionPlan, attention
from ...ops.linear import block_diag_b, lora_linear
from ...ops.logprob import linear_logprob_entropy
from ...ops.moe_layer import ExpertWeights, moe_forward
from ...ops.norm import rmsnorm
from ...ops.rope import apply_rope_, rope_tables
from .config import GptOssConfig, LoraConfig


class _RopeFn(torch.autograd.Function):
    """Out-of-place RoPE on the q and k heads of a fused qkv tensor; backward rotates back."""

    @staticmethod
    def forward(ctx, qkv, n_rot, d, pos, cos, sin):
        out = qkv.clone()
        apply_rope_(out, n_rot, d, pos, cos, sin)
        ctx.save_for_backward(pos, cos, sin)
        ctx.cfg = (n_rot, d)
        return out

    @staticmethod
    def backward(ctx, g):
        pos, cos, sin = ctx.saved_tensors
        n_rot, d = ctx.cfg
        g = g.clone()
        apply_rope_(g, n_rot, d, pos, cos, sin, inverse=True)
        return g, None, None, None, None, None


class GptOssAttention(nn.Module):
    def __init__(self, cfg: GptOssConfig, layer: int, lora: LoraConfig | None, device, dtype):
        super().__init__()
        self.cfg = cfg
        self.layer = layer
        self.window = cfg.window(layer)
        self.layer_idx = layer
        H, D = cfg.hidden_size, cfg.head_dim
        self.qkv_weight = nn.Parameter(torch.empty(cfg.qkv_size, H, device=device, dtype=dtype),
                                       requires_grad=False)
        self.qkv_bias = nn.Parameter(torch.zeros(cfg.qkv_size, device=device, dtype=torch.float32),
                                     requires_grad=False)
        self.o_weight = nn.Parameter(torch.empty(H, cfg.q_size, device=device, dtype=dtype),
                                     requires_grad=False)
        self.o_bias = nn.Parameter(torch.zeros(H, device=device, dtype=torch.float32),
                                   requires_grad=False)
        self.sinks = nn.Parameter(torch.zeros(cfg.num_attention_heads, device=device,
                                              dtype=torch.float32), requires_grad=False)
        self.lora = nn.ParameterDict()
        self.lora_scaling = lora.scaling if lora else 1.0
        if lora:
            r = lora.r
            outs = {"q_proj": cfg.q_size, "k_proj": cfg.kv_size, "v_proj": cfg.kv_size}
            for name, out in outs.items():
                if lora.targets(name):
                    self.lora[f"{name}_A"] = nn.Parameter(torch.empty(r, H, device=device))
                    self.lora[f"{name}_B"] = nn.Parameter(torch.zeros(out, r, device=device))
            if lora.targets("o_proj"):
                self.lora["o_proj_A"] = nn.Parameter(torch.empty(r, cfg.q_size, device=device))
                self.lora["o_proj_B"] = nn.Parameter(torch.zeros(H, r, device=device))

    def _qkv_lora(self):
        """Stacked A [sum r, H] and block-diagonal B [qkv, sum r] over the q/k/v branches."""
        if not any(k.endswith("_A") and not k.startswith("o_") for k in self.lora.keys()):
            return None, None
        cfg = self.cfg
        As, Bs = [], []
        sizes = {"q_proj": cfg.q_size, "k_proj": cfg.kv_size, "v_proj": cfg.kv_size}
        r = next(p for k, p in self.lora.items() if k.endswith("_A")).shape[0]
        for name, out in sizes.items():
            if f"{name}_A" in self.lora:
                As.append(self.lora[f"{name}_A"])
                Bs.append(self.lora[f"{name}_B"])
            else:  # untargeted branch: zero block keeps the layout fixed
                As.append(torch.zeros(r, cfg.hidden_size, device=self.qkv_weight.device))
                Bs.append(torch.zeros(out, r, device=self.qkv_weight.device))
        return torch.cat(As, 0), block_diag_b(Bs)

    def forward(self, xn, residual, pos, cos, sin, cu_seqlens, plan):
        cfg = self.cfg
        A, B = self._qkv_lora()
        qkv = lora_linear(xn, self.qkv_weight, self.qkv_bias, A, B, None, self.lora_scaling)
        qkv = _RopeFn.apply(qkv, cfg.num_attention_heads + cfg.num_key_value_heads,
                            cfg.head_dim, pos, cos, sin)
        # full-attention layers may hand their output to the checkpoint recompute
        o = attention(qkv, self.sinks, cu_seqlens, cfg.num_attention_heads,
                      cfg.num_key_value_heads, cfg.head_dim, self.window, None, plan,
                      cache_key=self.layer_idx if self.window == 0 else None)
        oA = self.lora["o_proj_A"] if "o_proj_A" in self.lora else None
        oB = self.lora["o_proj_B"] if "o_proj_B" in self.lora else None
        return lora_linear(o, self.o_weight, self.o_bias, oA, oB, residual, self.lora_scaling)


class GptOssMoE(nn.Module):
    def __init__(self, cfg: GptOssConfig, lora: LoraConfig | None, device, dtype):
        super().__init__()
        self.cfg = cfg
        E, H, I = cfg.num_local_experts, cfg.hidden_size, cfg.intermediate_size
        self.router_weight = nn.Parameter(torch.empty(E, H, device=device, dtype=dtype),
                                          requires_grad=False)
        self.router_bias = nn.Parameter(torch.zeros(E, device=device, dtype=torch.float32),
                                        requires_grad=False)
        u8 = torch.uint8
        self.register_buffer("gate_up_blocks", torch.zeros(E, 2 * I, H // 32, 16, dtype=u8, device=device))
        self.register_buffer("gate_up_scales", torch.full((E, 2 * I, H // 32), 127, dtype=u8, device=device))
        self.register_buffer("down_blocks", torch.zeros(E, H, I // 32, 16, dtype=u8, device=device))
        self.register_buffer("down_scales", torch.full((E, H, I // 32), 127, dtype=u8, device=device))
        self.gate_up_bias = nn.Parameter(torch.zeros(E, 2 * I, device=device), requires_grad=False)
        self.down_bias = nn.Parameter(torch.zeros(E, H, device=device), requires_grad=False)
        self.lora = nn.ParameterDict()
        self.lora_scaling = lora.scaling if lora else 1.0
        if lora:
            r = lora.r
            if lora.targets("gate_up_proj"):
                self.lora["gu_A"] = nn.Parameter(torch.empty(E, r, H, device=device))
                self.lora["gu_B"] = nn.Parameter(torch.zeros(E, 2 * I, r, device=device))
            if lora.targets("down_proj"):
                self.lora["dn_A"] = nn.Parameter(torch.empty(E, r, I, device=device))
                self.lora["dn_B"] = nn.Parameter(torch.zeros(E, H, r, device=device))

    def experts(self) -> ExpertWeights:
        return ExpertWeights(self.gate_up_blocks, self.gate_up_scales, self.gate_up_bias,
                             self.down_blocks, self.down_scales, self.down_bias,
                             shards=getattr(self, "expert_shards", None),
                             dequant_dtype=getattr(self, "dequant_dtype", "bf16"))

    def forward(self, xn, residual, replay_ids=None, routing_out=None):
        cfg = self.cfg
        return moe_forward(xn, residual, self.router_weight, self.router_bias, self.experts(),
                           cfg.num_experts_per_tok, dict(self.lora.items()), self.lora_scaling,
                           replay_ids, cfg.swiglu_alpha, cfg.swiglu_limit, routing_out)


class GptOssDecoderLayer(nn.Module):
    def __init__(self, cfg: GptOssConfig, layer: int, lora, device, dtype):
        super().__init__()
        self.cfg = cfg
        self.layer = layer
        self.input_layernorm = nn.Parameter(torch.ones(cfg.hidden_size, device=device),
                                            requires_grad=False)
        self.post_attention_layernorm = nn.Parameter(torch.ones(cfg.hidden_size, device=device),
                                                     requires_grad=False)
        self.self_attn = GptOssAttention(cfg, layer, lora, device, dtype)
        self.mlp = GptOssMoE(cfg, lora, device, dtype)

    def forward(self, x, pos, cos, sin, cu_seqlens, plan, replay_ids=None, routing_out=None):
        eps = self.cfg.rms_norm_eps
        xn = rmsnorm(x, self.input_layernorm, eps)
        h = self.self_attn(xn, x, pos, cos, sin, cu_seqlens, plan)
        hn = rmsnorm(h, self.post_attention_layernorm, eps)
        return self.mlp(hn, h, replay_ids, routing_out)


class GptOssForCausalLM(nn.Module):
    def __init__(self, cfg: GptOssConfig, lora: LoraConfig | None = None, device="cpu",
                 dtype=torch.bfloat16):
        super().__init__()
        self.cfg = cfg
        self.lora_config = lora
        self.embed_tokens = nn.Parameter(torch.empty(cfg.vocab_size, cfg.hidden_size, device=device,
                                                     dtype=dtype), requires_grad=False)
        self.layers = nn.ModuleList(GptOssDecoderLayer(cfg, i, lora, device, dtype)
                                    for i in range(cfg.num_hidden_layers))
        self.norm = nn.Parameter(torch.ones(cfg.hidden_size, device=device), requires_grad=False)
        self.lm_head = nn.Parameter(torch.empty(cfg.vocab_size, cfg.hidden_size, device=device,
                                                dtype=dtype), requires_grad=False)
        self.gradient_checkpointing = True
        # bytes of full-attention outputs kept for the checkpoint recompute (0 = recompute all)
        self.attention_cache_bytes = 0
        self._rope_cache = None

    # ------------------------------------------------------------------ init / params
    @torch.no_grad()
    def init_random(self, seed: int = 0, std: float | None = None,
                    keep_embeddings: bool = False) -> "GptOssForCausalLM":
        """Random-init weights (normal(0, std)), experts quantized to MXFP4; LoRA A random
        (Kaiming-uniform like PEFT), LoRA B zero.  ``keep_embeddings`` leaves the embedding
        and LM head untouched (a draft model sharing the target's)."""
        cfg = self.cfg
        std = cfg.initializer_range if std is None else std
        dev = self.embed_tokens.device
        # generate where the weights live: a 120b init on the GPU takes seconds
        g = torch.Generator(device=dev).manual_seed(seed)

        def randn(*shape):
            return torch.randn(*shape, generator=g, device=dev) * std

        if not keep_embeddings:
            self.embed_tokens.copy_(randn(*self.embed_tokens.shape).to(dev))
            self.lm_head.copy_(randn(*self.lm_head.shape).to(dev))
        for layer in self.layers:
            a, m = layer.self_attn, layer.mlp
            a.qkv_weight.copy_(randn(*a.qkv_weight.shape).to(dev))
            a.o_weight.copy_(randn(*a.o_weight.shape).to(dev))
            a.sinks.copy_(randn(*a.sinks.shape).to(dev))
            m.router_weight.copy_(randn(*m.router_weight.shape).to(dev))
            m.router_bias.copy_(randn(*m.router_bias.shape).to(dev))
            for e in range(cfg.num_local_experts):
                gu = randn(2 * cfg.intermediate_size, cfg.hidden_size)
                b, s = mxfp4.quantize(gu)
                m.gate_up_blocks[e].copy_(b.to(dev))
                m.gate_up_scales[e].copy_(s.to(dev))
                dn = randn(cfg.hidden_size, cfg.intermediate_size)
                b, s = mxfp4.quantize(dn)
                m.down_blocks[e].copy_(b.to(dev))
                m.down_scales[e].copy_(s.to(dev))
            for mod in (a, m):
                for name, p in mod.lora.items():
                    if name.endswith("_A"):
                        bound = 1.0 / math.sqrt(p.shape[-1])
                        p.copy_((torch.rand(*p.shape, generator=g, device=dev) * 2 - 1).mul_(bound))
                    else:
                        p.zero_()
        return self

    @torch.no_grad()
    def lora_param_dict(self) -> dict:
        """LoRA factors by internal name (``layers.{i}.self_attn.{name}`` /
        ``layers.{i}.mlp.{name}``), in the model's own layouts -- the unit of direct GPU weight
        sync between two copies of this model."""
        out = {}
        for i, layer in enumerate(self.layers):
            for n, p in layer.self_attn.lora.items():
                out[f"layers.{i}.self_attn.{n}"] = p
            for n, p in layer.mlp.lora.items():
                out[f"layers.{i}.mlp.{n}"] = p
        return out

    @torch.no_grad()
    def init_lora(self, seed: int = 0) -> "GptOssForCausalLM":
        """PEFT-style LoRA init only (A uniform(-1/sqrt(in), 1/sqrt(in)), B = 0)."""
        g = torch.Generator(device="cpu").manual_seed(seed)
        for layer in self.layers:
            for mod in (layer.self_attn, layer.mlp):
                for name, p in mod.lora.items():
                    if name.endswith("_A"):
                        bound = 1.0 / math.sqrt(p.shape[-1])
                        p.copy_((torch.rand(*p.shape, generator=g) * 2 - 1).mul_(bound).to(p.device))
                    else:
                        p.zero_()
        return self

    def lora_parameters(self):
        return [p for n, p in self.named_parameters() if ".lora." in f".{n}" or "lora" in n.split(".")]

    def trainable_parameters(self):
        return [p for p in self.parameters() if p.requires_grad]

    # ------------------------------------------------------------------ forward
    def rope(self, device):
        if self._rope_cache is None or self._rope_cache[0].device != torch.device(device):
            cfg = self.cfg
            cos, sin = rope_tables(cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta,
                                   cfg.rope_scaling, device=device)
            self._rope_cache = (cos, sin)
        return self._rope_cache

    def embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        return torch.nn.functional.embedding(input_ids, self.embed_tokens)

    def forward_hidden(self, input_ids, position_ids, cu_seqlens, routing_indices=None,
                       record_routing: bool = False, plan: AttentionPlan | None = None):
        """Packed forward.  input_ids/position_ids [T]; cu_seqlens int32 [S+1];
        routing_indices [T, L, K] (replay) or None.  Returns final-norm hidden [T, H] (and the
        chosen expert ids [T, L, K] when ``record_routing``)."""
        cfg = self.cfg
        dev = input_ids.device
        cos, sin = self.rope(dev)
        pos = position_ids.to(torch.int32).contiguous()
        cu = cu_seqlens.to(device=dev, dtype=torch.int32)
        if plan is None and dev.type == "cuda":
            plan = AttentionPlan(cu_seqlens, dev)
            if (self.gradient_checkpointing and torch.is_grad_enabled() and not record_routing
                    and self.attention_cache_bytes > 0):
                plan.cache = AttentionOutputCache(self.attention_cache_bytes)
        x = self.embed(input_ids)
        if torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters()):
            x = x.detach().requires_grad_(True)  # checkpoint segments need a grad-carrying input
        rec = [] if record_routing else None
        for li, layer in enumerate(self.layers):
            rid = None
            if routing_indices is not None:
                rid = routing_indices[:, li, :].to(device=dev, dtype=torch.int32).contiguous()
            if self.gradient_checkpointing and torch.is_grad_enabled() and not record_routing:
                x = ckpt.checkpoint(layer, x, pos, cos, sin, cu, plan, rid, None,
                                    use_reentrant=False)
            else:
                x = layer(x, pos, cos, sin, cu, plan, rid, rec)
        h = rmsnorm(x, self.norm, cfg.rms_norm_eps)
        if record_routing:
            return h, torch.stack(rec, dim=1)
        return h

    def token_logprobs(self, hidden, labels, temperature=1.0):
        return linear_logprob_entropy(hidden, self.lm_head, labels, temperature)

    def logits(self, hidden):
        return hidden.float() @ self.lm_head.float().t()
