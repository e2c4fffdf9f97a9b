"""Forward pass of the rollout engine over a mixed batch of prefill chunks and decode tokens.

All new tokens of a step are packed into one row block so every projection and MoE GEMM runs
once per layer for the whole batch.  Attention splits by kind:
  * decode tokens (one new token on top of cached pages) -> paged decode attention kernel;
  * prefill chunks -> the packed flash-attention kernel on a buffer holding each sequence's
    full context (cached K/V gathered from pages, queries only for the new rows; the tile list
    covers just the new rows).
New K/V go straight into their page slots; the MoE expert ids chosen for every new token are
written next to them so routed experts can be returned for prefix-cache hits later.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from ..models.gpt_oss.model import GptOssForCausalLM
from ..ops import decode as D
from ..ops._ext import ext, use_cuda_kernels
from ..ops.attention import attention_reference
from ..ops.gemm import matmul
from ..ops.linear import block_diag_b, lora_linear, lora_linear_masked
from ..ops.norm import rmsnorm
from ..ops.rope import apply_rope_
from .kv_cache import PagedKVCache


@dataclass
class StepItem:
    ids: list[int]          # new tokens
    start: int              # number of tokens already in the cache for this sequence
    pages: list[int]        # pages covering start + len(ids) tokens
    want_logits: bool = True
    all_logits: bool = False   # logits of every new token (speculative verify), not just the last
    adapter: str | None = None  # LoRA adapter of this sequence (mixed-adapter batches)


@dataclass
class StepOutput:
    logits: torch.Tensor            # [n_rows, V] fp32: per item with want_logits, its last new
                                    # token, or all its new tokens when all_logits
    routing: torch.Tensor | None    # [N, L, K] uint8 of the new tokens
    item_rows: list[tuple[int, int]] = field(default_factory=list)
    logit_offsets: list[int] = field(default_factory=list)   # first logits row of each item (-1: none)


class ModelRunner:
    def __init__(self, model: GptOssForCausalLM, kv: PagedKVCache, lora_active: bool = True):
        self.model = model
        self.kv = kv
        self.cfg = model.cfg
        self.lora_active = lora_active
        self.device = model.embed_tokens.device
        self._bd_cache: dict = {}
        self._multi_cache: dict = {}
        self.graphs = None      # engine.cuda_graph.DecodeGraphs when decode steps are captured

    def _qkv_lora(self, attn):
        if not self.lora_active:
            return None, None
        return attn._qkv_lora()

    def _meta(self, items: list[StepItem]) -> "_Meta":
        """Host-side step metadata: packed token ids / positions / KV slots, the decode rows with
        their page tables, and the prefill contexts with their attention tiles."""
        dev = self.device
        P = self.kv.page_size
        m = _Meta()
        ids, pos, slots, rows = [], [], [], []
        dec_idx, pre_idx = [], []
        for i, it in enumerate(items):
            n = len(it.ids)
            r0 = len(ids)
            ids += it.ids
            for j in range(n):
                p = it.start + j
                pos.append(p)
                slots.append(it.pages[p // P] * P + p % P)
            rows.append((r0, r0 + n))
            # a speculative verify block on top of cached pages is decoded row by row: its K/V
            # are stored first, so token j attends to start + j + 1 cached positions
            decode = it.start > 0 and (n == 1 or it.all_logits)
            (dec_idx if decode else pre_idx).append(i)
        m.N, m.rows, m.dec_idx, m.pre_idx = len(ids), rows, dec_idx, pre_idx
        m.ids_t = torch.tensor(ids, device=dev, dtype=torch.long)
        m.pos_t = torch.tensor(pos, device=dev, dtype=torch.int32)
        m.slots_t = torch.tensor(slots, device=dev, dtype=torch.int32)
        if dec_idx:
            maxp = max(len(items[i].pages) for i in dec_idx)
            n_dec = sum(len(items[i].ids) for i in dec_idx)
            pt = torch.zeros(n_dec, maxp, dtype=torch.int32)
            lens, drows, r = [], [], 0
            for i in dec_idx:
                it = items[i]
                pg = torch.tensor(it.pages, dtype=torch.int32)
                for j in range(len(it.ids)):
                    pt[r, :len(it.pages)] = pg
                    lens.append(it.start + j + 1)
                    drows.append(rows[i][0] + j)
                    r += 1
            m.dec_pt = pt.to(dev)
            m.dec_lens = torch.tensor(lens, device=dev, dtype=torch.int32)
            m.dec_rows = torch.tensor(drows, device=dev, dtype=torch.long)
            m.dec_max = int(max(lens))
            m.dec_identity = (not pre_idx) and drows == list(range(len(ids)))
        if pre_idx:   # packed full contexts of the prefill chunks
            ctx_slots, new_in_ctx, new_rows, tiles, cu = [], [], [], [], [0]
            for i in pre_idx:
                it = items[i]
                L = it.start + len(it.ids)
                base = cu[-1]
                for p in range(L):
                    ctx_slots.append(it.pages[p // P] * P + p % P)
                new_in_ctx += list(range(base + it.start, base + L))
                new_rows += list(range(*rows[i]))
                for q0 in range(it.start, L, 256):   # forward kernel spans of <= 256 rows
                    tiles.append((base, base + q0, base + min(q0 + 256, L)))
                cu.append(base + L)
            tiles.sort(key=lambda t: -(t[2] - t[0]))
            m.ctx_slots_t = torch.tensor(ctx_slots, device=dev, dtype=torch.int32)
            m.new_in_ctx_t = torch.tensor(new_in_ctx, device=dev, dtype=torch.long)
            m.new_rows_t = torch.tensor(new_rows, device=dev, dtype=torch.long)
            m.tiles_t = torch.tensor(tiles, device=dev, dtype=torch.int32)
            m.cu_t = torch.tensor(cu, device=dev, dtype=torch.int32)
            m.n_ctx = cu[-1]
        return m

    def _attention(self, li: int, m: "_Meta", xn, qkv_w, qkv_b, A, B, lora_s, sinks, window,
                   hq: int, hkv: int, pos_cos_sin, qkv_mask=None) -> torch.Tensor:
        """qkv projection, RoPE, KV store and attention of layer ``li`` for ``hq`` query and
        ``hkv`` KV heads (all heads, or one tensor-parallel rank's slice).  Returns [N, hq*d]."""
        d = self.cfg.head_dim
        qs, kvs = hq * d, hkv * d
        cos, sin = pos_cos_sin
        dev = self.device
        scale = 1.0 / math.sqrt(d)
        if qkv_mask is not None and A is not None:
            qkv = lora_linear_masked(xn, qkv_w, qkv_b, A, B, None, lora_s, qkv_mask)
        else:
            qkv = lora_linear(xn, qkv_w, qkv_b, A, B, None, lora_s)
        apply_rope_(qkv, hq + hkv, d, m.pos_t, cos, sin)
        kp, vp = self.kv.k[li], self.kv.v[li]
        D.kv_store(qkv, qs, qs + kvs, m.slots_t, kp, vp)
        if m.dec_idx and not m.pre_idx and getattr(m, "dec_identity", False):
            # every row is a decode row, in order: no gather / scatter around the kernel
            return D.decode_attention(qkv[:, :qs], kp, vp, m.dec_pt, m.dec_lens, sinks, hq, hkv,
                                      window, scale, m.dec_max)
        o = torch.empty(m.N, qs, device=dev, dtype=qkv.dtype)
        if m.dec_idx:
            q = qkv.index_select(0, m.dec_rows)
            od = D.decode_attention(q[:, :qs], kp, vp, m.dec_pt, m.dec_lens, sinks, hq, hkv,
                                    window, scale, m.dec_max)
            o.index_copy_(0, m.dec_rows, od)
        if m.pre_idx:
            ctx = torch.zeros(m.n_ctx, qkv.shape[1], device=dev, dtype=qkv.dtype)
            D.kv_gather(ctx, qs, qs + kvs, m.ctx_slots_t, kp, vp)
            ctx.index_copy_(0, m.new_in_ctx_t, qkv.index_select(0, m.new_rows_t))
            if use_cuda_kernels(ctx) and d == 64:
                oc = torch.empty(m.n_ctx, qs, device=dev, dtype=qkv.dtype)
                lse = torch.empty(hq, m.n_ctx, device=dev, dtype=torch.float32)
                ext().attn_fwd(ctx, sinks.float().contiguous(), m.tiles_t, m.cu_t, oc, lse, hq,
                               hkv, d, window, scale)
            else:
                oc = attention_reference(ctx, m.cu_t, sinks, hq, hkv, d, window, scale)
            o.index_copy_(0, m.new_rows_t, oc.index_select(0, m.new_in_ctx_t))
        return o

    def _finish(self, m: "_Meta", items, x, rec) -> StepOutput:
        cfg = self.cfg
        dev = self.device
        routing = torch.stack(rec, dim=1).to(torch.uint8)       # [N, L, K]
        self.kv.routing.view(-1, cfg.num_hidden_layers, cfg.num_experts_per_tok)[m.slots_t.long()] = routing
        sel, offs = [], []
        for (r0, r1), it in zip(m.rows, items):
            if not it.want_logits:
                offs.append(-1)
                continue
            offs.append(len(sel))
            sel += list(range(r0, r1)) if it.all_logits else [r1 - 1]
        if not sel:  # only partial prefill chunks this step
            return StepOutput(logits=torch.empty(0, cfg.vocab_size, device=dev), routing=routing,
                              item_rows=m.rows, logit_offsets=offs)
        last = torch.tensor(sel, device=dev, dtype=torch.long)
        hl = rmsnorm(x.index_select(0, last), self.model.norm, cfg.rms_norm_eps)
        logits = matmul(hl, self.model.lm_head, out_dtype=torch.float32)
        return StepOutput(logits=logits, routing=routing, item_rows=m.rows, logit_offsets=offs)

    def _layers(self, m: "_Meta", x: torch.Tensor) -> tuple[torch.Tensor, list]:
        """All decoder layers over the packed new tokens; returns the final hidden states and
        the per-layer routed expert ids."""
        cfg = self.cfg
        rope = self.model.rope(self.device)
        rec: list = []
        for li, layer in enumerate(self.model.layers):
            a, mlp = layer.self_attn, layer.mlp
            xn = rmsnorm(x, layer.input_layernorm, cfg.rms_norm_eps)
            A, B = self._qkv_lora(a)
            o = self._attention(li, m, xn, a.qkv_weight, a.qkv_bias, A, B, a.lora_scaling,
                                a.sinks, a.window, cfg.num_attention_heads,
                                cfg.num_key_value_heads, rope)
            oA = a.lora["o_proj_A"] if (self.lora_active and "o_proj_A" in a.lora) else None
            oB = a.lora["o_proj_B"] if (self.lora_active and "o_proj_B" in a.lora) else None
            h = lora_linear(o, a.o_weight, a.o_bias, oA, oB, x, a.lora_scaling)
            hn = rmsnorm(h, layer.post_attention_layernorm, cfg.rms_norm_eps)
            lay_rec: list = []
            if self.lora_active:
                x = mlp(hn, h, None, lay_rec)
            else:
                from ..ops.moe_layer import moe_forward
                x = moe_forward(hn, h, mlp.router_weight, mlp.router_bias, mlp.experts(),
                                cfg.num_experts_per_tok, None, 1.0, None, cfg.swiglu_alpha,
                                cfg.swiglu_limit, lay_rec)
            rec.append(lay_rec[0])
        return x, rec

    # ------------------------------------------------------------ mixed-adapter batches
    def _multi_tensors(self, names: tuple, bank: dict) -> list:
        """Per layer: the adapters' LoRA factors stacked along the rank, in ``names`` order
        (cached per adapter set).  bank[name] holds the adapter's factors in the model's own
        layout (``GptOssForCausalLM.lora_param_dict`` names)."""
        key = (names, tuple(id(bank[n]) for n in names))
        hit = self._multi_cache.get("key")
        if hit is not None and hit[0] == key:
            return hit[1]
        cfg = self.cfg
        dev = self.device
        bf = torch.bfloat16
        layers = []
        for li, layer in enumerate(self.model.layers):
            a, mlp = layer.self_attn, layer.mlp

            def get(kind, n, name, like):
                t = bank[n].get(f"layers.{li}.{kind}.{name}")
                return (t if t is not None else torch.zeros_like(like)).to(dev, bf)
            ent = {}
            alist = a.lora
            if any(k.endswith("_A") and not k.startswith("o_") for k in alist.keys()):
                As, Bs = [], []
                r = next(p for k, p in alist.items() if k.endswith("_A")).shape[0]
                sizes = {"q_proj": cfg.q_size, "k_proj": cfg.kv_size, "v_proj": cfg.kv_size}
                for n in names:
                    pa, pb = [], []
                    for br, out in sizes.items():
                        za = torch.zeros(r, cfg.hidden_size, device=dev)
                        zb = torch.zeros(out, r, device=dev)
                        pa.append(get("self_attn", n, f"{br}_A", za) if f"{br}_A" in alist else za.to(bf))
                        pb.append(get("self_attn", n, f"{br}_B", zb) if f"{br}_B" in alist else zb.to(bf))
                    As.append(torch.cat(pa, 0))
                    Bs.append(block_diag_b(pb))
                ent["qkv"] = (torch.cat(As, 0).contiguous(), torch.cat(Bs, 1).contiguous(), As[0].shape[0])
            if "o_proj_A" in alist:
                oa = [get("self_attn", n, "o_proj_A", alist["o_proj_A"]) for n in names]
                ob = [get("self_attn", n, "o_proj_B", alist["o_proj_B"]) for n in names]
                ent["o"] = (torch.cat(oa, 0).contiguous(), torch.cat(ob, 1).contiguous(), oa[0].shape[0])
            el = {}
            for k, dim in (("gu_A", 1), ("gu_B", 2), ("dn_A", 1), ("dn_B", 2)):
                if k in mlp.lora:
                    el[k] = torch.cat([get("mlp", n, k, mlp.lora[k]) for n in names], dim).contiguous()
            if el:
                ent["experts"] = (el, mlp.lora["gu_A"].shape[1] if "gu_A" in mlp.lora
                                  else mlp.lora["dn_A"].shape[1])
            layers.append(ent)
        self._multi_cache["key"] = (key, layers)
        return layers

    @staticmethod
    def _rank_mask(row_adapter: torch.Tensor, block: int, n: int) -> torch.Tensor:
        """[N, n*block] bf16: ones on the rank columns of each row's adapter (row_adapter -1:
        no adapter, all zeros)."""
        col = torch.arange(n * block, device=row_adapter.device) // block
        return (col[None, :] == row_adapter[:, None]).to(torch.bfloat16)

    def _layers_multi(self, m: "_Meta", x: torch.Tensor, row_adapter: torch.Tensor,
                      tensors: list, n: int) -> tuple[torch.Tensor, list]:
        from ..ops.moe_layer import moe_forward
        cfg = self.cfg
        rope = self.model.rope(self.device)
        rec: list = []
        masks: dict = {}

        def mask(block):
            if block not in masks:
                masks[block] = self._rank_mask(row_adapter, block, n)
            return masks[block]
        for li, layer in enumerate(self.model.layers):
            a, mlp = layer.self_attn, layer.mlp
            ent = tensors[li]
            xn = rmsnorm(x, layer.input_layernorm, cfg.rms_norm_eps)
            if "qkv" in ent:
                A, B, blk = ent["qkv"]
                o = self._attention(li, m, xn, a.qkv_weight, a.qkv_bias, A, B, a.lora_scaling,
                                    a.sinks, a.window, cfg.num_attention_heads,
                                    cfg.num_key_value_heads, rope, qkv_mask=mask(blk))
            else:
                o = self._attention(li, m, xn, a.qkv_weight, a.qkv_bias, None, None, 1.0,
                                    a.sinks, a.window, cfg.num_attention_heads,
                                    cfg.num_key_value_heads, rope)
            if "o" in ent:
                oA, oB, blk = ent["o"]
                h = lora_linear_masked(o, a.o_weight, a.o_bias, oA, oB, x, a.lora_scaling, mask(blk))
            else:
                h = lora_linear(o, a.o_weight, a.o_bias, None, None, x, 1.0)
            hn = rmsnorm(h, layer.post_attention_layernorm, cfg.rms_norm_eps)
            lay_rec: list = []
            if "experts" in ent:
                el, blk = ent["experts"]
                x = moe_forward(hn, h, mlp.router_weight, mlp.router_bias, mlp.experts(),
                                cfg.num_experts_per_tok, el, mlp.lora_scaling, None,
                                cfg.swiglu_alpha, cfg.swiglu_limit, lay_rec,
                                lora_row_mask=mask(blk))
            else:
                x = moe_forward(hn, h, mlp.router_weight, mlp.router_bias, mlp.experts(),
                                cfg.num_experts_per_tok, None, 1.0, None, cfg.swiglu_alpha,
                                cfg.swiglu_limit, lay_rec)
            rec.append(lay_rec[0])
        return x, rec

    @torch.inference_mode()
    def forward_mixed(self, items: list[StepItem], bank: dict) -> StepOutput:
        """One step over sequences that use different adapters (or none): every adapter's
        LoRA factors are stacked along the rank and each row keeps its own adapter's columns,
        so the base projections, attention and experts run once for the whole batch."""
        names = tuple(sorted({it.adapter for it in items if it.adapter is not None}))
        tensors = self._multi_tensors(names, bank)
        m = self._meta(items)
        idx = {n: i for i, n in enumerate(names)}
        row_adapter = torch.full((m.N,), -1, dtype=torch.long)
        for (r0, r1), it in zip(m.rows, items):
            if it.adapter is not None:
                row_adapter[r0:r1] = idx[it.adapter]
        row_adapter = row_adapter.to(self.device)
        x = torch.nn.functional.embedding(m.ids_t, self.model.embed_tokens)
        x, rec = self._layers_multi(m, x, row_adapter, tensors, len(names))
        return self._finish(m, items, x, rec)

    @torch.inference_mode()
    def forward(self, items: list[StepItem]) -> StepOutput:
        if self.graphs is not None:
            out = self.graphs.run(items)
            if out is not None:
                return out
        m = self._meta(items)
        x = torch.nn.functional.embedding(m.ids_t, self.model.embed_tokens)
        x, rec = self._layers(m, x)
        return self._finish(m, items, x, rec)


class _Meta:
    """Per-step metadata shared by every layer (see ``ModelRunner._meta``)."""
    N: int
    rows: list
    dec_idx: list
    pre_idx: list
