"""Tensor-parallel rollout engine: one process per GPU, heads and experts split over the ranks.

The reference serves rollouts from sglang with ``--tp`` (examples/*/run_train.sh launch the
server; rollout/sglang_backend.py talks to it).  Here the engine's own forward pass is split:

  * attention: rank r owns query heads [r*Hq/P, (r+1)*Hq/P) and the KV heads they read
    (GQA groups stay whole), its slice of q/k/v rows and of the o_proj input columns, and a
    KV cache holding only its KV heads;
  * MoE: expert parallel -- rank r owns experts [r*E/P, (r+1)*E/P); the router is replicated,
    so every rank derives the same routing, and runs only its experts' rows;
  * after o_proj and after the MoE combine each rank holds a partial [T, H] sum.  The GEMM /
    combine write it straight into a buffer every rank has mapped (CUDA IPC), and one kernel
    (``tp_allreduce_norm``) sums the partials of all ranks over NVLink, adds the residual and
    applies the next RMSNorm -- the all-reduce is fused with the compute that follows it and
    needs no separate copy-in;
  * embeddings, final norm and LM head are replicated; rank 0 runs the scheduler and samples,
    and ships each step's batch description to the other ranks (``broadcast_object_list`` on
    a CPU group) before running its own share.

On CPU (tests) or without the extension the same code runs with ``torch.distributed``
all-reduce (gloo) in place of the fused kernel.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops import gemm as G
from ..ops import moe as M
from ..ops import mxfp4
from ..ops._ext import ext, use_cuda_kernels
from ..ops.moe_layer import ExpertWeights, _token_tile, mxfp4_int_cvt
from ..ops.norm import rmsnorm, rmsnorm_reference
from .model_runner import ModelRunner, StepItem, StepOutput


@dataclass
class LayerShard:
    qkv_w: torch.Tensor
    qkv_b: torch.Tensor
    o_w: torch.Tensor
    o_b: torch.Tensor | None       # rank 0 only: the bias is added once
    sinks: torch.Tensor
    window: int
    router_w: torch.Tensor
    router_b: torch.Tensor
    experts: ExpertWeights         # this rank's experts
    e0: int
    e1: int
    in_norm: torch.Tensor
    post_norm: torch.Tensor


def shard_model(model, rank: int, world: int, free_full: bool = False) -> list[LayerShard]:
    """This rank's slices of every decoder layer (copies; with ``free_full`` the full layer
    weights are released afterwards)."""
    cfg = model.cfg
    hq, hkv, d, E = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.num_local_experts
    if hq % world or hkv % world or E % world:
        raise ValueError(f"TP={world} must divide {hq} query heads, {hkv} KV heads and {E} experts")
    qh, kh, ne = hq // world, hkv // world, E // world
    qs, kvs = cfg.q_size, cfg.kv_size
    q0, q1 = rank * qh * d, (rank + 1) * qh * d
    k0, k1 = qs + rank * kh * d, qs + (rank + 1) * kh * d
    v0, v1 = qs + kvs + rank * kh * d, qs + kvs + (rank + 1) * kh * d
    e0, e1 = rank * ne, (rank + 1) * ne
    shards = []
    with torch.no_grad():
        for layer in model.layers:
            a, m = layer.self_attn, layer.mlp
            W, b = a.qkv_weight, a.qkv_bias
            ex = ExpertWeights(m.gate_up_blocks[e0:e1].clone(), m.gate_up_scales[e0:e1].clone(),
                               m.gate_up_bias[e0:e1].clone(), m.down_blocks[e0:e1].clone(),
                               m.down_scales[e0:e1].clone(), m.down_bias[e0:e1].clone())
            shards.append(LayerShard(
                qkv_w=torch.cat([W[q0:q1], W[k0:k1], W[v0:v1]]).contiguous(),
                qkv_b=torch.cat([b[q0:q1], b[k0:k1], b[v0:v1]]).contiguous(),
                o_w=a.o_weight[:, q0:q1].contiguous(),
                o_b=a.o_bias.detach().clone() if rank == 0 else None,
                sinks=a.sinks[rank * qh:(rank + 1) * qh].detach().clone(),
                window=a.window,
                router_w=m.router_weight.detach(), router_b=m.router_bias.detach(),
                experts=ex, e0=e0, e1=e1,
                in_norm=layer.input_layernorm.detach(),
                post_norm=layer.post_attention_layernorm.detach()))
            if free_full:
                for t in (a.qkv_weight, a.o_weight, m.gate_up_blocks, m.gate_up_scales,
                          m.down_blocks, m.down_scales):
                    t.data = torch.empty(0, dtype=t.dtype, device=t.device)
    return shards


@dataclass
class LoraShard:
    """This rank's LoRA factors of one layer (bf16): query/KV-head rows of the fused q/k/v B,
    the o_proj input columns of its A, and the local experts' up-projections B; the expert
    down-projections A are kept whole (the LoRA activations of every routed row are computed,
    only the local experts' rows are read)."""
    qkv_A: torch.Tensor | None
    qkv_B: torch.Tensor | None
    o_A: torch.Tensor | None
    o_B: torch.Tensor | None
    gu_A: torch.Tensor | None
    gu_B: torch.Tensor | None
    dn_A: torch.Tensor | None
    dn_B: torch.Tensor | None
    s_attn: float
    s_mlp: float


def shard_lora(model, rank: int, world: int) -> list[LoraShard]:
    cfg = model.cfg
    hq, hkv, d, E = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.num_local_experts
    qh, kh, ne = hq // world, hkv // world, E // world
    qs, kvs = cfg.q_size, cfg.kv_size
    q0, q1 = rank * qh * d, (rank + 1) * qh * d
    k0, k1 = qs + rank * kh * d, qs + (rank + 1) * kh * d
    v0, v1 = qs + kvs + rank * kh * d, qs + kvs + (rank + 1) * kh * d
    e0, e1 = rank * ne, (rank + 1) * ne

    def bf(t):
        return None if t is None else t.detach().to(torch.bfloat16).contiguous()

    out = []
    with torch.no_grad():
        for layer in model.layers:
            a, m = layer.self_attn, layer.mlp
            A, B = a._qkv_lora()
            if B is not None:
                B = torch.cat([B[q0:q1], B[k0:k1], B[v0:v1]])
            oA = a.lora["o_proj_A"][:, q0:q1] if "o_proj_A" in a.lora else None
            oB = a.lora["o_proj_B"] if "o_proj_B" in a.lora else None
            lo = m.lora
            out.append(LoraShard(
                qkv_A=bf(A), qkv_B=bf(B), o_A=bf(oA), o_B=bf(oB),
                gu_A=bf(lo["gu_A"]) if "gu_A" in lo else None,
                gu_B=bf(lo["gu_B"][e0:e1]) if "gu_B" in lo else None,
                dn_A=bf(lo["dn_A"]) if "dn_A" in lo else None,
                dn_B=bf(lo["dn_B"][e0:e1]) if "dn_B" in lo else None,
                s_attn=a.lora_scaling, s_mlp=m.lora_scaling))
    return out


def broadcast_model(model, group=None, src: int = 0) -> None:
    """Make every rank's weights equal to rank ``src``'s (random init or a checkpoint loaded on
    one rank) before sharding."""
    with torch.no_grad():
        for t in list(model.parameters()) + list(model.buffers()):
            dist.broadcast(t.data, group=group, group_src=src)


class TPContext:
    """Process-group plumbing of one tensor-parallel engine rank.

    ``group``: the ranks of this engine (NCCL on GPU, gloo on CPU); ``cpu_group``: a gloo group
    over the same ranks for the per-step batch broadcast.  With CUDA kernels available the
    partial sums live in a ``SymmetricWorkspace`` of ``max_tokens`` x ``hidden`` bf16 rows."""

    def __init__(self, group=None, cpu_group=None, device=None, max_tokens: int = 0,
                 hidden: int = 0, timeout_s: float = 30.0):
        self.group = group
        self.cpu_group = cpu_group if cpu_group is not None else group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.timeout_s = timeout_s
        self.symm = None
        self.fused_calls = 0
        if self.device.type == "cuda" and use_cuda_kernels(torch.empty(0, device=self.device)):
            from ..parallel.symm import SymmetricWorkspace
            self.symm = SymmetricWorkspace(max_tokens * hidden * 2, group, self.device)

    # -- the partial-sum buffer the next reduction reads ----------------------------------
    def partial_buffer(self, T: int, H: int) -> torch.Tensor:
        if self.symm is not None:
            return self.symm.local_set((self.symm.epoch + 1) % self.symm.sets, (T, H))
        return torch.empty(T, H, device=self.device, dtype=torch.bfloat16)

    def allreduce_norm(self, partial: torch.Tensor, residual: torch.Tensor,
                       w: torch.Tensor | None, eps: float):
        """x = residual + sum over ranks of ``partial`` (bf16), xn = RMSNorm(x) * w (or None)."""
        T, H = partial.shape
        if self.symm is not None:
            self.symm.epoch += 1
            s = self.symm.epoch % self.symm.sets
            x = torch.empty(T, H, device=partial.device, dtype=torch.bfloat16)
            xn = torch.empty_like(x) if w is not None else None
            ext().tp_allreduce_norm(self.symm.set_ptrs(s), self.symm.flag_ptrs(), self.rank,
                                    self.symm.epoch, H, residual.contiguous(),
                                    None if w is None else w.float().contiguous(), eps, x, xn,
                                    T, H, self.timeout_s)
            self.fused_calls += 1
            return x, xn
        acc = partial.float()
        dist.all_reduce(acc, group=self.group)
        x = (residual.float() + acc).to(torch.bfloat16)
        xn = rmsnorm_reference(x, w, eps) if w is not None else None
        return x, xn

    def raise_on_device_error(self) -> None:
        """Read (and clear) the device error word after a step's fused reductions.  A peer
        that did not arrive within ``timeout_s`` makes the reduction kernel give up without
        writing its outputs; the step's hidden states are then garbage, so the step fails here
        instead of decoding on.  The read synchronises the stream once per step."""
        code = int(ext().device_error())
        if code != 0:
            raise RuntimeError(
                f"tensor-parallel rank {self.rank}: fused all-reduce reported device error "
                f"{code} (a peer rank did not arrive within {self.timeout_s} s); step aborted")

    # -- step broadcast (rank 0 -> others) -------------------------------------------------
    def send(self, msg) -> None:
        dist.broadcast_object_list([msg], group=self.cpu_group, group_src=0)

    def recv(self):
        obj = [None]
        dist.broadcast_object_list(obj, group=self.cpu_group, group_src=0)
        return obj[0]

    def send_items(self, items: list[StepItem] | None, lora_active: bool = False,
                   replay: bool = False) -> None:
        self.send(None if items is None else
                  ("step", [(it.ids, it.start, it.pages, it.want_logits, it.all_logits)
                            for it in items], lora_active, replay))

    @staticmethod
    def items_of(msg) -> list[StepItem]:
        return [StepItem(list(i), s, list(p), w, a) for i, s, p, w, a in msg[1]]

    def broadcast_tensors(self, tensors: list[torch.Tensor]) -> None:
        """Rank 0's values of ``tensors`` (same shapes on every rank) to every rank, over the
        device group."""
        for t in tensors:
            dist.broadcast(t.data, group=self.group, group_src=0)

    def close(self) -> None:
        if self.symm is not None:
            self.symm.close()

    def shutdown(self) -> None:
        """Collective: wait until no rank can still be reading another rank's buffer, then
        unmap.  Every rank must call it (a rank that exits early would free memory a peer's
        last reduction may still be reading over NVLink)."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.cpu_group)
        self.close()


def moe_ep_partial(xn: torch.Tensor, sh: LayerShard, n_experts: int, top_k: int, alpha: float,
                   limit: float, out: torch.Tensor, routing_out: list | None = None,
                   lora: LoraShard | None = None, replay_ids: torch.Tensor | None = None
                   ) -> torch.Tensor:
    """This rank's share of the MoE output: sum over the token's top-k experts that live on
    this rank of gate * expert(x), written into ``out`` [T, H] (no residual).  With ``lora``
    the experts' adapters join as in the single-GPU path: x A_e^T s as extra K columns against
    the local experts' B_e rows."""
    T, H = xn.shape
    logits = G.matmul(xn, sh.router_w, bias=sh.router_b, out_dtype=torch.float32)
    rt = M.route(logits, top_k, n_experts, replay_ids=replay_ids)
    if routing_out is not None:
        routing_out.append(rt.ids)
    mx = xn.is_cuda and use_cuda_kernels(xn) and sh.experts.f16_exact()
    x_s = M.gather_rows(xn, rt.row_src, zero_pad=not mx)   # the MXFP4 path never reads padding
    R = x_s.shape[0]
    ex = sh.experts
    y_s = torch.zeros(R, H, device=xn.device, dtype=torch.bfloat16)
    gu_lora = lora is not None and lora.gu_A is not None
    dn_lora = lora is not None and lora.dn_A is not None
    if mx:
        offs = rt.offsets[sh.e0:sh.e1 + 1]
        cnts = rt.counts[sh.e0:sh.e1]
        I2 = ex.gu_blocks.shape[1]
        h = torch.empty(R, I2 // 2, device=xn.device, dtype=torch.bfloat16)
        bn = _token_tile(T * top_k, n_experts)
        xa = G.grouped_matmul(x_s, lora.gu_A, rt.offsets, alpha=lora.s_mlp)[0] if gu_lora else None
        ic = mxfp4_int_cvt(ex)
        ext().moe_mxfp4_gemm(x_s, ex.gu_blocks, ex.gu_scales, ex.gu_bias, offs, cnts, 0, None, h,
                             alpha, limit, bn, lora_b=lora.gu_B if gu_lora else None, xa=xa,
                             int_cvt=ic)
        ha = G.grouped_matmul(h, lora.dn_A, rt.offsets, alpha=lora.s_mlp)[0] if dn_lora else None
        ext().moe_mxfp4_gemm(h, ex.dn_blocks, ex.dn_scales, ex.dn_bias, offs, cnts, 1,
                             rt.row_gate, y_s, alpha, limit, bn,
                             lora_b=lora.dn_B if dn_lora else None, xa=ha, int_cvt=ic)
    else:
        W_gu = mxfp4.dequantize(ex.gu_blocks, ex.gu_scales)
        W_dn = mxfp4.dequantize(ex.dn_blocks, ex.dn_scales)
        offs, cnts = rt.offsets.tolist(), rt.counts.tolist()
        for e in range(sh.e0, sh.e1):
            r0, n = offs[e], cnts[e]
            if n == 0:
                continue
            j = e - sh.e0
            xe = x_s[r0:r0 + n].float()
            gu = xe @ W_gu[j].float().t() + ex.gu_bias[j].float()
            if gu_lora:
                xa = (xe @ lora.gu_A[e].float().t() * lora.s_mlp).to(torch.bfloat16).float()
                gu = gu + xa @ lora.gu_B[j].float().t()
            h = G.swiglu_reference(gu.to(torch.bfloat16), alpha, limit).to(torch.bfloat16)
            y = h.float() @ W_dn[j].float().t() + ex.dn_bias[j].float()
            if dn_lora:
                ha = (h.float() @ lora.dn_A[e].float().t() * lora.s_mlp).to(torch.bfloat16).float()
                y = y + ha @ lora.dn_B[j].float().t()
            y = y * rt.row_gate[r0:r0 + n, None]
            y_s[r0:r0 + n] = y.to(torch.bfloat16)
    return M.combine_rows(y_s, rt.dest, top_k, out=out)


class TPModelRunner(ModelRunner):
    """Engine forward pass over this rank's shard; see the module docstring.

    LoRA: the engine loads an adapter into rank 0's model and calls ``sync_lora()``; the full
    factors are broadcast over the device group into every rank's model and each rank keeps its
    slices (``shard_lora``).  Every step message carries whether the adapter is active."""

    def __init__(self, model, kv, ctx: TPContext, shards: list[LayerShard] | None = None):
        super().__init__(model, kv, lora_active=False)
        self.ctx = ctx
        self.shards = shards if shards is not None else shard_model(model, ctx.rank, ctx.world)
        self.lora_shards: list[LoraShard] | None = None
        cfg = self.cfg
        self.hq = cfg.num_attention_heads // ctx.world
        self.hkv = cfg.num_key_value_heads // ctx.world

    def sync_lora(self) -> None:
        """Rank 0: publish the adapter now in the model's LoRA parameters to every rank."""
        params = list(self.model.lora_param_dict().values())
        if not params:
            raise ValueError("the model was built without LoRA capacity")
        if self.ctx.world > 1:
            self.ctx.send(("lora",))
            self.ctx.broadcast_tensors(params)
        self.lora_shards = shard_lora(self.model, self.ctx.rank, self.ctx.world)

    def _recv_lora(self) -> None:
        self.ctx.broadcast_tensors(list(self.model.lora_param_dict().values()))
        self.lora_shards = shard_lora(self.model, self.ctx.rank, self.ctx.world)

    def forward(self, items: list[StepItem], replay: torch.Tensor | None = None) -> StepOutput:
        """One engine step.  ``replay`` (int [N, L, K], rank 0): expert ids to use instead of
        the router's choice for every new token and layer (routing replay, e.g. to reproduce a
        recorded rollout); it is broadcast to the other ranks with the step."""
        if self.lora_active and self.lora_shards is None:
            raise RuntimeError("LoRA active but not synced to the tensor-parallel ranks")
        if self.ctx.rank == 0 and self.ctx.world > 1:
            self.ctx.send_items(items, self.lora_active, replay is not None)
            if replay is not None:
                self.ctx.broadcast_tensors([replay.to(self.device, torch.int32).contiguous()])
        return self._forward(items, self.lora_active, replay)

    def follow(self) -> int:
        """Non-zero ranks: run the steps rank 0 broadcasts until it sends None; returns the
        number of steps run."""
        n = 0
        while True:
            msg = self.ctx.recv()
            if msg is None:
                return n
            if msg[0] == "lora":
                self._recv_lora()
                continue
            items = TPContext.items_of(msg)
            replay = None
            if len(msg) > 3 and msg[3]:
                cfg = self.cfg
                replay = torch.empty(sum(len(it.ids) for it in items), cfg.num_hidden_layers,
                                     cfg.num_experts_per_tok, device=self.device,
                                     dtype=torch.int32)
                self.ctx.broadcast_tensors([replay])
            self._forward(items, bool(msg[2]), replay)
            n += 1

    def stop_followers(self) -> None:
        if self.ctx.rank == 0 and self.ctx.world > 1:
            self.ctx.send_items(None)

    @torch.inference_mode()
    def _forward(self, items: list[StepItem], lora_active: bool = False,
                 replay: torch.Tensor | None = None) -> StepOutput:
        cfg = self.cfg
        eps = cfg.rms_norm_eps
        H = cfg.hidden_size
        m = self._meta(items)
        rope = self.model.rope(self.device)
        x = torch.nn.functional.embedding(m.ids_t, self.model.embed_tokens)
        xn = rmsnorm(x, self.shards[0].in_norm, eps)
        rec: list = []
        L = len(self.shards)
        for li, sh in enumerate(self.shards):
            lo = self.lora_shards[li] if lora_active else None
            o = self._attention(li, m, xn, sh.qkv_w, sh.qkv_b,
                                lo.qkv_A if lo else None, lo.qkv_B if lo else None,
                                lo.s_attn if lo else 1.0, sh.sinks, sh.window, self.hq,
                                self.hkv, rope)
            part = self.ctx.partial_buffer(m.N, H)
            if lo is not None and lo.o_A is not None:
                oa = G.matmul(o, lo.o_A, alpha=lo.s_attn)                  # [N, r]
                G.matmul(o, sh.o_w, bias=sh.o_b, a2=oa, b2=lo.o_B, out=part)
            else:
                G.matmul(o, sh.o_w, bias=sh.o_b, out=part)
            h, hn = self.ctx.allreduce_norm(part, x, sh.post_norm, eps)
            part = self.ctx.partial_buffer(m.N, H)
            lay_rec: list = []
            rid = None
            if replay is not None:
                rid = replay[:, li, :].to(device=hn.device, dtype=torch.int32).contiguous()
            moe_ep_partial(hn, sh, cfg.num_local_experts, cfg.num_experts_per_tok,
                           cfg.swiglu_alpha, cfg.swiglu_limit, part, lay_rec, lo, replay_ids=rid)
            rec.append(lay_rec[0])
            nxt = self.shards[li + 1].in_norm if li + 1 < L else None
            x, xn = self.ctx.allreduce_norm(part, h, nxt, eps)
        if self.ctx.rank != 0:   # only rank 0 samples
            items = [StepItem(it.ids, it.start, it.pages, False, False) for it in items]
        out = self._finish(m, items, x, rec)
        if self.ctx.symm is not None:
            self.ctx.raise_on_device_error()
        return out
