"""ModelTrainer: LoRA (or full-parameter) RL training of gpt-oss on B200s.

Parity with the reference's ModelTrainer (trainer/model_trainer.py:108-929): the same public
methods (``train_step``, ``reset_optimizer_state``, ``save_model``, ``load_model``,
``save_merged_weights``, ``save_training_state``, ``load_training_state``), the same loss
(DDIS over the fused log-prob/entropy of the packed batch), AdamW with HF-style schedules, and
PEFT-format adapters.

What differs (B200 design):
  * one process per GPU; the frozen MXFP4 experts are either resident on every GPU (180 GB HBM
    holds gpt-oss-120b's 65 GB of weights plus 131k-token activations) or, with
    ``shard_base_weights``, split over the ranks and gathered over NVLink inside the kernel
    that dequantises a layer's experts (parallel/fsdp.py); only trainable state is reduced;
  * gradients of all trainable tensors live in one flat fp32 buffer so the data-parallel
    reduction is a single NCCL all-reduce (or reduce-scatter when the optimizer state is
    sharded) instead of per-parameter collectives;
  * loss/metric reductions are packed into one all-reduce;
  * rank 0 plans the step's packing and scatters to each rank only the samples of that rank's
    buckets, with their arrays sent as raw bytes (parallel/payload.py); no rank receives the
    whole step.
"""
from __future__ import annotations

import json
import logging
import math
import os
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..models.gpt_oss import GptOssConfig, GptOssForCausalLM, LoraConfig
from ..models.gpt_oss import checkpoint as ckpt
from ..parallel import payload
from ..parallel.rpc import RPCMixin, rpc_method
from .data.collator import DataCollatorWithPacking, shift_completion_mask
from .data.sampler import DeterministicPackedBatchSampler
from .losses.ddis_loss import DDISLoss
from .losses.metric_state import MeanMetricState, all_reduce_metric_states
from .scheduler import get_scheduler
from .training_config import TrainingConfig
from .types import TrainingSample

logger = logging.getLogger(__name__)


def build_model(config: TrainingConfig, device, model_config: GptOssConfig | None = None
                ) -> GptOssForCausalLM:
    lora = None
    if config.training_mode == "lora":
        lora = LoraConfig(r=config.lora_r, lora_alpha=config.lora_alpha,
                          target_modules=list(config.lora_target_modules),
                          lora_dropout=config.lora_dropout)
    path = Path(config.model_id)
    if model_config is None:
        if path.is_dir() and (path / "config.json").exists():
            model_config = GptOssConfig.load(path / "config.json")
        else:
            model_config = GptOssConfig.preset(config.model_id)
    model = GptOssForCausalLM(model_config, lora=lora, device=device)
    if path.is_dir() and any(path.glob("*.safetensors")):
        missing = ckpt.load_checkpoint(path, model)
        if missing:
            raise RuntimeError(f"checkpoint {path} is missing {len(missing)} tensors, e.g. {missing[:3]}")
        model.init_lora(seed=config.random_init_seed or 0)
    else:
        model.init_random(seed=config.random_init_seed or 0)
    model.gradient_checkpointing = config.gradient_checkpointing
    for layer in model.layers:
        layer.mlp.dequant_dtype = config.dequant_dtype
    model.attention_cache_bytes = int(config.attention_cache_gb * 1e9)
    if config.training_mode == "full":
        for n, p in model.named_parameters():
            train = config.trainable_modules is None or any(m in n for m in config.trainable_modules)
            p.requires_grad_(train and p.dtype.is_floating_point)
    return model


class ModelTrainer(RPCMixin):
    def __init__(self, config: TrainingConfig, model: GptOssForCausalLM | None = None, *,
                 model_config: GptOssConfig | None = None, device: str | torch.device | None = None,
                 rpc_group=None):
        self.config = config
        self.distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank() if self.distributed else 0
        self.world_size = dist.get_world_size() if self.distributed else 1
        if device is None:
            device = (f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}" if torch.cuda.is_available()
                      else "cpu")
        self.device = torch.device(device)
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        self.model = model if model is not None else build_model(config, self.device, model_config)
        self.expert_shards = None
        if config.shard_base_weights and self.distributed and self.world_size > 1:
            # FSDP-style: each rank keeps 1/W of every layer's frozen MXFP4 experts; a layer's
            # full stack is gathered over NVLink inside its dequantisation kernel
            from ..parallel.fsdp import shard_expert_weights
            self.expert_shards = shard_expert_weights(self.model)
        self.trainable = [p for p in self.model.parameters() if p.requires_grad]
        if not self.trainable:
            raise RuntimeError("no trainable parameters (check lora_target_modules / trainable_modules)")
        self._flatten_grads()
        self.optimizer = self._create_optimizer()
        self.lr_scheduler = get_scheduler(config.lr_scheduler_type, self.optimizer,
                                          num_warmup_steps=config.lr_warmup_steps,
                                          num_training_steps=1_000_000)
        self.loss_calculator = DDISLoss(eps_low=config.ddis_eps_low, eps_high=config.ddis_eps_high,
                                        use_opsm=config.use_opsm, opsm_delta=config.opsm_delta,
                                        entropy_top_pct=config.entropy_top_pct)
        self.collator = DataCollatorWithPacking(pad_token_id=self.model.cfg.pad_token_id,
                                                pad_to_multiple_of=config.pad_to_multiple_of_training,
                                                pin_memory=self.device.type == "cuda",
                                                vocab_size=self.model.cfg.vocab_size,
                                                num_experts=self.model.cfg.num_local_experts)
        self.step_count = 0
        self.last_step_events = None
        self._outbox = None
        self.last_step_h2d_bytes = self.last_step_d2h_bytes = self.last_step_tokens = 0
        RPCMixin.__init__(self, group=rpc_group)

    # ------------------------------------------------------------------ setup
    def _flatten_grads(self):
        """All trainable tensors and their gradients are views into one flat fp32 buffer each
        (one collective per step).  With ``shard_optimizer_state`` and several ranks, rank r
        owns the slice [r*S, (r+1)*S) of the flat parameters: AdamW keeps the moments of that
        slice only, gradients are reduce-scattered into it and the updated slices all-gathered
        back into every rank's flat parameters."""
        n = sum(p.numel() for p in self.trainable)
        w = self.world_size if self.distributed else 1
        self.sharded = (self.config.shard_optimizer_state and w > 1 and
                        all(p.dtype == torch.float32 for p in self.trainable))
        n_pad = (n + w * 8 - 1) // (w * 8) * (w * 8) if self.sharded else n
        self.flat_grad = torch.zeros(n_pad, device=self.device, dtype=torch.float32)
        if self.sharded:
            self.flat_param = torch.zeros(n_pad, device=self.device, dtype=torch.float32)
        off = 0
        for p in self.trainable:
            k = p.numel()
            if self.sharded:
                self.flat_param[off:off + k].copy_(p.detach().reshape(-1))
                p.data = self.flat_param[off:off + k].view_as(p)
            p.grad = self.flat_grad[off:off + k].view_as(p)
            off += k
        if self.sharded:
            S = n_pad // w
            self.shard_param = torch.nn.Parameter(self.flat_param[self.rank * S:(self.rank + 1) * S])
            self.shard_grad = torch.zeros(S, device=self.device, dtype=torch.float32)
            self.shard_param.grad = self.shard_grad
        self.grad_pusher = None
        if self.sharded and self.device.type == "cuda" and self.config.grad_reduce == "push":
            # reduce-scatter by copy-engine pushes overlapped with the backward (no NCCL)
            from ..parallel.grad_push import GradientPusher
            offs, o = [], 0
            for p in self.trainable:
                offs.append(o)
                o += p.numel()
            self.grad_pusher = GradientPusher(self.trainable, offs, self.flat_grad, self.shard_grad)

    def _create_optimizer(self):
        if self.config.optimizer_type != "AdamW":
            raise ValueError(f"Unsupported optimizer type: {self.config.optimizer_type}")
        kw = dict(lr=self.config.learning_rate, weight_decay=self.config.weight_decay,
                  betas=(self.config.adam_beta1, self.config.adam_beta2), eps=self.config.adam_epsilon)
        if self.device.type == "cuda":
            kw["fused"] = True
        return torch.optim.AdamW([self.shard_param] if self.sharded else self.trainable, **kw)

    # ------------------------------------------------------------------ step
    def _to_device(self, batch: dict) -> dict:
        out = {}
        for k, v in batch.items():
            if isinstance(v, torch.Tensor) and k not in ("cu_seqlens",):
                out[k] = v.to(self.device, non_blocking=True)
            else:
                out[k] = v
        return out

    def _microbatch(self, batch: dict) -> tuple[torch.Tensor, dict[str, MeanMetricState]]:
        m = self.model
        routing = batch.get("routing_indices") if self.config.use_routing_replay else None
        if self.config.use_routing_replay and routing is None:
            raise RuntimeError("use_routing_replay=True but the batch has no routing_indices")
        hidden = m.forward_hidden(batch["input_ids"], batch["position_ids"], batch["cu_seqlens"],
                                  routing_indices=routing)
        lp, ent = m.token_logprobs(hidden, batch["labels"], self.config.loss_temperature)
        # position t scores token t+1: shift the per-token fields to the predicting position
        comp = shift_completion_mask(batch["completion_mask"])
        gen = torch.zeros_like(batch["gen_logprobs"])
        gen[:-1] = batch["gen_logprobs"][1:]
        adv = torch.zeros_like(batch["advantages"])
        adv[:-1] = batch["advantages"][1:]
        seg = batch["segment_ids"]
        out = self.loss_calculator.compute_packed(
            log_probs=lp, completion_mask=comp, advantages=adv, gen_log_probs=gen,
            segment_ids=seg, divisors=batch["divisor"],
            entropies=ent if self.config.entropy_top_pct is not None else None)
        states = out.metric_states
        mask = comp.float()
        states["algo/response_entropy"] = MeanMetricState(
            (ent.detach() * mask).sum(), mask.sum(), "token")
        if "gen_entropy" in batch:
            ge = torch.zeros_like(batch["gen_entropy"])
            ge[:-1] = batch["gen_entropy"][1:]
            states["algo/gen_entropy"] = MeanMetricState((ge * mask).sum(), mask.sum(), "token")
        return out.loss_unscaled, states

    def _rank_microbatches(self, samples: list[TrainingSample]) -> list[list[int]]:
        sampler = self._sampler([len(s) for s in samples])
        self._packing_stats = sampler.stats
        return sampler.plan_for_rank(self.rank)

    def _reduce_gradients(self):
        """Data-parallel gradient reduction; returns this rank's shard sum of squares when the
        reduction computed it on the way (the overlapped push path), else None."""
        if self.distributed and self.world_size > 1:
            if self.grad_pusher is not None:
                return self.grad_pusher.finish()
            if self.sharded:
                dist.reduce_scatter_tensor(self.shard_grad, self.flat_grad)
            else:
                dist.all_reduce(self.flat_grad)
        return None

    def _arm_gradient_push(self) -> None:
        """Called before the step's last backward: gradients are pushed to their owners as
        soon as each is final."""
        if self.grad_pusher is not None:
            self.grad_pusher.arm()

    def _apply_gradients(self) -> torch.Tensor | None:
        """Reduce, clip and apply this step's gradients; returns the global gradient norm
        (device tensor) when clipping is on."""
        sq_shard = self._reduce_gradients()
        g = self.shard_grad if self.sharded else self.flat_grad
        grad_norm = None
        if self.config.max_grad_norm > 0:
            if self.sharded:
                sq = (sq_shard.reshape(()) if sq_shard is not None else g.pow(2).sum()).clone()
                dist.all_reduce(sq)
                grad_norm = sq.sqrt()
            else:
                grad_norm = torch.linalg.vector_norm(g)
            g.mul_((self.config.max_grad_norm / (grad_norm + 1e-6)).clamp(max=1.0))
        self.optimizer.step()
        self.lr_scheduler.step()
        if self.sharded:
            dist.all_gather_into_tensor(self.flat_param, self.shard_param.data)
        self.flat_grad.zero_()
        return grad_norm

    def _optimizer_step(self, loss_sum: torch.Tensor, states: dict) -> dict[str, float]:
        grad_norm = self._apply_gradients()
        extra = torch.stack([loss_sum.detach().float(),
                             grad_norm.float() if grad_norm is not None else torch.zeros((), device=self.device)])
        red = all_reduce_metric_states(states, extra=extra)
        keys = sorted(states)
        # the reduced extras and every metric's mean in one tensor: the step's single
        # device->host read
        packed = [red.float().reshape(-1)]
        if keys:
            packed.append(torch.stack([(states[k].sum / states[k].count.clamp_min(1.0)).float()
                                       for k in keys]))
        host = torch.cat(packed).tolist()
        self.last_step_d2h_bytes = 4 * len(host)
        vals = host[:red.numel()]
        metrics = {"loss": vals[0], "learning_rate": float(self.optimizer.param_groups[0]["lr"])}
        if grad_norm is not None:
            metrics["grad_norm"] = vals[1] / self.world_size  # every rank holds the global norm
        for k, v in zip(keys, host[red.numel():]):
            metrics[k] = float(v)
        return metrics

    def train_step(self, step_samples: list[TrainingSample]) -> dict[str, float]:
        """One optimizer step over ``step_samples``.  Called on rank 0; the other ranks sit in
        ``rpc_worker_loop``.  Rank 0 runs the deterministic packing plan over the whole list and
        sends every rank only the samples of its own buckets (one scatter over the control
        group: each rank receives its own payload, never the whole step); each rank collates
        and trains its buckets, and the gradients meet in the data-parallel reduction."""
        if not step_samples:
            raise ValueError("train_step received empty step_samples")
        if any(s.divisor is None or s.divisor == 0 for s in step_samples):
            raise ValueError("train_step requires all samples to have a non-null, non-zero divisor.")
        t0 = time.perf_counter()
        sampler = self._sampler([len(s) for s in step_samples])
        self._packing_stats = sampler.stats
        outbox = []
        for r in range(self.world_size):
            mbs = sampler.plan_for_rank(r)
            order = sorted({i for mb in mbs for i in mb})
            local = {g: j for j, g in enumerate(order)}
            outbox.append(([step_samples[i] for i in order], [[local[i] for i in mb] for mb in mbs]))
        self._outbox = outbox
        try:
            metrics = self._train_own_buckets()
        finally:
            self._outbox = None
        dt = time.perf_counter() - t0
        seq = [len(s) for s in step_samples]
        comp = [s.num_loss_tokens() for s in step_samples]
        metrics["step_time"] = dt
        metrics["train/tokens_per_sec"] = sum(seq) / dt
        metrics["train/seq_len_mean"] = sum(seq) / len(seq)
        metrics["train/seq_len_max"] = float(max(seq))
        metrics["train/completion_len_mean"] = sum(comp) / len(comp)
        metrics["train/completion_len_max"] = float(max(comp))
        return metrics

    def _sampler(self, lengths: list[int]) -> DeterministicPackedBatchSampler:
        return DeterministicPackedBatchSampler(
            lengths, max_capacity=self.config.max_capacity, world_size=self.world_size,
            balance=self.config.packing_balance,
            attention_tokens=self.config.packing_attention_tokens)

    @rpc_method(gather=False)
    def _train_own_buckets(self) -> dict[str, float]:
        """Every rank: receive this rank's (samples, microbatch index lists) from rank 0,
        then forward/backward each microbatch and take the optimizer step."""
        if self._rpc_active():
            samples, plan = payload.scatter(self._outbox if self.rank == 0 else None,
                                            group=self._rpc_group, src=0)
        else:
            samples, plan = self._outbox[0]
        self.model.train()
        loss_sum = torch.zeros((), device=self.device)
        states: dict[str, MeanMetricState] = {}
        self.last_step_h2d_bytes = 0
        self.last_step_tokens = 0
        for n_mb, idx in enumerate(plan):
            if n_mb == len(plan) - 1:
                self._arm_gradient_push()
            host = self.collator([samples[i] for i in idx])
            self.last_step_h2d_bytes += sum(v.numel() * v.element_size() for k, v in host.items()
                                            if isinstance(v, torch.Tensor) and k != "cu_seqlens")
            self.last_step_tokens += int(host["num_tokens"])
            batch = self._to_device(host)
            loss, st = self._microbatch(batch)
            loss.backward()
            loss_sum = loss_sum + loss.detach()
            for k, v in st.items():
                states[k] = states[k].merge(v) if k in states else v
        metrics = self._optimizer_step(loss_sum, states)
        self.step_count += 1
        return metrics

    def train_packed_batch(self, host_batch: dict) -> torch.Tensor:
        """Forward/backward/optimizer step of one pre-packed host batch (pinned tensors).
        Returns the loss as a device tensor (no host synchronisation)."""
        self.model.train()
        batch = self._to_device(host_batch)
        loss, states = self._microbatch(batch)
        self._arm_gradient_push()
        loss.backward()
        self._apply_gradients()
        self.step_count += 1
        return loss.detach()

    # ------------------------------------------------------------------ state
    @rpc_method(gather=False)
    def reset_optimizer_state(self):
        for st in self.optimizer.state.values():
            for k in ("exp_avg", "exp_avg_sq"):
                if k in st:
                    st[k].zero_()

    def lora_state_dict(self) -> dict[str, torch.Tensor]:
        """PEFT key names: base_model.model.model.layers.N.self_attn.q_proj.lora_A.weight
        [r, in], ...lora_B.weight [out, r]; expert factors under
        ...mlp.experts.{gate_up_proj,down_proj}.lora_{A,B}.weight with shapes [E*r, in] and
        [out, E*r] (expert e owns rows/columns e*r .. e*r+r-1)."""
        sd = {}
        for i, layer in enumerate(self.model.layers):
            pre = f"base_model.model.model.layers.{i}."
            for name, p in layer.self_attn.lora.items():
                mod, ab = name.rsplit("_", 1)
                sd[f"{pre}self_attn.{mod}.lora_{ab}.weight"] = p.detach().float().cpu()
            for name, p in layer.mlp.lora.items():
                mod = {"gu": "gate_up_proj", "dn": "down_proj"}[name.split("_")[0]]
                ab = name.split("_")[1]
                t = p.detach().float().cpu()
                E, a, b = t.shape
                if ab == "A":   # [E, r, in] -> [E*r, in]
                    t = t.reshape(E * a, b)
                else:           # [E, out, r] -> [out, E*r]
                    t = t.permute(1, 0, 2).reshape(a, E * b)
                sd[f"{pre}mlp.experts.{mod}.lora_{ab}.weight"] = t
        return sd

    @torch.no_grad()
    def load_lora_state_dict(self, sd: dict[str, torch.Tensor]):
        for i, layer in enumerate(self.model.layers):
            pre = f"base_model.model.model.layers.{i}."
            for name, p in layer.self_attn.lora.items():
                mod, ab = name.rsplit("_", 1)
                p.copy_(sd[f"{pre}self_attn.{mod}.lora_{ab}.weight"].to(p.device, p.dtype))
            for name, p in layer.mlp.lora.items():
                mod = {"gu": "gate_up_proj", "dn": "down_proj"}[name.split("_")[0]]
                ab = name.split("_")[1]
                t = sd[f"{pre}mlp.experts.{mod}.lora_{ab}.weight"]
                E, a, b = p.shape
                t = t.reshape(E, a, b) if ab == "A" else t.reshape(a, E, b).permute(1, 0, 2)
                p.copy_(t.to(p.device, p.dtype))

    @rpc_method(gather=False)
    def save_model(self, output_dir: str) -> None:
        """PEFT adapter: adapter_model.bin + adapter_config.json (rank 0 writes)."""
        if self.rank != 0:
            return
        out = Path(output_dir)
        out.mkdir(parents=True, exist_ok=True)
        lc = self.model.lora_config
        if lc is None:
            from safetensors.torch import save_file
            save_file({n: p.detach().cpu().contiguous() for n, p in self.model.named_parameters()
                       if p.requires_grad}, str(out / "trainable_params.safetensors"))
            return
        torch.save(self.lora_state_dict(), out / "adapter_model.bin")
        (out / "adapter_config.json").write_text(json.dumps(lc.to_peft_dict(self.config.model_id), indent=2))

    @rpc_method(gather=False)
    def load_model(self, input_dir: str) -> None:
        path = Path(input_dir)
        if (path / "adapter_model.bin").exists():
            sd = torch.load(path / "adapter_model.bin", map_location="cpu", weights_only=True)
            self.load_lora_state_dict(sd)
        elif (path / "adapter_model.safetensors").exists():
            from safetensors.torch import load_file
            self.load_lora_state_dict(load_file(str(path / "adapter_model.safetensors")))
        elif (path / "trainable_params.safetensors").exists():
            from safetensors.torch import load_file
            sd = load_file(str(path / "trainable_params.safetensors"))
            params = dict(self.model.named_parameters())
            with torch.no_grad():
                for k, v in sd.items():
                    params[k].copy_(v.to(params[k].device, params[k].dtype))
        else:
            raise FileNotFoundError(f"no adapter or trainable params under {path}")

    @rpc_method(gather=False)
    def save_merged_weights(self, output_dir: str) -> None:
        """HF-named attention weights with LoRA folded in (merged weight-sync mode)."""
        merged = ckpt.merged_state_dict(self.model)
        if self.rank != 0:
            return
        from safetensors.torch import save_file
        out = Path(output_dir)
        out.mkdir(parents=True, exist_ok=True)
        save_file({k: v.contiguous().cpu() for k, v in merged.items()}, str(out / "model.safetensors"))

    @rpc_method(gather=False)
    def save_training_state(self, output_dir: str) -> None:
        """Optimizer + scheduler state; a sharded optimizer writes one file per rank
        (training_state_rank{r}.pt, each holding that rank's slice of the moments)."""
        state = {"optimizer": self.optimizer.state_dict(), "lr_scheduler": self.lr_scheduler.state_dict(),
                 "step_count": self.step_count}
        Path(output_dir).mkdir(parents=True, exist_ok=True)
        if self.sharded:
            state["world_size"] = self.world_size
            torch.save(state, Path(output_dir) / f"training_state_rank{self.rank}.pt")
        elif self.rank == 0:
            torch.save(state, Path(output_dir) / "training_state.pt")

    def training_state_layout(self, input_dir: str) -> str:
        """"ok" when ``input_dir`` holds optimizer state in the layout this trainer loads
        (per-rank files for the sharded optimizer, one file otherwise), "missing" when it has
        none; raises when it only has the other layout (a sharded run resumed unsharded, or
        the reverse), which would otherwise drop the AdamW moments without a word."""
        d = Path(input_dir)
        mine = d / (f"training_state_rank{self.rank}.pt" if self.sharded else "training_state.pt")
        if mine.exists():
            return "ok"
        other = sorted(d.glob("training_state_rank*.pt")) if not self.sharded else \
            ([d / "training_state.pt"] if (d / "training_state.pt").exists() else [])
        if other:
            raise ValueError(f"{d} holds {'sharded' if not self.sharded else 'replicated'} "
                             f"optimizer state ({other[0].name}) but this trainer "
                             f"{'shards' if self.sharded else 'does not shard'} its optimizer "
                             f"state; resume with the same shard_optimizer_state and world size")
        return "missing"

    @rpc_method(gather=False)
    def load_training_state(self, input_dir: str) -> None:
        path = Path(input_dir) / (f"training_state_rank{self.rank}.pt" if self.sharded
                                  else "training_state.pt")
        state = torch.load(path, map_location=self.device, weights_only=False)
        if self.sharded and state.get("world_size") != self.world_size:
            raise ValueError(f"{path} was saved by {state.get('world_size')} ranks, "
                             f"this job has {self.world_size}")
        self.optimizer.load_state_dict(state["optimizer"])
        self.lr_scheduler.load_state_dict(state["lr_scheduler"])
        self.step_count = int(state.get("step_count", 0))
