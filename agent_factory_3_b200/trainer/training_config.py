"""Trainer configuration (field names of the reference's TrainingConfig,
trainer/training_config.py:19-192, plus the B200 engine's own knobs)."""
from __future__ import annotations

from pathlib import Path
from typing import Literal

from pydantic import BaseModel, computed_field, model_validator

LRSchedulerType = Literal["linear", "cosine", "cosine_with_restarts", "polynomial", "constant",
                          "constant_with_warmup", "inverse_sqrt"]


class TrainingConfig(BaseModel):
    # model
    model_id: str = "gpt-oss-120b"          # preset name or HF-format checkpoint directory
    attn_implementation: str = "sm100"       # kept for config compatibility; one kernel path
    gradient_checkpointing: bool = True
    # GB of full-attention layer outputs (O + LSE) kept from the forward so the checkpoint
    # recompute skips those attention kernels; 0 recomputes everything
    attention_cache_gb: float = 0.0
    use_reentrant: bool = False
    model_use_cache: bool = False
    model_init_kwargs: dict | None = None
    random_init_seed: int | None = None      # preset models: random-init weights (MXFP4 experts)
    # training mode
    training_mode: str = "lora"
    trainable_modules: list[str] | None = None
    # LoRA
    lora_r: int = 8
    lora_alpha: int = 32
    lora_target_modules: list[str] = ["q_proj", "k_proj", "v_proj", "o_proj"]
    lora_dropout: float = 0.0
    autocast_adapter_dtype: bool = True
    lora_kwargs: dict | None = None
    # optimizer
    learning_rate: float = 2e-4
    weight_decay: float = 0.0
    optimizer_type: str = "AdamW"
    adam_beta1: float = 0.9
    adam_beta2: float = 0.95
    adam_epsilon: float = 1e-8
    max_grad_norm: float = 1.0
    # data parallelism: shard the fp32 master copy and AdamW moments of the trainable tensors
    # over the ranks (gradients reduce-scattered, updated shards all-gathered), the optimizer
    # state sharding of FSDP2 / ZeRO-2; the frozen base model stays replicated
    shard_optimizer_state: bool = True
    # with the sharded optimizer on GPUs: "nccl" runs one reduce-scatter after the backward;
    # "push" copies each gradient to its owner rank over NVLink (copy engines) as soon as the
    # backward finalises it and reduces locally (parallel/grad_push.py).  Measured on 2 B200
    # with gpt-oss-120b (131k tokens per GPU): 19.4 s per step with "nccl", 21.9 s with "push"
    # -- the pushes' HBM and NVLink traffic slows the backward more than the overlap saves
    grad_reduce: Literal["push", "nccl"] = "nccl"
    # expert GEMMs of training: "bf16" dequantised experts, or "fp8" (e4m3 experts with one
    # scale per expert, e4m3 activations and gradients with one scale per row; the
    # reference's quantizer_config.dequant_dtype)
    dequant_dtype: Literal["bf16", "fp8"] = "bf16"
    lr_scheduler_type: LRSchedulerType = "constant_with_warmup"
    lr_warmup_steps: int = 20
    # DDIS / OPSM / entropy mask
    ddis_eps_low: float = 0.2
    ddis_eps_high: float = 0.2
    use_opsm: bool = False
    opsm_delta: float = 1e-4
    entropy_top_pct: float | None = None
    # loss
    loss_temperature: float = 1.0
    loss_backend: str = "sm100"              # fused tcgen05 linear-logprob ("torch" = chunked oracle)
    loss_aggregation_mode: str = "seq-mean-token-sum"
    # multi-step
    num_inner_steps: int = 1
    # packing
    max_capacity: int = 20000
    pad_to_multiple_of_training: int = 1024
    # rank balancing of the packing plan: "tokens" (the reference's rule) or "cost" (tokens
    # plus the quadratic attention work, n + n^2 / packing_attention_tokens per sample).  The
    # default is the sequence length at which a sample's attention time equals the rest of its
    # step time. It comes from a gpt-oss-120b step on one B200 (131072 tokens in two samples of
    # 112105 and 18967):
    #   - attention forward + backward: 11.2 s, over sum(n^2) = 1.29e10;
    #   - everything else: 4.7 s, over 131072 tokens;
    #   - (4.7 / 131072) / (11.2 / 1.29e10) = about 41k tokens.
    packing_balance: Literal["tokens", "cost"] = "cost"
    packing_attention_tokens: int = 40960
    dataloader_num_workers: int = 0
    # routing replay
    use_routing_replay: bool = True
    save_routing_indices: bool | None = None
    # weight sync
    weight_sync_interval: int = 1
    min_weight_sync_secs: float = 0.0
    weight_sync_mode: str = "lora"
    flush_cache_on_sync: bool = True
    flush_cache_every_n_steps: int = 0
    reset_optimizer_on_sync: bool = False
    lora_adapter_name: str = "policy"
    # staleness
    max_staleness: int = 2
    # paths / checkpoints
    run_dir: str = "./runs/default"
    save_checkpoint_every: int = 5
    save_latest_checkpoint: bool = True
    resume_from_checkpoint: str | None = None
    max_checkpoints_to_keep: int = 0
    # wandb
    use_wandb: bool = False
    wandb_project: str = "agent-factory-3"
    wandb_run_name: str | None = None
    wandb_tags: list[str] = []
    wandb_notes: str = ""
    wandb_resume: bool = True
    # parallelism (B200 engine)
    # FSDP-style sharding of the frozen MXFP4 experts over the data-parallel ranks; a layer's
    # experts are gathered over NVLink inside their dequantisation kernel (parallel/fsdp.py)
    shard_base_weights: bool = False

    @computed_field
    @property
    def checkpoint_dir(self) -> str:
        return str(Path(self.run_dir) / "checkpoints")

    @computed_field
    @property
    def rollout_dir(self) -> str:
        return str(Path(self.run_dir) / "rollouts")

    @computed_field
    @property
    def weight_sync_dir(self) -> str:
        return str(Path(self.run_dir) / "weight_sync")

    @model_validator(mode="after")
    def _validate(self) -> "TrainingConfig":
        if self.training_mode not in ("lora", "full"):
            raise ValueError(f"training_mode must be 'lora' or 'full', got {self.training_mode!r}")
        if self.weight_sync_mode not in ("lora", "merged"):
            raise ValueError("weight_sync_mode must be 'lora' or 'merged'")
        if self.training_mode == "full" and self.weight_sync_mode == "lora":
            raise ValueError("full-parameter training needs weight_sync_mode='merged'")
        if self.num_inner_steps < 1:
            raise ValueError("num_inner_steps must be >= 1")
        if self.max_capacity <= 0 or self.pad_to_multiple_of_training <= 0:
            raise ValueError("max_capacity and pad_to_multiple_of_training must be positive")
        if self.max_capacity % self.pad_to_multiple_of_training and self.pad_to_multiple_of_training > 1:
            pass  # padding may exceed capacity by < pad multiple; allowed as in the reference
        if self.loss_aggregation_mode not in ("seq-mean-token-sum", "seq-mean-token-mean",
                                              "token-mean", "prompt-mean-token-mean"):
            raise ValueError(f"unknown loss_aggregation_mode {self.loss_aggregation_mode!r}")
        if self.entropy_top_pct is not None and not (0 < self.entropy_top_pct <= 100):
            raise ValueError("entropy_top_pct must be in (0, 100]")
        return self
