#!/usr/bin/env python
"""Headline benchmark: gpt-oss-120b MXFP4 LoRA RL training step on B200s.

Config: gpt-oss-120b architecture with random-init weights (experts
quantized to MXFP4), LoRA r=32 / alpha=64 on attention and experts, per GPU one packed
microbatch of 131072 tokens made of samples with lengths uniform in [4096, 131072], R3 replay of
recorded (synthetic) top-4 expert ids, activation checkpointing, fused linear-logprob/entropy
over the 201088 vocabulary, DDIS loss against synthetic rollout log-probs, AdamW step.
Weak scaling: every rank trains its own 131072 tokens; gradients are all-reduced over NCCL.

    python bench.py --gpus N --steps K --warmup W            (N>1 under torch.distributed.run)
    python bench.py --impl reference ...                     (the reference's own stack)

Prints one JSON line on rank 0.  ``value`` is the device-timed throughput (CUDA events around
K steps, max over ranks); ``e2e`` is the same K steps measured by the host clock through the
public API (``ModelTrainer.train_packed_batch``) including the host->device copy of each step's
pinned inputs and the device->host read of each step's loss.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

METRIC = "gpt-oss-120b MXFP4 LoRA RL train tok/s + TP rollout decode tok/s, 1/2/4/8 B200"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="gpt-oss-120b")
    ap.add_argument("--tokens", type=int, default=131072, help="packed tokens per GPU")
    ap.add_argument("--min-len", type=int, default=4096)
    ap.add_argument("--max-len", type=int, default=131072)
    ap.add_argument("--lora-r", type=int, default=32)
    ap.add_argument("--lora-alpha", type=int, default=64)
    ap.add_argument("--layers", type=int, default=None, help="(debug only) override layer count")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--shard-optimizer", action="store_true",
                    help="shard the LoRA optimizer state over the ranks (reduce-scatter + "
                         "all-gather) instead of one all-reduce")
    ap.add_argument("--trace", default=None,
                    help="after the timed steps, run one more step under torch.profiler and write "
                         "its per-kernel device-time table (text) to this path")
    return ap.parse_args()


def write_trace(step, path: str) -> None:
    """One untimed step under torch.profiler: kernel table sorted by device time."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    table = prof.key_averages().table(sort_by="self_device_time_total", row_limit=60,
                                      max_name_column_width=90)
    with open(path, "w") as f:
        f.write(table)


def reference_unavailable(args) -> None:
    reason = ("reference training path cannot run offline: it imports triton_kernels "
              "(matmul_ogs, routing) and accelerate/peft, which are not installed and not in "
              "the wheelhouse (pip --no-deps install into baseline/_ref succeeds, import fails)")
    try:
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref"))
        import agent_factory_3.models.gpt_oss.quantization  # noqa: F401
        import agent_factory_3.trainer.model_trainer  # noqa: F401
        reason = "reference imports but its FSDP2/accelerate launch path is not wired in this bench"
    except Exception as e:  # noqa: BLE001
        reason += f" ({type(e).__name__}: {e})"
    print(json.dumps({"impl": "reference", "unavailable": reason}))


class ClockSampler:
    """nvidia-smi clocks / throttle reasons of this process's GPU while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.samples: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm = []
        maxes = []
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            try:
                sm.append(float(s[0]))
                maxes.append(float(s[1]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, s[4:8]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_samples(args, rank: int, n_layers: int, n_experts: int, top_k: int, vocab: int, device):
    """Synthetic agentic traces of one rank: random ids, a prompt prefix, rollout log-probs,
    group-normalised Bernoulli advantages and recorded top-k expert ids per layer."""
    import numpy as np
    import torch

    from agent_factory_3_b200.trainer.types import TrainingSample

    rng = np.random.default_rng(args.seed * 1000 + rank)
    lens = []
    left = args.tokens
    while left > 0:
        n = int(rng.integers(args.min_len, args.max_len + 1))
        n = min(n, left)
        lens.append(n)
        left -= n
    rewards = rng.integers(0, 2, size=len(lens)).astype(np.float32)
    adv = rewards - rewards.mean()
    if adv.std() > 0:
        adv = adv / (adv.std() + 1e-6)
    else:
        adv = np.where(np.arange(len(lens)) % 2 == 0, 1.0, -1.0).astype(np.float32)
    g = torch.Generator(device=device).manual_seed(args.seed * 1000 + rank)
    samples = []
    for i, n in enumerate(lens):
        prompt = min(2048, n // 4)
        comp = np.zeros(n, np.int32)
        comp[prompt:] = 1
        ids = rng.integers(0, vocab, n).astype(np.int64)
        gen = np.where(comp > 0, -np.log(vocab) + rng.normal(0, 0.05, n), 0).astype(np.float32)
        # distinct random experts per (token, layer)
        r = torch.rand(n * n_layers, n_experts, generator=g, device=device)
        routing = r.topk(top_k, dim=-1).indices.to(torch.uint8).reshape(n, n_layers, top_k).cpu().numpy()
        samples.append(TrainingSample(
            sample_id=f"r{rank}s{i}", input_ids=ids, completion_mask=comp, gen_logprobs=gen,
            advantages=(comp * adv[i]).astype(np.float32), routing_indices=routing,
            seq_token_count=int(comp.sum()), prompt_sequence_count=8, prompt_id=f"g{i // 8}",
            divisor=8.0))
    return samples, lens


def main():
    args = parse_args()
    if args.impl == "reference":
        reference_unavailable(args)
        return
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=device)

    from agent_factory_3_b200.models.gpt_oss import GptOssConfig
    from agent_factory_3_b200.ops import _ext
    from agent_factory_3_b200.trainer.model_trainer import ModelTrainer
    from agent_factory_3_b200.trainer.training_config import TrainingConfig

    mcfg = GptOssConfig.preset(args.model)
    if args.layers:
        mcfg = GptOssConfig.preset(args.model)
        mcfg.num_hidden_layers = args.layers
        mcfg.layer_types = mcfg.layer_types[: args.layers]
    tcfg = TrainingConfig(
        model_id=args.model, lora_r=args.lora_r, lora_alpha=args.lora_alpha,
        lora_target_modules=["q_proj", "k_proj", "v_proj", "o_proj", "gate_up_proj", "down_proj"],
        max_capacity=args.tokens, pad_to_multiple_of_training=1024, random_init_seed=0,
        use_routing_replay=True, gradient_checkpointing=True, lr_warmup_steps=0,
        learning_rate=1e-5, shard_optimizer_state=args.shard_optimizer)
    t_init = time.perf_counter()
    trainer = ModelTrainer(tcfg, model_config=mcfg, device=device)
    torch.cuda.synchronize()
    t_init = time.perf_counter() - t_init
    samples, lens = make_samples(args, rank, mcfg.num_hidden_layers, mcfg.num_local_experts,
                                 mcfg.num_experts_per_tok, mcfg.vocab_size, device)
    host_batch = trainer.collator(samples)
    tokens_per_rank = int(host_batch["num_tokens"])
    h2d_bytes = sum(v.numel() * v.element_size() for k, v in host_batch.items()
                    if isinstance(v, torch.Tensor) and k != "cu_seqlens")

    def step():
        loss = trainer.train_packed_batch(host_batch)
        return loss.item()  # device->host read of the step's result

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    clocks = ClockSampler(uuid)
    clocks.start()
    launches0 = _ext.launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    ev0.record()
    losses = []
    for _ in range(args.steps):
        losses.append(step())
    ev1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = _ext.launch_count() - launches0
    dev_ms = ev0.elapsed_time(ev1) / args.steps
    wall_ms = wall * 1000.0 / args.steps
    stats = torch.tensor([dev_ms, wall_ms], device=device, dtype=torch.float64)
    tok = torch.tensor([float(tokens_per_rank)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        dist.all_reduce(tok, op=dist.ReduceOp.SUM)
    dev_ms, wall_ms = stats.tolist()
    total_tokens = tok.item()
    value = total_tokens / (dev_ms / 1000.0)
    e2e = total_tokens / (wall_ms / 1000.0)
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "tokens/s (train, whole job)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_ms, 2),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random token ids, random-init weights, MXFP4 experts)",
            "impl": "ours",
            "config": {"model": args.model, "global_batch": int(total_tokens),
                       "tokens_per_gpu": tokens_per_rank, "seq_len": args.max_len,
                       "sample_lengths": f"uniform[{args.min_len},{args.max_len}] packed",
                       "samples_per_gpu": len(lens), "lora": f"r{args.lora_r}/a{args.lora_alpha} attn+experts",
                       "routing_replay": True, "activation_checkpointing": True,
                       "parallelism": f"dp{world}" if world > 1 else "single",
                       "layers": mcfg.num_hidden_layers,
                       "l2": "inputs larger than L2 (65 GB of weights stream every step)"},
            "clocks": clk,
            "e2e": {"value": round(e2e, 1), "unit": "tokens/s (train, whole job)",
                    "h2d_bytes_per_step": int(h2d_bytes), "d2h_bytes_per_step": 4,
                    "api": "ModelTrainer.train_packed_batch"},
            "gpu_launches": int(launches),
            "init_s": round(t_init, 1),
            "max_mem_gb": round(torch.cuda.max_memory_allocated(device) / 1e9, 1),
            "loss": losses[-1],
        }
        print(json.dumps(out), flush=True)
    if args.trace:
        write_trace(step, args.trace if world == 1 else f"{args.trace}.rank{rank}")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
