"""Shared driver of the examples: async agentic RL of gpt-oss with LoRA against the built-in
rollout engine (the reference's examples/*/train.py:136-264 build the same pieces around
accelerate + sglang).

Launch the engine first (``serve.sh``), then the trainer (``run_train.sh``).  Under torchrun,
rank 0 runs the RL loop and drives the other ranks' trainers through the RPC control plane;
the other ranks only serve training steps.
"""
from __future__ import annotations

import argparse
import os
import sys

PY = sys.executable


def base_args(default_model: str = "gpt-oss-20b") -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default=os.environ.get("MODEL_PATH", default_model),
                    help="preset name (random-init weights) or HF-format checkpoint directory")
    ap.add_argument("--run-dir", default=os.environ.get("RUN_DIR", "./runs/example"))
    ap.add_argument("--server-urls", default=os.environ.get("SGLANG_URLS", "http://127.0.0.1:30000"),
                    help="comma-separated engine server URLs")
    ap.add_argument("--batch-size", type=int, default=64, help="rollouts per training step")
    ap.add_argument("--group-size", type=int, default=8)
    ap.add_argument("--max-batches", type=int, default=None)
    ap.add_argument("--lora-r", type=int, default=32)
    ap.add_argument("--lora-alpha", type=int, default=64)
    ap.add_argument("--learning-rate", type=float, default=2e-5)
    ap.add_argument("--max-capacity", type=int, default=65536, help="packed tokens per microbatch")
    ap.add_argument("--max-rounds", type=int, default=8, help="tool-call rounds per rollout")
    ap.add_argument("--max-total-tokens", type=int, default=16384)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--num-workers", type=int, default=8)
    ap.add_argument("--worker-concurrency", type=int, default=16)
    ap.add_argument("--seed", type=int, default=0)
    return ap


def run(a, dataset: list[dict], reward, env_name: str) -> None:
    """Build the trainer and the RL loop from the parsed ``a`` and run it."""
    from agent_factory_3_b200.models.gpt_oss import GptOssConfig
    from agent_factory_3_b200.orchestrator.types import per_rollout
    from agent_factory_3_b200.rollout.config import LoopConfig, RecordConfig, SamplingParams
    from agent_factory_3_b200.trainer.model_trainer import ModelTrainer
    from agent_factory_3_b200.trainer.rl_flow import RLFlow
    from agent_factory_3_b200.trainer.training_config import TrainingConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(hours=6))
    targets = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_up_proj", "down_proj"]
    tc = TrainingConfig(model_id=a.model, lora_r=a.lora_r, lora_alpha=a.lora_alpha,
                        lora_target_modules=targets, learning_rate=a.learning_rate,
                        max_capacity=a.max_capacity, run_dir=a.run_dir, random_init_seed=a.seed,
                        use_routing_replay=True)
    trainer = ModelTrainer(tc)
    if rank != 0:
        trainer.rpc_worker_loop()
        return
    cfg: GptOssConfig = trainer.model.cfg
    loop = LoopConfig(max_rounds=a.max_rounds, max_total_tokens=a.max_total_tokens,
                      max_round_tokens=min(8192, a.max_total_tokens),
                      num_hidden_layers=cfg.num_hidden_layers,
                      num_experts_per_tok=cfg.num_experts_per_tok, lora_adapter_name="policy",
                      sampling=SamplingParams(temperature=a.temperature))
    flow = RLFlow(training_config=tc, model_trainer=trainer, dataset=dataset,
                  reward_fn=per_rollout(reward), server_urls=a.server_urls.split(","),
                  num_workers=a.num_workers, worker_concurrency=a.worker_concurrency,
                  batch_size=a.batch_size, group_size=a.group_size, loop_config=loop,
                  record_config=RecordConfig(logprobs=True, routing_indices=True),
                  max_batches=a.max_batches, base_seed=a.seed)
    try:
        flow.run(on_step=lambda m, i: print(f"[{env_name}] step {i}: loss {m.get('loss'):.4f} "
                                              f"reward {m.get('reward/mean', float('nan')):.3f}",
                                              flush=True))
    finally:
        if world > 1:
            trainer.rpc_shutdown()
    print(f"[{env_name}] done; checkpoints in {tc.checkpoint_dir}", flush=True)


def mcp_server(module: str, *args: str) -> dict:
    """An MCP config running one of this package's environment servers over stdio."""
    return {"mcpServers": {module.rsplit(".", 1)[-1]: {"command": PY, "args": ["-m", module, *args]}}}
