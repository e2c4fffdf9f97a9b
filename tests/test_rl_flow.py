"""End-to-end async RL loop on CPU: tiny gpt-oss engine behind the HTTP API, orchestrator,
rewards, sample processing, DDIS train steps, LoRA weight sync into the engine, checkpoints
and resume of the dataset position."""
import hashlib
import json

import torch

from agent_factory_3_b200.engine.local import LocalEngineServer
from agent_factory_3_b200.engine.scheduler import Engine
from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM, LoraConfig
from agent_factory_3_b200.orchestrator.types import per_rollout
from agent_factory_3_b200.rollout.config import LoopConfig, RecordConfig, SamplingParams
from agent_factory_3_b200.trainer.checkpoint_utils import read_meta
from agent_factory_3_b200.trainer.model_trainer import ModelTrainer
from agent_factory_3_b200.trainer.rl_flow import RLFlow
from agent_factory_3_b200.trainer.training_config import TrainingConfig
from agent_factory_3_b200.trainer.training_data_reader import iter_samples


def _reward(r, meta):
    toks = r.result.tokens if r.result is not None else []
    return float(int(hashlib.md5(str(toks).encode()).hexdigest(), 16) % 2)


def _tiny_full_vocab():
    # harmony special tokens (ids 199998-200012) need the real 201088-entry vocabulary
    cfg = GptOssConfig.tiny()
    cfg.vocab_size = 201088
    cfg.pad_token_id, cfg.eos_token_id = 199999, 200002
    return cfg


def test_rl_flow_end_to_end(tmp_path):
    targets = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_up_proj", "down_proj"]
    tc = TrainingConfig(model_id="tiny", lora_r=4, lora_alpha=8, lora_target_modules=targets,
                        max_capacity=4096, pad_to_multiple_of_training=64, random_init_seed=0,
                        run_dir=str(tmp_path / "run"), save_checkpoint_every=2, max_staleness=4,
                        lr_warmup_steps=0, use_routing_replay=True)
    trainer = ModelTrainer(tc, model_config=_tiny_full_vocab(), device="cpu")
    served = GptOssForCausalLM(_tiny_full_vocab(), LoraConfig(r=4, lora_alpha=8, target_modules=targets),
                               dtype=torch.float32)
    served.load_state_dict(trainer.model.state_dict())
    served.eval()
    srv = LocalEngineServer(Engine(served, num_pages=256, page_size=16).start()).start()
    loop_cfg = LoopConfig(max_rounds=1, max_round_tokens=24, max_total_tokens=64, max_aborts=5,
                          use_streaming=False, num_hidden_layers=2, num_experts_per_tok=2,
                          lora_adapter_name="policy", sampling=SamplingParams(temperature=1.0))
    dataset = [{"prompt": f"task {i}"} for i in range(6)]
    steps = []
    try:
        flow = RLFlow(training_config=tc, model_trainer=trainer, dataset=dataset,
                      reward_fn=per_rollout(_reward), server_urls=[srv.url], num_workers=1,
                      worker_concurrency=4, batch_size=8, group_size=4, loop_config=loop_cfg,
                      record_config=RecordConfig(logprobs=True, routing_indices=True),
                      max_batches=2, orchestrator_mode="thread", worker_mode="inproc",
                      filter_all_failed=False, filter_all_solved=False)
        metrics = flow.run(on_step=lambda m, i: steps.append(i))
    finally:
        srv.stop()
    assert len(metrics) >= 1 and steps
    assert all(torch.isfinite(torch.tensor(m["loss"])) for m in metrics)
    assert "algo/ratio_mean" in metrics[0] and "reward/mean" in metrics[0]
    # the engine received the trained adapter
    assert srv.engine.loras.get("policy") is not None
    assert srv.engine.weight_version in ("1", "2")
    ckpt = tmp_path / "run" / "checkpoints" / "checkpoint_latest"
    meta = read_meta(ckpt)
    fs = meta.factory_state     # progress counts whole epochs (the iterator may have wrapped)
    assert meta.batch_idx == 2 and fs["current_epoch"] * fs["dataset_size"] + fs["current_position"] >= 4
    assert (ckpt / "adapter_model.bin").exists() and (ckpt / "training_state.pt").exists()
    npz = sorted((tmp_path / "run" / "rollouts").glob("batch_*.npz"))
    assert npz and (tmp_path / "run" / "rollouts" / "batch_0000.html").exists()
    rec = next(iter_samples(npz[0]))
    assert rec["token_ids"].shape == rec["completion_mask"].shape
    assert rec["routing_indices"].shape[1:] == (2, 2)
