"""Sharded frozen experts on two GPUs: every rank keeps half of each layer's MXFP4 experts in a
peer-mapped buffer, the dequantisation kernel gathers the other half over NVLink, the gathered
bf16 stack equals the replicated one bit for bit, and training gives the same parameters."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg():
    from agent_factory_3_b200.models.gpt_oss import GptOssConfig
    return GptOssConfig(vocab_size=2048, hidden_size=256, intermediate_size=256,
                        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                        head_dim=64, num_local_experts=8, num_experts_per_tok=2,
                        sliding_window=64, rope_scaling=None, max_position_embeddings=4096,
                        pad_token_id=0, eos_token_id=1)


def _worker(rank, world, port, q):
    import numpy as np
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    out = {}
    try:
        from agent_factory_3_b200.trainer.model_trainer import ModelTrainer
        from agent_factory_3_b200.trainer.training_config import TrainingConfig
        from agent_factory_3_b200.trainer.types import TrainingSample
        mcfg = _cfg()
        rng = np.random.default_rng(5)
        samples = []
        for i in range(4):
            n = int(rng.integers(100, 300))
            comp = np.zeros(n, np.int32)
            comp[n // 3:] = 1
            samples.append(TrainingSample(
                sample_id=str(i), input_ids=rng.integers(0, mcfg.vocab_size, n),
                completion_mask=comp, gen_logprobs=np.where(comp > 0, -7.6, 0).astype(np.float32),
                advantages=(comp * (1.0 if i % 2 else -1.0)).astype(np.float32),
                seq_token_count=int(comp.sum()), prompt_sequence_count=2, divisor=2.0))
        params, stacks = {}, {}
        for shard in (False, True):
            cfg = TrainingConfig(model_id="t", lora_r=8, lora_alpha=16,
                                 lora_target_modules=["q_proj", "o_proj", "gate_up_proj", "down_proj"],
                                 max_capacity=1024, pad_to_multiple_of_training=128,
                                 random_init_seed=0, lr_warmup_steps=0, learning_rate=1e-3,
                                 use_routing_replay=False, shard_base_weights=shard)
            tr = ModelTrainer(cfg, model_config=mcfg, device=dev)
            mlp = tr.model.layers[1].mlp
            out[f"local_experts_{shard}"] = mlp.gate_up_blocks.shape[0]
            stacks[shard] = (mlp.experts().gate_up().clone(), mlp.experts().down().clone())
            if rank == 0:
                for _ in range(2):
                    tr.train_step(samples)
                tr.rpc_shutdown()
            else:
                tr.rpc_worker_loop()
            torch.cuda.synchronize()
            params[shard] = torch.cat([p.detach().reshape(-1) for p in tr.trainable]).cpu()
            del tr
        out["stack_equal"] = all(torch.equal(a, b) for a, b in zip(stacks[False], stacks[True]))
        out["param_diff"] = (params[False] - params[True]).abs().max().item()
        out["param_scale"] = params[False].abs().max().item()
    except Exception as e:  # noqa: BLE001
        out["error"] = repr(e)
    q.put((rank, out))
    dist.destroy_process_group()


def test_sharded_experts_gathered_over_nvlink_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q), daemon=True) for r in range(2)]
    for p in ps:
        p.start()
    try:
        outs = dict(q.get(timeout=600) for _ in range(2))
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, o in outs.items():
        assert "error" not in o, o
        assert o["local_experts_False"] == 8 and o["local_experts_True"] == 4
        assert o["stack_equal"]
        assert o["param_diff"] <= 1e-6 * max(1.0, o["param_scale"]), o
