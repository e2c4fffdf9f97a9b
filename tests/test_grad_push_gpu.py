"""Overlapped gradient reduce-scatter (copy-engine pushes into peer-mapped inboxes + local
reduction) against NCCL reduce_scatter, on two GPUs: the reduced shards and their sums of
squares agree to fp32 rounding, and a sharded-optimizer trainer ends with the same parameters
with either reduction."""
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
        from agent_factory_3_b200.parallel.grad_push import GradientPusher
        S = 1 << 16
        g = torch.Generator(device=dev).manual_seed(rank + 1)
        flat = torch.randn(world * S, generator=g, device=dev)
        shard = torch.zeros(S, device=dev)
        dummy = torch.zeros(world * S, device=dev, requires_grad=True)
        pusher = GradientPusher([dummy], [0], flat, shard, timeout_s=60.0)
        errs = []
        for _ in range(2):       # second call reuses the inbox and the next epoch
            sq = pusher.finish().clone()
            ref = torch.empty(S, device=dev)
            dist.reduce_scatter_tensor(ref, flat.clone())
            torch.cuda.synchronize()
            errs.append(((shard - ref).abs().max().item(), ref.abs().max().item(),
                         abs(sq.item() - float(ref.pow(2).sum())) / float(ref.pow(2).sum())))
            flat.mul_(0.5)
        pusher.check()
        pusher.close()
        out["unit"] = errs

        from agent_factory_3_b200.models.gpt_oss import GptOssConfig
        from agent_factory_3_b200.trainer.model_trainer import ModelTrainer
        from agent_factory_3_b200.trainer.training_config import TrainingConfig
        from agent_factory_3_b200.trainer.types import TrainingSample
        mcfg = GptOssConfig(vocab_size=2048, hidden_size=256, intermediate_size=256,
                            num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                            head_dim=64, num_local_experts=8, num_experts_per_tok=2,
                            sliding_window=64, rope_scaling=None, max_position_embeddings=4096,
                            pad_token_id=0, eos_token_id=1)
        rng = np.random.default_rng(3)
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
        params = {}
        for mode in ("nccl", "push"):
            cfg = TrainingConfig(model_id="t", lora_r=8, lora_alpha=16,
                                 lora_target_modules=["q_proj", "k_proj", "v_proj", "o_proj",
                                                      "gate_up_proj", "down_proj"],
                                 max_capacity=1024, pad_to_multiple_of_training=128,
                                 random_init_seed=0, lr_warmup_steps=0, learning_rate=1e-3,
                                 use_routing_replay=False, shard_optimizer_state=True,
                                 grad_reduce=mode)
            tr = ModelTrainer(cfg, model_config=mcfg, device=dev)
            assert (tr.grad_pusher is not None) == (mode == "push")
            if rank == 0:
                for _ in range(2):
                    tr.train_step(samples)
                tr.rpc_shutdown()
            else:
                tr.rpc_worker_loop()
            torch.cuda.synchronize()
            params[mode] = torch.cat([p.detach().reshape(-1) for p in tr.trainable]).cpu()
            if tr.grad_pusher is not None:
                out["pushes"] = tr.grad_pusher.pushes
                tr.grad_pusher.check()
                tr.grad_pusher.close()
            del tr
        out["param_diff"] = (params["nccl"] - params["push"]).abs().max().item()
        out["param_scale"] = params["nccl"].abs().max().item()
    except Exception as e:  # noqa: BLE001
        out["error"] = repr(e)
    q.put((rank, out))
    dist.destroy_process_group()


def test_pushed_reduce_scatter_matches_nccl_two_gpus():
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
        for diff, scale, rel_sq in o["unit"]:
            assert diff <= 1e-5 * max(1.0, scale), (rank, diff)
            assert rel_sq < 1e-5
        assert o["pushes"] > 0
        assert o["param_diff"] <= 1e-5 * max(1.0, o["param_scale"]), o
