"""Data-parallel trainer with the sharded optimizer state (gradients reduce-scattered, AdamW on
each rank's slice, updated slices all-gathered) against the replicated optimizer (one
all-reduce), on two gloo ranks: same parameters after several steps, per-rank optimizer state
holds only the rank's slice, and the per-rank training state round-trips."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _samples(vocab):
    from agent_factory_3_b200.trainer.types import TrainingSample
    rng = np.random.default_rng(10)
    out = []
    for i, n in enumerate([40, 56, 24, 48, 32, 16]):
        comp = np.zeros(n, np.int32)
        comp[n // 3:] = 1
        out.append(TrainingSample(
            sample_id=f"s{i}", input_ids=rng.integers(0, vocab, n).astype(np.int64),
            completion_mask=comp, gen_logprobs=(comp * -6.9).astype(np.float32),
            advantages=(comp * (1.0 if i % 2 else -1.0)).astype(np.float32),
            seq_token_count=int(comp.sum()), prompt_sequence_count=2, prompt_id=f"g{i // 2}",
            divisor=2.0))
    return out


def _run(rank, port, q, tmp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    try:
        from agent_factory_3_b200.models.gpt_oss import GptOssConfig
        from agent_factory_3_b200.trainer.model_trainer import ModelTrainer
        from agent_factory_3_b200.trainer.training_config import TrainingConfig
        mcfg = GptOssConfig.tiny()
        res = {}
        for sharded in (False, True):
            cfg = TrainingConfig(model_id="tiny", lora_r=4, lora_alpha=8,
                                 lora_target_modules=["q_proj", "o_proj", "gate_up_proj", "down_proj"],
                                 random_init_seed=0, use_routing_replay=False, lr_warmup_steps=0,
                                 learning_rate=1e-2, max_capacity=256, pad_to_multiple_of_training=8,
                                 shard_optimizer_state=sharded, gradient_checkpointing=False)
            tr = ModelTrainer(cfg, model_config=mcfg, device="cpu")
            if rank == 0:   # rank 0 drives, rank 1 serves the broadcast calls
                for _ in range(3):
                    tr.train_step(_samples(mcfg.vocab_size))
                if sharded:
                    tr.save_training_state(tmp)
                    before = {k: v.clone() for k, v in tr.optimizer.state[tr.shard_param].items()}
                    tr.reset_optimizer_state()
                    tr.load_training_state(tmp)
                    after = tr.optimizer.state[tr.shard_param]
                    res["roundtrip"] = all(torch.equal(before[k], after[k]) for k in before)
                tr.rpc_shutdown()
            else:
                tr.rpc_worker_loop()
            flat = torch.cat([p.detach().reshape(-1) for p in tr.trainable])
            n_state = sum(v.numel() for st in tr.optimizer.state.values() for v in st.values()
                          if torch.is_tensor(v) and v.dim() > 0)
            res[sharded] = (flat, n_state, tr.sharded)
        q.put((rank, (res[False][0] - res[True][0]).abs().max().item(),
               res[False][0].abs().max().item(), res[False][1], res[True][1], res[True][2],
               res.get("roundtrip", True)))
    finally:
        dist.destroy_process_group()


def test_sharded_optimizer_matches_replicated(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_run, args=(r, port, q, str(tmp_path))) for r in range(2)]
    for p in ps:
        p.start()
    outs = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, diff, scale, n_rep, n_shard, sharded, roundtrip in outs:
        assert sharded
        assert diff <= 1e-5 * max(1.0, scale), (diff, scale)
        assert n_shard * 2 <= n_rep + 64          # each rank keeps ~half of the moments
        assert roundtrip
    assert (tmp_path / "training_state_rank0.pt").exists()
    assert (tmp_path / "training_state_rank1.pt").exists()


def _run_resume(rank, port, q, tmp):
    """Sharded optimizer state saved and restored through RLFlow's checkpoint code."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    try:
        from pathlib import Path

        from agent_factory_3_b200.models.gpt_oss import GptOssConfig
        from agent_factory_3_b200.orchestrator.types import per_rollout
        from agent_factory_3_b200.rollout.config import LoopConfig
        from agent_factory_3_b200.trainer.model_trainer import ModelTrainer
        from agent_factory_3_b200.trainer.rl_flow import RLFlow
        from agent_factory_3_b200.trainer.training_config import TrainingConfig
        mcfg = GptOssConfig.tiny()
        cfg = TrainingConfig(model_id="tiny", lora_r=4, lora_alpha=8,
                             lora_target_modules=["q_proj", "o_proj", "gate_up_proj", "down_proj"],
                             random_init_seed=0, use_routing_replay=False, lr_warmup_steps=0,
                             learning_rate=1e-2, max_capacity=256, pad_to_multiple_of_training=8,
                             shard_optimizer_state=True, gradient_checkpointing=False,
                             run_dir=os.path.join(tmp, "run"))
        tr = ModelTrainer(cfg, model_config=mcfg, device="cpu")
        ck = Path(tmp) / "ckpt"
        if rank == 0:
            flow = RLFlow(training_config=cfg, model_trainer=tr, dataset=[{"prompt": "x"}],
                          reward_fn=per_rollout(lambda r, m: 0.0), server_urls=["http://unused"],
                          loop_config=LoopConfig(), group_size=2, batch_size=2)
            for _ in range(2):
                tr.train_step(_samples(mcfg.vocab_size))
            flow._checkpoint(ck, step=2, batch_idx=2, factory_state=None, run_id=None)
            tr.reset_optimizer_state()
            meta = flow._restore(ck)
            assert meta.step == 2
            tr.rpc_shutdown()
        else:
            tr.rpc_worker_loop()
        saved = torch.load(ck / f"training_state_rank{rank}.pt", weights_only=False)
        mine = tr.optimizer.state_dict()["state"]
        ok = all(torch.equal(saved["optimizer"]["state"][k][n], v[n])
                 for k, v in mine.items() for n in v if torch.is_tensor(v[n]) and v[n].dim() > 0)
        nonzero = any(bool((v["exp_avg_sq"] != 0).any()) for v in mine.values())
        q.put((rank, ok, nonzero, tr.step_count))
    finally:
        dist.destroy_process_group()


def test_sharded_optimizer_resume_through_rl_flow(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_run_resume, args=(r, port, q, str(tmp_path))) for r in range(2)]
    for p in ps:
        p.start()
    outs = sorted(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    for rank, ok, nonzero, steps in outs:
        assert ok and nonzero, (rank, ok, nonzero)
        assert steps == 2


def _run_base_shard(rank, port, q):
    """Experts sharded over the ranks (gathered on use) train exactly like replicated ones."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    try:
        from agent_factory_3_b200.models.gpt_oss import GptOssConfig
        from agent_factory_3_b200.trainer.model_trainer import ModelTrainer
        from agent_factory_3_b200.trainer.training_config import TrainingConfig
        mcfg = GptOssConfig.tiny()
        res = {}
        for shard in (False, True):
            cfg = TrainingConfig(model_id="tiny", lora_r=4, lora_alpha=8,
                                 lora_target_modules=["q_proj", "o_proj", "gate_up_proj", "down_proj"],
                                 random_init_seed=0, use_routing_replay=False, lr_warmup_steps=0,
                                 learning_rate=1e-2, max_capacity=256, pad_to_multiple_of_training=8,
                                 shard_base_weights=shard, gradient_checkpointing=False)
            tr = ModelTrainer(cfg, model_config=mcfg, device="cpu")
            E = mcfg.num_local_experts
            n_local = tr.model.layers[0].mlp.gate_up_blocks.shape[0]
            losses = []
            if rank == 0:
                for _ in range(2):
                    losses.append(tr.train_step(_samples(mcfg.vocab_size))["loss"])
                tr.rpc_shutdown()
            else:
                tr.rpc_worker_loop()
            flat = torch.cat([p.detach().reshape(-1) for p in tr.trainable])
            res[shard] = (flat, losses, n_local, E)
        q.put((rank, (res[False][0] - res[True][0]).abs().max().item(), res[False][1],
               res[True][1], res[False][2], res[True][2], res[True][3]))
    finally:
        dist.destroy_process_group()


def test_sharded_base_weights_match_replicated():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_run_base_shard, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    outs = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, diff, loss_rep, loss_sh, n_rep, n_sh, E in outs:
        assert n_rep == E and n_sh == E // 2          # each rank holds half of the experts
        assert diff <= 1e-6, diff
        if rank == 0:
            assert loss_rep == loss_sh
