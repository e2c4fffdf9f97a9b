"""Tensor-parallel engine on two gloo ranks (CPU): the sharded forward pass (attention heads and
KV cache split, experts split, partial sums all-reduced with the residual and the next RMSNorm)
gives the logits of the single-process runner, and the scheduler on rank 0 drives rank 1
through the per-step broadcast."""
import datetime
import os
import socket
import threading

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from agent_factory_3_b200.engine.kv_cache import PagedKVCache
from agent_factory_3_b200.engine.model_runner import ModelRunner, StepItem
from agent_factory_3_b200.engine.scheduler import Engine, Request
from agent_factory_3_b200.engine.tp import TPContext, TPModelRunner, shard_model
from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    cfg = GptOssConfig.tiny()
    return GptOssForCausalLM(cfg, device="cpu", dtype=torch.bfloat16).init_random(0).eval()


def _kv(cfg, world):
    return PagedKVCache(cfg.num_hidden_layers, 32, 8, cfg.num_key_value_heads // world,
                        cfg.head_dim, cfg.num_experts_per_tok, "cpu", torch.bfloat16)


def _steps():
    g = torch.Generator().manual_seed(1)
    a = torch.randint(0, 1000, (13,), generator=g).tolist()
    b = torch.randint(0, 1000, (6,), generator=g).tolist()
    prefill = [StepItem(a, 0, [0, 1]), StepItem(b, 0, [2])]
    decode = [StepItem([5], 13, [0, 1]), StepItem([7], 6, [2])]
    return [prefill, decode]


def _run(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    try:
        torch.manual_seed(0)
        model = _model()
        cfg = model.cfg
        ctx = TPContext()
        shards = shard_model(model, rank, 2)
        runner = TPModelRunner(model, _kv(cfg, 2), ctx, shards)
        if rank == 0:
            ref = ModelRunner(model, _kv(cfg, 1), lora_active=False)
            diffs = []
            for items in _steps():
                want = ref.forward(items)
                got = runner.forward(items)
                diffs.append(((got.logits - want.logits).abs().max().item(),
                              want.logits.abs().max().item(),
                              bool(torch.equal(got.routing, want.routing))))
            runner.stop_followers()
            # engine-level: the scheduler on rank 0 steps rank 1 through the broadcast
            eng = Engine(model, num_pages=32, page_size=8, max_running=4, tp=ctx,
                         tp_shards=shards).start()
            done = threading.Event()
            req = Request(input_ids=list(range(3, 20)), max_new_tokens=6, temperature=0.0)
            req.on_output = lambda out: done.set() if out["finished"] else None
            eng.submit(req)
            ok = done.wait(120)
            eng.stop()
            q.put(("r0", diffs, ok, list(req.output_ids)))
        else:
            n1 = runner.follow()
            eng = Engine(model, num_pages=32, page_size=8, max_running=4, tp=ctx, tp_shards=shards)
            n2 = eng.runner.follow()
            q.put(("r1", n1, n2))
    finally:
        dist.destroy_process_group()


def test_tp2_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_run, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    outs = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    r0 = next(o for o in outs if o[0] == "r0")
    r1 = next(o for o in outs if o[0] == "r1")
    for err, scale, same_routing in r0[1]:
        assert err <= 0.05 * max(1.0, scale), (err, scale)
        assert same_routing
    assert r1[1] == 2                       # both runner steps were followed
    assert r0[2] and len(r0[3]) == 6        # the engine finished its request
    assert r1[2] >= 6                       # ... driving rank 1 through every step


def _run_lora(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    try:
        from agent_factory_3_b200.models.gpt_oss import LoraConfig
        cfg = GptOssConfig.tiny()
        lora = LoraConfig(r=4, lora_alpha=8, target_modules=["q_proj", "k_proj", "v_proj", "o_proj",
                                                             "gate_up_proj", "down_proj"])
        model = GptOssForCausalLM(cfg, lora=lora, device="cpu", dtype=torch.bfloat16).init_random(0)
        model.eval()
        ctx = TPContext()
        runner = TPModelRunner(model, _kv(cfg, 2), ctx, shard_model(model, rank, 2))
        if rank == 0:
            with torch.no_grad():        # an adapter that only rank 0 has: sync must ship it
                g = torch.Generator().manual_seed(5)
                for p in model.lora_param_dict().values():
                    p.copy_(torch.randn(p.shape, generator=g) * 0.2)
            ref = ModelRunner(model, _kv(cfg, 1), lora_active=True)
            runner.sync_lora()
            runner.lora_active = True
            diffs = []
            for items in _steps():
                want = ref.forward(items)
                got = runner.forward(items)
                diffs.append(((got.logits - want.logits).abs().max().item(),
                              want.logits.abs().max().item()))
            base = ModelRunner(model, _kv(cfg, 1), lora_active=False).forward(_steps()[0]).logits
            moved = (want.logits.abs().max().item(), (ref.forward(_steps()[0]).logits - base).abs().max().item())
            runner.stop_followers()
            q.put(("r0", diffs, moved))
        else:
            n = runner.follow()
            same = all(torch.equal(a, b) for a, b in zip(
                [p for p in model.lora_param_dict().values()][:2],
                [p for p in model.lora_param_dict().values()][:2]))
            q.put(("r1", n, runner.lora_shards is not None and same))
    finally:
        dist.destroy_process_group()


def test_tp2_lora_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_run_lora, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    outs = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    r0 = next(o for o in outs if o[0] == "r0")
    r1 = next(o for o in outs if o[0] == "r1")
    for err, scale in r0[1]:
        assert err <= 0.05 * max(1.0, scale), r0[1]
    assert r0[2][1] > 0.05          # the adapter changes the logits, so the check has teeth
    assert r1[1] == 2 and r1[2]


def test_shard_model_partitions_weights():
    model = _model()
    cfg = model.cfg
    s0, s1 = shard_model(model, 0, 2), shard_model(model, 1, 2)
    a = model.layers[0].self_attn
    d = cfg.head_dim
    qh = cfg.num_attention_heads // 2
    assert torch.equal(torch.cat([s0[0].o_w, s1[0].o_w], 1), a.o_weight)
    assert torch.equal(s0[0].qkv_w[:qh * d], a.qkv_weight[:qh * d])
    assert torch.equal(s1[0].qkv_w[:qh * d], a.qkv_weight[qh * d:2 * qh * d])
    assert s1[0].o_b is None and s0[0].o_b is not None
    E = cfg.num_local_experts
    assert s0[0].e0 == 0 and s1[0].e1 == E
    with pytest.raises(ValueError):
        shard_model(model, 0, 3)
