"""Import paths of the reference package that scripts written against it use: each resolves
here to this package's implementation."""
import importlib

import pytest


@pytest.mark.parametrize("module,names", [
    ("agent_factory_3_b200.trainer.data.data_collator_with_packing", ["DataCollatorWithPacking"]),
    ("agent_factory_3_b200.trainer.data.rl_deterministic_packed_sampler",
     ["DeterministicPackedBatchSampler", "pack_samples_into_bucket_groups", "SampleInfo"]),
    ("agent_factory_3_b200.trainer.sglang_controller", ["SglangController"]),
    ("agent_factory_3_b200.trainer.sglang_metrics", ["SglangMetricsDrainer", "parse_loads_response"]),
    ("agent_factory_3_b200.trainer.losses.logprobs_computer", ["LogprobsComputer"]),
    ("agent_factory_3_b200.models.gpt_oss.quantizer_config", ["Mxfp4Bf16DequantConfig"]),
    ("agent_factory_3_b200.models.gpt_oss.routing_replay", ["enable_routing_replay"]),
    ("agent_factory_3_b200.models.gpt_oss.fsdp2_fix", []),
    ("agent_factory_3_b200.inference", ["AgentHandle"]),
    ("agent_factory_3_b200.orchestrator", ["Orchestrator", "GroupConfig", "GroupResult", "per_rollout"]),
    ("agent_factory_3_b200.visualizer", ["create_groups_viewer"]),
])
def test_reference_import_paths(module, names):
    m = importlib.import_module(module)
    for n in names:
        assert getattr(m, n) is not None, (module, n)


def test_aliases_are_the_implementations():
    from agent_factory_3_b200.trainer.data.collator import DataCollatorWithPacking
    from agent_factory_3_b200.trainer.data.data_collator_with_packing import \
        DataCollatorWithPacking as D2
    from agent_factory_3_b200.trainer.engine_controller import EngineController
    from agent_factory_3_b200.trainer.sglang_controller import SglangController
    assert D2 is DataCollatorWithPacking and SglangController is EngineController
    c = SglangController(["http://127.0.0.1:1"], mode="merged", lora_name="policy", flush_cache=False)
    assert c.mode == "merged" and c.settle_s == 0.0
    with pytest.raises(ValueError):
        SglangController(["http://127.0.0.1:1"], mode="full")


def test_logprobs_computer_matches_dense_softmax():
    """Batched [B, T] inputs: log P(token_i | tokens_<i) per row, 0 at position 0, the same from
    both backends and from a dense softmax over the model's logits."""
    import torch
    from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM
    from agent_factory_3_b200.trainer.losses.logprobs_computer import LogprobsComputer
    m = GptOssForCausalLM(GptOssConfig.tiny(), dtype=torch.float32).init_random(0)
    m.gradient_checkpointing = False
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, m.cfg.vocab_size, (2, 13), generator=g)
    with torch.no_grad():
        out = LogprobsComputer(temperature=0.7).compute_logprobs(m, {"input_ids": ids})
        out_t = LogprobsComputer(temperature=0.7, backend="torch").compute_logprobs(
            m, {"input_ids": ids})
        ref = []
        for b in range(2):
            h = m.forward_hidden(ids[b], torch.arange(13), torch.tensor([0, 13], dtype=torch.int32))
            logp = torch.log_softmax(m.logits(h) / 0.7, dim=-1)
            row = torch.zeros(13)
            row[1:] = logp[:-1].gather(1, ids[b, 1:, None])[:, 0]
            ref.append(row)
        ref = torch.stack(ref)
    assert out["logps"].shape == (2, 13) and out["entropies"].shape == (2, 13)
    assert (out["logps"][:, 0] == 0).all()
    torch.testing.assert_close(out["logps"], ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(out_t["logps"], out["logps"], atol=1e-5, rtol=1e-5)
    with pytest.raises(ValueError):
        LogprobsComputer(backend="vllm")
