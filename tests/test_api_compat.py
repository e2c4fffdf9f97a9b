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
