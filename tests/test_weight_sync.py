"""Direct weight sync: staging layout and write/apply round trip on CPU (plain copies), then on
two GPUs across two processes (CUDA IPC mapping + the fused cast / NVLink-store kernel)."""
import os
import pickle

import pytest
import torch
import torch.multiprocessing as mp

from agent_factory_3_b200.parallel.weight_sync import PeerWriter, StagingBuffer


def _shapes():
    return {"a": (4, 6), "b": (3, 5), "c": (16,)}


def test_staging_layout_and_local_write():
    st = StagingBuffer.for_tensors(_shapes(), "cpu")
    offs = [e.offset for e in st.layout]
    assert offs == [0, 24, 40] and all(o % 8 == 0 for o in offs)
    g = torch.Generator().manual_seed(0)
    src = {k: torch.randn(*v, generator=g) for k, v in _shapes().items()}
    w = PeerWriter(st)
    n = w.write(src)
    assert n == sum(t.numel() * 2 for t in src.values())
    for k, t in st.tensors().items():
        assert torch.equal(t, src[k].bfloat16())
    with pytest.raises(ValueError):
        w.write({"a": torch.zeros(6, 4)})


def test_engine_applies_staged_params():
    from agent_factory_3_b200.engine.scheduler import Engine
    from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM, LoraConfig
    cfg = GptOssConfig.preset("tiny")
    lora = LoraConfig(r=8, lora_alpha=16, target_modules=["q_proj", "o_proj", "gate_up_proj"])
    trainer_model = GptOssForCausalLM(cfg, lora=lora, device="cpu").init_random(0).init_lora(1)
    engine_model = GptOssForCausalLM(cfg, lora=lora, device="cpu").init_random(0)
    with torch.no_grad():
        for p in trainer_model.lora_param_dict().values():
            p.normal_(0, 0.1)
    src = trainer_model.lora_param_dict()
    st = StagingBuffer.for_tensors({k: tuple(v.shape) for k, v in src.items()}, "cpu")
    PeerWriter(st).write(src)
    eng = Engine(engine_model, num_pages=16, page_size=16).start()
    try:
        assert eng.control("apply_lora_params", "policy", st.tensors()) is True
    finally:
        eng.stop()
    got = engine_model.lora_param_dict()
    for k, v in src.items():
        torch.testing.assert_close(got[k].float(), v.detach().bfloat16().float())
    assert eng.active_lora == "policy"


def _receiver(q_out, q_in, shapes):
    torch.cuda.set_device(1)
    st = StagingBuffer.for_tensors(shapes, "cuda:1")
    q_out.put(st.export())
    q_in.get(timeout=120)           # the writer is done (bounded: never outlive a failed test)
    # numpy arrays pickle by value; CPU torch tensors would travel as shared-memory file
    # descriptors that the parent can only fetch while this process is still alive
    q_out.put({k: v.float().cpu().numpy() for k, v in st.tensors().items()})
    q_in.get(timeout=120)           # keep the buffer alive until the parent has read


def _writer(exported, shapes, q_done):
    torch.cuda.set_device(0)
    g = torch.Generator().manual_seed(3)
    src = {k: torch.randn(*v, generator=g).cuda() for k, v in shapes.items()}
    w = PeerWriter(exported)
    w.write(src)
    torch.cuda.synchronize()
    # by value (numpy): this process exits right after the put
    q_done.put({k: v.bfloat16().float().cpu().numpy() for k, v in src.items()})


@pytest.mark.gpu
def test_peer_write_across_processes_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    shapes = {"x": (128, 2880), "y": (5760, 32), "z": (8,)}
    ctx = mp.get_context("spawn")
    q_out, q_in, q_done = ctx.Queue(), ctx.Queue(), ctx.Queue()
    rec = ctx.Process(target=_receiver, args=(q_out, q_in, shapes), daemon=True)
    rec.start()
    wr = None
    try:
        exported = q_out.get(timeout=120)
        wr = ctx.Process(target=_writer, args=(exported, shapes, q_done), daemon=True)
        wr.start()
        want = q_done.get(timeout=120)
        wr.join(60)
        q_in.put(1)
        got = q_out.get(timeout=120)
        q_in.put(1)
        rec.join(60)
    finally:
        for p in (rec, wr):
            if p is not None and p.is_alive():
                p.kill()
    for k in shapes:
        assert got[k].shape == want[k].shape and (got[k] == want[k]).all(), k

