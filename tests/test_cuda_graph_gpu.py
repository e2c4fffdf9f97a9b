"""Decode steps replayed from CUDA graphs give the logits of the eager engine forward (same
kernels, padded batch), across growing context lengths and batch buckets."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model():
    from agent_factory_3_b200.models.gpt_oss import GptOssConfig, GptOssForCausalLM
    cfg = GptOssConfig.preset("gpt-oss-20b")
    cfg.num_hidden_layers = 2
    cfg.layer_types = cfg.layer_types[:2]
    return GptOssForCausalLM(cfg, device="cuda").init_random(0).eval()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_graph_decode_matches_eager():
    from agent_factory_3_b200.engine.cuda_graph import DecodeGraphs
    from agent_factory_3_b200.engine.kv_cache import PagedKVCache
    from agent_factory_3_b200.engine.model_runner import ModelRunner, StepItem
    model = _model()
    cfg = model.cfg

    def runner():
        kv = PagedKVCache(2, 32, 64, cfg.num_key_value_heads, cfg.head_dim, cfg.num_experts_per_tok,
                          "cuda", torch.bfloat16)
        return ModelRunner(model, kv, lora_active=False)

    eager, graphed = runner(), runner()
    graphed.graphs = DecodeGraphs(graphed)
    g = torch.Generator().manual_seed(1)
    lens = [70, 130, 20]
    pages = [[0, 1], [2, 3, 4], [5]]
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    pre = [StepItem(p, 0, pg) for p, pg in zip(prompts, pages)]
    for r in (eager, graphed):
        r.forward(pre)
    starts = list(lens)
    for step in range(4):
        n = 3 if step < 2 else 2                      # batch bucket changes too
        items = [StepItem([int(torch.randint(0, 1000, (1,), generator=g))], starts[i], pages[i])
                 for i in range(n)]
        want = eager.forward(items)
        got = graphed.forward(items)
        torch.cuda.synchronize()
        assert got.logits.shape == want.logits.shape
        err = (got.logits - want.logits).abs().max().item()
        assert err <= 1e-3 * max(1.0, want.logits.abs().max().item()), (step, err)
        assert torch.equal(got.routing, want.routing)
        for i in range(n):
            starts[i] += 1
    assert graphed.graphs.replays == 4 and len(graphed.graphs.graphs) >= 2


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_engine_with_graphs_generates():
    import threading

    from agent_factory_3_b200.engine.scheduler import Engine, Request
    model = _model()
    eng = Engine(model, num_pages=64, page_size=64, max_running=4, cuda_graphs=True).start()
    done = threading.Event()
    req = Request(input_ids=list(range(10, 60)), max_new_tokens=12, temperature=0.0)
    req.on_output = lambda out: done.set() if out["finished"] else None
    eng.submit(req)
    assert done.wait(300)
    eng.stop()
    assert len(req.output_ids) == 12
    assert eng.runner.graphs.replays >= 10
    ids = list(range(10, 60)) + req.output_ids[:-1]
    with torch.no_grad():
        h = model.forward_hidden(torch.tensor(ids, device="cuda"),
                                 torch.arange(len(ids), device="cuda", dtype=torch.int32),
                                 torch.tensor([0, len(ids)], device="cuda", dtype=torch.int32))
        lg = model.logits(h[49:]).float()
    chosen = lg[torch.arange(12), torch.tensor(req.output_ids, device="cuda")]
    assert bool((chosen >= lg.max(-1).values - 0.1).all())
