"""Speculative decoding in the engine (CPU): greedy verification keeps plain greedy decoding
(each token a near-argmax of a full recompute) whatever the drafter proposes; an oracle drafter
gets its blocks accepted; the sampling rule emits tokens distributed as the target's samples."""
import threading

import torch

from agent_factory_3_b200.engine.scheduler import Engine, Request
from agent_factory_3_b200.engine.spec import (BlockDraftModel, NgramDrafter, verify_batch,
                                              verify_block)
from tests.test_engine import assert_greedy, tiny_model


class _ListDrafter:
    def __init__(self, fn, block=4):
        self.fn, self.block = fn, block

    def propose(self, contexts, sizes):
        return [self.fn(c, k) for c, k in zip(contexts, sizes)]


def _generate(model, prompt, n, drafter=None):
    eng = Engine(model, num_pages=64, page_size=8, max_running=4, drafter=drafter).start()
    done = threading.Event()
    req = Request(input_ids=list(prompt), max_new_tokens=n, temperature=0.0)
    req.on_output = lambda out: done.set() if out["finished"] else None
    eng.submit(req)
    assert done.wait(120)
    eng.stop()
    return list(req.output_ids), eng


def test_verify_block_greedy():
    lg = torch.full((4, 10), -5.0)
    for i, t in enumerate([3, 4, 7, 1]):
        lg[i, t] = 5.0
    a, toks, lps, ents = verify_block(lg, [3, 4, 9], 0.0)
    assert a == 2 and toks == [3, 4, 7] and len(lps) == 3 and len(ents) == 3
    a, toks, _, _ = verify_block(lg, [3, 4, 7], 0.0)
    assert a == 3 and toks == [3, 4, 7, 1]
    a, toks, _, _ = verify_block(lg, [0, 4, 7], 0.0)
    assert a == 0 and toks == [3]


def test_verify_batch_matches_per_request():
    torch.manual_seed(3)
    lg = torch.randn(12, 9) * 3
    drafts = [[int(lg[0].argmax()), 1], [int(lg[3].argmax()), int(lg[4].argmax()), 2], [5]]
    offs = [0, 3, 7]
    got = verify_batch(lg, offs, drafts, [0.0, 0.0, 0.0])
    for (a, toks, lps, ents), o, d in zip(got, offs, drafts):
        ra, rt, rl, re = verify_block(lg[o:o + len(d) + 1], d, 0.0)
        assert (a, toks) == (ra, rt)
        assert torch.allclose(torch.tensor(lps), torch.tensor(rl), atol=1e-5)
        assert torch.allclose(torch.tensor(ents), torch.tensor(re), atol=1e-4)
    # sampling: the first emitted token of a block follows the target distribution
    T = 0.7
    p = torch.softmax(lg[3] / T, -1)
    counts = torch.zeros(9)
    g = torch.Generator().manual_seed(2)
    n = 6000
    for _ in range(n):
        res = verify_batch(lg, offs, drafts, [T, T, T], g)
        counts[res[1][1][0]] += 1
    assert (counts / n - p).abs().max() < 0.025


def test_verify_block_sampling_matches_target():
    # first emitted token must follow softmax(logits[0] / T) whatever the draft is
    torch.manual_seed(0)
    lg = torch.randn(3, 6) * 1.5
    T = 0.8
    p = torch.softmax(lg[0] / T, -1)
    counts = torch.zeros(6)
    g = torch.Generator().manual_seed(1)
    n = 20000
    for _ in range(n):
        _, toks, _, _ = verify_block(lg, [2, 5], T, g)
        counts[toks[0]] += 1
    assert (counts / n - p).abs().max() < 0.015


def test_spec_greedy_matches_plain_decoding():
    model = tiny_model()
    prompt = list(range(5, 22))
    base, _ = _generate(model, prompt, 14)
    assert_greedy(model, prompt, base)
    cont = list(prompt) + base

    def oracle(ctx, k):      # the true greedy continuation
        n = len(ctx)
        return (cont[n:n + k] + [0] * k)[:k]

    out, eng = _generate(model, prompt, 14, _ListDrafter(oracle))
    assert_greedy(model, prompt, out)
    assert eng.spec_accept_length > 2.0
    out, eng = _generate(model, prompt, 14, _ListDrafter(lambda c, k: [1] * k))
    assert_greedy(model, prompt, out)
    out, _ = _generate(model, prompt, 14, NgramDrafter(block=4))
    assert_greedy(model, prompt, out)


def test_block_draft_model_runs_in_engine():
    model = tiny_model()
    draft = BlockDraftModel.from_target(model, n_layers=1, block=4, window=8)
    ctxs = [list(range(3, 15)), list(range(20, 25))]
    props = draft.propose(ctxs, [4, 2])
    assert [len(p) for p in props] == [4, 2]
    assert all(0 <= t < model.cfg.vocab_size for p in props for t in p)
    prompt = list(range(7, 20))
    out, eng = _generate(model, prompt, 10, draft)
    assert len(out) == 10 and eng.spec_verifies > 0
    assert_greedy(model, prompt, out)
