"""CPU unit tests of the trainer pieces: MXFP4 codec, packing collator, deterministic packed
sampler, DDIS loss (against a direct padded implementation of the reference formula),
divisors and staleness, sample processor, group-config factory, LR schedules."""
import math

import numpy as np
import pytest
import torch

from agent_factory_3_b200.ops import mxfp4
from agent_factory_3_b200.trainer.data.collator import DataCollatorWithPacking
from agent_factory_3_b200.trainer.data.sampler import (DeterministicPackedBatchSampler, SampleInfo,
                                                       pack_samples_into_bucket_groups)
from agent_factory_3_b200.trainer.flow_utils import (assign_divisors, compute_staleness_metrics,
                                                     filter_stale_samples)
from agent_factory_3_b200.trainer.losses.ddis_loss import DDISLoss
from agent_factory_3_b200.trainer.scheduler import get_scheduler
from agent_factory_3_b200.trainer.types import TrainingSample


def test_mxfp4_lut_and_roundtrip():
    blocks = torch.tensor([[[0x21, 0xF8] + [0] * 14]], dtype=torch.uint8)   # nibbles 1,2,8,15
    scales = torch.tensor([[128]], dtype=torch.uint8)                        # x2
    out = mxfp4.dequantize_reference(blocks, scales, torch.float32)
    assert out[0, :4].tolist() == [1.0, 2.0, -0.0, -12.0]
    w = torch.randn(8, 64)
    b, s = mxfp4.quantize(w)
    d = mxfp4.dequantize_reference(b, s, torch.float32)
    # every value is the nearest representable one: error <= half the grid step of its block
    assert (d - w).abs().max() <= w.abs().max() / 4 + 1e-6
    b2, s2 = mxfp4.quantize(d)
    assert torch.equal(mxfp4.dequantize_reference(b2, s2, torch.float32), d)


def _sample(n, comp_from, sid="s", adv=1.0, lr=None, version=0):
    comp = np.zeros(n, np.int32)
    comp[comp_from:] = 1
    return TrainingSample(sample_id=sid, input_ids=np.arange(n) % 50, completion_mask=comp,
                          gen_logprobs=(comp * -1.0).astype(np.float32),
                          advantages=(comp * adv).astype(np.float32),
                          routing_indices=lr, seq_token_count=int(comp.sum()),
                          prompt_sequence_count=2, prompt_token_count=10, prompt_id="g",
                          oldest_weight_version=version,
                          weight_version_token_counts={version: int(comp.sum())})


def test_collator_packing():
    L, K = 3, 2
    s1 = _sample(6, 2, "a", lr=np.ones((6, L, K), np.uint8))
    s2 = _sample(3, 1, "b", lr=np.full((3, L, K), 2, np.uint8))
    b = DataCollatorWithPacking(pad_token_id=0, pad_to_multiple_of=4)([s1, s2])
    assert b["input_ids"].shape == (12,) and b["num_padding"] == 3
    assert b["position_ids"].tolist() == [0, 1, 2, 3, 4, 5, 0, 1, 2, 0, 1, 2]
    assert b["cu_seqlens"].tolist() == [0, 6, 9, 12]
    assert b["segment_ids"].tolist()[:9] == [0] * 6 + [1] * 3
    assert b["completion_mask"].tolist() == [0, 0, 1, 1, 1, 1, 0, 1, 1, 0, 0, 0]
    assert b["labels"][:5].tolist() == b["input_ids"][1:6].tolist()
    assert b["routing_indices"].shape == (12, L, K) and int(b["routing_indices"][7, 0, 0]) == 2
    with pytest.raises(ValueError):
        DataCollatorWithPacking(vocab_size=4)([s1])
    # replayed routing ids must index real experts: the saved-batch sentinel 255 is rejected
    assert DataCollatorWithPacking(num_experts=3)([s1, s2])["routing_indices"].shape[1:] == (L, K)
    with pytest.raises(ValueError, match="255"):
        DataCollatorWithPacking(num_experts=2)([s1, s2])
    bad = _sample(3, 1, "c", lr=np.full((3, L, K), 255, np.uint8))
    with pytest.raises(ValueError):
        DataCollatorWithPacking(num_experts=128)([s1, bad])


def test_packed_sampler_best_fit_and_zigzag():
    lens = [900, 100, 500, 500, 300, 200, 800, 50]
    groups, stats = pack_samples_into_bucket_groups(
        [SampleInfo(i, n) for i, n in enumerate(lens)], max_capacity=1000, world_size=2)
    placed = sorted(s.index for g in groups for b in g for s in b)
    assert placed == list(range(len(lens)))
    assert all(sum(s.length for s in b) <= 1000 for g in groups for b in g)
    assert all(len(g) == 2 and all(b for b in g) for g in groups)
    sm = DeterministicPackedBatchSampler(lens, max_capacity=1000, world_size=2)
    r0, r1 = sm.plan_for_rank(0), sm.plan_for_rank(1)
    assert len(r0) == len(r1)
    assert DeterministicPackedBatchSampler(lens, max_capacity=1000, world_size=2).plan == sm.plan
    with pytest.raises(ValueError):
        pack_samples_into_bucket_groups([SampleInfo(0, 2000), SampleInfo(1, 1)], max_capacity=1000,
                                        world_size=1)


def _ddis_reference(logp, comp, adv, gen, div, eps_low, eps_high):
    """Padded formula of the reference DDIS loss (trainer/losses/ddis_loss.py:118-164)."""
    total = 0.0
    for i in range(len(logp)):
        lr = (logp[i] - gen[i]).clamp(-20, 20)
        r = torch.exp(torch.where(comp[i] > 0, lr, torch.zeros_like(lr)))
        m = ((r > 1 - eps_low) & (r < 1 + eps_high)).float() * comp[i]
        total = total + (-(r.detach() * adv[i] * logp[i] * m)).sum() / div[i]
    return total


def test_ddis_matches_reference_formula_and_grad():
    torch.manual_seed(0)
    lens = [7, 4, 9]
    logp = [(-torch.rand(n) * 3).requires_grad_(True) for n in lens]
    gen = [lp.detach() + torch.randn(n) * 0.3 for lp, n in zip(logp, lens)]
    comp = [torch.tensor([0] * 2 + [1] * (n - 2), dtype=torch.float32) for n in lens]
    adv = [c * a for c, a in zip(comp, [1.0, -0.5, 2.0])]
    div = torch.tensor([2.0, 3.0, 1.0])
    out = DDISLoss(eps_low=0.2, eps_high=0.3).compute_unpacked(
        log_probs=logp, completion_mask=comp, advantages=adv, divisors=div, gen_log_probs=gen)
    ref = _ddis_reference(logp, comp, adv, gen, div, 0.2, 0.3)
    torch.testing.assert_close(out.loss_unscaled, ref)
    g1 = torch.autograd.grad(out.loss_unscaled, logp, retain_graph=True)
    g2 = torch.autograd.grad(ref, logp)
    for a, b in zip(g1, g2):
        torch.testing.assert_close(a, b)
    st = out.metric_states["algo/ddis_mask_rate"]
    assert 0 <= float(st.mean()) <= 1
    # OPSM drops negative-advantage sequences with large KL
    out2 = DDISLoss(use_opsm=True, opsm_delta=0.0).compute_unpacked(
        log_probs=logp, completion_mask=comp, advantages=adv, divisors=div,
        gen_log_probs=[lp.detach() + 1.0 for lp in logp])
    assert "opsm/drop_rate" in out2.metric_states


def test_divisors_and_staleness():
    s = [_sample(6, 2, f"s{i}", version=v) for i, v in enumerate([1, 3, 5])]
    assign_divisors(s, "seq-mean-token-sum")
    assert [x.divisor for x in s] == [2.0] * 3
    assign_divisors(s, "token-mean")
    assert s[0].divisor == 4.0
    assign_divisors(s, "seq-mean-token-mean")
    assert s[0].divisor == 8.0
    assign_divisors(s, "prompt-mean-token-mean")
    assert s[0].divisor == 10.0
    kept = filter_stale_samples(s, current_step=5, max_staleness=2)
    assert [x.oldest_weight_version for x in kept] == [3, 5]
    m, pct = compute_staleness_metrics(kept, 5, 3)
    assert m["flow/stale_drop_count"] == 1.0 and m["flow/staleness_max"] == 2.0
    assert math.isclose(sum(pct.values()), 1.0)


def test_lr_schedules():
    p = torch.nn.Parameter(torch.zeros(1))
    opt = torch.optim.SGD([p], lr=1.0)
    s = get_scheduler("constant_with_warmup", opt, num_warmup_steps=4)
    lrs = []
    for _ in range(6):
        lrs.append(opt.param_groups[0]["lr"])
        opt.step()
        s.step()
    assert lrs == [0.0, 0.25, 0.5, 0.75, 1.0, 1.0]
    opt2 = torch.optim.SGD([p], lr=1.0)
    s2 = get_scheduler("cosine", opt2, num_warmup_steps=0, num_training_steps=10)
    for _ in range(5):
        opt2.step()
        s2.step()
    assert abs(opt2.param_groups[0]["lr"] - 0.5) < 1e-6
