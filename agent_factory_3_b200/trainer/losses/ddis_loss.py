"""DDIS: double-sided hard-masked importance-weighted policy-gradient loss.

Per completion token t of sample i (anchor = rollout-time log-prob, no extra forward):
    r_t      = exp(clamp(logp_t - gen_t, -20, 20))
    keep_t   = (1 - eps_low < r_t < 1 + eps_high) and completion_t
    loss     = - sum_i (1/d_i) sum_t sg(r_t) * A_t * logp_t * keep_t
with optional entropy top-x% token masking (per-sample rescale) and OPSM (zero sequences with
negative mean advantage whose KL(gen || train) exceeds delta).  Semantics and metric names are
those of the reference (trainer/losses/ddis_loss.py:40-245).

``compute_packed`` works directly on the packed token stream with segment ids (scatter
reductions, no padding to [B, T_max]); ``compute_unpacked`` keeps the reference's list API.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .metric_state import MeanMetricState


@dataclass(frozen=True)
class DDISLossOutputs:
    loss_unscaled: torch.Tensor
    metric_states: dict[str, MeanMetricState]


def _seg_sum(x: torch.Tensor, seg: torch.Tensor, n: int) -> torch.Tensor:
    return torch.zeros(n, device=x.device, dtype=torch.float32).index_add_(0, seg, x.float())


def _seg_max(x: torch.Tensor, seg: torch.Tensor, n: int, fill: float) -> torch.Tensor:
    out = torch.full((n,), fill, device=x.device, dtype=torch.float32)
    return out.scatter_reduce_(0, seg, x.float(), reduce="amax", include_self=True)


def _seg_min(x: torch.Tensor, seg: torch.Tensor, n: int, fill: float) -> torch.Tensor:
    out = torch.full((n,), fill, device=x.device, dtype=torch.float32)
    return out.scatter_reduce_(0, seg, x.float(), reduce="amin", include_self=True)


def _state(values: torch.Tensor, valid: torch.Tensor) -> MeanMetricState:
    v = values.detach()
    return MeanMetricState(sum=v[valid].sum(), count=valid.sum().to(torch.float32),
                           weighting="sample")


class DDISLoss:
    def __init__(self, *, eps_low: float = 0.2, eps_high: float = 0.2, use_opsm: bool = False,
                 opsm_delta: float = 1e-4, entropy_top_pct: float | None = None):
        if eps_low < 0:
            raise ValueError(f"eps_low must be >= 0, got {eps_low}")
        if eps_high < 0:
            raise ValueError(f"eps_high must be >= 0, got {eps_high}")
        self.eps_low = eps_low
        self.eps_high = eps_high
        self.use_opsm = use_opsm
        self.opsm_delta = opsm_delta
        self.entropy_top_pct = entropy_top_pct

    # ------------------------------------------------------------------ packed
    def compute_packed(self, *, log_probs: torch.Tensor, completion_mask: torch.Tensor,
                       advantages: torch.Tensor, gen_log_probs: torch.Tensor,
                       segment_ids: torch.Tensor, divisors: torch.Tensor,
                       entropies: torch.Tensor | None = None) -> DDISLossOutputs:
        """All token tensors are [T] over the packed stream; segment_ids[t] in [0, B) is the
        sample of token t (tokens of padding may use any id with completion_mask 0)."""
        B = divisors.numel()
        if B == 0:
            raise ValueError("compute_packed received no samples")
        dev = log_probs.device
        seg = segment_ids.to(device=dev, dtype=torch.long)
        logp = log_probs.float()
        comp = completion_mask.to(device=dev).float()
        adv = advantages.to(device=dev).float()
        gen = gen_log_probs.to(device=dev).float().detach()
        compb = comp > 0
        ccount = _seg_sum(comp, seg, B)
        has_comp = ccount > 0
        denom = ccount.clamp_min(1.0)

        log_ratio = (logp - gen).clamp(-20, 20)
        ratio = torch.exp(torch.where(compb, log_ratio, torch.zeros_like(log_ratio)))
        rd = ratio.detach()
        ddis_mask = ((rd > 1.0 - self.eps_low) & (rd < 1.0 + self.eps_high)).float()
        eff = ddis_mask * comp

        ent_scale = None
        if self.entropy_top_pct is not None:
            if entropies is None:
                raise RuntimeError("entropy_top_pct is set but entropies were not provided")
            ent = entropies.detach().float()
            thr = torch.full((B,), float("inf"), device=dev)
            k = (ccount * self.entropy_top_pct / 100.0).clamp(min=1).long()
            # per-sample k-th largest completion entropy (samples are few; loop on host ids)
            for i in torch.nonzero(has_comp).flatten().tolist():
                vals = ent[(seg == i) & compb]
                thr[i] = torch.topk(vals, int(min(k[i].item(), vals.numel()))).values[-1]
            keep = (ent >= thr[seg]).float() * comp
            eff = eff * keep
            ent_scale = ccount / _seg_sum(keep, seg, B).clamp_min(1.0)

        per_tok = -(rd * adv * logp * eff)
        per_sample = _seg_sum(per_tok, seg, B) if per_tok.requires_grad is False else \
            torch.zeros(B, device=dev, dtype=torch.float32).index_add(0, seg, per_tok)
        if ent_scale is not None:
            per_sample = per_sample * ent_scale
        opsm_mask = None
        if self.use_opsm:
            mean_adv = _seg_sum(adv * comp, seg, B) / denom
            kl = _seg_sum((gen - logp.detach()) * comp, seg, B) / denom
            opsm_mask = (mean_adv < 0) & (kl > self.opsm_delta)
            per_sample = per_sample * (~opsm_mask).float()
        d = divisors.to(device=dev, dtype=torch.float32)
        if not bool((d > 0).all()):
            raise ValueError("divisors must be positive")
        loss = (per_sample / d).sum()

        m: dict[str, MeanMetricState] = {}
        m["algo/ddis_mask_rate"] = _state(_seg_sum(comp * (1 - ddis_mask), seg, B) / denom, has_comp)
        pos = (adv > 0).float() * comp
        neg = (adv < 0).float() * comp
        pc, nc = _seg_sum(pos, seg, B), _seg_sum(neg, seg, B)
        m["algo/mask_rate_pos"] = _state(_seg_sum(pos * (1 - ddis_mask), seg, B) / pc.clamp_min(1), pc > 0)
        m["algo/mask_rate_neg"] = _state(_seg_sum(neg * (1 - ddis_mask), seg, B) / nc.clamp_min(1), nc > 0)
        m["algo/mask_rate_low"] = _state(_seg_sum((rd <= 1 - self.eps_low).float() * comp, seg, B) / denom, has_comp)
        m["algo/mask_rate_high"] = _state(_seg_sum((rd >= 1 + self.eps_high).float() * comp, seg, B) / denom, has_comp)
        rmean = _seg_sum(rd * comp, seg, B) / denom
        m["algo/ratio_mean"] = _state(rmean, has_comp)
        m["algo/ratio_max"] = _state(_seg_max(torch.where(compb, rd, torch.full_like(rd, -torch.inf)), seg, B, -float("inf")), has_comp)
        m["algo/ratio_min"] = _state(_seg_min(torch.where(compb, rd, torch.full_like(rd, torch.inf)), seg, B, float("inf")), has_comp)
        r2 = _seg_sum(rd * rd * comp, seg, B) / denom
        m["algo/ratio_std"] = _state(torch.sqrt((r2 - rmean ** 2).clamp(min=0)), has_comp)
        ld = logp.detach()
        m["algo/logprobs_mean"] = _state(_seg_sum(ld * comp, seg, B) / denom, has_comp)
        m["algo/logprobs_mean_pos"] = _state(_seg_sum(ld * pos, seg, B) / pc.clamp_min(1), pc > 0)
        m["algo/logprobs_mean_neg"] = _state(_seg_sum(ld * neg, seg, B) / nc.clamp_min(1), nc > 0)
        m["algo/gen_logprobs_mean"] = _state(_seg_sum(gen * comp, seg, B) / denom, has_comp)
        m["algo/kl_gen_train"] = _state(_seg_sum((gen - ld) * comp, seg, B) / denom, has_comp)
        if opsm_mask is not None:
            m["opsm/drop_rate"] = _state(opsm_mask.float(), has_comp)
            m["opsm/drop_count"] = MeanMetricState(opsm_mask.float().sum(), torch.tensor(1.0, device=dev), "token")
        remain = _seg_sum(eff, seg, B) / denom
        m["loss/token_remain_rate"] = _state(remain, has_comp)
        m["loss/token_mask_rate"] = _state(1.0 - remain, has_comp)
        return DDISLossOutputs(loss_unscaled=loss, metric_states=m)

    # ------------------------------------------------------------------ list API
    def compute_unpacked(self, *, log_probs: list[torch.Tensor], completion_mask: list[torch.Tensor],
                         advantages: list[torch.Tensor], divisors: torch.Tensor,
                         gen_log_probs: list[torch.Tensor],
                         entropies: list[torch.Tensor] | None = None) -> DDISLossOutputs:
        B = len(log_probs)
        if B == 0:
            raise ValueError("compute_unpacked received empty log_probs list")
        for name, lst in (("completion_mask", completion_mask), ("advantages", advantages),
                          ("gen_log_probs", gen_log_probs)):
            if len(lst) != B:
                raise ValueError(f"Mismatched list lengths in compute_unpacked inputs ({name})")
        if divisors.numel() != B:
            raise ValueError(f"divisors must have shape [B], got numel={divisors.numel()} B={B}")
        dev = log_probs[0].device
        seg = torch.cat([torch.full((lp.shape[0],), i, dtype=torch.long, device=dev)
                         for i, lp in enumerate(log_probs)])
        cat = lambda xs: torch.cat([x.to(dev) for x in xs])  # noqa: E731
        return self.compute_packed(log_probs=cat(log_probs), completion_mask=cat(completion_mask),
                                   advantages=cat(advantages), gen_log_probs=cat(gen_log_probs),
                                   segment_ids=seg, divisors=divisors,
                                   entropies=cat(entropies) if entropies is not None else None)
