"""Speculative decoding for the rollout engine: a drafter proposes a block of tokens for every
decoding request, the target model scores the block in one forward pass (the request's last
token + the drafts, logits at every position), and the longest acceptable prefix is kept.

The reference runs DFlash block speculation inside its sglang fork (examples/wordle/serve.sh:
80-84: a draft model proposing blocks of 10 tokens verified by the target).  Here:

  * ``BlockDraftModel``: a small gpt-oss-style model (1 decoder layer by default) that shares
    the target's embeddings and LM head and proposes a whole block in ONE forward: the last
    ``window`` context tokens followed by ``block`` mask tokens, logits read at the mask
    positions (greedy);
  * ``NgramDrafter``: prompt-lookup drafting (the continuation that followed the latest
    occurrence of the context's last n-gram), free to run and effective on repetitive tool
    traffic;
  * ``verify_block``: greedy acceptance at temperature 0 (the output equals plain greedy
    decoding); at temperature > 0 exact speculative sampling for a deterministic draft: draft
    token d is kept with probability p(d), and on the first rejection the replacement is drawn
    from p with d removed, so every emitted token is distributed as the target's sample.
"""
from __future__ import annotations

from typing import Protocol

import torch


class Drafter(Protocol):
    block: int

    def propose(self, contexts: list[list[int]], sizes: list[int]) -> list[list[int]]:
        """Draft ``sizes[i]`` tokens continuing ``contexts[i]``."""


class NgramDrafter:
    def __init__(self, block: int = 8, max_ngram: int = 4, min_ngram: int = 1):
        self.block, self.max_ngram, self.min_ngram = block, max_ngram, min_ngram

    def propose(self, contexts, sizes):
        out = []
        for ctx, k in zip(contexts, sizes):
            prop: list[int] = []
            for n in range(min(self.max_ngram, len(ctx) - 1), self.min_ngram - 1, -1):
                tail = ctx[-n:]
                # latest earlier occurrence of the tail
                for s in range(len(ctx) - n - 1, -1, -1):
                    if ctx[s:s + n] == tail:
                        prop = ctx[s + n:s + n + k]
                        break
                if prop:
                    break
            # pad with the last token (a rejected guess costs nothing extra in the verify pass)
            prop = (prop + [ctx[-1]] * k)[:k]
            out.append(prop)
        return out


class BlockDraftModel:
    """One-forward block drafter.  ``model`` is a ``GptOssForCausalLM`` (e.g. 1 layer) whose
    embeddings / LM head may be the target's tensors."""

    def __init__(self, model, block: int = 8, window: int = 32, mask_id: int | None = None):
        self.model, self.block, self.window = model, block, window
        self.mask_id = model.cfg.vocab_size - 1 if mask_id is None else mask_id

    @classmethod
    def from_target(cls, target, n_layers: int = 1, block: int = 8, seed: int = 1, **kw):
        """Random-init draft with ``n_layers`` layers of the target's shape, sharing the
        target's embedding and LM head."""
        import copy

        from ..models.gpt_oss import GptOssForCausalLM
        cfg = copy.deepcopy(target.cfg)
        cfg.num_hidden_layers = n_layers
        cfg.layer_types = cfg.layer_types[:n_layers]
        dev = target.embed_tokens.device
        d = GptOssForCausalLM(cfg, device=dev, dtype=target.embed_tokens.dtype)
        d.embed_tokens = target.embed_tokens
        d.lm_head = target.lm_head
        d.norm = torch.nn.Parameter(target.norm.detach().clone(), requires_grad=False)
        d.init_random(seed, keep_embeddings=True)
        return cls(d.eval(), block=block, **kw)

    @torch.inference_mode()
    def propose(self, contexts, sizes):
        dev = self.model.embed_tokens.device
        ids, pos, cu, picks = [], [], [0], []
        for ctx, k in zip(contexts, sizes):
            tail = ctx[-self.window:]
            base = len(ctx) - len(tail)
            seq = tail + [self.mask_id] * k
            ids += seq
            pos += list(range(base, base + len(seq)))
            picks += list(range(cu[-1] + len(tail), cu[-1] + len(seq)))
            cu.append(cu[-1] + len(seq))
        h = self.model.forward_hidden(torch.tensor(ids, device=dev),
                                      torch.tensor(pos, device=dev, dtype=torch.int32),
                                      torch.tensor(cu, device=dev, dtype=torch.int32))
        rows = h.index_select(0, torch.tensor(picks, device=dev, dtype=torch.long))
        toks = self.model.logits(rows).argmax(-1).tolist()
        out, o = [], 0
        for k in sizes:
            out.append(toks[o:o + k])
            o += k
        return out


def verify_block(logits: torch.Tensor, drafts: list[int], temperature: float,
                 generator: torch.Generator | None = None):
    """``logits`` [len(drafts) + 1, V]: the target's logits after the last token and after each
    draft.  Returns (n_accepted, emitted tokens (accepted drafts + one more), their log-probs and
    the entropies of the distributions they came from)."""
    B = len(drafts)
    lg = logits.float()
    if temperature <= 0:
        logp = torch.log_softmax(lg, -1)
        pred = lg.argmax(-1).tolist()
        a = 0
        while a < B and pred[a] == drafts[a]:
            a += 1
        toks = drafts[:a] + [pred[a]]
    else:
        logp = torch.log_softmax(lg / temperature, -1)
        p = logp.exp()
        u = torch.rand(B, generator=generator, device=lg.device) if B else None
        a = 0
        nxt = None
        while a < B:
            d = drafts[a]
            if float(u[a]) < float(p[a, d]):
                a += 1
                continue
            resid = p[a].clone()
            resid[d] = 0.0
            s = resid.sum()
            if float(s) <= 0:       # p is a point mass on d, so d was accepted with prob 1
                a += 1
                continue
            nxt = int(torch.multinomial(resid / s, 1, generator=generator))
            break
        if nxt is None:
            nxt = int(torch.multinomial(p[a], 1, generator=generator))
        toks = drafts[:a] + [nxt]
    idx = torch.arange(len(toks), device=lg.device)
    sel = torch.tensor(toks, device=lg.device)
    lps = logp[idx, sel].tolist()
    ents = (-(logp[:len(toks)].exp() * logp[:len(toks)]).sum(-1)).tolist()
    return a, toks, lps, ents


def verify_batch(logits: torch.Tensor, offsets: list[int], drafts: list[list[int]],
                 temperatures: list[float], generator: torch.Generator | None = None):
    """``verify_block`` for every request of a step at once: request i's block occupies logits
    rows offsets[i] .. offsets[i] + len(drafts[i]).  Same acceptance rules; the work stays on
    the device and crosses to the host three times per step (not per request)."""
    dev = logits.device
    lg = logits.float()
    rows_t, draft_rows, draft_tok = [], [], []
    for o, d, t in zip(offsets, drafts, temperatures):
        rows_t += [t] * (len(d) + 1)
        draft_rows += list(range(o, o + len(d)))
        draft_tok += list(d)
    # per-row temperature over the rows the blocks occupy (absolute row indices)
    all_rows = []
    for o, d in zip(offsets, drafts):
        all_rows += list(range(o, o + len(d) + 1))
    ar = torch.tensor(all_rows, device=dev, dtype=torch.long)
    temp_rows = torch.ones(lg.shape[0], device=dev, dtype=torch.float32)
    temp_rows[ar] = torch.tensor(rows_t, device=dev, dtype=torch.float32)
    scaled = torch.where(temp_rows[:, None] > 0, lg / temp_rows.clamp_min(1e-6)[:, None], lg)
    logp = torch.log_softmax(scaled, -1)
    pred = lg.argmax(-1)
    if draft_rows:
        dr = torch.tensor(draft_rows, device=dev, dtype=torch.long)
        dt = torch.tensor(draft_tok, device=dev, dtype=torch.long)
        p_d = logp[dr, dt].exp()
        u = torch.rand(len(draft_rows), device=dev, generator=generator)
        host = torch.stack([pred[dr].float(), p_d, u]).tolist()          # transfer 1
    else:
        host = [[], [], []]
    # acceptance on the host
    res, k = [], 0
    need_rows, need_excl = [], []
    for i, (o, d, t) in enumerate(zip(offsets, drafts, temperatures)):
        a = 0
        while a < len(d):
            j = k + a
            ok = (int(host[0][j]) == d[a]) if t <= 0 else (host[2][j] < host[1][j])
            if not ok:
                break
            a += 1
        k += len(d)
        res.append([a, o, t, d])
        need_rows.append(o + a)
        need_excl.append(d[a] if (a < len(d) and t > 0) else -1)
    # the token after the accepted prefix: greedy pick, or a sample (draft removed on rejection)
    nr = torch.tensor(need_rows, device=dev, dtype=torch.long)
    probs = logp[nr].exp()
    excl = torch.tensor(need_excl, device=dev, dtype=torch.long)
    has = excl >= 0
    if bool(has.any()):
        probs[has.nonzero().squeeze(1), excl[has]] = 0.0
    sampled = torch.multinomial(probs / probs.sum(-1, keepdim=True).clamp_min(1e-30), 1,
                                generator=generator).squeeze(1)
    greedy_next = pred[nr]
    is_greedy = torch.tensor([t <= 0 for _, _, t, _ in res], device=dev)
    nxt = torch.where(is_greedy, greedy_next, sampled).tolist()              # transfer 2
    # log-probs and entropies of every emitted token
    em_rows, em_tok = [], []
    for (a, o, t, d), x in zip(res, nxt):
        toks = d[:a] + [int(x)]
        em_rows += list(range(o, o + len(toks)))
        em_tok += toks
    er = torch.tensor(em_rows, device=dev, dtype=torch.long)
    et = torch.tensor(em_tok, device=dev, dtype=torch.long)
    lp_rows = logp[er]
    lps = lp_rows.gather(1, et[:, None]).squeeze(1)
    ents = -(lp_rows.exp() * lp_rows).sum(-1)
    lps_h, ents_h = torch.stack([lps, ents]).tolist()                          # transfer 3
    out, q = [], 0
    for (a, o, t, d), x in zip(res, nxt):
        n = a + 1
        out.append((a, d[:a] + [int(x)], lps_h[q:q + n], ents_h[q:q + n]))
        q += n
    return out
