"""Per-token log-probabilities and entropies of a batch under ``GptOssForCausalLM``, with the
interface of the reference's ``LogprobsComputer`` (trainer/losses/logprobs_computer.py:20-371):
``compute_logprobs(model, inputs) -> {"logps": [B, T], "entropies": [B, T]}`` where
``logps[b, i] = log P(token_i | tokens_<i)`` and position 0 is 0.

The reference picks one of four loss backends (Triton, torch, cut-cross-entropy, Liger).  Here
there are two: the fused sm_100a linear -> log-prob / entropy kernel on CUDA (every GPU backend
name selects it) and the chunked PyTorch reference (``backend="torch"``, and the path on CPU).
Both compute softmax(hidden W^T / temperature) over the whole vocabulary without materialising
the [T, V] logits."""
from __future__ import annotations

import torch

from ...ops import logprob as L

_BACKENDS = ("triton", "torch", "cce", "liger", "fused")


class LogprobsComputer:
    def __init__(self, temperature: float = 1.0, backend: str = "fused"):
        self.temperature = float(temperature)
        self.backend = backend.lower()
        if self.backend not in _BACKENDS:
            raise ValueError(f"backend must be one of {_BACKENDS}, got {backend!r}")

    def _token_stats(self, model, hidden: torch.Tensor, labels: torch.Tensor):
        if self.backend == "torch":
            return L.linear_logprob_entropy_torch(hidden, model.lm_head, labels, self.temperature)
        return L.linear_logprob_entropy(hidden, model.lm_head, labels, self.temperature)

    def compute_logprobs(self, model, inputs: dict, return_entropy: bool = True) -> dict:
        """``inputs``: ``input_ids`` [B, T] (one sequence per row) or [T] with ``cu_seqlens``
        (packed); optional ``position_ids`` (same shape; default: restarting per sequence) and
        ``routing_indices`` ([B, T, L, K] or [T, L, K], replayed)."""
        if "input_ids" not in inputs:
            raise ValueError("inputs must contain 'input_ids'.")
        ids = inputs["input_ids"]
        batched = ids.dim() == 2
        dev = ids.device
        if batched:
            B, T = ids.shape
            flat = ids.reshape(-1)
            cu = torch.arange(0, (B + 1) * T, T, dtype=torch.int32)
        else:
            flat = ids
            cu = inputs.get("cu_seqlens")
            if cu is None:
                cu = torch.tensor([0, ids.numel()], dtype=torch.int32)
            cu = cu.to(torch.int32).cpu()
        pos = inputs.get("position_ids")
        if pos is None:
            pos = torch.cat([torch.arange(int(e - s)) for s, e in zip(cu[:-1], cu[1:])])
        pos = pos.reshape(-1).to(dev)
        routing = inputs.get("routing_indices")
        if routing is not None and batched:
            routing = routing.reshape(-1, *routing.shape[2:])
        hidden = model.forward_hidden(flat, pos, cu, routing_indices=routing)
        # hidden[i] predicts token i+1 inside each sequence; the last position of a sequence
        # predicts nothing and its label is replaced by a valid id (its value is discarded)
        labels = torch.empty_like(flat)
        labels[:-1] = flat[1:]
        labels[-1] = 0
        lp, ent = self._token_stats(model, hidden, labels)
        # shift right by one within each sequence: position s (a sequence start) gets 0
        out_lp = torch.zeros_like(lp)
        out_ent = torch.zeros_like(ent)
        starts = cu[:-1].tolist()
        ends = cu[1:].tolist()
        for s, e in zip(starts, ends):
            if e - s > 1:
                out_lp[s + 1:e] = lp[s:e - 1]
                out_ent[s + 1:e] = ent[s:e - 1]
        if batched:
            out_lp, out_ent = out_lp.reshape(B, T), out_ent.reshape(B, T)
        result = {"logps": out_lp.float()}
        if return_entropy:
            result["entropies"] = out_ent.float()
        return result
