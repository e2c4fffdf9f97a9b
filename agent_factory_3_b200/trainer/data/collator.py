"""Sequence packing of training samples into one flat token stream (reference:
trainer/data/data_collator_with_packing.py:5-92).

The batch is one row of T tokens: samples back to back, then padding up to a multiple of
``pad_to_multiple_of``.  Position ids restart at 0 for every sample and the padding forms its
own sequence; ``cu_seqlens`` lists the boundaries (padding included), ``segment_ids`` maps
every token to its sample (padding -> the last sample id with completion_mask 0).  Arrays are
built with numpy in one pass and handed over as (optionally pinned) host tensors so the
host->device copy is one asynchronous transfer per field.
"""
from __future__ import annotations

import numpy as np
import torch

from ..types import TrainingSample


class DataCollatorWithPacking:
    def __init__(self, pad_token_id: int = 0, pad_to_multiple_of: int = 128, pin_memory: bool = False,
                 vocab_size: int | None = None, num_experts: int | None = None):
        if vocab_size is not None and not 0 <= pad_token_id < vocab_size:
            raise ValueError(f"pad_token_id {pad_token_id} outside vocabulary of {vocab_size}")
        self.vocab_size = vocab_size
        self.num_experts = num_experts
        self.pad_token_id = pad_token_id
        self.pad_to_multiple_of = pad_to_multiple_of
        self.pin_memory = pin_memory

    def __call__(self, samples: list[TrainingSample | dict]) -> dict:
        get = (lambda s, k: s[k]) if isinstance(samples[0], dict) else (lambda s, k: getattr(s, k))
        lens = np.array([len(get(s, "input_ids")) for s in samples], dtype=np.int64)
        total = int(lens.sum())
        m = self.pad_to_multiple_of
        npad = (m - total % m) % m if m > 1 else 0
        T = total + npad

        def pack(key, dtype, pad_value=0):
            out = np.full(T, pad_value, dtype=dtype)
            off = 0
            for s, n in zip(samples, lens):
                out[off:off + n] = np.asarray(get(s, key), dtype=dtype)
                off += n
            return out

        ids = pack("input_ids", np.int64, self.pad_token_id)
        if self.vocab_size is not None and T and (ids.min() < 0 or ids.max() >= self.vocab_size):
            raise ValueError(f"token id outside [0, {self.vocab_size}) in the batch")
        pos = np.empty(T, dtype=np.int64)
        seg = np.empty(T, dtype=np.int64)
        off = 0
        for i, n in enumerate(lens):
            pos[off:off + n] = np.arange(n)
            seg[off:off + n] = i
            off += n
        pos[off:] = np.arange(npad)
        seg[off:] = len(samples) - 1
        cu = np.concatenate([[0], np.cumsum(lens)] + ([[T]] if npad else [])).astype(np.int32)
        # labels: next token within the packed row (boundary positions are masked by the
        # completion mask of the token *after* them being a prompt token or padding)
        labels = np.empty(T, dtype=np.int64)
        labels[:-1] = ids[1:]
        labels[-1] = self.pad_token_id
        batch = {
            "input_ids": ids, "position_ids": pos, "labels": labels, "segment_ids": seg,
            "cu_seqlens": cu, "num_samples": len(samples), "num_tokens": total, "num_padding": npad,
        }
        adv0 = get(samples[0], "advantages")
        if adv0 is not None:
            batch["advantages"] = pack("advantages", np.float32, 0.0)
        batch["completion_mask"] = pack("completion_mask", np.int32, 0)
        batch["gen_logprobs"] = pack("gen_logprobs", np.float32, 0.0)
        if get(samples[0], "gen_entropy") is not None:
            batch["gen_entropy"] = pack("gen_entropy", np.float32, 0.0)
        r0 = get(samples[0], "routing_indices")
        if r0 is not None:
            L, K = r0.shape[1], r0.shape[2]
            rt = np.zeros((T, L, K), dtype=np.uint8)
            off = 0
            for s, n in zip(samples, lens):
                rt[off:off + n] = get(s, "routing_indices")
                off += n
            # replayed ids index the router logits and the expert histograms on the device, so
            # an id outside [0, num_experts) is rejected here, on the host; saved batches mark
            # positions without a recorded route with 255, which must be filled before training
            if self.num_experts is not None and rt.size and int(rt.max()) >= self.num_experts:
                raise ValueError(f"routing id {int(rt.max())} outside [0, {self.num_experts}) in "
                                 "the batch (255 marks an unrecorded position in saved batches)")
            batch["routing_indices"] = rt
        if not isinstance(samples[0], dict) or "divisor" in samples[0]:
            batch["divisor"] = np.array([get(s, "divisor") or 1.0 for s in samples], np.float32)
        for k, v in list(batch.items()):
            if isinstance(v, np.ndarray):
                t = torch.from_numpy(v)
                batch[k] = t.pin_memory() if self.pin_memory and torch.cuda.is_available() else t
        return batch


def shift_completion_mask(completion_mask: torch.Tensor) -> torch.Tensor:
    """Loss mask for next-token log-probs: position t predicts token t+1, so it counts when
    token t+1 is a generated token (the reference shifts hidden[:-1] against ids[1:])."""
    out = torch.zeros_like(completion_mask)
    out[:-1] = completion_mask[1:]
    return out
