"""CUDA graphs for the engine's decode steps (one GPU).

A decode step runs ~25 kernels per layer (norms, projections, RoPE, KV store, paged attention,
router, grouping, MXFP4 expert GEMMs, combine) for every one of the 36 layers; launched one by
one from Python, the host falls behind the GPU.  A step whose items are all single-token decodes
is instead replayed from a captured graph:

  * the batch is padded to a bucket size; pad rows use KV slot -1 (the KV store skips it),
    sequence length 1 on page 0, and their outputs are ignored;
  * token ids, positions, slots, page tables and lengths live in static device buffers that are
    filled (one host->device copy each) before the replay;
  * the paged attention kernel sizes its grid from the longest context, so the graph key is
    (bucket, number of 1024-token attention chunks, page-table width, LoRA active);
  * the routed-expert record is copied into the KV-side table outside the graph, for the real
    rows only.

Graphs of all keys share one memory pool.  LoRA tensors are updated in place by the engine, so a
captured graph reads the current adapter.  The tensor-parallel runner is not captured: its
all-reduce kernel takes the call's arrival epoch as an argument, which a replay would repeat.
"""
from __future__ import annotations

import torch

from .model_runner import StepItem, StepOutput, _Meta

BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 256, 384, 512)


def _bucket(n: int, buckets=BUCKETS) -> int | None:
    for b in buckets:
        if b >= n:
            return b
    return None


def _pow2(n: int) -> int:
    p = 1
    while p < n:
        p *= 2
    return p


class _Graph:
    def __init__(self, runner, B: int, chunks: int, maxp: int, lora: bool, pool):
        dev = runner.device
        cfg = runner.cfg
        P = runner.kv.page_size
        self.B, self.maxp = B, maxp
        self.ids = torch.zeros(B, device=dev, dtype=torch.long)
        self.pos = torch.zeros(B, device=dev, dtype=torch.int32)
        self.slots = torch.full((B,), -1, device=dev, dtype=torch.int32)
        self.pt = torch.zeros(B, maxp, device=dev, dtype=torch.int32)
        self.lens = torch.ones(B, device=dev, dtype=torch.int32)
        m = _Meta()
        m.N, m.rows, m.dec_idx, m.pre_idx = B, [(i, i + 1) for i in range(B)], list(range(B)), []
        m.ids_t, m.pos_t, m.slots_t = self.ids, self.pos, self.slots
        m.dec_pt, m.dec_lens = self.pt, self.lens
        m.dec_rows = torch.arange(B, device=dev, dtype=torch.long)
        m.dec_max = chunks * 16 * P
        m.dec_identity = True
        self.m = m
        self.runner = runner

        def body():
            x = torch.nn.functional.embedding(self.ids, runner.model.embed_tokens)
            x, rec = runner._layers(m, x)
            from ..ops.gemm import matmul
            from ..ops.norm import rmsnorm
            hl = rmsnorm(x, runner.model.norm, cfg.rms_norm_eps)
            logits = matmul(hl, runner.model.lm_head, out_dtype=torch.float32)
            return logits, torch.stack(rec, dim=1).to(torch.uint8)

        # warm-up outside the capture (first-call host work, cached checks, kernel attributes)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                body()
        torch.cuda.current_stream(dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool):
            self.logits, self.routing = body()

    def replay(self, items: list[StepItem]) -> StepOutput:
        B, n = self.B, len(items)
        P = self.runner.kv.page_size
        ids = torch.zeros(B, dtype=torch.long)
        pos = torch.zeros(B, dtype=torch.int32)
        slots = torch.full((B,), -1, dtype=torch.int32)
        lens = torch.ones(B, dtype=torch.int32)
        pt = torch.zeros(B, self.maxp, dtype=torch.int32)
        for i, it in enumerate(items):
            p = it.start
            ids[i] = it.ids[0]
            pos[i] = p
            slots[i] = it.pages[p // P] * P + p % P
            lens[i] = p + 1
            pt[i, :len(it.pages)] = torch.tensor(it.pages, dtype=torch.int32)
        for dst, src in ((self.ids, ids), (self.pos, pos), (self.slots, slots), (self.lens, lens),
                         (self.pt, pt)):
            dst.copy_(src.pin_memory(), non_blocking=True)
        self.graph.replay()
        cfg = self.runner.cfg
        routing = self.routing[:n]
        real = self.slots[:n].long()
        self.runner.kv.routing.view(-1, cfg.num_hidden_layers, cfg.num_experts_per_tok)[real] = routing
        return StepOutput(logits=self.logits[:n], routing=routing,
                          item_rows=[(i, i + 1) for i in range(n)], logit_offsets=list(range(n)))


class DecodeGraphs:
    """Captured decode steps of one ``ModelRunner`` (see the module docstring)."""

    def __init__(self, runner, max_graphs: int = 32):
        self.runner = runner
        self.graphs: dict = {}
        self.pool = torch.cuda.graph_pool_handle()
        self.max_graphs = max_graphs
        self.replays = 0

    def run(self, items: list[StepItem]) -> StepOutput | None:
        if not items or any(len(it.ids) != 1 or it.start <= 0 or it.all_logits or not it.want_logits
                            for it in items):
            return None
        B = _bucket(len(items))
        if B is None:
            return None
        P = self.runner.kv.page_size
        longest = max(it.start + 1 for it in items)
        chunks = max(1, (longest + 16 * P - 1) // (16 * P))
        maxp = _pow2(max(len(it.pages) for it in items))
        key = (B, chunks, maxp, bool(self.runner.lora_active))
        g = self.graphs.get(key)
        if g is None:
            if len(self.graphs) >= self.max_graphs:
                return None
            g = _Graph(self.runner, B, chunks, maxp, key[3], self.pool)
            self.graphs[key] = g
        self.replays += 1
        return g.replay(items)
