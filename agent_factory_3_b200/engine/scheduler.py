"""Continuous-batching engine core (one GPU thread).

Each iteration: apply control commands (pause / continue / flush / weights / LoRA), admit
waiting requests while KV pages last (matching the longest cached prefix first), run one
forward over prefill chunks (bounded by ``max_prefill_tokens``) plus one decode token for every
running request, sample, append, stream, and retire finished requests.

Pause semantics follow the sglang API the reference drives (trainer/sglang_controller.py):
``abort`` finishes every in-flight request immediately with finish_reason "abort" and its
partial output, and holds new requests until ``continue``; ``in_place`` only stops scheduling,
keeping running requests and their KV for resumption.
"""
from __future__ import annotations

import base64
import itertools
import logging
import os
import queue
import threading
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import numpy as np
import torch

from ..ops import decode as D
from .kv_cache import OutOfPages, PagedKVCache
from .model_runner import ModelRunner, StepItem

logger = logging.getLogger(__name__)
_ids = itertools.count()


@dataclass
class Request:
    input_ids: list[int]
    max_new_tokens: int = 128
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    min_p: float = 0.0
    seed: Optional[int] = None
    stop_token_ids: list[int] = field(default_factory=list)
    return_logprob: bool = False
    return_entropy: bool = False
    top_logprobs_num: int = 0
    return_routed_experts: bool = False
    lora_path: Optional[str] = None
    extra_key: Optional[str] = None
    stream: bool = False
    on_output: Optional[Callable[[dict], None]] = None   # called from the engine thread
    abort_after_tokens: Optional[int] = None   # injected fault: abort once this many are out
    rid: int = field(default_factory=lambda: next(_ids))
    # state
    output_ids: list[int] = field(default_factory=list)
    output_logprobs: list[float] = field(default_factory=list)
    output_entropy: list[float] = field(default_factory=list)
    output_top: list = field(default_factory=list)
    pages: list[int] = field(default_factory=list)
    page_hashes: list[bytes] = field(default_factory=list)
    n_cached: int = 0          # tokens with K/V in the cache
    cached_tokens: int = 0     # prefix-cache hits at admission
    finish_reason: Optional[dict] = None
    created: float = field(default_factory=time.time)
    sent: int = 0              # streamed tokens so far

    @property
    def all_ids(self) -> list[int]:
        return self.input_ids + self.output_ids

    @property
    def salt(self) -> str:
        return f"{self.extra_key or ''}|{self.lora_path or ''}"


class Engine:
    def __init__(self, model, *, num_pages: int = 4096, page_size: int = 64,
                 max_running: int = 128, max_prefill_tokens: int = 16384,
                 max_context_tokens: Optional[int] = None, weight_version: str = "0",
                 tp=None, tp_shards=None, drafter=None, cuda_graphs: Optional[bool] = None):
        """``tp``: an ``engine.tp.TPContext`` to run tensor-parallel (this process is one rank;
        rank 0 runs the scheduler, the others call ``self.runner.follow()``)."""
        self.model = model
        cfg = model.cfg
        dev = model.embed_tokens.device
        world = tp.world if tp is not None else 1
        self.kv = PagedKVCache(cfg.num_hidden_layers, num_pages, page_size,
                               cfg.num_key_value_heads // world, cfg.head_dim,
                               cfg.num_experts_per_tok, dev, dtype=model.embed_tokens.dtype)
        if tp is not None:
            from .tp import TPModelRunner
            self.runner = TPModelRunner(model, self.kv, tp, tp_shards)
        else:
            self.runner = ModelRunner(model, self.kv, lora_active=False)
            if cuda_graphs is None:
                cuda_graphs = os.environ.get("AF3_CUDA_GRAPHS") == "1"
            if cuda_graphs and dev.type == "cuda":
                from .cuda_graph import DecodeGraphs
                self.runner.graphs = DecodeGraphs(self.runner)
        self.tp = tp
        # one GPU: requests of different adapters share a batch (ModelRunner.forward_mixed);
        # tensor parallel keeps one applied adapter per batch
        self.mixed_lora = tp is None
        self.lora_bank: dict = {}
        self.drafter = drafter          # engine.spec drafter: speculative decoding when set
        self.spec_verifies = 0
        self.spec_accepted = 0
        self.max_running = max_running
        self.max_prefill_tokens = max_prefill_tokens
        self.max_context = max_context_tokens or cfg.max_position_embeddings
        self.weight_version = weight_version
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.inbox: queue.Queue = queue.Queue()
        self.paused: Optional[str] = None
        self.loras: dict[str, dict] = {}
        self.active_lora: Optional[str] = None
        self.step_count = 0
        self.gen_tokens_window: deque = deque(maxlen=64)
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.lock = threading.Lock()
        self.spec_accept_length = 0.0
        self.spec_accept_rate = 0.0

    # ------------------------------------------------------------------ public (any thread)
    def submit(self, req: Request) -> None:
        self.inbox.put(("req", req))

    def control(self, cmd: str, *args, wait: bool = True, timeout: float = 600.0):
        done = threading.Event()
        box: dict[str, Any] = {}
        self.inbox.put((cmd, (args, done, box)))
        if wait and not done.wait(timeout):
            raise TimeoutError(f"engine did not process {cmd} within {timeout}s")
        if "error" in box:
            raise box["error"]
        return box.get("result")

    def start(self) -> "Engine":
        self._thread = threading.Thread(target=self._loop, name="af3-engine", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        self.inbox.put(("noop", None))
        if self._thread is not None:
            self._thread.join(timeout=30)
        if self.tp is not None:
            self.runner.stop_followers()

    def loads(self) -> dict:
        now = time.time()
        toks = sum(n for t, n in self.gen_tokens_window if now - t < 10.0)
        span = max(1e-3, min(10.0, now - min((t for t, _ in self.gen_tokens_window), default=now)))
        used = sum(len(r.all_ids) for r in self.running)
        return {"num_used_tokens": used, "gen_throughput": toks / span,
                "token_usage": self.kv.usage(), "memory": {"kv_cache_gb": self.kv.gb()},
                "cache_hit_rate": self.kv.cache_hit_rate(),
                "speculative": {"accept_length": self.spec_accept_length,
                                "accept_rate": self.spec_accept_rate},
                "num_running_reqs": len(self.running), "num_waiting_reqs": len(self.waiting),
                "queues": {"paused": 1 if self.paused else 0, "retracted": 0, "grammar": 0},
                "utilization": min(1.0, len(self.running) / max(1, self.max_running))}

    # ------------------------------------------------------------------ control (engine thread)
    def _do_control(self, cmd, args):
        if cmd == "pause":
            mode = args[0] if args else "abort"
            self.paused = mode
            if mode == "abort":
                for r in list(self.running) + list(self.waiting):
                    self._finish(r, {"type": "abort"})
                self.running.clear()
                self.waiting.clear()
        elif cmd == "abort_request":       # one request (its client went away)
            req = args[0]
            for q in (self.running, self.waiting):
                if req in q:
                    q.remove(req)
                    self._finish(req, {"type": "abort"})
                    break
        elif cmd == "continue":
            self.paused = None
        elif cmd == "flush_cache":
            if self.running:
                raise RuntimeError("cannot flush the cache while requests are running")
            self.kv.flush()
        elif cmd == "update_weight_version":
            self.weight_version = str(args[0])
        elif cmd == "load_lora":
            name, path = args
            self.loras[name] = self._read_adapter(path)
            self.lora_bank.pop(name, None)
            return True
        elif cmd == "unload_lora":
            self.loras.pop(args[0], None)
            self.lora_bank.pop(args[0], None)
            if self.active_lora == args[0]:
                self.active_lora = None
                self.runner.lora_active = False
        elif cmd == "update_weights":
            path, flush = args
            self._load_merged(path)
            if flush:
                self.kv.flush()
        elif cmd == "apply_lora_params":    # staged tensors in the model's own LoRA layout
            name, sd = args
            self.loras[name] = ("params", sd)
            self.lora_bank.pop(name, None)
            self._apply_lora(name)
            return True
        elif cmd == "set_lora_tensors":     # in-memory adapter (direct weight sync)
            name, sd = args
            self.loras[name] = sd
            self.lora_bank.pop(name, None)
            if self.active_lora == name:
                self._apply_lora(name)
        return None

    def _read_adapter(self, path: str) -> dict:
        from pathlib import Path
        p = Path(path)
        if (p / "adapter_model.bin").exists():
            return torch.load(p / "adapter_model.bin", map_location="cpu", weights_only=True)
        from safetensors.torch import load_file
        return load_file(str(p / "adapter_model.safetensors"))

    def _bank(self, name: str) -> dict:
        """Adapter ``name``'s factors in the model's own layout (bf16 on the device), for
        mixed-adapter steps; built once per adapter version.  A PEFT state dict is converted by
        loading it into the model's LoRA parameters and restoring the applied adapter after."""
        hit = self.lora_bank.get(name)
        if hit is not None:
            return hit
        ad = self.loras[name]
        dev = self.model.embed_tokens.device
        if isinstance(ad, tuple) and ad[0] == "params":
            params = self.model.lora_param_dict()
            bank = {k: t.to(dev, torch.bfloat16).view(params[k].shape) for k, t in ad[1].items()}
        else:
            params = self.model.lora_param_dict()
            saved = {k: p.detach().clone() for k, p in params.items()}
            _load_lora_into(self.model, ad)
            bank = {k: p.detach().to(torch.bfloat16).clone() for k, p in params.items()}
            with torch.no_grad():
                for k, p in params.items():
                    p.copy_(saved[k])
        self.lora_bank[name] = bank
        return bank

    def _apply_lora(self, name: str) -> None:
        ad = self.loras[name]
        if isinstance(ad, tuple) and ad[0] == "params":   # internal layout (GPU weight sync)
            params = self.model.lora_param_dict()
            with torch.no_grad():
                for k, t in ad[1].items():
                    params[k].copy_(t.view_as(params[k]))
        else:
            _load_lora_into(self.model, ad)
        if self.tp is not None:
            self.runner.sync_lora()     # slices on every tensor-parallel rank
        self.active_lora = name
        self.runner.lora_active = True

    def _load_merged(self, path: str) -> None:
        from pathlib import Path

        from safetensors import safe_open
        cfg = self.model.cfg
        q, kv = cfg.q_size, cfg.kv_size
        split = {"q_proj": (0, q), "k_proj": (q, q + kv), "v_proj": (q + kv, q + 2 * kv)}
        for f in sorted(Path(path).glob("*.safetensors")):
            with safe_open(str(f), framework="pt") as h:
                for k in h.keys():
                    parts = k.split(".")
                    if len(parts) < 6 or parts[0] != "model" or parts[1] != "layers":
                        continue
                    li = int(parts[2])
                    a = self.model.layers[li].self_attn
                    t = h.get_tensor(k)
                    with torch.no_grad():
                        if parts[3] == "self_attn" and parts[4] in split and parts[5] == "weight":
                            lo, hi = split[parts[4]]
                            a.qkv_weight[lo:hi].copy_(t.to(a.qkv_weight.device, a.qkv_weight.dtype))
                        elif parts[3] == "self_attn" and parts[4] == "o_proj" and parts[5] == "weight":
                            a.o_weight.copy_(t.to(a.o_weight.device, a.o_weight.dtype))

    # ------------------------------------------------------------------ loop
    def _loop(self):
        torch.cuda.set_device(self.model.embed_tokens.device) if self.model.embed_tokens.is_cuda else None
        while not self._stop.is_set():
            block = not self.running and (not self.waiting or self.paused)
            try:
                item = self.inbox.get(timeout=0.05 if block else 0.0) if block else self.inbox.get_nowait()
            except queue.Empty:
                item = None
            while item is not None:
                kind, payload = item
                if kind == "req":
                    self.waiting.append(payload)   # held while paused, scheduled on continue
                elif kind != "noop":
                    args, done, box = payload
                    try:
                        box["result"] = self._do_control(kind, args)
                    except Exception as e:  # noqa: BLE001
                        box["error"] = e
                    done.set()
                try:
                    item = self.inbox.get_nowait()
                except queue.Empty:
                    item = None
            if self.paused or (not self.running and not self.waiting):
                continue
            try:
                self._step()
            except Exception as e:  # noqa: BLE001 - fail the batch, keep serving
                logger.exception("engine step failed: %s", e)
                for r in list(self.running):
                    self._finish(r, {"type": "abort", "message": str(e)})
                self.running.clear()

    def _admit(self) -> None:
        P = self.kv.page_size
        while self.waiting and len(self.running) < self.max_running:
            r = self.waiting[0]
            if self.mixed_lora:
                # one GPU: sequences of different adapters share a batch (stacked-rank LoRA)
                if r.lora_path is not None and r.lora_path not in self.loras:
                    self.waiting.popleft()
                    self._finish(r, {"type": "abort", "message": f"unknown lora {r.lora_path}"})
                    continue
            elif r.lora_path != self.active_lora:
                if self.running:       # tensor parallel: adapters switch only between batches
                    break
                if r.lora_path is None:
                    self.active_lora = None
                    self.runner.lora_active = False
                elif r.lora_path in self.loras:
                    self._apply_lora(r.lora_path)
                else:
                    self.waiting.popleft()
                    self._finish(r, {"type": "abort", "message": f"unknown lora {r.lora_path}"})
                    continue
            if len(r.input_ids) + 1 > self.max_context:
                self.waiting.popleft()
                self._finish(r, {"type": "length"})
                continue
            pages, hashes = self.kv.match_prefix(r.input_ids[:-1], r.salt)
            need = (len(r.input_ids) + P - 1) // P - len(pages)
            if not self.kv.can_allocate(need + 1):
                self.kv.release(pages)
                break
            self.waiting.popleft()
            r.pages = pages + self.kv.allocate(need)
            r.page_hashes = hashes
            r.n_cached = len(pages) * P
            r.cached_tokens = r.n_cached
            self.running.append(r)

    def _ensure_page(self, r: Request, n_tokens: int) -> None:
        P = self.kv.page_size
        while len(r.pages) * P < n_tokens:
            r.pages += self.kv.allocate(1)

    def _register_full_pages(self, r: Request) -> None:
        P = self.kv.page_size
        ids = r.all_ids
        while len(r.page_hashes) < min(r.n_cached // P, len(r.pages)):
            i = len(r.page_hashes)
            prev = r.page_hashes[-1] if r.page_hashes else b""
            h = self.kv.chain(prev, ids[i * P:(i + 1) * P], r.salt)
            self.kv.register(r.pages[i], h)
            r.page_hashes.append(h)

    def _spec_ok(self, r: Request) -> bool:
        return (self.drafter is not None and r.top_k <= 0 and r.top_p >= 1.0 and r.min_p <= 0)

    def _append(self, r: Request, t: int, lp: float, ent: float, top=None) -> bool:
        """Record one generated token (``top``: its top-k alternatives, when computed);
        returns True when the request has finished."""
        if r.return_logprob and r.top_logprobs_num > 0:
            r.output_top.append(top if top is not None else [(float(lp), int(t))])
        r.output_ids.append(int(t))
        r.output_logprobs.append(float(lp))
        r.output_entropy.append(float(ent))
        if r.stop_token_ids and t in r.stop_token_ids:
            r.finish_reason = {"type": "stop", "matched": int(t)}
        elif r.abort_after_tokens is not None and len(r.output_ids) >= r.abort_after_tokens:
            r.finish_reason = {"type": "abort", "message": "injected fault"}
        elif len(r.output_ids) >= r.max_new_tokens:
            r.finish_reason = {"type": "length"}
        elif len(r.all_ids) >= self.max_context:
            r.finish_reason = {"type": "length"}
        return r.finish_reason is not None

    def _step(self) -> None:
        self._admit()
        if not self.running:
            return
        items, owners, budget = [], [], self.max_prefill_tokens
        spec_reqs, spec_sizes = [], []
        for r in self.running:
            ids = r.all_ids
            pending = len(ids) - r.n_cached
            if pending <= 0:
                continue
            if pending == 1 and r.n_cached > 0 and self._spec_ok(r):
                k = min(self.drafter.block, r.max_new_tokens - len(r.output_ids) - 1,
                        self.max_context - len(ids) - 1)
                if k > 0:
                    try:
                        self._ensure_page(r, r.n_cached + 1 + k)
                    except OutOfPages:
                        k = 0
                if k > 0:
                    spec_reqs.append(r)
                    spec_sizes.append(k)
                    continue
            n = pending if pending == 1 else min(pending, max(1, budget))
            if pending > 1:
                if budget <= 0:
                    continue
                budget -= n
            try:
                self._ensure_page(r, r.n_cached + n)
            except OutOfPages:
                continue
            items.append(StepItem(ids=ids[r.n_cached:r.n_cached + n], start=r.n_cached,
                                  pages=list(r.pages), want_logits=(r.n_cached + n == len(ids)),
                                  adapter=r.lora_path))
            owners.append(r)
        n_plain = len(items)
        if spec_reqs:
            drafts = self.drafter.propose([r.all_ids for r in spec_reqs], spec_sizes)
            for r, d in zip(spec_reqs, drafts):
                items.append(StepItem(ids=[r.all_ids[-1]] + list(d), start=r.n_cached,
                                      pages=list(r.pages), want_logits=True, all_logits=True,
                                      adapter=r.lora_path))
                owners.append(r)
        if not items:
            return
        out = self._forward(items)
        self.step_count += 1
        plain = [i for i in range(n_plain) if items[i].want_logits]
        sample_owners = [owners[i] for i in plain]
        for r, it in zip(owners[:n_plain], items[:n_plain]):
            r.n_cached += len(it.ids)
        if sample_owners:
            dev = out.logits.device
            temps = torch.tensor([r.temperature for r in sample_owners], device=dev)
            minp = torch.tensor([r.min_p for r in sample_owners], device=dev)
            seeds = torch.tensor([(r.seed if r.seed is not None else r.rid) for r in sample_owners],
                                 device=dev, dtype=torch.int64)
            logits = out.logits
            if spec_reqs:
                logits = logits.index_select(0, torch.tensor([out.logit_offsets[i] for i in plain],
                                                             device=dev, dtype=torch.long))
            raw = logits
            if any(r.top_k > 0 or r.top_p < 1.0 for r in sample_owners):
                logits = _apply_top_k_top_p(logits, sample_owners)
            steps = [len(r.output_ids) for r in sample_owners]
            tok, lp, ent = D.sample(logits, temps, seeds + torch.tensor(steps, device=dev) * 1000003,
                                    self.step_count, minp if float(minp.max()) > 0 else None)
            tops = _top_logprobs(raw, temps, sample_owners)
            tok, lp, ent = tok.tolist(), lp.tolist(), ent.tolist()
            self.gen_tokens_window.append((time.time(), len(tok)))
            for j, (r, t, l, e) in enumerate(zip(sample_owners, tok, lp, ent)):
                self._append(r, t, l, e, tops.get(j))
                if r.stream and r.finish_reason is None:
                    self._emit(r, final=False)
        if spec_reqs:
            from .spec import verify_batch
            idx = [n_plain + j for j in range(len(spec_reqs))]
            g = None
            if any(r.temperature > 0 for r in spec_reqs):
                g = torch.Generator(device=out.logits.device)
                g.manual_seed((self.step_count * 1000003 + sum(r.rid for r in spec_reqs)) % (2 ** 63))
            results = verify_batch(out.logits, [out.logit_offsets[i] for i in idx],
                                   [items[i].ids[1:] for i in idx],
                                   [r.temperature for r in spec_reqs], g)
            n_new = 0
            for r, (a, toks, lps, ents) in zip(spec_reqs, results):
                r.n_cached += a + 1          # the last token and the accepted drafts now have KV
                self.spec_verifies += 1
                self.spec_accepted += a
                for t, l, e in zip(toks, lps, ents):
                    n_new += 1
                    if self._append(r, t, l, e):
                        break
                if r.stream and r.finish_reason is None:
                    self._emit(r, final=False)
            self.gen_tokens_window.append((time.time(), n_new))
            self.spec_accept_length = 1.0 + self.spec_accepted / max(1, self.spec_verifies)
            self.spec_accept_rate = self.spec_accepted / max(1, self.spec_verifies * self.drafter.block)
        still = []
        for r in self.running:
            self._register_full_pages(r)
            if r.finish_reason is not None:
                self._finish(r, r.finish_reason)
            else:
                still.append(r)
        self.running = still

    def _forward(self, items: list[StepItem]):
        if not self.mixed_lora:
            return self.runner.forward(items)
        adapters = {it.adapter for it in items}
        if len(adapters) > 1:
            return self.runner.forward_mixed(items, {n: self._bank(n) for n in adapters if n})
        (name,) = adapters
        if name is None:
            self.runner.lora_active = False
        elif name != self.active_lora or not self.runner.lora_active:
            self._apply_lora(name)
        return self.runner.forward(items)

    # ------------------------------------------------------------------ outputs
    def _meta(self, r: Request, final: bool) -> dict:
        meta = {"id": str(r.rid), "finish_reason": r.finish_reason if final else None,
                "prompt_tokens": len(r.input_ids), "completion_tokens": len(r.output_ids),
                "cached_tokens": r.cached_tokens, "weight_version": self.weight_version,
                "e2e_latency": time.time() - r.created}
        if r.return_logprob:
            meta["output_token_logprobs"] = [[lp, t, None] for lp, t in zip(r.output_logprobs, r.output_ids)]
            if r.top_logprobs_num:
                # per generated token: its top-k alternatives [logprob, token_id, None] under
                # the request's temperature (tokens accepted by speculative verification carry
                # only themselves)
                meta["output_top_logprobs"] = [[[float(v), int(t), None] for v, t in row]
                                               for row in r.output_top]
        if r.return_entropy:
            meta["output_token_entropy"] = list(r.output_entropy)
        if final and r.return_routed_experts and r.pages:
            n = len(r.all_ids) - 1
            P = self.kv.page_size
            L, K = self.model.cfg.num_hidden_layers, self.model.cfg.num_experts_per_tok
            pos = np.arange(max(0, min(n, r.n_cached)))
            if len(pos):
                slots = torch.tensor([r.pages[p // P] * P + p % P for p in pos],
                                     device=self.kv.routing.device, dtype=torch.long)
                arr = self.kv.routing.view(-1, L, K)[slots].cpu().numpy().astype(np.int32)
            else:
                arr = np.zeros((0, L, K), np.int32)
            meta["routed_experts"] = base64.b64encode(arr.tobytes()).decode()
        return meta

    def _emit(self, r: Request, final: bool) -> None:
        if r.on_output is None:
            return
        new = r.output_ids[r.sent:]
        r.sent = len(r.output_ids)
        r.on_output({"output_ids": new if r.stream else list(r.output_ids),
                     "meta_info": self._meta(r, final), "finished": final})

    def _finish(self, r: Request, reason: dict) -> None:
        r.finish_reason = reason
        self.kv.release(r.pages)
        self._emit(r, final=True)
        r.pages = []


def _load_lora_into(model, sd: dict) -> None:
    """PEFT-format adapter tensors -> the model's LoRA parameters (same mapping as
    ModelTrainer.load_lora_state_dict)."""
    with torch.no_grad():
        for i, layer in enumerate(model.layers):
            pre = f"base_model.model.model.layers.{i}."
            for name, p in layer.self_attn.lora.items():
                mod, ab = name.rsplit("_", 1)
                k = f"{pre}self_attn.{mod}.lora_{ab}.weight"
                if k in sd:
                    p.copy_(sd[k].to(p.device, p.dtype))
            for name, p in layer.mlp.lora.items():
                mod = {"gu": "gate_up_proj", "dn": "down_proj"}[name.split("_")[0]]
                ab = name.split("_")[1]
                k = f"{pre}mlp.experts.{mod}.lora_{ab}.weight"
                if k not in sd:
                    continue
                t = sd[k]
                E, a, b = p.shape
                t = t.reshape(E, a, b) if ab == "A" else t.reshape(a, E, b).permute(1, 0, 2)
                p.copy_(t.to(p.device, p.dtype))


def _top_logprobs(logits: torch.Tensor, temps: torch.Tensor, owners: list) -> dict:
    """{row: [(logprob, token), ...]} -- the top ``top_logprobs_num`` tokens of every row whose
    request asked for them, log-softmax under the request's temperature (greedy rows use 1)."""
    rows = [j for j, r in enumerate(owners) if r.return_logprob and r.top_logprobs_num > 0]
    if not rows:
        return {}
    k = max(owners[j].top_logprobs_num for j in rows)
    idx = torch.tensor(rows, device=logits.device, dtype=torch.long)
    t = temps.index_select(0, idx).float()
    t = torch.where(t > 0, t, torch.ones_like(t))
    lp = torch.log_softmax(logits.index_select(0, idx).float() / t[:, None], dim=-1)
    vals, ids = lp.topk(min(k, lp.shape[-1]), dim=-1)
    vals, ids = vals.tolist(), ids.tolist()
    return {j: list(zip(vals[n][:owners[j].top_logprobs_num], ids[n][:owners[j].top_logprobs_num]))
            for n, j in enumerate(rows)}


def _apply_top_k_top_p(logits: torch.Tensor, reqs: list[Request]) -> torch.Tensor:
    """Mask logits outside each row's top-k / top-p set (sort-based)."""
    out = logits.clone()
    for i, r in enumerate(reqs):
        row = out[i] / max(r.temperature, 1e-6)
        if r.top_k > 0:
            kth = torch.topk(row, min(r.top_k, row.numel())).values[-1]
            out[i][row < kth] = -float("inf")
            row = out[i] / max(r.temperature, 1e-6)
        if r.top_p < 1.0:
            sv, si = torch.sort(row, descending=True)
            cp = torch.softmax(sv, 0).cumsum(0)
            drop = cp - torch.softmax(sv, 0) > r.top_p
            out[i][si[drop]] = -float("inf")
    return out
