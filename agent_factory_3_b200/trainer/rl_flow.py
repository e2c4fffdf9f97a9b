"""RLFlow: the async RL pipeline (reference: trainer/rl_flow.py:516-1068).

Rank 0 runs the training loop; other ranks serve RPC calls.  A separate orchestrator
(process, or thread with ``orchestrator_mode="thread"``) streams batches of training samples:

    GroupConfigFactory -> Orchestrator (workers -> engines) -> rewards -> SampleProcessor
    -> RolloutSaver (JSON/HTML/NPZ) -> sample_queue (maxsize 2: back-pressure)

Training loop per batch: staleness filter (samples older than ``max_staleness`` batches are
dropped), split into ``num_inner_steps`` mini-batches, divisors per aggregation mode,
``train_step``; every ``weight_sync_interval`` batches (and at least ``min_weight_sync_secs``
apart) the adapter (or merged attention weights) is written to a double-buffered directory
and the orchestrator is told to sync the engines (``WeightsUpdated``); ``checkpoint_latest``
every batch and ``checkpoint_step_N`` periodically, with the dataset-factory position for
exact resume.  On resume the adapter, optimizer/scheduler state, factory position and wandb
run id are restored and the engines re-synced before rollouts start.
"""
from __future__ import annotations

import asyncio
import logging
import multiprocessing as mp
import queue
import random
import threading
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Literal, Optional

from ..orchestrator.orchestrator import Orchestrator
from ..orchestrator.types import RewardFn
from ..rollout.config import ConversationConfig, LoopConfig, RecordConfig
from .checkpoint_utils import CheckpointMeta, cleanup_old_checkpoints, resolve_resume_path, write_meta
from .engine_controller import EngineController
from .engine_metrics import EngineMetricsDrainer
from .flow_utils import assign_divisors, compute_staleness_metrics, filter_stale_samples
from .group_config_factory import GroupConfigFactory
from .rollout_saver import RolloutSaver
from .sample_processor import SampleProcessor

logger = logging.getLogger(__name__)


@dataclass
class WeightsUpdated:
    path: str
    step: int
    flush: bool = False


@dataclass
class Shutdown:
    pass


def _orchestrator_main(sample_queue, control_queue, metrics_queue, *, server_urls, num_workers,
                       worker_concurrency, batch_size, reward_fn, dataset, group_size, loop_config,
                       conv_config, record_config, prompt_key, base_seed, normalize_advantages,
                       filter_all_failed, filter_all_solved, excluded_error_kinds, rollout_save_dir,
                       save_routing_indices, weight_sync_mode, lora_name, flush_cache_on_sync,
                       factory_initial_state, prompt_fn, cache_salt_mode, server_affinity,
                       worker_mode="process", rollout_fn=None, stop_flag=None, sync_settle_s=0.0):
    factory = GroupConfigFactory(dataset=dataset, group_size=group_size, loop_config=loop_config,
                                 conv_config=conv_config, record_config=record_config,
                                 prompt_key=prompt_key, base_seed=base_seed, prompt_fn=prompt_fn,
                                 cache_salt_mode=cache_salt_mode, server_affinity=server_affinity)
    if factory_initial_state:
        factory.load_state_dict(factory_initial_state)
    processor = SampleProcessor(normalize_advantages=normalize_advantages,
                                filter_all_failed=filter_all_failed,
                                filter_all_solved=filter_all_solved,
                                excluded_error_kinds=excluded_error_kinds)
    orch = Orchestrator(server_urls, num_workers=num_workers, worker_concurrency=worker_concurrency,
                        batch_size=batch_size, reward_fn=reward_fn, metrics_queue=metrics_queue,
                        worker_mode=worker_mode, rollout_fn=rollout_fn)
    saver = RolloutSaver(rollout_save_dir, save_routing_indices=save_routing_indices)
    controller = EngineController(server_urls, mode=weight_sync_mode, lora_name=lora_name,
                                  flush_cache=flush_cache_on_sync, settle_s=sync_settle_s)
    asyncio.run(_orchestrator_loop(orch, factory, processor, saver, controller, sample_queue,
                                   control_queue, stop_flag))


async def _orchestrator_loop(orch, factory, processor, saver, controller, sample_queue,
                             control_queue, stop_flag):
    stop = asyncio.Event()
    loop = asyncio.get_running_loop()

    async def control_listener():
        while not stop.is_set():
            try:
                msg = await loop.run_in_executor(None, lambda: control_queue.get(timeout=1.0))
            except (queue.Empty, EOFError, OSError):
                if stop_flag is not None and stop_flag.is_set():
                    stop.set()
                continue
            if isinstance(msg, Shutdown):
                stop.set()
                return
            if isinstance(msg, WeightsUpdated):
                try:
                    await controller.sync_weights(msg.path, str(msg.step), flush=msg.flush)
                except Exception:  # noqa: BLE001
                    logger.exception("weight sync failed")

    listener = asyncio.create_task(control_listener())
    batch_idx = 0
    try:
        async for groups in orch.run(iter(factory), stop_event=stop):
            samples, stats = processor.process(groups)
            _, _, html = saver.save_batch(groups, batch_idx)
            saver.save_training_data(groups, batch_idx)
            batch_idx += 1
            item = (samples, stats, html, factory.state_dict())
            while not stop.is_set():
                try:
                    await loop.run_in_executor(None, lambda: sample_queue.put(item, timeout=1.0))
                    break
                except queue.Full:
                    continue
            if stop.is_set():
                break
    finally:
        stop.set()
        listener.cancel()


class RLFlow:
    def __init__(self, *, training_config, model_trainer, dataset, reward_fn: RewardFn,
                 prompt_key: str = "prompt", server_urls: list[str], num_workers: int = 8,
                 worker_concurrency: int = 8, batch_size: int = 128, group_size: int = 8,
                 loop_config: LoopConfig, conv_config: ConversationConfig = ConversationConfig(),
                 record_config: RecordConfig = RecordConfig(), normalize_advantages: bool = False,
                 filter_all_failed: bool = True, filter_all_solved: bool = True,
                 excluded_error_kinds: list[str] | None = None, max_batches: int | None = None,
                 base_seed: int = 42, prompt_fn: Any = None,
                 cache_salt_mode: Literal["none", "per_group", "per_rollout"] = "none",
                 server_affinity: bool = False,
                 orchestrator_mode: Literal["process", "thread"] = "process",
                 worker_mode: Literal["process", "inproc"] = "process",
                 rollout_fn: Optional[Callable] = None, sync_settle_s: float = 0.0,
                 log_fn: Optional[Callable[[dict], None]] = None):
        tc = training_config
        self.training_config = tc
        self.model_trainer = model_trainer
        self.dataset = dataset
        self.reward_fn = reward_fn
        self.server_urls = server_urls
        self.batch_size = batch_size
        self.group_size = group_size
        self.max_batches = max_batches
        self.orch_kwargs = dict(
            server_urls=server_urls, num_workers=num_workers, worker_concurrency=worker_concurrency,
            batch_size=batch_size, reward_fn=reward_fn, dataset=dataset, group_size=group_size,
            loop_config=loop_config, conv_config=conv_config, record_config=record_config,
            prompt_key=prompt_key, base_seed=base_seed, normalize_advantages=normalize_advantages,
            filter_all_failed=filter_all_failed, filter_all_solved=filter_all_solved,
            excluded_error_kinds=excluded_error_kinds, rollout_save_dir=tc.rollout_dir,
            save_routing_indices=(tc.save_routing_indices if tc.save_routing_indices is not None
                                  else tc.use_routing_replay),
            weight_sync_mode=tc.weight_sync_mode, lora_name=tc.lora_adapter_name,
            flush_cache_on_sync=tc.flush_cache_on_sync, prompt_fn=prompt_fn,
            cache_salt_mode=cache_salt_mode, server_affinity=server_affinity,
            worker_mode=worker_mode, rollout_fn=rollout_fn, sync_settle_s=sync_settle_s)
        self.orchestrator_mode = orchestrator_mode
        self.log_fn = log_fn
        self.sync_settle_s = sync_settle_s
        if tc.training_mode == "full" and loop_config.lora_adapter_name is not None:
            raise ValueError("training_mode='full' needs loop_config.lora_adapter_name=None")
        if (tc.use_routing_replay or record_config.routing_indices) and (
                loop_config.num_hidden_layers is None or loop_config.num_experts_per_tok is None):
            raise ValueError("routing replay needs loop_config.num_hidden_layers and "
                             "num_experts_per_tok (gpt-oss-120b: 36 and 4)")
        if tc.use_routing_replay and not record_config.routing_indices:
            raise ValueError("use_routing_replay=True needs record_config.routing_indices=True")
        if loop_config.use_streaming and record_config.routing_indices:
            raise ValueError("use_streaming=True cannot capture routing indices; set use_streaming=False")
        if loop_config.segment_temperature is not None and (record_config.logprobs or
                                                            record_config.routing_indices):
            raise ValueError("segment_temperature cannot record logprobs or routing indices")
        if batch_size <= 0 or batch_size % group_size:
            raise ValueError(f"batch_size ({batch_size}) must be a positive multiple of group_size ({group_size})")

    def _save_for_sync(self, path: str) -> None:
        if self.training_config.weight_sync_mode == "lora":
            self.model_trainer.save_model(path)
        else:
            self.model_trainer.save_merged_weights(path)

    def _checkpoint(self, path: Path, step: int, batch_idx: int, factory_state, run_id):
        self.model_trainer.save_model(str(path))
        self.model_trainer.save_training_state(str(path))
        write_meta(path, CheckpointMeta(step=step, batch_idx=batch_idx, factory_state=factory_state,
                                        wandb_run_id=run_id, weight_version=str(batch_idx)))

    def _restore(self, path: Path) -> CheckpointMeta:
        """Load a checkpoint written by ``_checkpoint``: adapter weights, then the optimizer
        and scheduler state in whichever layout the trainer uses (one file, or one file per
        rank for the sharded optimizer; every rank loads its own slice).  A checkpoint that
        has optimizer state only in the other layout is an error, not a silent fresh start."""
        from .checkpoint_utils import read_meta
        meta = read_meta(path)
        tr = self.model_trainer
        tr.load_model(str(path))
        kind = tr.training_state_layout(str(path))
        if kind == "missing":
            logger.warning("checkpoint %s has no optimizer state; AdamW restarts from zero", path)
        else:
            tr.load_training_state(str(path))
        return meta

    def run(self, on_step: Callable[[dict, int], None] | None = None) -> list[dict]:
        tr = self.model_trainer
        tc = self.training_config
        if getattr(tr, "rank", 0) != 0:
            tr.rpc_worker_loop()
            return []
        for d in (tc.checkpoint_dir, tc.rollout_dir):
            Path(d).mkdir(parents=True, exist_ok=True)
        ckpt_root = Path(tc.checkpoint_dir).resolve()
        resume = resolve_resume_path(tc.resume_from_checkpoint, ckpt_root)
        step_count = batch_idx = 0
        factory_state = None
        run_id = None
        if resume is not None:
            meta = self._restore(resume)
            step_count, batch_idx = meta.step, meta.batch_idx
            factory_state, run_id = meta.factory_state, meta.wandb_run_id
        # initial weight sync (engines start from the trainer's weights / resumed adapter)
        ctrl = EngineController(self.server_urls, mode=tc.weight_sync_mode, lora_name=tc.lora_adapter_name,
                                flush_cache=True, settle_s=self.sync_settle_s)
        init_path = str(Path(tc.run_dir) / "weight_init")
        self._save_for_sync(init_path)
        asyncio.run(ctrl.sync_weights(init_path, str(batch_idx)))
        last_sync = time.time()
        self.exposed_sync_s = [ctrl.last_sync_s]
        kw = dict(self.orch_kwargs, factory_initial_state=factory_state)
        if self.orchestrator_mode == "process":
            ctx = mp.get_context("spawn")
            sample_q, control_q = ctx.Queue(maxsize=2), ctx.Queue()
            metrics_q = ctx.Queue(maxsize=10000)
            proc = ctx.Process(target=_orchestrator_main, args=(sample_q, control_q, metrics_q),
                               kwargs=kw, daemon=False)
        else:
            sample_q, control_q, metrics_q = queue.Queue(maxsize=2), queue.Queue(), queue.Queue(maxsize=10000)
            stop_flag = threading.Event()
            kw["stop_flag"] = stop_flag
            proc = threading.Thread(target=_orchestrator_main, args=(sample_q, control_q, metrics_q),
                                    kwargs=kw, daemon=True)
        proc.start()
        drainer = EngineMetricsDrainer(metrics_q, self.log_fn).start()
        all_metrics: list[dict] = []
        t0 = time.time()
        try:
            while self.max_batches is None or batch_idx < self.max_batches:
                try:
                    item = sample_q.get(timeout=30)
                except queue.Empty:
                    if not proc.is_alive():
                        break
                    continue
                samples, stats, html, latest_factory = item
                batch_idx += 1
                pre = len(samples)
                samples = filter_stale_samples(samples, batch_idx, tc.max_staleness)
                if not samples:
                    continue
                stale_metrics, _ = compute_staleness_metrics(samples, batch_idx, pre)
                n_inner = tc.num_inner_steps
                if n_inner > 1:
                    random.shuffle(samples)
                n = len(samples)
                chunks = [c for c in (samples[i * n // n_inner:(i + 1) * n // n_inner]
                                      for i in range(n_inner)) if c]
                for inner, chunk in enumerate(chunks):
                    if len(chunk) < getattr(tr, "world_size", 1):
                        continue
                    assign_divisors(chunk, tc.loss_aggregation_mode)
                    n_groups = len({s.prompt_id for s in chunk})
                    if n_groups > 1:
                        for s in chunk:
                            s.divisor *= n_groups
                    m = tr.train_step(chunk)
                    step_count += 1
                    m.update({"flow/batch_idx": float(batch_idx), "flow/step_count": float(step_count),
                              "flow/inner_step": float(inner), "flow/num_inner_steps": float(len(chunks)),
                              "flow/num_samples": float(len(chunk)), "flow/elapsed": time.time() - t0})
                    if inner == 0:
                        m.update(stale_metrics)
                        m.update(stats.to_metrics_dict())
                    all_metrics.append(m)
                    if on_step is not None:
                        on_step(m, step_count)
                    if self.log_fn is not None:
                        self.log_fn(m)
                if batch_idx % tc.weight_sync_interval == 0 and \
                        time.time() - last_sync >= tc.min_weight_sync_secs:
                    path = str(Path(tc.weight_sync_dir + ("_a" if batch_idx % 2 == 0 else "_b")))
                    self._save_for_sync(path)
                    if tc.reset_optimizer_on_sync:
                        tr.reset_optimizer_state()
                    k = tc.flush_cache_every_n_steps
                    control_q.put(WeightsUpdated(path=path, step=batch_idx, flush=k > 0 and batch_idx % k == 0))
                    last_sync = time.time()
                if tc.save_latest_checkpoint:
                    self._checkpoint(ckpt_root / "checkpoint_latest", step_count, batch_idx,
                                     latest_factory, run_id)
                if tc.save_checkpoint_every > 0 and batch_idx % tc.save_checkpoint_every == 0:
                    self._checkpoint(ckpt_root / f"checkpoint_step_{step_count}", step_count,
                                     batch_idx, latest_factory, run_id)
                    cleanup_old_checkpoints(ckpt_root, tc.max_checkpoints_to_keep)
        finally:
            drainer.stop()
            control_q.put(Shutdown())
            if self.orchestrator_mode == "thread":
                kw["stop_flag"].set()
            deadline = time.time() + 60
            while proc.is_alive() and time.time() < deadline:
                try:
                    sample_q.get_nowait()
                except queue.Empty:
                    pass
                proc.join(timeout=0.5)
            if self.orchestrator_mode == "process" and proc.is_alive():
                proc.terminate()
            tr.rpc_shutdown()
        return all_metrics
