"""Multi-process rollout orchestrator (reference: orchestrator/orchestrator.py:46-471).

* N worker processes with bounded concurrency pull rollout tasks from one shared queue.
* A group is dispatched only when ``in_flight + group_size <= workers * concurrency``.
* Each rollout goes to the engine with the lowest estimated KV load: the real token count from
  ``/v1/loads`` (polled every ``poll_interval`` seconds) plus an EWMA of tokens per rollout for
  every task in transit; ``server_affinity`` keeps a whole group on one engine (shared prefix).
* Completed groups are rewarded; a batch is yielded once ``batch_size`` rollouts from groups
  with reward variance ("signal") have arrived, or when 3x ``batch_size`` rollouts pile up.
* Dead workers are detected; when all are dead the run fails.

``worker_mode="inproc"`` runs rollouts as tasks of the calling event loop instead of worker
processes (tests and single-process tools); ``rollout_fn`` overrides the rollout call.
"""
from __future__ import annotations

import asyncio
import logging
import multiprocessing as mp
import queue
import time
from dataclasses import dataclass, field
from typing import Any, AsyncIterator, Callable, Iterable, Optional

import aiohttp

from ..rollout.parallel.config import RolloutResult
from ..rollout.parallel.executor import execute_rollout
from .types import GroupConfig, GroupResult, RewardFn, RolloutTask, per_rollout
from .worker import worker_main

logger = logging.getLogger(__name__)

POLL_INTERVAL_S = 10.0
EWMA_ALPHA = 0.05


@dataclass
class _GroupState:
    group_size: int
    metadata: dict
    results: dict = field(default_factory=dict)
    completed: int = 0


def parse_loads_response(data: dict) -> dict[str, float]:
    """Flatten the /v1/loads payload into metric fields (see trainer/engine_metrics.py)."""
    from ..trainer.engine_metrics import parse_loads_response as p
    return p(data)


class Orchestrator:
    def __init__(self, server_urls: list[str], num_workers: int = 8, worker_concurrency: int = 8,
                 batch_size: int = 128, reward_fn: Optional[RewardFn] = None,
                 metrics_queue: Optional[mp.Queue] = None, worker_mode: str = "process",
                 rollout_fn: Optional[Callable] = None, poll_interval: float = POLL_INTERVAL_S):
        if not server_urls:
            raise ValueError("server_urls cannot be empty")
        self.server_urls = list(server_urls)
        self.num_workers = num_workers
        self.worker_concurrency = worker_concurrency
        self.batch_size = batch_size
        self.reward_fn = reward_fn or per_rollout(lambda r, m: 0.0)
        self.metrics_queue = metrics_queue
        self.worker_mode = worker_mode
        self.rollout_fn = rollout_fn or execute_rollout
        self.poll_interval = poll_interval
        self.stats = {"dispatched_groups": 0, "completed_groups": 0}

    async def run(self, groups: Iterable[GroupConfig],
                  stop_event: Optional[asyncio.Event] = None) -> AsyncIterator[list[GroupResult]]:
        if self.worker_mode == "inproc":
            async for b in self._main_loop(groups, None, None, [], stop_event):
                yield b
            return
        ctx = mp.get_context("spawn")
        in_q, out_q = ctx.Queue(), ctx.Queue()
        workers = []
        for i in range(self.num_workers):
            p = ctx.Process(target=worker_main, args=(in_q, out_q, self.worker_concurrency, i),
                            daemon=True)
            p.start()
            workers.append(p)
        stopped = False
        try:
            async for b in self._main_loop(groups, in_q, out_q, workers, stop_event):
                yield b
                if stop_event is not None and stop_event.is_set():
                    stopped = True
                    break
        finally:
            self._shutdown_workers(in_q, workers, force=stopped)

    @staticmethod
    def _has_signal(g: GroupResult) -> bool:
        return len(g.rewards) > 1 and max(g.rewards) - min(g.rewards) > 1e-9

    def _finalize_group(self, gid: str, st: _GroupState) -> GroupResult:
        results = [st.results[i] for i in range(st.group_size)]
        try:
            rewards = list(self.reward_fn(results, st.metadata))
        except Exception as e:  # noqa: BLE001
            logger.exception("reward_fn failed for group %s: %s", gid, e)
            rewards = [0.0] * len(results)
        for r, w in zip(results, rewards):
            r.weighted_reward = w
        return GroupResult(group_id=gid, results=results, rewards=rewards, metadata=st.metadata)

    async def _main_loop(self, groups, in_q, out_q, workers, stop_event):
        loop = asyncio.get_running_loop()
        max_in_flight = self.num_workers * self.worker_concurrency
        load = {u: 0.0 for u in self.server_urls}
        in_transit = {u: 0 for u in self.server_urls}
        est = 10000.0
        it = iter(groups)
        tracker: dict[str, _GroupState] = {}
        pool: list[GroupResult] = []
        pool_n = signal_n = in_flight = 0
        exhausted = False
        pending: Optional[GroupConfig] = None
        local_q: asyncio.Queue = asyncio.Queue()
        local_tasks: set = set()

        def submit(task: RolloutTask):
            if in_q is not None:
                in_q.put(task)
                return

            async def run():
                try:
                    r = await self.rollout_fn(task.config, task.server_url)
                except Exception as e:  # noqa: BLE001
                    now = time.time()
                    r = RolloutResult(rollout_id=task.config.rollout_id, start_time=now,
                                      end_time=now, elapsed_time=0, server_url=task.server_url,
                                      success=False, error=str(e))
                await local_q.put((task.group_id, task.index_in_group, r))

            t = asyncio.create_task(run())
            local_tasks.add(t)
            t.add_done_callback(local_tasks.discard)

        def assign() -> str:
            u = min(self.server_urls, key=lambda x: load[x])
            load[u] += est
            in_transit[u] += 1
            return u

        def dispatch(g: GroupConfig):
            nonlocal in_flight
            n = len(g.rollout_configs)
            tracker[g.group_id] = _GroupState(n, g.metadata)
            if g.server_affinity:
                u = min(self.server_urls, key=lambda x: load[x])
                load[u] += est * n
                in_transit[u] += n
                urls = [u] * n
            else:
                urls = [assign() for _ in range(n)]
            for i, (c, u) in enumerate(zip(g.rollout_configs, urls)):
                submit(RolloutTask(config=c, server_url=u, group_id=g.group_id, index_in_group=i))
            in_flight += n
            self.stats["dispatched_groups"] += 1

        def fill():
            nonlocal pending, exhausted
            while not exhausted and not (stop_event is not None and stop_event.is_set()):
                if pending is None:
                    pending = next(it, None)
                    if pending is None:
                        exhausted = True
                        break
                if in_flight + len(pending.rollout_configs) <= max_in_flight:
                    dispatch(pending)
                    pending = None
                else:
                    break

        poll_stop = asyncio.Event()

        async def poller():
            timeout = aiohttp.ClientTimeout(total=1.5)
            while not poll_stop.is_set():
                try:
                    async with aiohttp.ClientSession(timeout=timeout) as s:
                        while not poll_stop.is_set():
                            rs = await asyncio.gather(*(s.get(f"{u}/v1/loads") for u in self.server_urls),
                                                      return_exceptions=True)
                            for u, r in zip(self.server_urls, rs):
                                if isinstance(r, BaseException):
                                    continue
                                try:
                                    data = await r.json()
                                    real = float(data["loads"][0]["num_used_tokens"])
                                    load[u] = real + in_transit[u] * est
                                    if self.metrics_queue is not None:
                                        flat = parse_loads_response(data)
                                        if flat:
                                            try:
                                                self.metrics_queue.put_nowait((time.time(), u, flat))
                                            except queue.Full:
                                                pass
                                except Exception:  # noqa: BLE001
                                    pass
                                finally:
                                    r.close()
                            try:
                                await asyncio.wait_for(poll_stop.wait(), timeout=self.poll_interval)
                                return
                            except asyncio.TimeoutError:
                                pass
                except Exception:  # noqa: BLE001
                    try:
                        await asyncio.wait_for(poll_stop.wait(), timeout=5.0)
                        return
                    except asyncio.TimeoutError:
                        pass

        poll_task = asyncio.create_task(poller())
        try:
            fill()
            while in_flight > 0:
                if stop_event is not None and stop_event.is_set():
                    break
                try:
                    if out_q is not None:
                        raw = await asyncio.wait_for(
                            loop.run_in_executor(None, lambda: out_q.get(timeout=10)), timeout=15)
                    else:
                        raw = await asyncio.wait_for(local_q.get(), timeout=15)
                except (asyncio.TimeoutError, queue.Empty):
                    if workers and sum(p.is_alive() for p in workers) == 0:
                        raise RuntimeError(f"All {self.num_workers} workers died. in_flight={in_flight}")
                    continue
                gid, idx, res = raw
                in_flight -= 1
                if res.server_url in in_transit:
                    in_transit[res.server_url] -= 1
                if res.num_generated_tokens > 0:
                    est = EWMA_ALPHA * res.num_generated_tokens + (1 - EWMA_ALPHA) * est
                st = tracker[gid]
                st.results[idx] = res
                st.completed += 1
                if st.completed == st.group_size:
                    g = self._finalize_group(gid, st)
                    pool.append(g)
                    pool_n += len(g.results)
                    if self._has_signal(g):
                        signal_n += len(g.results)
                    del tracker[gid]
                    self.stats["completed_groups"] += 1
                    if signal_n >= self.batch_size or pool_n >= 3 * self.batch_size:
                        yield pool
                        pool, pool_n, signal_n = [], 0, 0
                fill()
            if pool and not (stop_event is not None and stop_event.is_set()):
                yield pool
        finally:
            poll_stop.set()
            poll_task.cancel()
            for t in list(local_tasks):
                t.cancel()

    def _shutdown_workers(self, in_q, workers, force: bool = False) -> None:
        if not force:
            for _ in workers:
                in_q.put(None)
            deadline = time.time() + 30
            for p in workers:
                p.join(timeout=max(0.1, deadline - time.time()))
        for p in workers:
            if p.is_alive():
                p.terminate()
                p.join(timeout=5)
            if p.is_alive():
                p.kill()
