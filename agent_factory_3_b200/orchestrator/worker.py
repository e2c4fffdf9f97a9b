"""Rollout worker process.

Behaviour (the reference's worker, orchestrator/worker.py:21-84, has the same contract): a
worker runs up to ``max_concurrent`` rollouts at once and takes a task from the shared input
queue only while it has a free lane, so tasks left in the queue stay available to idle workers
instead of piling up in one busy worker.  Every task produces exactly one
``(group_id, index_in_group, RolloutResult)`` on the output queue; an exception inside a
rollout becomes a failed result.  ``None`` on the input queue stops the worker after its
in-flight rollouts finish.

Design: a ``_LaneWorker`` keeps an explicit count of free lanes and a completion queue.  One
dispatcher coroutine blocks (in a helper thread) on the multiprocessing queue only after a lane
became free; each rollout runs as its own asyncio task and posts its result to the completion
queue; a single sender coroutine forwards completions to the output queue, so the blocking
``put`` of a large result never runs inside a rollout task.
"""
from __future__ import annotations

import asyncio
import logging
import multiprocessing as mp
import time
import traceback

from ..rollout.parallel.config import RolloutResult
from ..rollout.parallel.executor import execute_rollout
from .types import RolloutTask

logger = logging.getLogger(__name__)

_DONE = object()   # completion-queue end marker


def failed_result(task: RolloutTask, exc: BaseException) -> RolloutResult:
    """A RolloutResult that records ``exc`` for a rollout that raised."""
    t = time.time()
    return RolloutResult(rollout_id=task.config.rollout_id, start_time=t, end_time=t,
                         elapsed_time=0.0, server_url=task.server_url, success=False,
                         error=f"{type(exc).__name__}: {exc}",
                         traceback="".join(traceback.format_exception(exc)))


class _LaneWorker:
    def __init__(self, in_q: mp.Queue, out_q: mp.Queue, lanes: int, worker_id: int):
        if lanes < 1:
            raise ValueError("a worker needs at least one lane")
        self.in_q, self.out_q = in_q, out_q
        self.worker_id = worker_id
        self.free_lanes = lanes
        self.lane_freed = asyncio.Event()
        self.completions: asyncio.Queue = asyncio.Queue()
        self.running: set[asyncio.Task] = set()

    async def _wait_for_lane(self) -> None:
        while self.free_lanes == 0:
            self.lane_freed.clear()
            await self.lane_freed.wait()
        self.free_lanes -= 1

    def _release_lane(self) -> None:
        self.free_lanes += 1
        self.lane_freed.set()

    async def _rollout(self, task: RolloutTask) -> None:
        try:
            result = await execute_rollout(task.config, task.server_url)
        except Exception as exc:  # noqa: BLE001 - every task must yield a result
            logger.warning("worker %d: rollout %s failed: %s", self.worker_id,
                           task.config.rollout_id, exc)
            result = failed_result(task, exc)
        await self.completions.put((task.group_id, task.index_in_group, result))
        self._release_lane()

    async def _sender(self) -> None:
        while True:
            item = await self.completions.get()
            if item is _DONE:
                return
            await asyncio.to_thread(self.out_q.put, item)

    async def run(self) -> None:
        sender = asyncio.create_task(self._sender())
        while True:
            await self._wait_for_lane()
            task = await asyncio.to_thread(self.in_q.get)
            if task is None:                       # stop request: no new work
                self._release_lane()
                break
            t = asyncio.create_task(self._rollout(task))
            self.running.add(t)
            t.add_done_callback(self.running.discard)
        if self.running:
            await asyncio.wait(set(self.running))
        await self.completions.put(_DONE)
        await sender


def worker_main(input_queue: mp.Queue, output_queue: mp.Queue, max_concurrent: int,
                worker_id: int) -> None:
    """Process entry point: serve rollouts until a ``None`` arrives on ``input_queue``."""
    asyncio.run(_LaneWorker(input_queue, output_queue, max_concurrent, worker_id).run())
