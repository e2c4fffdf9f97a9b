"""Rollout worker process: an asyncio loop that takes tasks from the shared input queue only
when it has a free concurrency slot (semaphore acquired *before* ``get``), so idle workers can
pick up the remaining tasks; any failure becomes a failed RolloutResult (reference:
orchestrator/worker.py:21-84)."""
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


def worker_main(input_queue: mp.Queue, output_queue: mp.Queue, max_concurrent: int,
                worker_id: int) -> None:
    asyncio.run(_worker_loop(input_queue, output_queue, max_concurrent, worker_id))


async def _worker_loop(input_queue, output_queue, max_concurrent: int, worker_id: int) -> None:
    sem = asyncio.Semaphore(max_concurrent)
    loop = asyncio.get_running_loop()
    pending: set = set()

    async def run_task(task: RolloutTask):
        try:
            try:
                result = await execute_rollout(task.config, task.server_url)
            except Exception as e:  # noqa: BLE001
                now = time.time()
                result = RolloutResult(rollout_id=task.config.rollout_id, start_time=now,
                                       end_time=now, elapsed_time=0.0, server_url=task.server_url,
                                       success=False, error=str(e), traceback=traceback.format_exc())
            await loop.run_in_executor(None, output_queue.put,
                                       (task.group_id, task.index_in_group, result))
        finally:
            sem.release()

    while True:
        await sem.acquire()
        raw = await loop.run_in_executor(None, input_queue.get)
        if raw is None:
            sem.release()
            break
        t = asyncio.create_task(run_task(raw))
        pending.add(t)
        t.add_done_callback(pending.discard)
    if pending:
        await asyncio.gather(*pending, return_exceptions=True)
