"""Async serving engine over one or more GPU replicas (dan/engine.py:1-113).

Same contract as dan's ``AsyncEngine``: requests queue up; a worker packs them
into prefill batches FIFO up to ``max_batch_tokens`` (cost = prompt tokens +
question tokens), waiting at most ``max_wait_ms`` for company; a batch runs in a
thread (``runner.read_many``; ctypes launches release the GIL) and resolves its
requests' futures; a failing batch fails only its own requests; the queue is
capped (``Overloaded``).

Difference: ``runner`` may be a list of runners, one per GPU. Each replica has
its own worker pulling whole batches from the shared queue, so a batch goes to
whichever replica is free (least loaded). Replicas share nothing on the data
path (no collective). ``stats`` aggregates; ``replica_stats`` is per replica.
"""
import asyncio
import time
from dataclasses import dataclass, field

from .readout import answers, combine


class Overloaded(RuntimeError):
    pass


@dataclass
class Stats:
    requests: int = 0
    batches: int = 0
    tokens: int = 0
    busy_s: float = 0.0
    latency_s: float = 0.0
    errors: int = 0
    started: float = field(default_factory=time.time)


class AsyncEngine:
    def __init__(self, planner, runner, max_batch_tokens=8192, max_wait_ms=2.0, max_queue=1024):
        self.planner = planner
        self.runners = list(runner) if isinstance(runner, (list, tuple)) else [runner]
        self.runner = self.runners[0]  # dan's /metrics reads engine.runner.cache
        self.max_batch_tokens = max_batch_tokens
        self.max_wait = max_wait_ms / 1000
        self.max_queue = max_queue
        self.queue = asyncio.Queue()
        self.stats = Stats()
        self.replica_stats = [Stats() for _ in self.runners]
        self._workers = []

    def start(self):
        if not self._workers:
            loop = asyncio.get_running_loop()
            self._workers = [loop.create_task(self._loop(i)) for i in range(len(self.runners))]

    async def stop(self):
        for w in self._workers:
            w.cancel()
        for w in self._workers:
            try:
                await w
            except asyncio.CancelledError:
                pass
        self._workers = []

    async def decide(self, state, questions, profile=None):
        """Answers keyed by question id, and the input tokens the reads took (engine.py:55-72)."""
        plans = self.planner.plans(state, questions, profile)
        if not plans[0].branches:
            return answers(plans[0], []), 0
        if self.queue.qsize() + len(plans) > self.max_queue:
            raise Overloaded("dan is at capacity. Retry shortly.")
        self.start()
        loop, t0 = asyncio.get_running_loop(), time.perf_counter()
        futs = [loop.create_future() for _ in plans]
        for plan, fut in zip(plans, futs):
            await self.queue.put((plan, fut, t0))
        reads = await asyncio.gather(*futs)
        self.stats.requests += 1
        self.stats.latency_s += time.perf_counter() - t0
        logp = combine(plans, reads)
        return answers(plans[0], logp, profile, logits_canonical=True), sum(self.cost(p) for p in plans)

    @staticmethod
    def cost(plan):
        return len(plan.prefix) + sum(len(b.suffix) for b in plan.branches)

    async def _loop(self, replica):
        while True:
            batch = [await self.queue.get()]
            budget = self.cost(batch[0][0])
            deadline = time.perf_counter() + self.max_wait
            while budget < self.max_batch_tokens:
                if self.queue.empty():
                    left = deadline - time.perf_counter()
                    if left <= 0:
                        break
                    await asyncio.sleep(min(left, 0.0005))
                    continue
                plan = self.queue._queue[0][0]  # peek: stop before the budget is exceeded
                if budget + self.cost(plan) > self.max_batch_tokens:
                    break
                batch.append(self.queue.get_nowait())
                budget += self.cost(plan)
            await self._run(replica, batch, budget)

    async def _run(self, replica, batch, tokens):
        plans = [p for p, _, _ in batch]
        st = self.replica_stats[replica]
        t = time.perf_counter()
        try:
            logits = await asyncio.to_thread(self.runners[replica].read_many, plans)
        except Exception as e:  # noqa: BLE001 - fail this batch's requests, keep serving
            self.stats.errors += len(batch)
            st.errors += len(batch)
            for _, fut, _ in batch:
                if not fut.done():
                    fut.set_exception(e)
            return
        dt = time.perf_counter() - t
        for s in (self.stats, st):
            s.batches += 1
            s.tokens += tokens
            s.busy_s += dt
        for (_, fut, _), lg in zip(batch, logits):
            if not fut.done():
                fut.set_result(lg)

    def metrics(self):
        """Prometheus-style rows (dan/entrypoints/api_server.py:137-147) plus one set per replica."""
        s = self.stats
        rows = [("dan_requests_total", s.requests), ("dan_request_errors_total", s.errors),
                ("dan_batches_total", s.batches), ("dan_prompt_tokens_total", s.tokens),
                ("dan_busy_seconds_total", round(s.busy_s, 6)),
                ("dan_request_latency_seconds_sum", round(s.latency_s, 6)), ("dan_queue_size", self.queue.qsize())]
        for i, (r, rs) in enumerate(zip(self.runners, self.replica_stats)):
            rows += [(f'dan_replica_batches_total{{replica="{i}"}}', rs.batches),
                     (f'dan_replica_busy_seconds_total{{replica="{i}"}}', round(rs.busy_s, 6))]
            cache = getattr(r, "cache", None)
            if cache is not None:
                rows += [(f'dan_prefix_cache_hits_total{{replica="{i}"}}', cache.hits),
                         (f'dan_prefix_cache_misses_total{{replica="{i}"}}', cache.misses),
                         (f'dan_prefix_cache_bytes{{replica="{i}"}}', cache.used)]
        return "".join(f"{k} {v}\n" for k, v in rows)
