"""Async serving engine over one or more GPU replicas (dan/engine.py:1-113).

Same contract as dan's ``AsyncEngine``: requests queue up; a worker packs them
into prefill batches FIFO up to ``max_batch_tokens`` (cost = prompt tokens +
question tokens), waiting at most ``max_wait_ms`` for company; a batch runs in a
thread (``runner.read_many``; ctypes launches release the GIL) and resolves its
requests' futures; a failing batch fails only its own requests; the queue is
capped (``Overloaded``).

Batches are pipelined per replica: with a runner that has ``submit`` (queue the
batch on the device, return a handle whose ``result()`` waits), up to
``in_flight`` batches are queued at once, so the host collects and packs the
next batch while the device computes the current one. A runner with only
``read_many`` runs one batch at a time.

Planning (the prompt planner's tokenisation, dan/prompt.py:70-123; with
``dan_b200.planner.CachedPlanner`` the chat template is rendered once, not per
prompt) runs on a pool of ``planner_threads`` threads (default 1) instead of the event loop, so
one request's planning does not hold up the others' routing, batching and
result delivery; with a thread-safe planner and a tokenizer that releases the
GIL (Hugging Face fast tokenizers), more threads plan several requests at once.

Difference: ``runner`` may be a list of runners, one per GPU, each with its own
prefix pool and its own queue. A plan whose static prefix was routed before goes
to the same replica (prefix affinity: its cached K/V or recurrent state lives
there); any other plan goes to the least-loaded replica (queued tokens, plus a
batch for a busy one), which becomes that prefix's home. A replica with nothing
queued takes work from another replica's queue only when that queue holds more
than a batch or its oldest plan has waited ``steal_after_ms`` behind a busy
replica. Replicas share nothing on the data path (no collective). ``stats``
aggregates; ``replica_stats`` is per replica.
"""
import asyncio
import time
from collections import OrderedDict, deque
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field

from ._dan import answers, combine


class Overloaded(RuntimeError):
    pass


class _Done:
    """The handle of a batch a ``read_many``-only runner has already read."""

    __slots__ = ("value",)

    def __init__(self, value):
        self.value = value

    def result(self):
        return self.value


@dataclass
class Stats:
    requests: int = 0
    batches: int = 0
    tokens: int = 0
    busy_s: float = 0.0
    latency_s: float = 0.0
    errors: int = 0
    plans: int = 0
    stolen: int = 0
    started: float = field(default_factory=time.time)


class AsyncEngine:
    def __init__(self, planner, runner, max_batch_tokens=8192, max_wait_ms=2.0, max_queue=1024,
                 steal_after_ms=20.0, max_homes=65536, in_flight=2, planner_threads=1):
        self.planner = planner
        self.runners = list(runner) if isinstance(runner, (list, tuple)) else [runner]
        self.runner = self.runners[0]  # dan's /metrics reads engine.runner.cache
        self.max_batch_tokens = max_batch_tokens
        self.max_wait = max_wait_ms / 1000
        self.max_queue = max_queue
        self.steal_after = steal_after_ms / 1000
        self.max_homes = max_homes
        n = len(self.runners)
        self._queues = [deque() for _ in range(n)]  # (plan, future, enqueue time, cost)
        self._queued = [0] * n  # tokens waiting per replica
        self._busy = [0] * n  # per replica: batches being collected or in flight
        self._busy_since = [0.0] * n
        self.in_flight = max(1, int(in_flight))
        self._plan_pool = ThreadPoolExecutor(max(1, int(planner_threads)), thread_name_prefix="dan-plan")
        self._homes = OrderedDict()  # static-prefix key -> replica
        self._arrived = asyncio.Event()
        self.affinity_hits = 0
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

    def queued(self):
        return sum(len(q) for q in self._queues)

    async def decide(self, state, questions, profile=None):
        """Answers keyed by question id, and the input tokens the reads took (engine.py:55-72)."""
        loop = asyncio.get_running_loop()
        plans = await loop.run_in_executor(self._plan_pool, self.planner.plans, state, questions, profile)
        if not plans[0].branches:
            return answers(plans[0], []), 0
        if self.queued() + len(plans) > self.max_queue:
            raise Overloaded("dan is at capacity. Retry shortly.")
        self.start()
        t0 = time.perf_counter()
        futs = [loop.create_future() for _ in plans]
        for plan, fut in zip(plans, futs):
            r, cost = self.route(plan), self.cost(plan)
            self._queues[r].append((plan, fut, time.perf_counter(), cost))
            self._queued[r] += cost
        self._arrived.set()
        reads = await asyncio.gather(*futs)
        self.stats.requests += 1
        self.stats.latency_s += time.perf_counter() - t0
        logp = combine(plans, reads)
        return answers(plans[0], logp, profile, logits_canonical=True), sum(self.cost(p) for p in plans)

    @staticmethod
    def cost(plan):
        return len(plan.prefix) + sum(len(b.suffix) for b in plan.branches)

    @staticmethod
    def prefix_key(plan):
        """The prefix pool's key for ``plan`` (its static prefix, runner.py:56), or None."""
        return hash(tuple(plan.prefix[:plan.static])) if getattr(plan, "static", 0) else None

    def route(self, plan):
        """Replica for ``plan``: its static prefix's home, else the least-loaded replica."""
        key = self.prefix_key(plan)
        if key is not None and key in self._homes:
            self._homes.move_to_end(key)
            self.affinity_hits += 1
            return self._homes[key]
        load = [q + (self.max_batch_tokens if b else 0) for q, b in zip(self._queued, self._busy)]
        r = min(range(len(load)), key=load.__getitem__)
        if key is not None:
            self._homes[key] = r
            if len(self._homes) > self.max_homes:
                self._homes.popitem(last=False)
        return r

    def _source(self, i):
        """Queue replica ``i`` takes its next plan from: its own, else one it may steal from."""
        if self._queues[i]:
            return i
        now, best = time.perf_counter(), None
        for j, q in enumerate(self._queues):
            if j == i or not q:
                continue
            if self._queued[j] > self.max_batch_tokens or (self._busy[j] and now - q[0][2] >= self.steal_after):
                if best is None or self._queued[j] > self._queued[best]:
                    best = j
        return best

    def _pop(self, i, src):
        item = self._queues[src].popleft()
        self._queued[src] -= item[3]
        if src != i:
            self.replica_stats[i].stolen += 1
        return item

    async def _loop(self, replica):
        slots, finishing = asyncio.Semaphore(self.in_flight), set()
        try:
            await self._serve(replica, slots, finishing)
        finally:
            for task in list(finishing):
                task.cancel()

    async def _serve(self, replica, slots, finishing):
        while True:
            await slots.acquire()  # at most ``in_flight`` batches queued on this replica
            while True:
                self._arrived.clear()
                src = self._source(replica)
                if src is not None:
                    break
                try:
                    await asyncio.wait_for(self._arrived.wait(), timeout=self.steal_after)
                except asyncio.TimeoutError:
                    pass
            batch = [self._pop(replica, src)]
            budget = batch[0][3]
            self._mark_busy(replica, +1)  # collecting a batch counts as load for routing and stealing
            deadline = time.perf_counter() + self.max_wait
            while budget < self.max_batch_tokens:
                src = self._source(replica)
                if src is None:
                    left = deadline - time.perf_counter()
                    if left <= 0:
                        break
                    await asyncio.sleep(min(left, 0.0005))
                    continue
                if budget + self._queues[src][0][3] > self.max_batch_tokens:  # stop before the budget
                    break
                batch.append(self._pop(replica, src))
                budget += batch[-1][3]
            handed_off = False
            try:
                pending = await self._submit(replica, batch)
                if pending is not None:
                    task = asyncio.get_running_loop().create_task(
                        self._finish(replica, batch, budget, pending, slots))
                    finishing.add(task)
                    task.add_done_callback(finishing.discard)
                    handed_off = True
            finally:
                if not handed_off:
                    slots.release()
                    self._mark_busy(replica, -1)
                    self._arrived.set()

    def _mark_busy(self, replica, d):
        """Count a batch in (+1) or out (-1); busy seconds add up the time with any batch busy."""
        now = time.perf_counter()
        if d > 0 and self._busy[replica] == 0:
            self._busy_since[replica] = now
        self._busy[replica] += d
        if d < 0 and self._busy[replica] == 0:
            dt = now - self._busy_since[replica]
            self.stats.busy_s += dt
            self.replica_stats[replica].busy_s += dt

    def _fail(self, replica, batch, e):
        self.stats.errors += len(batch)
        self.replica_stats[replica].errors += len(batch)
        for item in batch:
            if not item[1].done():
                item[1].set_exception(e)

    async def _submit(self, replica, batch):
        """Queue ``batch`` on the replica's device; None if that failed (its requests fail)."""
        runner, plans = self.runners[replica], [item[0] for item in batch]
        try:
            if hasattr(runner, "submit"):
                return await asyncio.to_thread(runner.submit, plans)
            return _Done(await asyncio.to_thread(runner.read_many, plans))
        except Exception as e:  # noqa: BLE001 - fail this batch's requests, keep serving
            self._fail(replica, batch, e)
            return None

    async def _finish(self, replica, batch, tokens, pending, slots):
        try:
            try:
                logits = pending.result() if isinstance(pending, _Done) else await asyncio.to_thread(pending.result)
            except Exception as e:  # noqa: BLE001 - fail this batch's requests, keep serving
                self._fail(replica, batch, e)
                return
            for s in (self.stats, self.replica_stats[replica]):
                s.batches += 1
                s.tokens += tokens
                s.plans += len(batch)
            for item, lg in zip(batch, logits):
                if not item[1].done():
                    item[1].set_result(lg)
        finally:
            slots.release()
            self._mark_busy(replica, -1)
            self._arrived.set()  # a replica that just went idle may now be stolen from

    def metrics(self):
        """Prometheus-style rows (dan/entrypoints/api_server.py:137-147) plus one set per replica."""
        s = self.stats
        rows = [("dan_requests_total", s.requests), ("dan_request_errors_total", s.errors),
                ("dan_batches_total", s.batches), ("dan_prompt_tokens_total", s.tokens),
                ("dan_busy_seconds_total", round(s.busy_s, 6)),
                ("dan_request_latency_seconds_sum", round(s.latency_s, 6)), ("dan_queue_size", self.queued()),
                ("dan_route_affinity_total", self.affinity_hits)]
        for i, (r, rs) in enumerate(zip(self.runners, self.replica_stats)):
            rows += [(f'dan_replica_batches_total{{replica="{i}"}}', rs.batches),
                     (f'dan_replica_busy_seconds_total{{replica="{i}"}}', round(rs.busy_s, 6)),
                     (f'dan_replica_plans_total{{replica="{i}"}}', rs.plans),
                     (f'dan_replica_stolen_total{{replica="{i}"}}', rs.stolen),
                     (f'dan_replica_queued_tokens{{replica="{i}"}}', self._queued[i])]
            cache = getattr(r, "cache", None)
            if cache is not None:
                rows += [(f'dan_prefix_cache_hits_total{{replica="{i}"}}', cache.hits),
                         (f'dan_prefix_cache_misses_total{{replica="{i}"}}', cache.misses),
                         (f'dan_prefix_cache_bytes{{replica="{i}"}}', cache.used)]
        return "".join(f"{k} {v}\n" for k, v in rows)
