"""The serving engine on the CPU with fake replicas (no GPU); answers are formatted by dan's own
readout module, installed beside this package.

Mirrors the reference's serving tests (tests/test_api.py:51-68: concurrent decides are
batched and give the same answers as solo reads) and its failure isolation
(engine.py:102-107: a failing batch fails only its own requests), over several
replicas; fault injection is on the host (a replica that raises)."""
import asyncio
import random
import threading

import pytest
import torch

pytest.importorskip("dan.readout")  # dan's own answer formatting, installed beside this package

from dan.readout import answers  # noqa: E402

from dan_b200.engine import AsyncEngine, Overloaded  # noqa: E402
from dan_b200.plan import Branch, ReadPlan  # noqa: E402


class Spec:
    def __init__(self, key, type_, options, legend=None):
        self.key, self.type, self.options, self.legend = key, type_, options, legend


class FakePlanner:
    """Plans for a state string: trunk tokens from the text, one branch per question."""

    def plans(self, state, questions, profile=None):
        prefix = [ord(c) % 97 for c in state] or [1]
        specs = [Spec(k, q["type"], [(o, "") for o in q["options"]]) for k, q in questions.items()]
        branches = [Branch([len(k), 3], list(range(len(q["options"])))) for k, q in questions.items()]
        return [ReadPlan(prefix, specs=specs, branches=branches, order=list(questions), perms=[])]


class FakeRunner:
    """Deterministic 'logits' from the plan; optionally raises on chosen batches."""

    def __init__(self, fail_on=(), delay=0.0):
        self.calls, self.fail_on, self.delay = 0, set(fail_on), delay
        self.lock = threading.Lock()

    def read_many(self, plans):
        import time

        with self.lock:
            self.calls += 1
            n = self.calls
        time.sleep(self.delay)
        if n in self.fail_on:
            raise RuntimeError(f"injected failure on batch {n}")
        return [[torch.tensor([float(sum(p.prefix) % 7), float(len(b.suffix))] + [0.0] * (len(b.label_ids) - 2))
                 for b in p.branches] for p in plans]


QUESTIONS = {"urgent": {"type": "noul", "options": ["yes", "no"]},
             "topic": {"type": "choice", "options": ["a", "b", "c"]}}


def run(coro):
    return asyncio.run(coro)


def test_concurrent_decides_are_batched_and_match_solo_reads():
    runner = FakeRunner()
    eng = AsyncEngine(FakePlanner(), runner, max_wait_ms=20)

    async def main():
        states = [f"state number {i}" for i in range(12)]
        res = await asyncio.gather(*[eng.decide(s, QUESTIONS) for s in states])
        await eng.stop()
        return states, res

    states, res = run(main())
    assert eng.stats.batches < 12 and eng.stats.requests == 12
    for s, (ans, tokens) in zip(states, res):
        plan = FakePlanner().plans(s, QUESTIONS)[0]
        solo = answers(plan, FakeRunner().read_many([plan])[0])
        assert ans == solo and tokens == AsyncEngine.cost(plan)


def test_replicas_share_the_queue_and_failures_stay_in_their_batch():
    runners = [FakeRunner(fail_on={1}, delay=0.01), FakeRunner(delay=0.01)]
    eng = AsyncEngine(FakePlanner(), runners, max_batch_tokens=40, max_wait_ms=1)

    async def main():
        states = [f"s{i}" * 5 for i in range(16)]
        res = await asyncio.gather(*[eng.decide(s, QUESTIONS) for s in states], return_exceptions=True)
        await eng.stop()
        return res

    res = run(main())
    failed = [r for r in res if isinstance(r, Exception)]
    assert failed and all("injected" in str(e) for e in failed)
    assert len(failed) < len(res)  # the engine kept serving after the failing batch
    assert all(r.calls > 0 for r in runners)  # both replicas took batches
    assert eng.stats.errors == len(failed)
    assert 'replica="1"' in eng.metrics()


def test_overloaded_at_queue_cap():
    eng = AsyncEngine(FakePlanner(), FakeRunner(), max_queue=0)

    async def main():
        with pytest.raises(Overloaded):
            await eng.decide("x", QUESTIONS)

    run(main())


class PrefixPlanner(FakePlanner):
    """Plans whose prompt (the text before '|') is a cacheable static prefix."""

    def plans(self, state, questions, profile=None):
        plans = super().plans(state.split("|")[0], questions, profile)
        for p in plans:
            p.static = len(p.prefix)
        return plans


class RecordingRunner(FakeRunner):
    def __init__(self, delay=0.0):
        super().__init__(delay=delay)
        self.prefixes = []

    def read_many(self, plans):
        with self.lock:
            self.prefixes += [tuple(p.prefix) for p in plans]
        return super().read_many(plans)


def test_prefix_affinity_keeps_each_prefix_on_one_replica():
    """Plans sharing a static prefix go to the replica whose pool holds it (the prefix's home);
    new prefixes go to the least-loaded replica, so two prefixes land on different replicas."""
    runners = [RecordingRunner(delay=0.005), RecordingRunner(delay=0.005)]
    eng = AsyncEngine(PrefixPlanner(), runners, max_batch_tokens=10_000, max_wait_ms=1, steal_after_ms=10_000)

    async def main():
        for wave in range(4):
            await asyncio.gather(*[eng.decide(f"{tag} shared prompt|{wave}{i}", QUESTIONS)
                                   for tag in ("alpha", "beta") for i in range(3)])
        await eng.stop()

    run(main())
    homes = {}
    for i, r in enumerate(runners):
        for pre in r.prefixes:
            homes.setdefault(pre, set()).add(i)
    assert len(homes) == 2 and all(len(v) == 1 for v in homes.values())
    assert set().union(*homes.values()) == {0, 1}
    assert eng.affinity_hits == 4 * 6 - 2  # every plan but the first of each prefix
    assert "dan_route_affinity_total 22" in eng.metrics()


def test_idle_replica_steals_a_backlog_from_a_busy_one():
    """All plans share one prefix (home: replica 0, which is slow); once its queue holds more
    than a batch, the idle replica takes work from it, and every request is answered."""
    runners = [RecordingRunner(delay=0.05), RecordingRunner(delay=0.0)]
    eng = AsyncEngine(PrefixPlanner(), runners, max_batch_tokens=60, max_wait_ms=1, steal_after_ms=5)

    async def main():
        res = await asyncio.gather(*[eng.decide(f"same prefix|{i}", QUESTIONS) for i in range(12)])
        await eng.stop()
        return res

    res = run(main())
    assert len(res) == 12 and all(isinstance(r, tuple) for r in res)
    assert runners[1].calls > 0 and eng.replica_stats[1].stolen > 0
    assert sum(rs.plans for rs in eng.replica_stats) == 12


class PipelinedRunner(FakeRunner):
    """A runner with the two-phase interface: ``submit`` returns at once and its handle's
    ``result`` returns ``delay`` seconds after the previous batch's (a device that runs the
    queued batches in order); records how many batches were outstanding at most."""

    def __init__(self, fail_on=(), delay=0.0):
        super().__init__(fail_on=fail_on, delay=delay)
        self.outstanding = self.max_outstanding = 0
        self.ready_at = 0.0

    def submit(self, plans):
        import time

        with self.lock:
            self.calls += 1
            n = self.calls
            self.outstanding += 1
            self.max_outstanding = max(self.max_outstanding, self.outstanding)
            self.ready_at = max(time.perf_counter(), self.ready_at) + self.delay
            done_at = self.ready_at
        value = FakeRunner(delay=0.0).read_many(plans)
        runner = self

        class Handle:
            def result(self):
                time.sleep(max(0.0, done_at - time.perf_counter()))
                with runner.lock:
                    runner.outstanding -= 1
                if n in runner.fail_on:
                    raise RuntimeError(f"injected failure on batch {n}")
                return value

        return Handle()


@pytest.mark.parametrize("in_flight", [1, 2, 3])
def test_pipelined_batches_stay_bounded_and_answer_like_solo_reads(in_flight):
    """With a two-phase runner the engine queues up to ``in_flight`` batches at once (the host
    packs the next batch while the device runs one); answers equal solo reads, a failing batch
    fails only its own requests, and busy seconds count overlapping batches once."""
    import time

    runner = PipelinedRunner(fail_on={3}, delay=0.01)
    eng = AsyncEngine(FakePlanner(), runner, max_batch_tokens=40, max_wait_ms=1, in_flight=in_flight)

    async def main():
        states = [f"p{i}" * 5 for i in range(24)]
        t0 = time.perf_counter()
        res = await asyncio.gather(*[eng.decide(s, QUESTIONS) for s in states], return_exceptions=True)
        wall = time.perf_counter() - t0
        await eng.stop()
        return states, res, wall

    states, res, wall = run(main())
    assert 1 <= runner.max_outstanding <= in_flight
    if in_flight > 1:
        assert runner.max_outstanding == in_flight  # the 24 requests keep the pipeline full
    failed = [r for r in res if isinstance(r, Exception)]
    assert failed and all("injected failure on batch 3" in str(e) for e in failed)
    assert eng.stats.errors == len(failed) and eng.stats.batches == runner.calls - 1
    for s, r in zip(states, res):
        if isinstance(r, Exception):
            continue
        plan = FakePlanner().plans(s, QUESTIONS)[0]
        assert r[0] == answers(plan, FakeRunner().read_many([plan])[0])
    assert 0 < eng.stats.busy_s <= wall + 1e-3
    assert runner.outstanding == 0


class SlowPlanner(FakePlanner):
    """Planning that takes 50 ms outside the GIL (as a fast tokenizer's encode does)."""

    def plans(self, state, questions, profile=None):
        import time

        time.sleep(0.05)
        return super().plans(state, questions, profile)


def test_planning_runs_off_the_event_loop():
    """The engine plans on its planner pool: the event loop stays free while a request is being
    planned (a ticker keeps running), and with a thread-safe planner several plan at once."""
    import time

    def measure(threads):
        eng = AsyncEngine(SlowPlanner(), FakeRunner(), max_wait_ms=1, planner_threads=threads)
        ticks = []

        async def ticker(stop):
            while not stop.is_set():
                ticks.append(time.perf_counter())
                await asyncio.sleep(0.005)

        async def main():
            stop = asyncio.Event()
            tick = asyncio.create_task(ticker(stop))
            t0 = time.perf_counter()
            res = await asyncio.gather(*[eng.decide(f"state {i}", QUESTIONS) for i in range(8)])
            dt = time.perf_counter() - t0
            stop.set()
            await tick
            await eng.stop()
            return res, dt

        res, dt = run(main())
        gaps = [b - a for a, b in zip(ticks, ticks[1:])]
        return res, dt, max(gaps) if gaps else 0.0

    res1, dt1, gap1 = measure(1)
    res4, dt4, gap4 = measure(4)
    assert len(res1) == len(res4) == 8 and [r[1] for r in res1] == [r[1] for r in res4]
    assert gap1 < 0.045 and gap4 < 0.045  # the loop never waited out a 50 ms planning call
    assert dt4 < 0.7 * dt1  # four planning threads overlap the 8 x 50 ms of planning
