"""Several GPU replicas driven from one process (the engine's multi-replica mode): each
device gets its own kernel attributes and status word, and two threads reading at once give
the same answers as one replica alone. Needs two GPUs; skipped otherwise."""
from concurrent.futures import ThreadPoolExecutor

import pytest
import torch
from conftest import golden, plans_from_json

from dan_b200.runner import Runner
from oracle import weights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    g = golden("tiny_llama.json")
    path = tmp_path_factory.mktemp("tiny_llama_replicas")
    weights.save_checkpoint(str(path), g["config"], weights.random_state(g["config"], g["seed"]))
    return str(path), g


def test_two_replicas_in_one_process(tiny_dir):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path, g = tiny_dir
    runners = [Runner(path, torch.device("cuda", i), cache_bytes=0) for i in (0, 1)]
    batches = [plans_from_json(b["plans"]) for b in g["batches"]]
    solo = [runners[0].read_many(p, probabilities=True) for p in batches]

    def read_all(r):
        return [r.read_many(p, probabilities=True) for p in batches]

    with ThreadPoolExecutor(2) as ex:
        both = list(ex.map(read_all, runners))
    for outs in both:
        for (lg, pr), (lg0, pr0) in zip(outs, solo):
            for a, b in zip(lg + pr, lg0 + pr0):
                assert all(torch.equal(x, y) for x, y in zip(a, b))


def test_engine_over_gpu_replicas(tiny_dir):
    """dan's serving contract on the GPU: concurrent decides through ``AsyncEngine`` over one
    runner per visible GPU (two batches in flight per replica) give the answers solo reads give."""
    import asyncio

    from test_engine import QUESTIONS, FakePlanner

    from dan.readout import answers, combine
    from dan_b200.engine import AsyncEngine

    path, _ = tiny_dir
    n = min(2, torch.cuda.device_count())
    runners = [Runner(path, torch.device("cuda", i), cache_bytes=0) for i in range(n)]
    eng = AsyncEngine(FakePlanner(), runners, max_batch_tokens=96, max_wait_ms=1)
    states = [f"request {i} about billing " * (1 + i % 3) for i in range(24)]

    async def main():
        res = await asyncio.gather(*[eng.decide(s, QUESTIONS) for s in states])
        await eng.stop()
        return res

    res = asyncio.run(main())
    assert eng.stats.requests == len(states) and eng.stats.errors == 0 and eng.stats.batches > 1

    def close(a, b):
        if isinstance(a, dict):
            return a.keys() == b.keys() and all(close(a[k], b[k]) for k in a)
        if isinstance(a, float):
            return abs(a - b) < 1e-5
        return a == b

    for s, (ans, tokens) in zip(states, res):
        plans = FakePlanner().plans(s, QUESTIONS)
        reads = runners[0].read_many(plans)
        solo = answers(plans[0], combine(plans, reads), logits_canonical=True)
        assert close(ans, solo) and tokens == AsyncEngine.cost(plans[0])
