"""Seeded synthetic workloads with the shapes of the five benchmark configurations.

No public dataset is involved: token ids are uniform over the vocabulary and
lengths follow each configuration's stated distributions, all drawn from
``random.Random(seed)`` so a (config, seed) pair gives the same plans anywhere.

- cfg 1: one request, 256-token trunk, 4 branches of 32 tokens, 2-8 labels each.
- cfg 2/3: trunk U[128, 2048], U[1, 16] branches of U[16, 96] tokens; 2-26 labels.
- cfg 4: trunk U[256, 4096], U[1, 8] branches of U[24, 64] tokens; 2-26 labels.
- cfg 5: a fixed 1024-token shared static prefix, then a state of U[64, 1024]
  tokens, then 8 questions of U[16, 96] tokens with U[2, 255] labels.

Batches are formed like the serving engine forms them (dan/engine.py:74-94):
requests in draw order while ``len(prefix) + sum(len(suffix))`` stays within
the token budget (and at most ``max_requests``).
"""
import random

from .plan import Branch, ReadPlan


def _labels(rng, vocab, lo, hi):
    return rng.sample(range(vocab), rng.randint(lo, hi))


def _tokens(rng, vocab, n):
    return [rng.randrange(vocab) for _ in range(n)]


def request(cfg, rng, vocab, shared_prefix=None):
    """One synthetic read plan of configuration ``cfg`` (1-5)."""
    if cfg == 1:
        prefix = _tokens(rng, vocab, 256)
        branches = [Branch(_tokens(rng, vocab, 32), _labels(rng, vocab, 2, 8)) for _ in range(4)]
        return ReadPlan(prefix, branches=branches)
    if cfg in (2, 3):
        prefix = _tokens(rng, vocab, rng.randint(128, 2048))
        nb = rng.randint(1, 16)
        branches = [Branch(_tokens(rng, vocab, rng.randint(16, 96)), _labels(rng, vocab, 2, 26)) for _ in range(nb)]
        return ReadPlan(prefix, branches=branches)
    if cfg == 4:
        prefix = _tokens(rng, vocab, rng.randint(256, 4096))
        nb = rng.randint(1, 8)
        branches = [Branch(_tokens(rng, vocab, rng.randint(24, 64)), _labels(rng, vocab, 2, 26)) for _ in range(nb)]
        return ReadPlan(prefix, branches=branches)
    if cfg == 5:
        shared = shared_prefix if shared_prefix is not None else _tokens(random.Random(5), vocab, 1024)
        prefix = list(shared) + _tokens(rng, vocab, rng.randint(64, 1024))
        branches = [Branch(_tokens(rng, vocab, rng.randint(16, 96)), _labels(rng, vocab, 2, 255)) for _ in range(8)]
        return ReadPlan(prefix, branches=branches, static=len(shared))
    raise ValueError(cfg)


def cost(plan):
    """Tokens a plan takes in the engine's budget (dan/engine.py:74-76)."""
    return len(plan.prefix) + sum(len(b.suffix) for b in plan.branches)


def batch(cfg, seed=0, vocab=128256, max_tokens=8192, max_requests=16):
    """Requests in draw order until the next would exceed ``max_tokens`` or
    ``max_requests`` are taken (the engine's FIFO rule)."""
    rng = random.Random(seed)
    plans, used = [], 0
    while len(plans) < max_requests:
        p = request(cfg, rng, vocab)
        if plans and used + cost(p) > max_tokens:
            break
        plans.append(p)
        used += cost(p)
    return plans


def batches(cfg, count, seed=0, **kw):
    """``count`` consecutive batches drawn from one seeded request stream."""
    rng = random.Random(seed)
    vocab = kw.get("vocab", 128256)
    max_tokens, max_requests = kw.get("max_tokens", 8192), kw.get("max_requests", 16)
    out, pending = [], None
    for _ in range(count):
        plans, used = [], 0
        while len(plans) < max_requests:
            p = pending or request(cfg, rng, vocab)
            pending = None
            if plans and used + cost(p) > max_tokens:
                pending = p
                break
            plans.append(p)
            used += cost(p)
        out.append(plans)
    return out
