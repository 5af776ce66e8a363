"""Offline Python API (dan/entrypoints/llm.py:1-64) on the dan_b200 runner.

    llm = LLM("/models/Llama-3-8B-Instruct", planner=dan.prompt.Planner(tokenizer))
    llm.decide("I was charged twice", {"intent": {"type": "choice", "criteria": {"refund": None, "other": None}}})

The planner (tokenizer-bound prompt planning) is dan's own; by default it runs with the
template cache of ``dan_b200.planner.CachedPlanner`` (same plans, the chat template rendered
once instead of per prompt); any object with ``plans(state, questions, profile)`` returning read
plans works. All reads of all requests run in one packed forward per batch.
"""
import torch

from ._dan import answers, combine
from .planner import CachedPlanner
from .runner import Runner


class LLM:
    def __init__(self, model, planner=None, device="cuda", dtype=torch.bfloat16, quantization=None,
                 cache_bytes=2 << 30):
        if planner is None:  # dan installed alongside: its planner, with the template cache
            from transformers import AutoTokenizer

            planner = CachedPlanner(AutoTokenizer.from_pretrained(model))
        self.planner = planner
        self.runner = Runner(model, device, dtype, cache_bytes=cache_bytes, quantization=quantization)

    def decide(self, state, questions, profile=None):
        """Answers keyed by question id, in Jev's answer shapes (llm.py:36-38)."""
        return self.decide_batch([(state, questions)], profile)[0]

    def decide_batch(self, requests, profile=None):
        """[(state, questions), ...] -> answers per request (llm.py:40-44)."""
        groups, logp = self.read(requests, profile)
        return [answers(g[0], lp, profile, logits_canonical=True) for g, lp in zip(groups, logp)]

    def read(self, requests, profile=None, batch_size=None):
        """Per request: its read plans, and per question the rotation-averaged canonical
        log-probabilities before the profile's correction (llm.py:46-64)."""
        groups = [self.planner.plans(s, q, profile) for s, q in requests]
        flat = [p for g in groups for p in g]
        step = batch_size or len(flat) or 1
        reads = []
        for out in self.runner.read_stream(flat[i:i + step] for i in range(0, len(flat), step)):
            reads += out
        out, k = [], 0
        for g in groups:
            out.append(combine(g, reads[k:k + len(g)]))
            k += len(g)
        return groups, out
