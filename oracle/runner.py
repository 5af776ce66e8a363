"""Packing, prefix cache and label reads, restated on the CPU (test infrastructure only).

Follows the reference:
- ``pack``: dan/runner.py:38-64 (flat ids/positions, one segment per plan with
  branches, trunk first then each branch contiguous, branch positions restart
  at ``len(prefix)``, read row = last token of each branch, prefix-cache hit on
  ``prefix[:static]`` skips those tokens, a miss saves them) and ``segment``
  dan/attention.py:114-126 (trunk length = first non-zero branch id, branch
  spans = runs of equal ids);
- ``PrefixCache``: dan/cache.py:11-39 (exact-key LRU under a byte budget);
- ``read_many``: dan/runner.py:66-82 (hidden -> rows -> per-branch fp32 label
  logits -> split per plan; saved prefixes stored after the forward).
"""
from collections import OrderedDict

import torch

from . import llama, qwen3_5


class PrefixCache:
    """cache.py:11-39."""

    def __init__(self, max_bytes=2 << 30):
        self.max_bytes, self.used = max_bytes, 0
        self.entries = OrderedDict()
        self.hits = self.misses = 0

    def get(self, ids):
        key = tuple(ids)
        hit = self.entries.get(key)
        if hit is None:
            self.misses += 1
            return None
        self.hits += 1
        self.entries.move_to_end(key)
        return hit[0]

    def put(self, ids, kv):
        key = tuple(ids)
        if key in self.entries:
            return
        size = sum(t.numel() * t.element_size() for pair in kv.values() for t in pair)
        if size > self.max_bytes:
            return
        while self.used + size > self.max_bytes:
            _, (_, freed) = self.entries.popitem(last=False)
            self.used -= freed
        self.entries[key] = (kv, size)
        self.used += size


def segment(start, branch, past=None, save=0, past_len=0):
    """attention.py:114-126 as a dict."""
    trunk = next((i for i, b in enumerate(branch) if b), len(branch))
    spans, i = [], trunk
    while i < len(branch):
        j = i
        while j < len(branch) and branch[j] == branch[i]:
            j += 1
        spans.append((start + i, start + j))
        i = j
    return {"start": start, "end": start + len(branch), "trunk": trunk, "branches": spans, "past": past,
            "save": save, "past_len": past_len if past else 0, "branch": list(branch), "saved": {}}


def pack(plans, cache=None, use_cache=True):
    """runner.py:38-64 -> (ids, pos, segments, reads, stores)."""
    ids, pos, segs, reads, stores = [], [], [], [], []
    use_cache = use_cache and cache is not None
    for plan in plans:
        if not plan.branches:
            continue
        static = plan.prefix[:plan.static]
        past = cache.get(static) if use_cache and static else None
        skip = plan.static if past else 0
        start = len(ids)
        trunk = plan.prefix[skip:]
        ids += trunk
        pos += range(skip, len(plan.prefix))
        branch = [0] * len(trunk)
        for j, b in enumerate(plan.branches, 1):
            ids += b.suffix
            pos += range(len(plan.prefix), len(plan.prefix) + len(b.suffix))
            branch += [j] * len(b.suffix)
            reads.append((len(ids) - 1, list(b.label_ids)))
        save = plan.static if use_cache and static and not past else 0
        segs.append(segment(start, branch, past, save, skip))
        if save:
            stores.append((static, segs[-1]))
    return ids, pos, segs, reads, stores


def read_many(state, config, plans, cache=None, fp8=False, bf16=False, p_bf16=False):
    """Per plan, per branch: fp32 label logits (runner.py:66-82); ``fp8``: decoder linears
    through the FP8 restatement (Llama family only); ``bf16``: the reference's bf16 path
    (``Runner(dtype=torch.bfloat16)``, the dtype of its GPU and FP8 paths); ``p_bf16``:
    attention probabilities rounded to bf16 before the PV product (Llama family only)."""
    arch = qwen3_5 if config["model_type"].startswith("qwen3_5") else llama
    ids, pos, segs, reads, stores = pack(plans, cache)
    flat = []
    if reads:
        kw = {"bf16": True} if bf16 else {}
        if fp8:
            kw["fp8"] = True
        if p_bf16:
            kw["p_bf16"] = True
        h = arch.hidden(state, config, ids, pos, segs, **kw)
        flat = [arch.label_logits(state, h[r], labels, bf16=bf16) for r, labels in reads]
        for static, seg in stores:
            cache.put(static, seg["saved"])
    out, k = [], 0
    for plan in plans:
        n = len(plan.branches)
        out.append(flat[k:k + n])
        k += n
    return out


def probabilities(logits):
    """Per-question softmax over label logits (readout.py:13-17), fp64 -> fp32."""
    return torch.softmax(torch.as_tensor(logits).double(), 0).float()
