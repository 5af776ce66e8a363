"""Prefix cache as a paged HBM pool.

Same contract as the reference's ``PrefixCache`` (dan/cache.py:11-39): entries
are keyed by the exact static-prefix token ids, a hit is always exact,
``get`` counts ``hits`` / ``misses``, ``used`` is the bytes held, and eviction
is least-recently-used under a byte budget.

Instead of per-layer ``(k, v)`` tensors copied into every batch that reuses
them (attention.py:217-226), keys and values live in fixed 128-token pages of
one preallocated pool per model, ``k`` / ``v`` [layers, pages * 128, Hkv, D]
bf16. An entry is a list of pages; the attention kernel reads them in place
through a page table. Recurrent (DeltaNet) layers keep, per entry, one state
slot: the conv tail and the state of every DeltaNet layer, held as ``conv``
[layers, slots, k - 1, conv_dim] bf16 and ``state`` [layers, slots, Hv, Dk, Dv]
fp32 (qwen3_5.py:207-209).

Pages are reserved when a batch is packed (the reference stores after the
forward); entries used as ``past`` by the batch being packed are never evicted
for it, and a prefix that cannot fit is simply not cached (as the reference
skips entries larger than the budget).
"""
from collections import OrderedDict
from dataclasses import dataclass, field

import torch

PAGE = 128


@dataclass
class PoolEntry:
    pages: list
    length: int
    nbytes: int
    slot: int = -1  # recurrent state slot, -1 for attention-only models
    layers: dict = field(default_factory=dict, repr=False)

    def __bool__(self):
        return True


class PrefixPool:
    def __init__(self, max_bytes, layers, kv_heads, head_dim, device, recurrent=None):
        """``recurrent``: optional (n_delta_layers, conv_rows, conv_dim, hv, dk, dv) for hybrid models."""
        self.max_bytes = max_bytes
        self.page_bytes = PAGE * kv_heads * head_dim * 2 * 2 * max(layers, 1)
        self.slot_bytes = 0
        if recurrent:
            nl, kr, cd, hv, dk, dv = recurrent
            self.slot_bytes = nl * (kr * cd * 2 + hv * dk * dv * 4)
        budget = max_bytes
        self.n_slots = 0
        if recurrent:
            self.n_slots = max(0, min(64, budget // (4 * self.slot_bytes)))
            budget -= self.n_slots * self.slot_bytes
        self.n_pages = max(0, budget // self.page_bytes) if layers else 0
        dev = torch.device(device)
        # Zeroed once: the kernel masks the rows of an entry's last page past its length, and a
        # masked row still enters P V with weight 0, which must not meet a NaN bit pattern. Pages
        # reused after eviction hold earlier entries' (finite) keys and values.
        self.k = torch.zeros(layers, self.n_pages * PAGE, kv_heads, head_dim, dtype=torch.bfloat16, device=dev)
        self.v = torch.zeros_like(self.k)
        if recurrent:  # layer-major, so one layer's slots are one contiguous block
            nl, kr, cd, hv, dk, dv = recurrent
            self.conv = torch.zeros(nl, self.n_slots, kr, cd, dtype=torch.bfloat16, device=dev)
            self.state = torch.zeros(nl, self.n_slots, hv, dk, dv, dtype=torch.float32, device=dev)
        self.free_pages = list(range(self.n_pages))
        self.free_slots = list(range(self.n_slots))
        self.recurrent = bool(recurrent)
        self.entries = OrderedDict()
        self.hits = self.misses = 0
        self.used = 0

    def get(self, ids):
        key = tuple(ids)
        hit = self.entries.get(key)
        if hit is None:
            self.misses += 1
            return None
        self.hits += 1
        self.entries.move_to_end(key)
        return hit

    def _evict_one(self, pinned):
        for key, e in self.entries.items():
            if id(e) not in pinned:
                del self.entries[key]
                self._free(e)
                return True
        return False

    def _free(self, e):
        self.free_pages += e.pages
        if e.slot >= 0:
            self.free_slots.append(e.slot)
        self.used -= e.nbytes

    def reserve(self, ids, length, pinned=()):
        """Pages (and a state slot) for ``length`` tokens of prefix ``ids``, evicting LRU
        entries not in ``pinned``; None when the prefix cannot be cached."""
        if tuple(ids) in self.entries:
            return None
        need = -(-length // PAGE) if self.page_bytes and self.n_pages else 0
        nbytes = length * self.page_bytes // PAGE + self.slot_bytes
        if nbytes > self.max_bytes or need > self.n_pages or (self.recurrent and not self.n_slots):
            return None
        pinned = {id(e) for e in pinned}
        while len(self.free_pages) < need or (self.recurrent and not self.free_slots):
            if not self._evict_one(pinned):
                return None
        pages = [self.free_pages.pop() for _ in range(need)]
        slot = self.free_slots.pop() if self.recurrent else -1
        self.used += nbytes
        return PoolEntry(pages, length, nbytes, slot)

    def commit(self, ids, entry):
        self.entries[tuple(ids)] = entry

    def release(self, entry):
        self._free(entry)

    def rows(self, entry, count=None):
        """Pool rows of the first ``count`` tokens of ``entry``."""
        count = entry.length if count is None else count
        return [entry.pages[t // PAGE] * PAGE + t % PAGE for t in range(count)]

    def clear(self):
        for e in list(self.entries.values()):
            self._free(e)
        self.entries.clear()


class PrefixCache:
    """dan's prefix cache contract (dan/cache.py:11-39) for callers that keep per-layer
    ``{layer: (k, v)}`` tensors (``attend`` reads such pasts by staging them into pages):
    exact-key entries, ``get`` counting ``hits`` / ``misses``, ``used`` bytes under
    ``max_bytes`` with least-recently-used eviction, entries larger than the budget not kept.
    ``Runner`` uses the paged ``PrefixPool`` above instead, which the kernels read in place."""

    def __init__(self, max_bytes=2 << 30):
        self.max_bytes = max_bytes
        self.used = 0
        self.hits = self.misses = 0
        self._lru = OrderedDict()  # key -> (kv, nbytes), least recent first

    def get(self, ids):
        found = self._lru.get(tuple(ids))
        if found is None:
            self.misses += 1
            return None
        self.hits += 1
        self._lru.move_to_end(tuple(ids))
        return found[0]

    def put(self, ids, kv):
        key = tuple(ids)
        nbytes = sum(t.numel() * t.element_size() for pair in kv.values() for t in pair)
        if key in self._lru or nbytes > self.max_bytes:
            return
        while self._lru and self.used + nbytes > self.max_bytes:
            self.used -= self._lru.popitem(last=False)[1][1]
        self._lru[key] = (kv, nbytes)
        self.used += nbytes

    @property
    def entries(self):
        return self._lru
