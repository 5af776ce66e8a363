"""Tree attention for packed, prefill-only reads (host side of the CUDA kernel).

Same model as the reference (dan/attention.py:1-30): requests are packed into
one flat token sequence; each request is a *segment* whose new tokens are a
trunk followed by one branch per question; a query sees a key when the key
comes first and is trunk (cached past included) or in the same branch.

The reference runs three flash varlen calls, gathers and an LSE merge per
layer (attention.py:210-241). Here one kernel (``dan_tree_attention``) reads
the packed q/k/v rows and the cached prefix pages in place, driven by a tile
table built once per batch (``TreeLayout``) and shared by every layer.
"""
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib, ops
from .cache import PoolEntry

BLOCK = 128  # query rows per tile, keys per block, tokens per pool page
TILE_FIELDS = ("row0", "nrows", "seg_start", "past", "ppad", "split", "nblk_a", "blk_b0", "blk_b1", "page0", "q0v",
               "pad")


def tree_mask(branch):
    """[N, N] boolean mask (True = attend) from per-token branch ids (0 = trunk) (attention.py:54-59)."""
    n = branch.shape[0]
    idx = torch.arange(n, device=branch.device)
    causal = idx[None, :] <= idx[:, None]
    return causal & ((branch[None, :] == 0) | (branch[None, :] == branch[:, None]))


def branch_rows_mask(branch, trunk):
    """The tree mask's rows for branch tokens only (== tree_mask(branch)[trunk:]) (attention.py:62-69)."""
    n = branch.shape[0]
    cols = torch.arange(n, device=branch.device)
    rows = cols[trunk:]
    own = (branch[None, :] == branch[trunk:, None]) & (cols[None, :] <= rows[:, None])
    return (cols[None, :] < trunk) | own


@dataclass
class Segment:
    """One request of a packed batch (attention.py:72-95). ``past`` is a prefix-pool
    entry (its pages hold the cached keys/values of every layer) or None."""
    start: int
    end: int
    trunk: int = 0
    branches: list = field(default_factory=list)
    past: object = None
    save: int = 0
    saved: dict = field(default_factory=dict)
    past_len: int = 0
    branch_ids: list = field(default_factory=list, repr=False)
    device: str = "cpu"


class Batch(list):
    """The segments of one packed forward; caches the tile layout every attention
    layer shares (``layout``), the recurrent-layer layout (``recurrent``) and the paging of
    pasts given as tensors (``staged``)."""

    layout = None
    recurrent = None
    staged = None


def segment(start, branch, past=None, save=0, past_len=0, device="cpu"):
    """A segment over new tokens with ``branch`` ids (trunk first, then each branch
    contiguous), after ``past_len`` cached tokens (attention.py:114-126)."""
    trunk = next((i for i, b in enumerate(branch) if b), len(branch))
    spans, i = [], trunk
    while i < len(branch):
        j = i
        while j < len(branch) and branch[j] == branch[i]:
            j += 1
        spans.append((start + i, start + j))
        i = j
    return Segment(start, start + len(branch), trunk, spans, past, save, past_len=past_len if past else 0,
                   branch_ids=branch, device=device)


def useful_pairs(segments):
    """Visible (query, key) pairs: t(t+1)/2 + P t + sum_b (l_b (P + t) + l_b (l_b + 1) / 2) per segment."""
    total = 0
    for s in segments:
        t, p = s.trunk, s.past_len
        total += t * (t + 1) // 2 + p * t
        for a, b in s.branches:
            n = b - a
            total += n * (p + t) + n * (n + 1) // 2
    return total


@dataclass
class TreeLayout:
    """Device tables of one packed batch for ``dan_tree_attention``."""
    tiles: torch.Tensor  # int32 [n_tiles, 12], longest tiles first
    row_own: torch.Tensor  # int32 [N]: packed row where each row's own run starts
    pages: torch.Tensor  # int32: pool page of each cached 128-token block, per segment
    n_tiles: int
    n_rows: int
    pairs: int  # visible (query, key) pairs (the useful work)
    blocks: int  # key blocks the tiles visit (per head)

    @classmethod
    def build(cls, segments, n_rows, device):
        own = np.zeros(max(n_rows, 1), dtype=np.int32)
        pages, recs = [], []
        for s in segments:
            n = s.end - s.start
            p = s.past_len
            ppad = -(-p // BLOCK) * BLOCK
            split = ppad + s.trunk
            page0 = len(pages)
            if p:
                pg = list(s.past.pages)
                if len(pg) * BLOCK < p:
                    raise ValueError(f"segment at {s.start}: {len(pg)} pages cannot hold {p} cached tokens")
                pages += pg[:ppad // BLOCK]
            own[s.start:s.start + s.trunk] = s.start
            for a, b in s.branches:
                own[a:b] = a
            for t0 in range(0, n, BLOCK):
                nr = min(BLOCK, n - t0)
                q0v, q1v = ppad + t0, ppad + t0 + nr - 1
                nblk_a = -(-min(split, q1v + 1) // BLOCK)
                if q1v >= split:  # the tile holds branch rows
                    rb = max(t0, s.trunk)
                    own_v = ppad + (int(own[s.start + rb]) - s.start)
                    b0, b1 = max(own_v // BLOCK, nblk_a), q1v // BLOCK + 1
                    if b0 >= b1:
                        b0 = b1 = nblk_a
                else:
                    b0 = b1 = nblk_a
                recs.append((s.start + t0, nr, s.start, p, ppad, split, nblk_a, b0, b1, page0, q0v, 0))
        recs.sort(key=lambda r: -(r[6] + r[8] - r[7]))
        tiles = np.asarray(recs, dtype=np.int32).reshape(-1, len(TILE_FIELDS))
        blocks = int((tiles[:, 6] + tiles[:, 8] - tiles[:, 7]).sum()) if len(recs) else 0
        pg = np.asarray(pages or [0], dtype=np.int32)
        dev = torch.device(device)

        def up(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            return t.pin_memory().to(dev, non_blocking=True) if dev.type == "cuda" else t

        lay = cls(up(tiles), up(own[:n_rows] if n_rows else own), up(pg), len(recs), n_rows,
                  useful_pairs(segments), blocks)
        lay.costs = (tiles[:, 6] + tiles[:, 8] - tiles[:, 7]).astype(np.int64) if len(recs) else np.zeros(0, np.int64)
        lay.device = dev
        lay._sched = {}
        return lay

    # A work item (one tile x one pair of query heads) costs its key blocks plus a fixed
    # per-item share (Q load, pipeline fill, epilogue), in block units.
    ITEM_OVERHEAD = 1.5

    def schedule(self, n_pairs, n_ctas):
        """Greedy longest-processing-time assignment of the paired kernel's work items to
        ``n_ctas`` persistent CTAs: (device int32 CSR schedule, number of CTAs)."""
        key = (n_pairs, n_ctas)
        hit = self._sched.get(key)
        if hit is not None:
            return hit
        import heapq

        n_items = self.n_tiles * n_pairs
        ctas = min(n_ctas, n_items)
        cost = np.repeat(self.costs, n_pairs) + self.ITEM_OVERHEAD  # item w = tile * n_pairs + pair
        order = np.argsort(-cost, kind="stable")
        heap = [(0.0, c) for c in range(ctas)]
        lists = [[] for _ in range(ctas)]
        for w in order:
            load, c = heapq.heappop(heap)
            lists[c].append(int(w))
            heapq.heappush(heap, (load + float(cost[w]), c))
        offs = np.zeros(ctas + 1, dtype=np.int32)
        offs[1:] = np.cumsum([len(x) for x in lists])
        flat = np.concatenate([offs, np.asarray([w for x in lists for w in x], dtype=np.int32)])
        t = torch.from_numpy(flat)
        if self.device.type == "cuda":
            t = t.pin_memory().to(self.device, non_blocking=True)
        hit = self._sched[key] = (t, ctas)
        return hit


_SMS = {}


def _sm_count(device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def layout_of(segments, n_rows, device):
    lay = getattr(segments, "layout", None)
    if lay is None or lay.n_rows != n_rows:
        lay = TreeLayout.build(segments, n_rows, device)
        if isinstance(segments, Batch):
            segments.layout = lay
    return lay


def tree_attention(q, k, v, layout, out=None, pool=None, layer=0, scale=None):
    """q: [N, H, D], k/v: [N, Hkv, D] (any row/head strides, unit stride in D) -> out [N, H, D] bf16.

    ``pool``: the prefix pool holding cached keys/values (needed when any segment has a past)."""
    n, h, d = q.shape
    hkv = k.shape[1]
    if out is None:
        out = torch.empty(n, h, d, dtype=q.dtype, device=q.device)
    if layout.n_tiles == 0:
        return out
    scale = d ** -0.5 if scale is None else scale
    if pool is not None and pool.k[layer].shape[0] > 0:
        pk, pv = pool.k[layer], pool.v[layer]
        pool_args = (_lib.ptr(pk), _lib.ptr(pv), pk.stride(0), pk.stride(1), pk.shape[0])
    else:
        pool_args = (None, None, 0, 0, 0)
    sched, ctas = None, 0
    if (h // hkv) % 2 == 0 and d <= 128:  # the paired-head persistent kernel runs this shape
        sched, ctas = layout.schedule(h // 2, _sm_count(q.device))
    _lib.call("dan_tree_attention", _lib.ptr(q), q.stride(0), q.stride(1), _lib.ptr(k), k.stride(0), k.stride(1),
              _lib.ptr(v), v.stride(0), v.stride(1), *pool_args, _lib.ptr(out), out.stride(0), out.stride(1), n, h,
              hkv, d, _lib.ptr(layout.tiles), layout.n_tiles, _lib.ptr(layout.row_own), _lib.ptr(layout.pages),
              _lib.ptr(sched), ctas, float(scale), _lib.ptr(_lib.status_word(q.device)), _lib.stream(),
              work=4 * h * d * layout.pairs)
    return out


class _StagedPasts:
    """Cached prefixes given as dan's per-layer tensors, staged into 128-token pages for the
    kernel: ``segments`` re-stated with page entries (the tile layout is built once per batch
    from them) and one layer's staging pool at a time."""

    def __init__(self, segments):
        self.segments, page = Batch(), 0
        for s in segments:
            entry = None
            if s.past_len:
                npg = -(-s.past_len // BLOCK)
                entry = PoolEntry(list(range(page, page + npg)), s.past_len, 0)
                page += npg
            self.segments.append(Segment(s.start, s.end, s.trunk, s.branches, entry, 0, {}, s.past_len,
                                         s.branch_ids, s.device))
        self.n_pages = page
        self.layer, self.k, self.v = None, {}, {}

    def stage(self, originals, layer, like):
        """Copy every past's keys / values of ``layer`` ([Hkv, P, D] each) into the pages."""
        if self.layer == layer:
            return self
        hkv, d = like.shape[0], like.shape[2]
        # zeroed: rows past each past's length are masked but still multiply into P V
        pk = torch.zeros(self.n_pages * BLOCK, hkv, d, dtype=like.dtype, device=like.device)
        pv = torch.zeros_like(pk)
        for s, t in zip(originals, self.segments):
            if not s.past_len:
                continue
            k, v = s.past[layer]
            rows = torch.arange(s.past_len, dtype=torch.int32, device=like.device)
            dst = torch.as_tensor(t.past.pages, dtype=torch.int32, device=like.device).repeat_interleave(BLOCK)
            dst = (dst * BLOCK + torch.arange(BLOCK, dtype=torch.int32, device=like.device).repeat(len(t.past.pages)))
            kt, vt = k.transpose(0, 1), v.transpose(0, 1)  # [P, Hkv, D] views
            ops.kv_store(kt, vt, pk, pv, rows, dst[:s.past_len].contiguous())
        self.layer, self.k, self.v = layer, {layer: pk}, {layer: pv}
        return self


def attend(q, k, v, segments, layer, scale=None, pool=None):
    """q: [H, N, D]; k, v: [Hkv, N, D] (rotary applied) -> [H, N, D] (attention.py:200-207).

    Views of the packed [N, heads, D] projections are used in place (no copies). Segments
    with ``save`` record copies of their first ``save`` new tokens' k/v in
    ``s.saved[layer]`` as dan does. A segment's ``past`` is either a prefix-pool entry (read
    in place from ``pool``) or dan's per-layer ``{layer: (k, v)}`` tensors [Hkv, past, D],
    which are staged into pages once per layer."""
    for s in segments:
        if s.save:
            s.saved[layer] = (k[:, s.start:s.start + s.save].clone(), v[:, s.start:s.start + s.save].clone())
    segs = segments
    if pool is None and any(s.past_len and not isinstance(s.past, PoolEntry) for s in segments):
        staged = getattr(segments, "staged", None)
        if staged is None:
            staged = _StagedPasts(segments)
            if isinstance(segments, Batch):
                segments.staged = staged
        pool = staged.stage(segments, layer, k)
        segs = staged.segments
    lay = layout_of(segs, q.shape[1], q.device)
    out = tree_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1), lay, pool=pool, layer=layer,
                         scale=scale)
    return out.transpose(0, 1)
