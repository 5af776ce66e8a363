"""Shared test helpers: build packed segment batches with cached pasts."""
import random
import re

import numpy as np
import torch

from dan_b200.attention import BLOCK, Batch, segment
from dan_b200.cache import PoolEntry


def header_symbols(path):
    text = open(path).read()
    return sorted(set(re.findall(r"\b(dan_[a-z0-9_]+)\s*\(", text)))


def build_segments(shapes, device="cpu", page_base=0, shuffle_pages=True, seed=0):
    """shapes: [(trunk, [branch lens], past)] -> (Batch, n_rows, pages_needed).
    Pasts get pool pages (a permutation, so page order is not trivial)."""
    rng = random.Random(seed)
    segs, start, page = Batch(), 0, page_base
    for trunk, lens, past in shapes:
        branch = [0] * trunk + [j for j, n in enumerate(lens, 1) for _ in range(n)]
        entry = None
        if past:
            npg = -(-past // BLOCK)
            entry = PoolEntry(list(range(page, page + npg)), past, 0)
            page += npg
        segs.append(segment(start, branch, entry, 0, past, device))
        start += len(branch)
    if shuffle_pages:
        all_pages = list(range(page_base, page))
        perm = all_pages[:]
        rng.shuffle(perm)
        remap = dict(zip(all_pages, perm))
        for s in segs:
            if s.past:
                s.past.pages = [remap[p] for p in s.past.pages]
    return segs, start, page


def kernel_visible(layout, n_rows):
    """Replay the kernel's block enumeration and mask from a TreeLayout on the CPU.
    Returns {packed_row: sorted list of virtual key indices}, and asserts no block twice."""
    tiles = layout.tiles.cpu().numpy()
    own = layout.row_own.cpu().numpy()
    vis = {}
    for t in tiles:
        row0, nrows, seg_start, past, ppad, split, nblk_a, b0, b1, page0, q0v, _ = (int(x) for x in t)
        blocks = list(range(nblk_a)) + list(range(b0, b1))
        assert len(set(blocks)) == len(blocks)
        for i in range(nrows):
            r = row0 + i
            qv = q0v + i
            ov = ppad + (int(own[r]) - seg_start)
            keys = []
            for b in blocks:
                v = np.arange(b * BLOCK, (b + 1) * BLOCK)
                ok = (v <= qv) & ((v < split) | (v >= ov)) & ((v < past) | (v >= ppad))
                keys += v[ok].tolist()
            vis[r] = keys
    return vis


def expected_visible(segs):
    """Oracle: per packed row, the visible virtual key indices from the tree mask."""
    from oracle.attention import segment_mask

    out = {}
    for s in segs:
        p = s.past_len
        ppad = -(-p // BLOCK) * BLOCK
        m = segment_mask(s.branch_ids, p)
        for i in range(s.end - s.start):
            cols = torch.nonzero(m[i]).flatten().tolist()
            out[s.start + i] = [c if c < p else ppad + (c - p) for c in cols]
    return out


def attention_problem(shapes, h, hkv, d, device, dtype=torch.bfloat16, seed=0):
    """Seeded packed q/k/v [N, heads, D], a pool holding every segment's past, and the
    oracle segments (dicts) with the same past tensors."""
    segs, n, npages = build_segments(shapes, device)
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(n, h, d, generator=gen).to(dtype)
    k = torch.randn(n, hkv, d, generator=gen).to(dtype)
    v = torch.randn(n, hkv, d, generator=gen).to(dtype)
    pool_k = torch.zeros(max(npages, 1) * BLOCK, hkv, d, dtype=dtype)
    pool_v = torch.zeros_like(pool_k)
    oracle_segs = []
    for s in segs:
        past = None
        if s.past_len:
            pk = torch.randn(s.past_len, hkv, d, generator=gen).to(dtype)
            pv = torch.randn(s.past_len, hkv, d, generator=gen).to(dtype)
            for t in range(s.past_len):
                row = s.past.pages[t // BLOCK] * BLOCK + t % BLOCK
                pool_k[row], pool_v[row] = pk[t], pv[t]
            past = (pk.transpose(0, 1).float(), pv.transpose(0, 1).float())
        oracle_segs.append({"start": s.start, "end": s.end, "branch": s.branch_ids, "past": past})
    return segs, n, q, k, v, pool_k, pool_v, oracle_segs
