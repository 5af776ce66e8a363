"""Host-side logic on the CPU: the C-ABI library, packing, the tree-attention tile
table and the prefix pool policy. No GPU calls."""
import os
import random

import pytest
import torch
from conftest import ROOT, golden, plans_from_json
from helpers import build_segments, expected_visible, header_symbols, kernel_visible

from dan_b200 import synthetic
from dan_b200.attention import TreeLayout, useful_pairs
from dan_b200.cache import PrefixPool
from dan_b200.runner import Runner


@pytest.fixture(scope="session")
def built_lib():
    from dan_b200 import _lib, build

    build.build()
    return _lib


def test_library_exports_every_header_symbol(built_lib):
    lib = built_lib.lib()
    syms = header_symbols(os.path.join(ROOT, "include", "dan_b200.h"))
    assert len(syms) >= 12
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    assert b"sm_100a" in lib.dan_version()


def cpu_runner(cache_bytes=1 << 30):
    r = Runner.__new__(Runner)
    r.device = torch.device("cpu")
    r.cache = PrefixPool(cache_bytes, 1, 1, 8, "cpu") if cache_bytes else None
    return r


def test_pack_matches_reference_bit_exact():
    runner = cpu_runner()
    for rec in golden("pack.json"):
        plans = plans_from_json(rec["plans"])
        ids, pos, segs, reads, stores = runner.pack(plans)
        assert ids == rec["ids"] and pos == rec["pos"]
        assert [[r, list(l)] for r, l in reads] == rec["reads"]
        assert len(segs) == len(rec["segments"])
        for s, r in zip(segs, rec["segments"]):
            assert (s.start, s.end, s.trunk, s.past_len, s.save, bool(s.past)) == \
                (r["start"], r["end"], r["trunk"], r["past_len"], r["save"], r["has_past"])
            assert [list(x) for x in s.branches] == r["branches"]
            assert list(s.branch_ids) == r["branch_ids"]
        assert [[len(st), segs.index(sg)] for st, sg in stores] == rec["stores"]
        held, _, _ = runner._reserve(segs, stores)
        for static, seg, entry in held:
            runner.cache.commit(static, entry)


def test_read_layout_rows_match_reference():
    """The reference's varlen row sets and cumulative lengths (attention.py:155-172) follow
    from our segments exactly."""
    runner = cpu_runner()
    for rec in golden("pack.json"):
        plans = plans_from_json(rec["plans"])
        ids, pos, segs, reads, stores = runner.pack(plans)
        want = rec["read_layout"]
        trunk_rows = [r for s in segs for r in range(s.start, s.start + s.trunk)]
        branch_rows = [r for s in segs for r in range(s.start + s.trunk, s.end)]
        assert trunk_rows == want["trunk_rows"] and branch_rows == want["branch_rows"]
        cu = lambda xs: [0] + list(__import__("itertools").accumulate(xs))
        assert cu([s.trunk for s in segs]) == want["cu_trunk_q"]
        assert cu([s.past_len + s.trunk for s in segs]) == want["cu_trunk_k"]
        assert cu([s.end - s.start - s.trunk for s in segs]) == want["cu_branch_q"]
        bl = [b - a for s in segs for a, b in s.branches]
        assert (cu(bl) if bl else None) == want["cu_branch"]
        held, _, _ = runner._reserve(segs, stores)
        for static, seg, entry in held:
            runner.cache.commit(static, entry)


EDGE = [(40, [5, 9, 1], 0), (7, [30], 12), (1, [3, 3, 3, 3, 3, 3], 0), (64, [], 0), (13, [17, 2], 20)]


@pytest.mark.parametrize("shapes", [
    EDGE,
    [(300, [17, 200, 1], 0), (129, [128, 128], 250), (0, [5, 7], 130), (128, [1], 128), (1000, [96] * 12, 0)],
    [(0, [3], 1), (5, [], 300), (256, [0 + 64] * 5, 1024)],
])
def test_tree_layout_visits_exactly_the_tree_mask(shapes):
    segs, n, _ = build_segments(shapes)
    lay = TreeLayout.build(segs, n, "cpu")
    got = kernel_visible(lay, n)
    want = expected_visible(segs)
    assert got.keys() == want.keys()
    for r in want:
        assert sorted(got[r]) == want[r], r
    assert lay.pairs == sum(len(v) for v in want.values()) == useful_pairs(segs)


def test_tree_layout_random_batches():
    rng = random.Random(7)
    for trial in range(20):
        shapes = [(rng.randint(0, 400), [rng.randint(1, 150) for _ in range(rng.randint(0, 6))],
                   rng.choice([0, 0, rng.randint(1, 700)])) for _ in range(rng.randint(1, 5))]
        shapes = [s for s in shapes if s[0] + sum(s[1]) > 0]
        if not shapes:
            continue
        segs, n, _ = build_segments(shapes, seed=trial)
        lay = TreeLayout.build(segs, n, "cpu")
        got, want = kernel_visible(lay, n), expected_visible(segs)
        for r in want:
            assert sorted(got[r]) == want[r]


def test_tiles_are_longest_first_and_cover_all_rows():
    plans = synthetic.batch(2, seed=3)
    runner = cpu_runner(0)
    ids, pos, segs, reads, stores = runner.pack(plans)
    lay = TreeLayout.build(segs, len(ids), "cpu")
    t = lay.tiles.numpy()
    cost = t[:, 6] + t[:, 8] - t[:, 7]
    assert (cost[:-1] >= cost[1:]).all()
    assert t[:, 1].sum() == len(ids)


def test_synthetic_batches_follow_the_engine_rule():
    for seed in range(5):
        plans = synthetic.batch(2, seed=seed)
        used = sum(synthetic.cost(p) for p in plans)
        assert used <= 8192 and len(plans) <= 16
        for p in plans:
            assert 128 <= len(p.prefix) <= 2048 and 1 <= len(p.branches) <= 16
            assert all(16 <= len(b.suffix) <= 96 and 2 <= len(b.label_ids) <= 26 for b in p.branches)
    b = synthetic.batches(3, 3, seed=1)
    assert len(b) == 3 and all(sum(synthetic.cost(p) for p in x) <= 8192 for x in b)


def test_prefix_pool_lru_and_budget():
    page_bytes = 128 * 1 * 8 * 2 * 2
    pool = PrefixPool(page_bytes * 4, 1, 1, 8, "cpu")
    assert pool.n_pages == 4
    a = pool.reserve([1, 2], 200)  # 2 pages
    pool.commit([1, 2], a)
    b = pool.reserve([3], 130)  # 2 pages
    pool.commit([3], b)
    assert pool.get([1, 2]) is a and pool.hits == 1
    c = pool.reserve([4], 100)  # evicts the LRU entry ([3]); [1, 2] was just used
    pool.commit([4], c)
    assert pool.get([3]) is None and pool.misses == 1
    assert pool.get([1, 2]) is a
    assert pool.reserve([5], 10 ** 6) is None  # larger than the budget: not cached
    d = pool.reserve([6], 300, pinned=[a, c])  # needs 3 pages, only pinned entries left
    assert d is None
    assert pool.used == a.nbytes + c.nbytes


def test_lpt_schedule_covers_every_item_once():
    plans = synthetic.batch(2, seed=4)
    runner = cpu_runner(0)
    ids, pos, segs, reads, stores = runner.pack(plans)
    lay = TreeLayout.build(segs, len(ids), "cpu")
    sched, ctas = lay.schedule(16, 148)
    s = sched.numpy()
    offs, items = s[:ctas + 1], s[ctas + 1:]
    assert offs[0] == 0 and offs[-1] == len(items) == lay.n_tiles * 16
    assert sorted(items.tolist()) == list(range(lay.n_tiles * 16))
    cost = lay.costs.repeat(16) + lay.ITEM_OVERHEAD
    loads = [cost[items[offs[c]:offs[c + 1]]].sum() for c in range(ctas)]
    assert max(loads) <= sum(loads) / ctas + cost.max()  # greedy LPT bound


def test_recurrent_layout_chunks_follow_each_segments_runs():
    """The DeltaNet scan's chunk list: every run (trunk to the save cut, rest of the trunk, each
    branch) is cut into chunks of at most 64 rows that tile it exactly; a segment's chunks are
    contiguous in processing order from its record's first-chunk field; segment records are
    sorted longest first (the longest chains start first)."""
    from dan_b200.qwen3_5 import CHUNK, RecurrentLayout

    segs, n, _ = build_segments([(70, [3, 64, 65], 0), (300, [], 0), (1, [129], 0), (64, [1], 0)],
                                shuffle_pages=False)
    segs[1].save = 130  # a save cut inside the trunk splits it into two runs
    rl = RecurrentLayout.build(segs, n, 3, "cpu")
    recs, brs, chunks = rl.segs.numpy(), rl.branches.numpy(), rl.chunks.numpy()
    assert rl.n_chunks == len(chunks) and (chunks[:, 1] >= 1).all() and (chunks[:, 1] <= CHUNK).all()
    lens = [r[1] + sum(brs[r[5] + i][1] for i in range(r[6])) for r in recs]
    assert lens == sorted(lens, reverse=True)
    seen = []
    for r in recs:
        start, trunk, cut, b0, nb, c = r[0], r[1], r[2], r[5], r[6], r[7]
        runs = [(start, cut), (start + cut, trunk - cut)] + [(brs[b0 + i][0], brs[b0 + i][1]) for i in range(nb)]
        for i, (rs, rlen) in enumerate(runs):
            if i >= 2:
                assert brs[b0 + i - 2][2] == c  # a branch record points at its first chunk
            for t0 in range(0, rlen, CHUNK):
                assert tuple(chunks[c]) == (rs + t0, min(CHUNK, rlen - t0))
                seen.append(c)
                c += 1
    assert sorted(seen) == list(range(rl.n_chunks))  # every chunk belongs to exactly one run
    assert recs[[r[1] for r in recs].index(300)][2] == 130
    # each segment's (first chunk, chunk count), longest first, for the scan's split launch
    assert [c0 for c0, _ in rl.seg_chunks] == [int(r[7]) for r in recs]
    assert sum(k for _, k in rl.seg_chunks) == rl.n_chunks


def test_scan_split_rule():
    """The scan splits off segment 0's chain only when it leads the next segment by more than
    the overlap costs the rest of the pre-pass, and never for one segment or a short lead."""
    from dan_b200.qwen3_5 import RecurrentLayout

    rule = RecurrentLayout.split_lead
    assert rule([66, 40, 15], 32) and rule([18, 5, 3], 32)
    assert not rule([64, 63], 32) and not rule([43, 38, 34, 21], 32)
    assert not rule([100], 32) and not rule([7, 1], 32)
    assert rule([61, 50], 2) and not rule([61, 50], 64)  # more value heads: a longer pre-pass to hide
    segs, n, _ = build_segments([(1000, [40], 0), (100, [20], 0), (70, [], 0)], shuffle_pages=False)
    rl = RecurrentLayout.build(segs, n, 3, "cpu")
    assert rl.lead == (0, 0) and rl.choose_lead(32) == rl.seg_chunks[0] and rl.lead[1] == 17


def test_prefix_cache_contract():
    """dan's PrefixCache contract (dan/cache.py:11-39): exact keys, hit / miss counters, bytes
    used, least-recently-used eviction, entries larger than the budget not kept."""
    from dan_b200.cache import PrefixCache

    def kv(rows):
        return {0: (torch.zeros(rows, 50, dtype=torch.bfloat16), torch.zeros(rows, 50, dtype=torch.bfloat16))}

    c = PrefixCache(max_bytes=3000)
    assert c.get([1, 2]) is None and c.misses == 1
    big = kv(10)  # 2000 bytes
    c.put([1, 2], big)
    assert c.used == 2000 and c.get([1, 2]) is big and c.hits == 1
    c.put([1, 2], big)  # already present: unchanged
    assert c.used == 2000
    c.put([3], kv(2))  # 400 bytes
    assert c.used == 2400
    c.get([1, 2])  # [3] is now the least recently used
    c.put([4], kv(2))  # 2800: fits
    c.put([5], kv(6))  # 1200 more: evicts [3], then [1, 2]
    assert c.get([3]) is None and c.get([1, 2]) is None and c.get([4]) is not None and c.get([5]) is not None
    assert c.used == 1600
    c.put([6], kv(40))  # larger than the whole budget: not kept, nothing evicted
    assert c.get([6]) is None and c.used == 1600
