"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

The fixtures come from running the reference (tests/golden/make_golden.py);
these tests prove the oracle restates its algorithm before the oracle is used
to check the CUDA path.
"""
import pytest
import torch
from conftest import golden, plans_from_json

from oracle import attention as OA
from oracle import llama as OL
from oracle import qwen3_5 as OQ
from oracle import runner as OR
from oracle import weights


def test_tree_mask_golden():
    g = golden("tree_mask.json")
    assert OA.tree_mask(torch.tensor(g["branch"])).tolist() == g["mask"]
    assert OA.branch_rows_mask(torch.tensor(g["branch2"]), 3).tolist() == g["rows_mask2"]
    # the reference's own known-answer rows (tests/test_runner.py:16-22)
    m = OA.tree_mask(torch.tensor([0, 0, 1, 1, 2]))
    assert m[1].tolist() == [True, True, False, False, False]
    assert m[3].tolist() == [True, True, True, True, False]
    assert m[4].tolist() == [True, True, False, False, True]


def test_attention_edges_golden():
    from make_golden import attention_inputs

    g = golden("attention_edges.pt")
    q, k, v, pasts = attention_inputs(g["h"], g["hkv"], g["d"], g["seed"], g["shapes"])
    segs, start = [], 0
    for (trunk, lens, past), pkv in zip(g["shapes"], pasts):
        branch = [0] * trunk + [j for j, n in enumerate(lens, 1) for _ in range(n)]
        segs.append({"start": start, "end": start + len(branch), "branch": branch, "past": pkv})
        start += len(branch)
    out = OA.attend(q, k, v, segs)
    torch.testing.assert_close(out, g["out"], atol=2e-5, rtol=1e-5)


def test_attention_bf16_probabilities_within_rounding():
    """``p_bf16`` (probabilities rounded to bf16 before the PV product) moves each output by at
    most bf16 rounding of the weights: relative 2^-8 of sum |p v|."""
    from make_golden import attention_inputs

    g = golden("attention_edges.pt")
    q, k, v, pasts = attention_inputs(g["h"], g["hkv"], g["d"], g["seed"], g["shapes"])
    segs, start = [], 0
    for (trunk, lens, past), pkv in zip(g["shapes"], pasts):
        branch = [0] * trunk + [j for j, n in enumerate(lens, 1) for _ in range(n)]
        segs.append({"start": start, "end": start + len(branch), "branch": branch, "past": pkv})
        start += len(branch)
    exact, rounded = OA.attend(q, k, v, segs), OA.attend(q, k, v, segs, p_bf16=True)
    bound = 2.0 ** -8 * v.abs().max().item()
    assert 0 < (exact - rounded).abs().max().item() <= bound


def test_pack_golden():
    cache = OR.PrefixCache(1 << 30)
    for rec in golden("pack.json"):
        plans = plans_from_json(rec["plans"])
        ids, pos, segs, reads, stores = OR.pack(plans, cache)
        assert ids == rec["ids"] and pos == rec["pos"]
        assert [[r, l] for r, l in reads] == rec["reads"]
        assert len(segs) == len(rec["segments"])
        for s, r in zip(segs, rec["segments"]):
            assert (s["start"], s["end"], s["trunk"], s["past_len"], s["save"]) == \
                (r["start"], r["end"], r["trunk"], r["past_len"], r["save"])
            assert [list(x) for x in s["branches"]] == r["branches"]
            assert s["branch"] == r["branch_ids"]
        for static, seg in stores:
            cache.put(static, {0: (torch.zeros(1, len(static), 1), torch.zeros(1, len(static), 1))})


def _model_golden(name, arch):
    g = golden(name)
    cfg, state = g["config"], weights.random_state(g["config"], g["seed"])
    cache = OR.PrefixCache()
    for b in g["batches"]:
        plans = plans_from_json(b["plans"])
        got = OR.read_many(state, cfg, plans, cache)
        for per, want_r, want_h in zip(got, b["runner"], b["hf"]):
            for a, wr, wh in zip(per, want_r, want_h):
                torch.testing.assert_close(a, torch.tensor(wr), atol=2e-4, rtol=1e-4)
                torch.testing.assert_close(a, torch.tensor(wh), atol=2e-4, rtol=1e-4)
        assert cache.hits == b["hits"]


def test_tiny_llama_golden():
    _model_golden("tiny_llama.json", OL)


def test_tiny_hybrid_golden():
    _model_golden("tiny_hybrid.json", OQ)


@pytest.mark.parametrize("name", ["tiny_qwen2.json", "tiny_qwen3.json"])
def test_llama_family_variants_golden(name):
    """Qwen2 (q/k/v bias) and Qwen3 (per-head q/k RMSNorm) through the oracle's Llama path."""
    _model_golden(name, OL)


def test_useful_pairs_matches_mask_count():
    segs = [{"start": 0, "end": 10, "branch": [0] * 4 + [1] * 3 + [2] * 3,
             "past": (torch.zeros(1, 5, 2), torch.zeros(1, 5, 2))}]
    assert OA.useful_pairs(segs) == int(OA.segment_mask(segs[0]["branch"], 5).sum())


def _probs_gap(a, b):
    worst = 0.0
    for pa, pb in zip(a, b):
        for x, y in zip(pa, pb):
            px = torch.softmax(torch.as_tensor(x).double(), 0)
            worst = max(worst, (px - torch.softmax(torch.as_tensor(y).double(), 0)).abs().max().item())
    return worst


def _bf16_golden(name):
    """The oracle's bf16 mode against the reference run in bf16 (``runner_bf16``): both round to
    bf16 at the same module boundaries, so they land within the reference's own bf16-vs-fp32
    distance of each other (attention and matmul accumulation orders still differ)."""
    g = golden(name)
    cfg, state = g["config"], weights.random_state(g["config"], g["seed"])
    cache = OR.PrefixCache()
    for b in g["batches"]:
        got = OR.read_many(state, cfg, plans_from_json(b["plans"]), cache, bf16=True)
        own_gap = _probs_gap(b["runner_bf16"], b["runner"])
        assert _probs_gap(got, b["runner_bf16"]) <= max(own_gap, 1e-3), b["name"]
        assert _probs_gap(got, b["runner"]) <= 2 * own_gap + 1e-3, b["name"]


def test_tiny_llama_bf16_mode_golden():
    _bf16_golden("tiny_llama.json")


def test_tiny_hybrid_bf16_mode_golden():
    _bf16_golden("tiny_hybrid.json")


@pytest.mark.parametrize("name", ["tiny_qwen2.json", "tiny_qwen3.json"])
def test_llama_family_variants_bf16_mode_golden(name):
    _bf16_golden(name)


def test_rope_frequencies_golden():
    """RoPE inverse frequencies (default, linear, llama3 scaling; llama.py:18-40), bit for bit in
    both the oracle and the model's table builder."""
    from dan_b200.llama import inv_frequencies

    for case in golden("rope_frequencies.json"):
        want = torch.tensor(case["inv"], dtype=torch.float32)
        assert torch.equal(OL.inv_frequencies(case["config"], case["head_dim"]), want), case["name"]
        assert torch.equal(inv_frequencies(case["config"], case["head_dim"]), want), case["name"]

