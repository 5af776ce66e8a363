"""Parity at the benchmark configurations' full shapes (seeded synthetic batches, random-init
weights; the oracle runs on the host CPU in fp32 / fp64).

- configuration 2: one <= 8192-token batch of tree attention at Llama-3-8B heads (32 / 8 x
  128, trunks up to 2048, up to 16 branches) through ``dan_tree_attention`` against the dense
  masked oracle; the bar is BASELINE's "max relative error 2e-2" (max |got - want| over max
  |want|) and the reference's own assert_close(2e-2, 2e-2) (tests/test_runner.py:55-68);
- configuration 3: a 2-layer Llama-3-8B-shaped slice (hidden 4096, 32 / 8 x 128 heads, MLP
  14336, vocabulary 128,256) on one batch: answer probabilities within 5e-3;
- configuration 4: a 4-layer Qwen3.5-4B-shaped slice (3 Gated DeltaNet layers at 16 / 32 x 128
  heads, then one gated attention layer at 16 / 4 x 256 with partial RoPE 0.25), one batch:
  probabilities within 5e-3;
- configuration 5: the configuration-3 slice with FP8 e4m3 decoder linears over two batches
  of one request stream, the shared 1024-token prefix stored by the first and served from the
  prefix pool to the second: probabilities within 3e-2 of the FP8 oracle, and the same cache
  hits as the oracle's cache.

The vocabulary matrix is tied to lm_head (the forward reads the batch's embedding rows and the
label rows only; tying halves the host memory the oracle needs)."""
import pytest
import torch

from dan_b200 import synthetic
from dan_b200.attention import TreeLayout, tree_attention
from dan_b200.loader import arch_for, llama3_8b_config, qwen35_4b_config
from dan_b200.runner import Runner
from oracle import attention as OA
from oracle import runner as OR
from oracle import weights as OW

pytestmark = pytest.mark.gpu


def _packed(cfg_id, seed, vocab):
    r = Runner.__new__(Runner)
    r.device, r.cache = torch.device("cuda"), None
    return r.pack(synthetic.batch(cfg_id, seed=seed, vocab=vocab), use_cache=False)


def test_cfg2_attention_full_batch(cuda):
    ids, pos, segs, reads, _ = _packed(2, 11, 128256)
    n, h, hkv, d = len(ids), 32, 8, 128
    assert n > 4096 and max(s.trunk for s in segs) > 512
    g = torch.Generator().manual_seed(2)
    q = torch.randn(n, h, d, generator=g).bfloat16()
    k = torch.randn(n, hkv, d, generator=g).bfloat16()
    v = torch.randn(n, hkv, d, generator=g).bfloat16()
    lay = TreeLayout.build(segs, n, cuda)
    got = tree_attention(q.to(cuda), k.to(cuda), v.to(cuda), lay).float().cpu()  # [N, H, D]
    oracle_segs = [{"start": s.start, "end": s.end, "branch": s.branch_ids, "past": None} for s in segs]
    qt, kt, vt = q.transpose(0, 1).float(), k.transpose(0, 1).float(), v.transpose(0, 1).float()
    rep = h // hkv
    want = torch.empty(h, n, d)
    for grp in range(hkv):  # one kv head and its query heads at a time (bounded host memory)
        want[grp * rep:(grp + 1) * rep] = OA.attend(qt[grp * rep:(grp + 1) * rep], kt[grp:grp + 1],
                                                    vt[grp:grp + 1], oracle_segs)
    want = want.transpose(0, 1)
    rel = ((got - want).abs().max() / want.abs().max()).item()
    print(f"cfg2: {n} tokens, {len(segs)} segments, {len(reads)} branches, max relative error {rel:.3e}")
    assert rel <= 2e-2, rel
    torch.testing.assert_close(got, want, atol=2e-2, rtol=2e-2)


def _probs_vs_oracle(got_probs, got_logits, want_logits, bar):
    worst_p = worst_l = scale = 0.0
    for pp, gl, ww in zip(got_probs, got_logits, want_logits):
        assert len(pp) == len(ww)
        for p, lg, w in zip(pp, gl, ww):
            w = torch.as_tensor(w).float()
            worst_p = max(worst_p, (p - torch.softmax(w.double(), 0).float()).abs().max().item())
            worst_l = max(worst_l, (lg - w).abs().max().item())
            scale = max(scale, w.abs().max().item())
    assert worst_p < bar, (worst_p, worst_l, scale)
    return worst_p, worst_l / max(scale, 1e-9)


def _llama_slice():
    cfg = dict(llama3_8b_config(), num_hidden_layers=2, tie_word_embeddings=True)
    state = OW.random_state(cfg, seed=8)
    return cfg, state


def test_cfg3_llama3_8b_slice(cuda):
    cfg, state = _llama_slice()
    model = arch_for(cfg)(cfg, state, cuda, torch.bfloat16, None)
    runner = Runner(model, cuda, cache_bytes=0)
    plans = synthetic.batch(3, seed=21, vocab=cfg["vocab_size"])
    logits, probs = runner.read_many(plans, probabilities=True)
    want = OR.read_many(state, cfg, plans)
    p, lrel = _probs_vs_oracle(probs, logits, want, 5e-3)
    print(f"cfg3 slice: {sum(len(x) for x in want)} questions, max |dp| {p:.2e}, logits rel {lrel:.2e}")


def test_cfg4_qwen35_4b_slice(cuda):
    cfg = dict(qwen35_4b_config(), num_hidden_layers=4, tie_word_embeddings=True)
    cfg["layer_types"] = cfg["layer_types"][:4]
    assert cfg["layer_types"] == ["linear_attention"] * 3 + ["full_attention"]
    state = OW.random_state(cfg, seed=9)
    model = arch_for(cfg)(cfg, state, cuda, torch.bfloat16, None)
    runner = Runner(model, cuda, cache_bytes=0)
    plans = synthetic.batch(4, seed=22, vocab=cfg["vocab_size"])
    logits, probs = runner.read_many(plans, probabilities=True)
    want = OR.read_many(state, cfg, plans)
    p, lrel = _probs_vs_oracle(probs, logits, want, 5e-3)
    print(f"cfg4 slice: {sum(len(x) for x in want)} questions, max |dp| {p:.2e}, logits rel {lrel:.2e}")


def test_cfg5_fp8_slice_with_cached_prefix(cuda):
    cfg, state = _llama_slice()
    model = arch_for(cfg)(cfg, state, cuda, torch.bfloat16, "fp8")
    runner = Runner(model, cuda, cache_bytes=2 << 30)
    cache = OR.PrefixCache(2 << 30)
    worst = 0.0
    for i, plans in enumerate(synthetic.batches(5, 2, seed=23, vocab=cfg["vocab_size"])):
        assert all(p.static == 1024 for p in plans)
        logits, probs = runner.read_many(plans, probabilities=True)
        want = OR.read_many(state, cfg, plans, cache=cache, fp8=True)
        p, _ = _probs_vs_oracle(probs, logits, want, 3e-2)
        worst = max(worst, p)
        assert (runner.cache.hits, runner.cache.misses) == (cache.hits, cache.misses), i
    assert runner.cache.hits >= 2  # the second batch read the 1024-token prefix from the pool
    print(f"cfg5 slice: max |dp| {worst:.2e}, pool hits {runner.cache.hits}")
