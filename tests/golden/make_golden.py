"""Generate the golden fixtures in this directory by running the reference itself.

    python tests/golden/make_golden.py --reference <path to the dan source tree>

The reference (quangliz/dan, pure Python on PyTorch) is imported from the
given path and run on the CPU in fp32 on seeded inputs. Only its outputs are
written here; inputs are either stored too (token ids, plans) or regenerated
by the tests from the same seeds (random checkpoints via ``oracle.weights``,
attention inputs via ``attention_inputs`` below).

Fixtures:
- ``pack.json``: ``Runner.pack`` (runner.py:38-64) over three batches that go
  cold -> warm -> mixed through a prefix cache, with the index layouts the
  reference derives from the segments: ``ReadLayout`` (attention.py:138-172)
  and ``RecurrentLayout`` (qwen3_5.py:240-298).
- ``attention_edges.pt``: ``_attend_dense`` (attention.py:244-270) on the five
  edge shapes of the reference's own varlen test (tests/test_runner.py:55).
- ``tiny_llama.json``: per-branch label logits from ``Runner.read_many`` (dense
  masked path, fp32) and from ``HFReference`` (reference.py:16-23) for the
  configuration-1 model, plus a cold/warm/mixed prefix-cache sequence.
- ``rope_frequencies.json``: RoPE inverse frequencies (default, linear, llama3 scaling);
- ``tiny_qwen2.json`` / ``tiny_qwen3.json``: the same for small Qwen2 (q/k/v bias) and Qwen3
  (per-head q/k RMSNorm) models;
- ``tiny_hybrid.json``: the same for a small Qwen3.5 hybrid (3 DeltaNet + 1
  gated attention layer) whose trunks exceed one 64-token delta-rule chunk.
- ``tree_mask.json``: ``tree_mask`` / ``branch_rows_mask`` rows
  (tests/test_runner.py:16-22).
- ``fullsize.json``: ``Runner.read_many`` label logits in fp32 and in bf16 (the reference's
  GPU dtype, here on the CPU) for a 2-layer Llama-3-8B-shaped slice on one configuration-3
  batch and a 4-layer Qwen3.5-4B-shaped slice on one configuration-4 batch.

The model fixtures also hold the bf16 runner's logits (``runner_bf16``), which pin the
oracle's bf16 rounding mode.
"""
import argparse
import json
import os
import random
import sys
import tempfile

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from dan_b200 import synthetic  # noqa: E402
from oracle import weights  # noqa: E402

SHM = "/dev/shm" if os.path.isdir("/dev/shm") else None  # checkpoints of GBs: write to memory
EDGE_SHAPES = [(40, [5, 9, 1], 0), (7, [30], 12), (1, [3, 3, 3, 3, 3, 3], 0), (64, [], 0), (13, [17, 2], 20)]


def attention_inputs(h=8, hkv=2, d=64, seed=0, shapes=EDGE_SHAPES):
    """Seeded fp32 inputs for the edge-shape attention case: q, k, v and per-segment past (k, v)."""
    gen = torch.Generator().manual_seed(seed)
    n = sum(t + sum(lens) for t, lens, _ in shapes)
    q = torch.randn(h, n, d, generator=gen)
    k = torch.randn(hkv, n, d, generator=gen)
    v = torch.randn(hkv, n, d, generator=gen)
    pasts = []
    for _, _, past in shapes:
        pasts.append((torch.randn(hkv, past, d, generator=gen), torch.randn(hkv, past, d, generator=gen))
                     if past else None)
    return q, k, v, pasts


def plan_json(p):
    return {"prefix": list(p.prefix), "static": p.static,
            "branches": [{"suffix": list(b.suffix), "label_ids": list(b.label_ids)} for b in p.branches]}


def ref_plans(dan_prompt, plans):
    return [dan_prompt.ReadPlan(list(p.prefix), [], [], [dan_prompt.Branch(list(b.suffix), list(b.label_ids))
                                                         for b in p.branches], static=p.static) for p in plans]


def small_plans(rng, vocab, n, trunk=(5, 40), nb=(0, 4), blen=(1, 6), static=(0, 8)):
    from dan_b200.plan import Branch, ReadPlan

    out = []
    for _ in range(n):
        prefix = [rng.randrange(vocab) for _ in range(rng.randint(*trunk))]
        br = [Branch([rng.randrange(vocab) for _ in range(rng.randint(*blen))],
                     rng.sample(range(vocab), rng.randint(2, 5))) for _ in range(rng.randint(*nb))]
        st = min(rng.randint(*static), len(prefix) - 1)
        out.append(ReadPlan(prefix, branches=br, static=st))
    return out


def dump_pack(dan):
    from dan.attention import ReadLayout
    from dan.cache import PrefixCache
    from dan.models.qwen3_5 import RecurrentLayout
    from dan.runner import Runner

    rng = random.Random(11)
    plans = small_plans(rng, 1000, 10)
    plans[2].static = 0
    plans[3].branches = []
    warm = plans[:6]
    mixed = [plans[7], plans[1]] + small_plans(rng, 1000, 3) + [plans[4]]
    runner = Runner.__new__(Runner)
    runner.device, runner.cache = "cpu", PrefixCache(1 << 30)
    out = []
    for name, batch in (("cold", plans), ("warm", warm), ("mixed", mixed)):
        rp = ref_plans(dan.prompt, batch)
        ids, pos, segs, reads, stores = runner.pack(rp)
        rec = {"name": name, "plans": [plan_json(p) for p in batch], "ids": ids.tolist(), "pos": pos.tolist(),
               "segments": [{"start": s.start, "end": s.end, "trunk": s.trunk, "branches": [list(x) for x in s.branches],
                             "past_len": s.past_len, "save": s.save, "has_past": bool(s.past),
                             "branch_ids": list(s.branch_ids)} for s in segs],
               "reads": [[r, list(l)] for r, l in reads], "stores": [[len(st), segs.index(sg)] for st, sg in stores]}
        lay = ReadLayout.build(segs, "cpu")
        rec["read_layout"] = {"trunk_rows": lay.trunk_rows.tolist(), "branch_rows": lay.branch_rows.tolist(),
                              "cu_trunk_q": lay.cu_trunk_q.tolist(), "cu_trunk_k": lay.cu_trunk_k.tolist(),
                              "max_trunk_q": lay.max_trunk_q, "max_trunk_k": lay.max_trunk_k,
                              "cu_branch_q": lay.cu_branch_q.tolist(), "max_branch_q": lay.max_branch_q,
                              "cu_branch": None if lay.cu_branch is None else lay.cu_branch.tolist(),
                              "max_branch": lay.max_branch, "has_past": lay.has_past, "has_branches": lay.has_branches}
        rl = RecurrentLayout.build(segs, 3, len(ids), "cpu")

        def ph(p):
            return None if p is None else {"ext": p.ext.tolist(), "take": p.take.tolist(), "rows": p.rows.tolist(),
                                           "lens": list(p.lens)}

        rec["recurrent_layout"] = {
            "trunk1": ph(rl.trunk1), "trunk2": ph(rl.trunk2), "branches": ph(rl.branches),
            "split_segments": None if rl.split_segments is None else rl.split_segments.tolist(),
            "branch_segment": None if rl.branch_segment is None else rl.branch_segment.tolist(),
            "past_segments": list(rl.past_segments), "saves": [[i, t.tolist()] for i, t in rl.saves]}
        for static, seg in stores:  # the value is irrelevant to packing; its presence makes the next hit
            runner.cache.put(static, {0: (torch.zeros(1, len(static), 1), torch.zeros(1, len(static), 1))})
        out.append(rec)
    with open(os.path.join(HERE, "pack.json"), "w") as f:
        json.dump(out, f)


def dump_attention(dan):
    from dan import attention as A

    q, k, v, pasts = attention_inputs()
    segs, start = A.Batch(), 0
    for (trunk, lens, past), pkv in zip(EDGE_SHAPES, pasts):
        branch = [0] * trunk + [j for j, n in enumerate(lens, 1) for _ in range(n)]
        segs.append(A.segment(start, branch, {0: pkv} if past else None, 0, past, "cpu"))
        start += len(branch)
    out = A._attend_dense(q, k, v, segs, 0, None)
    torch.save({"out": out.contiguous(), "shapes": EDGE_SHAPES, "seed": 0, "h": 8, "hkv": 2, "d": 64},
               os.path.join(HERE, "attention_edges.pt"))


def run_model(dan, config, seed, batches, name, hf=True):
    from dan.reference import HFReference
    from dan.runner import Runner

    with tempfile.TemporaryDirectory(dir=SHM) as tmp:
        weights.save_checkpoint(tmp, config, weights.random_state(config, seed))
        runner = Runner(tmp, "cpu", torch.float32)
        runner16 = Runner(tmp, "cpu", torch.bfloat16)  # the reference's bf16 path (its GPU dtype)
        ref = HFReference(tmp) if hf else None
        recs = []
        for bname, plans in batches:
            rp = ref_plans(dan.prompt, plans)
            got = runner.read_many(rp)
            got16 = runner16.read_many(ref_plans(dan.prompt, plans))
            rec = {"name": bname, "plans": [plan_json(p) for p in plans],
                   "runner": [[x.tolist() for x in per] for per in got], "hits": runner.cache.hits,
                   "runner_bf16": [[x.tolist() for x in per] for per in got16]}
            if ref is not None:
                rec["hf"] = [[x.tolist() for x in ref.read(p)] for p in rp]
            recs.append(rec)
    with open(os.path.join(HERE, name), "w") as f:
        json.dump({"config": config, "seed": seed, "batches": recs}, f)


def plans_digest(plans):
    """A short hash of a batch's plans (the tests regenerate them from the same seed)."""
    import hashlib

    return hashlib.sha256(json.dumps([plan_json(p) for p in plans]).encode()).hexdigest()[:16]


def fullsize_cases():
    """(name, config, weight seed, plans) of the full-shape slices: 2 Llama-3-8B-shaped layers on
    one configuration-3 batch, and 4 Qwen3.5-4B-shaped layers (3 Gated DeltaNet + 1 gated
    attention) on one configuration-4 batch; vocabulary tied to lm_head."""
    from dan_b200.loader import llama3_8b_config, qwen35_4b_config

    c3 = dict(llama3_8b_config(), num_hidden_layers=2, tie_word_embeddings=True, architectures=["LlamaForCausalLM"],
              torch_dtype="float32", hidden_act="silu", max_position_embeddings=131072)
    c4 = dict(qwen35_4b_config(), num_hidden_layers=4, tie_word_embeddings=True, architectures=["Qwen3_5ForCausalLM"],
              torch_dtype="float32", hidden_act="silu", max_position_embeddings=32768, attention_bias=False)
    c4["layer_types"] = c4["layer_types"][:4]
    return [("cfg3_llama3_8b_2layers", c3, 8, synthetic.batch(3, seed=21, vocab=c3["vocab_size"])),
            ("cfg4_qwen35_4b_4layers", c4, 9, synthetic.batch(4, seed=22, vocab=c4["vocab_size"]))]


def dump_fullsize(dan):
    """The reference's own fp32 and bf16 label logits on the full-shape slices (CPU)."""
    from dan.runner import Runner

    out = {}
    for name, config, seed, plans in fullsize_cases():
        with tempfile.TemporaryDirectory(dir=SHM) as tmp:
            weights.save_checkpoint(tmp, config, weights.random_state(config, seed))
            rec = {"seed": seed, "digest": plans_digest(plans)}
            for key, dtype in (("runner", torch.float32), ("runner_bf16", torch.bfloat16)):
                runner = Runner(tmp, "cpu", dtype, cache_bytes=0)
                rec[key] = [[x.tolist() for x in per] for per in runner.read_many(ref_plans(dan.prompt, plans))]
                del runner
        out[name] = rec
    with open(os.path.join(HERE, "fullsize.json"), "w") as f:
        json.dump(out, f)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DAN_REFERENCE"), required=False,
                    help="path of the reference source tree (the directory holding the dan package)")
    ap.add_argument("--only", choices=["families", "rope"], help="regenerate only these fixtures")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or DAN_REFERENCE) is required")
    sys.path.insert(0, args.reference)
    import dan.prompt  # noqa: F401
    if args.only == "families":
        dump_families(dan)
        return
    if args.only == "rope":
        dump_rope(dan)
        return
    from dan.attention import branch_rows_mask, tree_mask

    torch.manual_seed(0)
    b = torch.tensor([0, 0, 1, 1, 2])
    b2 = torch.tensor([0, 0, 0, 1, 1, 2, 3, 3])
    with open(os.path.join(HERE, "tree_mask.json"), "w") as f:
        json.dump({"branch": b.tolist(), "mask": tree_mask(b).tolist(), "branch2": b2.tolist(),
                   "rows_mask2": branch_rows_mask(b2, 3).tolist()}, f)
    dump_pack(dan)
    dump_attention(dan)

    # configuration 1 (SmolLM2-135M shaped, tied embeddings) + a prefix-cache sequence
    cfg1 = weights.llama_config()
    b1 = [synthetic.request(1, random.Random(1), cfg1["vocab_size"])]
    rng = random.Random(2)
    cache_plans = small_plans(rng, cfg1["vocab_size"], 3, trunk=(60, 120), nb=(1, 3), blen=(3, 9), static=(20, 50))
    extra = small_plans(rng, cfg1["vocab_size"], 1, trunk=(60, 120), nb=(1, 3), blen=(3, 9), static=(20, 50))
    run_model(dan, cfg1, 0, [("cfg1", b1), ("cold", cache_plans), ("warm", cache_plans),
                             ("mixed", [cache_plans[1], extra[0], cache_plans[0]])], "tiny_llama.json")

    # a small Qwen3.5 hybrid; trunks longer than one 64-token delta-rule chunk
    # DeltaNet heads of 128 (the Qwen3.5 head size the scan kernel is built for), small elsewhere
    cfgh = weights.qwen35_config(heads=2, kv_heads=1, lin_k_heads=1, lin_v_heads=2, lin_k_dim=128, lin_v_dim=128)
    rng = random.Random(3)
    hp = small_plans(rng, cfgh["vocab_size"], 3, trunk=(70, 150), nb=(1, 3), blen=(3, 9), static=(20, 60))
    hx = small_plans(rng, cfgh["vocab_size"], 1, trunk=(70, 150), nb=(1, 3), blen=(3, 9), static=(20, 60))
    run_model(dan, cfgh, 0, [("cold", hp), ("warm", hp), ("mixed", [hp[2], hx[0], hp[0]])], "tiny_hybrid.json")
    dump_families(dan)
    dump_rope(dan)
    dump_fullsize(dan)


ROPE_CASES = [
    ("default", {"rope_theta": 500000.0}),
    ("linear", {"rope_theta": 10000.0, "rope_scaling": {"rope_type": "linear", "factor": 4.0}}),
    ("llama3", {"rope_theta": 500000.0, "rope_scaling": {
        "rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 8192}}),
    ("params", {"rope_parameters": {"rope_theta": 1000000.0, "rope_type": "default"}}),
]


def dump_rope(dan):
    """``rope_frequencies.json``: the reference's RoPE inverse frequencies (llama.py:18-40) for
    default, linear and llama3 scaling at head dims 64 / 128 / 256."""
    from types import SimpleNamespace

    from dan.models.llama import inv_frequencies

    out = []
    for name, fields in ROPE_CASES:
        for d in (64, 128, 256):
            inv = inv_frequencies(SimpleNamespace(**fields), d)
            out.append({"name": name, "config": fields, "head_dim": d, "inv": inv.tolist()})
    with open(os.path.join(HERE, "rope_frequencies.json"), "w") as f:
        json.dump(out, f)


def dump_families(dan):
    """``tiny_qwen2.json`` / ``tiny_qwen3.json``: the other Llama-family variants dan runs
    (llama.py:62-85, 129-135): Qwen2's q/k/v bias and Qwen3's per-head q/k RMSNorm."""
    for mt, seed in (("qwen2", 5), ("qwen3", 6)):
        cfg = weights.llama_config(vocab=512, hidden=256, inter=512, layers=2, heads=4, kv_heads=2, head_dim=64,
                                   model_type=mt, tie=False, theta=1000000.0, eps=1e-6)
        rng = random.Random(seed)
        plans = small_plans(rng, cfg["vocab_size"], 3, trunk=(60, 140), nb=(1, 3), blen=(3, 9), static=(20, 50))
        extra = small_plans(rng, cfg["vocab_size"], 1, trunk=(60, 140), nb=(1, 3), blen=(3, 9), static=(20, 50))
        run_model(dan, cfg, seed, [("cold", plans), ("warm", plans), ("mixed", [plans[1], extra[0], plans[0]])],
                  f"tiny_{mt}.json")


if __name__ == "__main__":
    main()
