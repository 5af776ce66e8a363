"""bf16 reads on the GPU against the reference's own bf16 GPU path, run side by side on the
same device from its offline install (``baseline/_ref``; skipped where that is absent).

The golden fixtures pin this build against the reference's fp32 (and CPU bf16) runs; these
tests add the reference's GPU arithmetic: dan's ``Runner`` in bf16 on CUDA over the same
checkpoint and plans, cold -> warm -> mixed prefix cache, with its tree attention through
torch's varlen flash kernel (attention.py:176-197, the default) or its dense masked path
(``DAN_VARLEN=0``, attention.py:244-270), and for the Qwen3.5 hybrid its torch chunked delta
rule on the GPU (qwen3_5.py:103-133; the flash-linear-attention kernels it prefers when
installed are a third-party library, left out). Batches here are below the 512 rows at which
dan compiles its fused ops, so those run eagerly (fused.py:20-31).

Bar: answer probabilities within max(5e-3, 2 g) of the reference's bf16 GPU run, where g is
that run's own distance from the reference's fp32 run (the fixture), the same form as the
full-shape bars; cache hits identical."""
import pytest
import torch
from conftest import golden, plans_from_json

from dan_b200.runner import Runner
from oracle import weights

pytestmark = pytest.mark.gpu


def _compare(cuda, tmp_path, name, monkeypatch, varlen=True):
    dan_runner = pytest.importorskip("dan.runner")
    import dan.attention
    import dan.models.qwen3_5

    monkeypatch.setattr(dan.attention, "VARLEN", varlen)
    monkeypatch.setattr(dan.models.qwen3_5, "fla_chunk_gated_delta_rule", None)
    g = golden(name)
    weights.save_checkpoint(str(tmp_path), g["config"], weights.random_state(g["config"], g["seed"]))
    ref = dan_runner.Runner(str(tmp_path), "cuda", torch.bfloat16)
    ours = Runner(str(tmp_path), cuda)
    worst = gap = 0.0
    for b in g["batches"]:
        plans = plans_from_json(b["plans"])
        want = ref.read_many(plans)
        _, probs = ours.read_many(plans, probabilities=True)
        for pp, ww, ff in zip(probs, want, b["runner"]):
            assert len(pp) == len(ww) == len(ff)
            for p, w, f in zip(pp, ww, ff):
                pw = torch.softmax(w.double(), 0)
                worst = max(worst, (p.double() - pw).abs().max().item())
                gap = max(gap, (pw - torch.softmax(torch.tensor(f).double(), 0)).abs().max().item())
        assert ours.cache.hits == ref.cache.hits == b["hits"], b["name"]
    print(f"{name} ({'varlen' if varlen else 'dense'}): vs dan's bf16 GPU run max |dp| {worst:.2e}; "
          f"that run vs dan's fp32 run {gap:.2e}")
    assert worst <= max(5e-3, 2 * gap), (worst, gap)


@pytest.mark.parametrize("varlen", [True, False], ids=["varlen", "dense"])
def test_tiny_llama_vs_reference_bf16_gpu(cuda, tmp_path, monkeypatch, varlen):
    _compare(cuda, tmp_path, "tiny_llama.json", monkeypatch, varlen)


@pytest.mark.parametrize("name", ["tiny_qwen2.json", "tiny_qwen3.json"])
def test_llama_family_vs_reference_bf16_gpu(cuda, tmp_path, monkeypatch, name):
    _compare(cuda, tmp_path, name, monkeypatch)


def test_tiny_hybrid_vs_reference_bf16_gpu(cuda, tmp_path, monkeypatch):
    _compare(cuda, tmp_path, "tiny_hybrid.json", monkeypatch)
