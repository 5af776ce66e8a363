"""End-to-end reads on the GPU vs the reference's own outputs (golden fixtures).

Configuration 1's model (SmolLM2-135M shaped, seeded weights) runs through
``Runner.read_many`` in bf16 on the dan_b200 kernels over a cold -> warm ->
mixed prefix-cache sequence. Bars: answer probabilities within 5e-3 of the
reference's fp32 path (north-star bf16 bound) and the same cache hits."""
import pytest
import torch
from conftest import golden, plans_from_json

from dan_b200.runner import Runner
from oracle import weights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    g = golden("tiny_llama.json")
    path = tmp_path_factory.mktemp("tiny_llama")
    weights.save_checkpoint(str(path), g["config"], weights.random_state(g["config"], g["seed"]))
    return str(path), g


def test_tiny_llama_matches_reference(cuda, tiny_dir):
    path, g = tiny_dir
    runner = Runner(path, cuda)
    worst_p = worst_l = 0.0
    for b in g["batches"]:
        plans = plans_from_json(b["plans"])
        got, probs = runner.read_many(plans, probabilities=True)
        for per, pp, want in zip(got, probs, b["runner"]):
            assert len(per) == len(want)
            for lg, p, w in zip(per, pp, want):
                w = torch.tensor(w)
                worst_l = max(worst_l, (lg - w).abs().max().item())
                worst_p = max(worst_p, (p - torch.softmax(w.double(), 0).float()).abs().max().item())
        assert runner.cache.hits == b["hits"], b["name"]
    assert worst_p < 5e-3, worst_p
    assert worst_l < 5e-2, worst_l


@pytest.mark.parametrize("name", ["tiny_qwen2.json", "tiny_qwen3.json"])
def test_llama_family_variants_match_reference(cuda, tmp_path, name):
    """Qwen2 (q/k/v bias in the q/k/v GEMM's epilogue, before RoPE) and Qwen3 (per-head q/k
    RMSNorm before RoPE) end to end against dan's own fp32 runner, cold -> warm -> mixed."""
    g = golden(name)
    weights.save_checkpoint(str(tmp_path), g["config"], weights.random_state(g["config"], g["seed"]))
    runner = Runner(str(tmp_path), cuda)
    worst_p = 0.0
    for b in g["batches"]:
        _, probs = runner.read_many(plans_from_json(b["plans"]), probabilities=True)
        for pp, want in zip(probs, b["runner"]):
            for p, w in zip(pp, want):
                worst_p = max(worst_p, (p - torch.softmax(torch.tensor(w).double(), 0).float()).abs().max().item())
        assert runner.cache.hits == b["hits"], b["name"]
    assert worst_p < 5e-3, worst_p


def test_without_cache_same_answers(cuda, tiny_dir):
    path, g = tiny_dir
    runner = Runner(path, cuda, cache_bytes=0)
    b = g["batches"][-1]
    got, probs = runner.read_many(plans_from_json(b["plans"]), probabilities=True)
    for pp, want in zip(probs, b["runner"]):
        for p, w in zip(pp, want):
            assert (p - torch.softmax(torch.tensor(w).double(), 0).float()).abs().max() < 5e-3


def test_tiny_llama_fp8_matches_fp8_oracle(cuda, tiny_dir):
    """FP8 e4m3 decoder linears (configuration 5's quantisation) vs the FP8 restatement of the
    reference (oracle.fp8, itself checked against the reference's FP8 path in the next test) at
    the north-star 3e-2 probability bound."""
    from oracle import runner as OR

    path, g = tiny_dir
    runner = Runner(path, cuda, quantization="fp8", cache_bytes=0)
    state = weights.random_state(g["config"], g["seed"])
    plans = plans_from_json(g["batches"][0]["plans"])
    _, probs = runner.read_many(plans, probabilities=True)
    want = OR.read_many(state, g["config"], plans, fp8=True)
    worst = 0.0
    for pp, ww in zip(probs, want):
        for p, w in zip(pp, ww):
            worst = max(worst, (p - torch.softmax(w.double(), 0).float()).abs().max().item())
    assert worst < 3e-2, worst


def test_tiny_llama_fp8_matches_reference_fp8_on_gpu(cuda, tiny_dir, monkeypatch):
    """FP8 pinned to the reference itself: dan's own Runner(quantization="fp8") from its
    offline install (torch._scaled_mm with row-wise scales, its varlen attention, eager
    activation quantisation: quant.py:23-42, fused.py:85-91) on the same GPU, same checkpoint
    and plans; probabilities within the north-star FP8 bound 3e-2, cold and warm cache."""
    dan_runner = pytest.importorskip("dan.runner")
    import dan.fused

    monkeypatch.setattr(dan.fused, "ENABLED", False)  # dan's eager rounding (its CPU / < 512-row path)
    from oracle import runner as OR

    path, g = tiny_dir
    ref = dan_runner.Runner(path, "cuda", torch.bfloat16, cache_bytes=2 << 30, quantization="fp8")
    ours = Runner(path, cuda, quantization="fp8")
    worst, first = 0.0, None
    for b in g["batches"]:
        plans = plans_from_json(b["plans"])
        want = ref.read_many(plans)
        first = want if first is None else first
        _, probs = ours.read_many(plans, probabilities=True)
        for pp, ww in zip(probs, want):
            assert len(pp) == len(ww)
            for p, w in zip(pp, ww):
                worst = max(worst, (p - torch.softmax(w.double(), 0).float()).abs().max().item())
        assert ours.cache.hits == ref.cache.hits, b["name"]
    # the FP8 restatement (oracle.fp8, CPU) against the same reference run, cold batch
    orc = OR.read_many(weights.random_state(g["config"], g["seed"]), g["config"],
                       plans_from_json(g["batches"][0]["plans"]), fp8=True)
    worst_o = max((torch.softmax(a.double(), 0) - torch.softmax(torch.as_tensor(w).double(), 0)).abs().max().item()
                  for pa, pw in zip(orc, first) for a, w in zip(pa, pw))
    print(f"fp8 vs dan's own fp8 path on this GPU: max |dp| {worst:.2e}; oracle.fp8 vs it: {worst_o:.2e}")
    assert worst < 3e-2, worst
    assert worst_o < 3e-2, worst_o


def test_read_stream_matches_read_many(cuda, tiny_dir):
    """``read_stream`` keeps one batch queued on the device while the host packs the next;
    each batch's results are bit-identical to a lone ``read_many`` of that batch, and a
    submitted batch's handle waits only for its own results."""
    path, g = tiny_dir
    runner = Runner(path, cuda, cache_bytes=0)
    batches = [plans_from_json(b["plans"]) for b in g["batches"]] * 2
    solo = [runner.read_many(p, probabilities=True) for p in batches]
    streamed = list(runner.read_stream(batches, probabilities=True))
    assert len(streamed) == len(solo)
    for (lg_s, pr_s), (lg_a, pr_a) in zip(streamed, solo):
        for a, b in zip(lg_s + pr_s, lg_a + pr_a):
            assert len(a) == len(b) and all(torch.equal(x, y) for x, y in zip(a, b))
    first, second = runner.submit(batches[0]), runner.submit(batches[1])
    assert second.result() is not None and first.ready()  # in-order device queue
    assert all(torch.equal(x, y) for x, y in zip(first.result()[0], solo[0][0][0]))


def test_submit_edges(cuda, tiny_dir):
    """A batch whose plans ask nothing reads nothing (one empty list per plan), an empty stream
    yields nothing, and such a batch between real ones does not disturb them."""
    from dan_b200.plan import ReadPlan

    path, g = tiny_dir
    runner = Runner(path, cuda, cache_bytes=0)
    empty = [ReadPlan([1, 2, 3], branches=[], static=0)]
    assert runner.read_many(empty) == [[]]
    assert list(runner.read_stream([])) == []
    real = plans_from_json(g["batches"][0]["plans"])
    outs = list(runner.read_stream([real, empty, real]))
    assert outs[1] == [[]]
    assert all(torch.equal(a, b) for pa, pb in zip(outs[0], outs[2]) for a, b in zip(pa, pb))
