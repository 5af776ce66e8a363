"""Qwen3.5 hybrid on the GPU: the DeltaNet conv + gated delta scan kernels against the
oracle's token-by-token recurrence, and end-to-end reads against the reference's own
outputs (golden fixture: cold -> warm -> mixed prefix-cache batches, trunks longer
than one 64-token chunk). Bars: answer probabilities within 5e-3 (bf16), the
reference's hybrid tolerance on logits is 5e-3 abs in fp32 (tests/test_qwen3_5.py:29),
here bf16 runs are held to 5e-2 on logits."""
import random

import pytest
import torch
from conftest import golden, plans_from_json

from dan_b200 import _lib
from dan_b200.runner import Runner
from oracle import qwen3_5 as OQ
from oracle import weights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def hybrid_dir(tmp_path_factory):
    g = golden("tiny_hybrid.json")
    path = tmp_path_factory.mktemp("tiny_hybrid")
    weights.save_checkpoint(str(path), g["config"], weights.random_state(g["config"], g["seed"]))
    return str(path), g


def test_tiny_hybrid_matches_reference(cuda, hybrid_dir):
    path, g = hybrid_dir
    runner = Runner(path, cuda)
    worst_p = worst_l = 0.0
    for b in g["batches"]:
        got, probs = runner.read_many(plans_from_json(b["plans"]), probabilities=True)
        for per, pp, want in zip(got, probs, b["runner"]):
            for lg, p, w in zip(per, pp, want):
                w = torch.tensor(w)
                worst_l = max(worst_l, (lg - w).abs().max().item())
                worst_p = max(worst_p, (p - torch.softmax(w.double(), 0).float()).abs().max().item())
        assert runner.cache.hits == b["hits"], b["name"]
    assert worst_p < 5e-3, worst_p
    assert worst_l < 5e-2, worst_l


def _scan_case(cuda, hk, hv, seg_shapes, seed=0, lead=None, oracle=True):
    """Conv + scan over a packed batch (no pasts) vs the oracle; q/k/v from random pre-conv rows.
    ``lead``: the scan's split range (default: the layout's own choice)."""
    from dan_b200.attention import Batch, segment
    from dan_b200.qwen3_5 import RecurrentLayout

    dk = dv = 128
    C = 2 * hk * dk + hv * dv
    gen = torch.Generator().manual_seed(seed)
    segs, start = Batch(), 0
    for trunk, lens in seg_shapes:
        branch = [0] * trunk + [j for j, n in enumerate(lens, 1) for _ in range(n)]
        segs.append(segment(start, branch, None, 0, 0, cuda))
        start += len(branch)
    n = start
    pre = (torch.randn(n, C, generator=gen) * 0.5).bfloat16()
    ba = torch.randn(n, 2 * hv, generator=gen).bfloat16()
    conv_w = (torch.randn(C, 4, generator=gen) * 0.5).bfloat16()
    a_log = torch.log(1 + 15 * torch.rand(hv, generator=gen))
    dt_bias = 0.5 + 0.5 * torch.rand(hv, generator=gen)
    rl = RecurrentLayout.build(segs, n, 3, cuda)
    lead = rl.choose_lead(hv) if lead is None else lead
    # every device buffer is held in a variable until the kernels ran: a temporary passed as
    # ``_lib.ptr(t.to(cuda))`` would be freed (and its memory reused) before the launch
    pre_d, conv = pre.to(cuda), torch.empty(n, C, dtype=torch.bfloat16, device=cuda)
    conv_w_d, ba_d, a_log_d, dt_d = conv_w.to(cuda), ba.to(cuda), a_log.to(cuda), dt_bias.to(cuda)
    _lib.call("dan_causal_conv", _lib.ptr(pre_d), C, None, 0, _lib.ptr(conv_w_d), _lib.ptr(rl.prev),
              _lib.ptr(conv), C, n, C, _lib.stream())
    out = torch.empty(n, hv * dv, dtype=torch.bfloat16, device=cuda)
    kd = hk * dk
    scratch = _lib.delta_scratch(rl.n_chunks, hk, hv, cuda)
    _lib.call("dan_gated_delta_scan", _lib.ptr(conv[:, :kd]), _lib.ptr(conv[:, kd:2 * kd]), _lib.ptr(conv[:, 2 * kd:]),
              C, _lib.ptr(ba_d[:, :hv]), _lib.ptr(ba_d[:, hv:]), 2 * hv, _lib.ptr(a_log_d), _lib.ptr(dt_d),
              _lib.ptr(rl.segs), rl.n_segs, _lib.ptr(rl.branches), _lib.ptr(rl.chunks), rl.n_chunks, None, 0,
              _lib.ptr(out), hv * dv, hk, hv, dk, dv, float(dk ** -0.5), _lib.ptr(scratch), scratch.numel(),
              *lead, _lib.ptr(_lib.status_word(cuda)), _lib.stream())
    torch.cuda.synchronize()
    if not oracle:
        return out.float().cpu().view(n, hv, dv), None
    # oracle: same tree runs, token by token, from the same bf16 inputs
    w = conv_w[:, None, :].float()
    b, a = ba[:, :hv].float(), ba[:, hv:].float()
    beta = torch.sigmoid(b)
    g = -a_log.exp() * torch.nn.functional.softplus(a + dt_bias)
    want = torch.zeros(n, hv, dv)
    conv_ref = torch.zeros(n, C)
    for s in segs:
        trunk_rows = list(range(s.start, s.start + s.trunk))
        virt = torch.cat([torch.zeros(3, C), pre[trunk_rows].float()])

        def run(hist, rows, init):
            ext = torch.cat([hist, pre[rows].float()])
            y = OQ.causal_conv_silu(ext, w)
            conv_ref[rows] = y
            qq = y[:, :kd].reshape(-1, hk, dk).repeat_interleave(hv // hk, 1)
            kk = y[:, kd:2 * kd].reshape(-1, hk, dk).repeat_interleave(hv // hk, 1)
            vv = y[:, 2 * kd:].reshape(-1, hv, dv)
            o, fin = OQ.delta_rule(qq, kk, vv, g[rows], beta[rows], init)
            want[rows] = o
            return fin

        fin = run(virt[:3], trunk_rows, torch.zeros(hv, dk, dv))
        for ba_, bb in s.branches:
            run(virt[-3:], list(range(ba_, bb)), fin)
    assert ((conv.float().cpu() - conv_ref).abs().max() / conv_ref.abs().max()).item() < 1e-2
    return out.float().cpu().view(n, hv, dv), want


@pytest.mark.parametrize("hk,hv", [(1, 2), (16, 32)])
def test_conv_and_scan_vs_oracle(cuda, hk, hv):
    rng = random.Random(hk)
    shapes = [(rng.randint(70, 200), [rng.randint(24, 64) for _ in range(rng.randint(1, 4))]) for _ in range(2)]
    shapes.append((5, [3]))
    got, want = _scan_case(cuda, hk, hv, shapes)
    # bf16 inputs of the scan (conv output) vs an fp32 oracle on the same pre-conv rows
    err = (got - want).abs().max().item() / want.abs().max().item()
    assert err < 2e-2, err


def test_long_chunk_chain_vs_oracle(cuda):
    """A 1500-token trunk (24 chunks of the WY-form scan, the state carried 23 times through
    bf16 operands) plus branches and a chunk-aligned 64-token trunk, vs the fp64 token
    recurrence: the chunked form must not drift over a long chain."""
    got, want = _scan_case(cuda, 1, 2, [(1500, [40, 64]), (64, [1])], seed=3)
    err = (got - want).abs().max().item() / want.abs().max().item()
    assert err < 2e-2, err


def test_split_scan_matches_unsplit_and_oracle(cuda):
    """A batch whose first segment's chain dominates (1000-token trunk) beside two short ones, at
    configuration-4 head counts: the layout splits the scan (that chain beside the other
    segments' pre-pass, on a second stream), and the outputs are bit-identical to the unsplit
    launch and within the oracle bar."""
    from dan_b200.qwen3_5 import RecurrentLayout

    shapes = [(1000, [40, 50]), (200, [30]), (100, [20])]
    assert RecurrentLayout.split_lead([18, 5, 3], 32) and not RecurrentLayout.split_lead([6, 5], 32)
    split, want = _scan_case(cuda, 16, 32, shapes, seed=5)
    whole, _ = _scan_case(cuda, 16, 32, shapes, seed=5, lead=(0, 0), oracle=False)
    assert torch.equal(split, whole)
    err = (split - want).abs().max().item() / want.abs().max().item()
    assert err < 2e-2, err


@pytest.mark.parametrize("rows,channels", [(1, 1032), (3, 512), (13, 1032), (25, 8192), (301, 1032)])
def test_causal_conv_row_sources(cuda, rows, channels):
    """dan_causal_conv against a float64 restatement of qwen3_5.py:218-220 row by row, at about
    one bf16 step. Each row's three sources are drawn at random among the previous packed row
    (taken from registers, including across the kernel's 12-row blocks), another packed row
    (gathered), a zero row (code -1) and a history row (code -2 - i), with a channel count that
    is not a multiple of the 1024 a block covers."""
    gen = torch.Generator().manual_seed(rows * 7 + channels)
    rng = random.Random(rows)
    src = (torch.randn(rows, channels, generator=gen) * 0.7).bfloat16()
    hist = (torch.randn(5, channels, generator=gen) * 0.7).bfloat16()
    w = (torch.randn(channels, 4, generator=gen) * 0.5).bfloat16()
    codes = torch.empty(rows, 3, dtype=torch.int32)
    for r in range(rows):
        for j in range(3):
            kind = rng.random()
            if kind < 0.6 and r - 1 - j >= 0:
                codes[r, j] = r - 1 - j
            elif kind < 0.75:
                codes[r, j] = rng.randrange(rows)
            elif kind < 0.9:
                codes[r, j] = -1
            else:
                codes[r, j] = -2 - rng.randrange(5)

    def row(code):
        if code >= 0:
            return src[code].double()
        if code == -1:
            return torch.zeros(channels, dtype=torch.float64)
        return hist[-code - 2].double()

    want = torch.empty(rows, channels, dtype=torch.float64)
    wd = w.double()
    for r in range(rows):
        ext = [row(int(codes[r, 2])), row(int(codes[r, 1])), row(int(codes[r, 0])), src[r].double()]
        acc = sum(wd[:, t] * ext[t] for t in range(4))
        want[r] = torch.nn.functional.silu(acc)
    src_d, hist_d, w_d, codes_d = src.to(cuda), hist.to(cuda), w.to(cuda), codes.to(cuda)
    out = torch.empty(rows, channels, dtype=torch.bfloat16, device=cuda)
    _lib.call("dan_causal_conv", _lib.ptr(src_d), channels, _lib.ptr(hist_d), channels, _lib.ptr(w_d),
              _lib.ptr(codes_d), _lib.ptr(out), channels, rows, channels, _lib.stream())
    got = out.double().cpu()
    err = (got - want).abs() - (want.abs() * 2.0 ** -7 + 1e-5)
    assert err.max().item() <= 0, (got - want).abs().max().item()
