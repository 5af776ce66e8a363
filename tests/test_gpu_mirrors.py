"""dan's op-level interfaces on the dan_b200 kernels, each against a CPU statement of dan's own
formula (the rounding points of dan/fused.py in bf16, or the fp64 oracle):

- the fused.py functions under their names and signatures (fused.py:35-101);
- ``FP8Linear(linear, rowwise).forward`` (quant.py:23-42), row-wise and per-tensor;
- ``delta_rule(q, k, v, g, beta, lengths, states)`` (qwen3_5.py:136-158);
- ``attend(q, k, v, segments, layer)`` with pasts as pool pages and as dan's per-layer
  tensors, and its saves (attention.py:200-207);
- ``model.hidden`` / ``model.label_logits`` (llama.py:152-165).

bf16 results are held to one bf16 step (relative 2^-7) of the reference formula, two where the
reference rounds twice and the kernel once."""
import random

import pytest
import torch
import torch.nn.functional as F

from dan_b200 import fused
from dan_b200.attention import Batch, attend, segment
from oracle import attention as OA
from oracle import fp8 as OF
from oracle import qwen3_5 as OQ

pytestmark = pytest.mark.gpu

BF16_STEP = 2.0 ** -7  # the largest relative spacing of bf16 values


def _close(got, want, rel=BF16_STEP, what=""):
    got, want = got.float().cpu(), want.float().cpu()
    err = ((got - want).abs() / want.abs().clamp(min=1e-3)).max().item()
    assert err <= rel * 1.01, f"{what}: relative error {err} > {rel}"


def _r(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).bfloat16()


def test_rms_norms(cuda):
    x, w = _r(37, 4096, seed=1), _r(4096, seed=2, scale=0.1) + 1
    y = x.float()
    y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-5)
    _close(fused.rms_norm(x.to(cuda), w.to(cuda), 1e-5), w * y.bfloat16(), what="rms_norm")  # fused.py:35-40
    wz = _r(2560, seed=3, scale=0.1)
    xz = _r(5, 3, 2560, seed=4)
    yz = xz.float()
    yz = yz * torch.rsqrt(yz.pow(2).mean(-1, keepdim=True) + 1e-6)
    _close(fused.rms_norm_zero_centered(xz.to(cuda), wz.to(cuda), 1e-6), (yz * (1 + wz.float())).bfloat16(),
           what="rms_norm_zero_centered")  # fused.py:43-48


@pytest.mark.parametrize("d", [128, 96])
def test_gated_rms_norm(cuda, d):
    x, z, w = _r(50, 4, d, seed=5), _r(50, 4, d, seed=6), _r(d, seed=7, scale=0.1) + 1
    y = x.float()
    y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-6)
    want = ((w * y.bfloat16()).float() * F.silu(z.float())).bfloat16()  # fused.py:51-56
    _close(fused.gated_rms_norm(x.to(cuda), z.to(cuda), w.to(cuda), 1e-6), want, rel=2 * BF16_STEP,
           what="gated_rms_norm")


def test_swiglu_and_sigmoid_gate(cuda):
    g, u = _r(33, 300, seed=8, scale=3), _r(33, 300, seed=9)
    _close(fused.swiglu(g.to(cuda), u.to(cuda)), F.silu(g) * u, rel=2 * BF16_STEP, what="swiglu")  # fused.py:59-61
    x, gate = _r(17, 2, 256, seed=10), _r(17, 2, 256, seed=11, scale=3)
    _close(fused.sigmoid_gate(x.to(cuda), gate.to(cuda)), x * torch.sigmoid(gate), rel=2 * BF16_STEP,
           what="sigmoid_gate")


@pytest.mark.parametrize("r", [128, 64])
def test_rotate_partial(cuda, r):
    n, h, d = 40, 6, 256 if r == 64 else 128
    x = _r(n, h, d, seed=12)
    pos = torch.arange(100, 100 + n, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, r, 2, dtype=torch.float32) / r))
    ang = pos[:, None] * inv[None, :]
    ang = torch.cat((ang, ang), -1)
    cos, sin = ang.cos().bfloat16(), ang.sin().bfloat16()
    xr, xp = x[..., :r], x[..., r:]
    a, b = xr.chunk(2, dim=-1)
    want = torch.cat([xr * cos[:, None] + torch.cat((-b, a), dim=-1) * sin[:, None], xp], dim=-1)  # fused.py:69-76
    got = fused.rotate_partial(x.to(cuda), cos.to(cuda), sin.to(cuda))
    _close(got, want, rel=2 * BF16_STEP, what="rotate_partial")
    assert torch.equal(got[..., r:].cpu(), x[..., r:])


def test_delta_gates(cuda):
    b, a = _r(70, 32, seed=13, scale=2), _r(70, 32, seed=14, scale=3)
    a_log = torch.log(1 + 15 * torch.rand(32, generator=torch.Generator().manual_seed(15)))
    dt = 0.5 + 0.5 * torch.rand(32, generator=torch.Generator().manual_seed(16))
    beta, g = fused.delta_gates(b.to(cuda), a.to(cuda), a_log.to(cuda), dt.to(cuda))
    _close(beta, b.sigmoid(), what="beta")  # fused.py:79-82
    want = -a_log.exp() * F.softplus(a.float() + dt)
    assert g.dtype == torch.float32
    assert ((g.cpu() - want).abs() / want.abs().clamp(min=1e-6)).max().item() < 1e-5


@pytest.mark.parametrize("rowwise", [True, False])
def test_fp8_quantize_and_linear(cuda, rowwise):
    x = _r(300, 512, seed=17)
    q, s = fused.fp8_quantize(x.to(cuda), 448.0, rowwise)
    xf = x.float()  # fused.py:85-91
    amax = xf.abs().amax(dim=-1, keepdim=True) if rowwise else xf.abs().amax().reshape(1, 1)
    scale = amax.clamp(min=1e-12) / 448.0
    assert torch.equal(s.cpu(), scale)
    assert torch.equal(q.cpu().view(torch.uint8), (xf / scale).to(torch.float8_e4m3fn).view(torch.uint8))

    from dan_b200.quant import FP8Linear

    lin = torch.nn.Linear(512, 768, bias=True)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(768, 512, generator=torch.Generator().manual_seed(18)) * 0.05)
        lin.bias.copy_(torch.randn(768, generator=torch.Generator().manual_seed(19)) * 0.1)
    lin = lin.to(cuda, torch.bfloat16)
    fl = FP8Linear(lin, rowwise=rowwise)
    assert fl.weight.dtype == torch.float8_e4m3fn and tuple(fl.weight_scale.shape) == ((1, 768) if rowwise else (1, 1))
    got = fl.forward(x.to(cuda).view(3, 100, 512))
    assert got.shape == (3, 100, 768) and got.dtype == torch.bfloat16
    # quant.py:37-42: both operands' e4m3 values times their scales, fp32 accumulation
    wq, ws = fl.weight.float().cpu(), fl.weight_scale.cpu().reshape(-1)
    xq = (xf / scale).to(torch.float8_e4m3fn).float()
    want = (xq.double() @ wq.double().T) * scale.double() * ws.double().reshape(1, -1) + lin.bias.double().cpu()
    err = (got.reshape(300, 768).float().cpu() - want.float()).abs().max().item() / want.abs().max().item()
    assert err < 1e-2, err
    if rowwise:  # and the row-wise path agrees with the oracle's FP8 linear
        ref = OF.linear(x, wq, ws, lin.bias.float().cpu())
        assert (got.reshape(300, 768).float().cpu() - ref).abs().max().item() / ref.abs().max().item() < 1e-2


def test_lse_merge(cuda):
    t, h, d = 45, 4, 64
    oa, ob = _r(t, h, d, seed=20), _r(t, h, d, seed=21)
    la = torch.randn(h, t, generator=torch.Generator().manual_seed(22)) * 3
    lb = torch.randn(h, t, generator=torch.Generator().manual_seed(23)) * 3
    got = fused.lse_merge(oa.to(cuda), la.to(cuda), ob.to(cuda), lb.to(cuda))
    xa, xb = la.t()[..., None], lb.t()[..., None]  # fused.py:94-101
    m = torch.maximum(xa, xb)
    wa, wb = (xa - m).exp(), (xb - m).exp()
    _close(got, ((oa.float() * wa + ob.float() * wb) / (wa + wb)).bfloat16(), what="lse_merge")


@pytest.mark.parametrize("lengths", [[70, 200, 1, 64], [0, 130]])
def test_delta_rule(cuda, lengths):
    h, dk = 4, 128
    n = sum(lengths)
    q, k, v = _r(n, h, dk, seed=24), _r(n, h, dk, seed=25), _r(n, h, dk, seed=26)
    g = -torch.rand(n, h, generator=torch.Generator().manual_seed(27)) * 0.5
    beta = torch.rand(n, h, generator=torch.Generator().manual_seed(28)).bfloat16()
    states = torch.randn(len(lengths), h, dk, dk, generator=torch.Generator().manual_seed(29)) * 0.1
    from dan_b200.qwen3_5 import delta_rule

    out, final = delta_rule(q.to(cuda), k.to(cuda), v.to(cuda), g.to(cuda), beta.to(cuda), lengths,
                            states.to(cuda))
    assert out.shape == (n, h, dk) and final.shape == states.shape and final.dtype == torch.float32
    i = 0
    for j, length in enumerate(lengths):
        o, f = OQ.delta_rule(q[i:i + length], k[i:i + length], v[i:i + length], g[i:i + length],
                             beta[i:i + length].float(), states[j])
        if length:
            err = (out[i:i + length].float().cpu() - o).abs().max().item() / o.abs().max().item()
            assert err < 2e-2, (j, err)
        ferr = (final[j].cpu() - f).abs().max().item() / f.abs().max().item()
        assert ferr < 2e-2, (j, ferr)
        i += length


def _dan_segments(shapes, h, hkv, d, seed):
    """Packed q/k/v and segments whose pasts are dan's per-layer tensors (layer 0), and the
    oracle's segment dicts."""
    gen = torch.Generator().manual_seed(seed)
    segs, oracle, start = Batch(), [], 0
    branch_all = []
    for trunk, lens, past in shapes:
        branch = [0] * trunk + [j for j, n in enumerate(lens, 1) for _ in range(n)]
        pk = torch.randn(hkv, past, d, generator=gen).bfloat16() if past else None
        pv = torch.randn(hkv, past, d, generator=gen).bfloat16() if past else None
        past_arg = {0: (pk.to("cuda"), pv.to("cuda"))} if past else None
        segs.append(segment(start, branch, past_arg, 0, past, "cuda"))
        oracle.append({"start": start, "end": start + len(branch), "branch": branch,
                       "past": (pk.float(), pv.float()) if past else None})
        branch_all += branch
        start += len(branch)
    q = torch.randn(h, start, d, generator=gen).bfloat16()
    k = torch.randn(hkv, start, d, generator=gen).bfloat16()
    v = torch.randn(hkv, start, d, generator=gen).bfloat16()
    return segs, oracle, q, k, v


@pytest.mark.parametrize("d", [64, 128])
def test_attend_with_dan_pasts(cuda, d):
    h, hkv = 8, 2
    shapes = [(200, [30, 1, 70], 300), (5, [3], 0), (129, [64, 64], 128), (40, [], 1)]
    segs, oracle, q, k, v = _dan_segments(shapes, h, hkv, d, 30)
    segs[0].save = 100
    got = attend(q.to(cuda), k.to(cuda), v.to(cuda), segs, 0)
    want = OA.attend(q.float(), k.float(), v.float(), oracle)
    err = (got.float().cpu() - want).abs().max().item()
    assert got.shape == q.shape and err < 2e-2, err
    sk, sv = segs[0].saved[0]  # attention.py:202-204: clones of the first ``save`` new tokens
    assert torch.equal(sk.cpu(), k[:, :100]) and torch.equal(sv.cpu(), v[:, :100])
    got2 = attend(q.to(cuda), k.to(cuda), v.to(cuda), segs, 0)  # cached layout and staging
    assert torch.equal(got, got2)


def test_attend_without_pasts_matches_oracle(cuda):
    rng = random.Random(3)
    shapes = [(rng.randint(100, 700), [rng.randint(16, 96) for _ in range(rng.randint(1, 9))], 0) for _ in range(3)]
    segs, oracle, q, k, v = _dan_segments(shapes, 32, 8, 128, 31)
    got = attend(q.to(cuda), k.to(cuda), v.to(cuda), segs, 0)
    want = OA.attend(q.float(), k.float(), v.float(), oracle)
    assert (got.float().cpu() - want).abs().max().item() < 2e-2


def test_hidden_and_label_logits(cuda, tmp_path):
    from dan_b200.plan import Branch, ReadPlan
    from dan_b200.runner import Runner
    from oracle import llama as OL
    from oracle import runner as OR
    from oracle import weights

    cfg = weights.llama_config(vocab=640, hidden=256, inter=512, layers=2, heads=4, kv_heads=2, head_dim=64, tie=False)
    state = weights.random_state(cfg, seed=4)
    weights.save_checkpoint(str(tmp_path), cfg, state)
    runner = Runner(str(tmp_path), cuda, cache_bytes=0)
    plans = [ReadPlan(list(range(5, 120)), branches=[Branch([7, 8, 9], [1, 2, 3]), Branch([4] * 9, [5, 600])])]
    ids, pos, segs, reads, _ = runner.pack(plans, use_cache=False)
    m = runner.model
    h = m.hidden(torch.as_tensor(ids, device=cuda), torch.as_tensor(pos, device=cuda), segs)
    oids, opos, osegs, _, _ = OR.pack(plans)
    want_h = OL.hidden(state, cfg, oids, opos, osegs)  # final-normed (llama.py:152-161)
    assert (h.float().cpu() - want_h).abs().max().item() / want_h.abs().max().item() < 3e-2
    for row, labels in reads:
        got = m.label_logits(h[row], labels)
        assert got.dtype == torch.float32 and got.shape == (len(labels),)
        want = m.lm_head[torch.as_tensor(labels, device=cuda)].float() @ h[row].float()  # llama.py:163-165
        assert (got - want).abs().max().item() < 1e-3 * max(1.0, want.abs().max().item())
