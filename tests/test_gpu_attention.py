"""Tree-attention kernel vs the CPU oracle (the reference's dense masked path restated)
and vs the reference's own output on its edge shapes. Tolerance: the reference's own
varlen-vs-dense bound, atol = rtol = 2e-2 (tests/test_runner.py:68)."""
import pytest
import torch
from conftest import golden
from helpers import attention_problem

from dan_b200.attention import TreeLayout, tree_attention
from oracle import attention as OA

pytestmark = pytest.mark.gpu

EDGE = [(40, [5, 9, 1], 0), (7, [30], 12), (1, [3, 3, 3, 3, 3, 3], 0), (64, [], 0), (13, [17, 2], 20)]
LONG = [(300, [17, 200, 1], 0), (129, [128, 128], 250), (0, [5, 7], 130), (128, [1], 128), (700, [96] * 9, 0)]


def run_case(shapes, h, hkv, d, cuda, seed=0):
    segs, n, q, k, v, pk, pv, osegs = attention_problem(shapes, h, hkv, d, "cpu", seed=seed)
    lay = TreeLayout.build(segs, n, cuda)

    class Pool:
        pass

    pool = Pool()
    pool.k, pool.v = [pk.to(cuda)], [pv.to(cuda)]
    out = tree_attention(q.to(cuda), k.to(cuda), v.to(cuda), lay, pool=pool, layer=0)
    torch.cuda.synchronize()
    want = OA.attend(q.float().transpose(0, 1), k.float().transpose(0, 1), v.float().transpose(0, 1), osegs)
    return out.float().cpu(), want.transpose(0, 1)


@pytest.mark.parametrize("d", [64, 128, 256])
def test_edge_shapes(cuda, d):
    got, want = run_case(EDGE, 8, 2, d, cuda)
    torch.testing.assert_close(got, want, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("d", [64, 128])
def test_long_segments_with_pages(cuda, d):
    got, want = run_case(LONG, 8, 2, d, cuda, seed=1)
    torch.testing.assert_close(got, want, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("h,hkv,d", [(9, 3, 64), (9, 3, 128), (8, 2, 256)])
def test_single_head_kernel_long_segments(cuda, h, hkv, d):
    """The single-head kernel (odd GQA ratio, or D = 256) on long paged segments: whole 32-row
    slabs leave by TMA store, ragged ones per row."""
    got, want = run_case(LONG, h, hkv, d, cuda, seed=3)
    torch.testing.assert_close(got, want, atol=2e-2, rtol=2e-2)


def test_llama3_heads_random_batch(cuda):
    import random

    rng = random.Random(5)
    shapes = [(rng.randint(128, 700), [rng.randint(16, 96) for _ in range(rng.randint(1, 8))], 0)
              for _ in range(3)]
    got, want = run_case(shapes, 32, 8, 128, cuda, seed=2)
    torch.testing.assert_close(got, want, atol=2e-2, rtol=2e-2)


def test_against_reference_output(cuda):
    """The reference's own _attend_dense output on its edge shapes (fp32 inputs, d=64)."""
    from make_golden import attention_inputs

    g = golden("attention_edges.pt")
    q, k, v, pasts = attention_inputs(g["h"], g["hkv"], g["d"], g["seed"], g["shapes"])
    from helpers import build_segments

    segs, n, npages = build_segments(g["shapes"], shuffle_pages=False)
    pk = torch.zeros(max(npages, 1) * 128, g["hkv"], g["d"])
    pv = torch.zeros_like(pk)
    for s, pkv in zip(segs, pasts):
        if pkv is not None:
            for t in range(s.past_len):
                row = s.past.pages[t // 128] * 128 + t % 128
                pk[row], pv[row] = pkv[0][:, t], pkv[1][:, t]

    class Pool:
        pass

    pool = Pool()
    pool.k, pool.v = [pk.to(cuda, torch.bfloat16)], [pv.to(cuda, torch.bfloat16)]
    lay = TreeLayout.build(segs, n, cuda)
    b = lambda t: t.transpose(0, 1).contiguous().to(cuda, torch.bfloat16)
    out = tree_attention(b(q), b(k), b(v), lay, pool=pool).float().cpu().transpose(0, 1)
    torch.testing.assert_close(out, g["out"], atol=2e-2, rtol=2e-2)


def test_reads_strided_qkv_in_place(cuda):
    """q/k/v as column slices of one fused projection buffer (how the model calls it)."""
    segs, n, q, k, v, pk, pv, osegs = attention_problem([(90, [20, 30], 0), (200, [64], 0)], 8, 2, 128, "cpu")
    qkv = torch.cat([q.reshape(n, -1), k.reshape(n, -1), v.reshape(n, -1)], 1).to(cuda)
    qs = qkv[:, :8 * 128].view(n, 8, 128)
    ks = qkv[:, 8 * 128:10 * 128].view(n, 2, 128)
    vs = qkv[:, 10 * 128:].view(n, 2, 128)
    lay = TreeLayout.build(segs, n, cuda)
    out = torch.empty(n, 8 * 128, dtype=torch.bfloat16, device=cuda)
    tree_attention(qs, ks, vs, lay, out=out.view(n, 8, 128))
    want = OA.attend(q.float().transpose(0, 1), k.float().transpose(0, 1), v.float().transpose(0, 1), osegs)
    torch.testing.assert_close(out.view(n, 8, 128).float().cpu(), want.transpose(0, 1), atol=2e-2, rtol=2e-2)
