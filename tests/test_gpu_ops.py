"""GEMM, norm, RoPE, embedding, quantisation and readout kernels vs fp32 references.

Tolerances: bf16 outputs are compared at a relative error of 1e-2 of the output
scale (one bf16 rounding is 2^-8); e4m3 GEMMs against the FP8 restatement
(oracle.fp8) at the same bound after identical quantisation."""
import pytest
import torch
import torch.nn.functional as F

from dan_b200 import _lib, ops
from oracle import fp8 as OF

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp(min=1e-6)).item()


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (200, 960, 576), (1000, 6144, 512), (77, 512, 1536),
                                   (1, 256, 128), (300, 1000, 200)])
def test_gemm_bf16(cuda, m, n, k):
    g = torch.Generator(device=cuda).manual_seed(m + n + k)
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = torch.randn(n, k, device=cuda, generator=g).bfloat16()
    y = ops.linear(x, w)
    assert rel_err(y, x.float() @ w.float().T) < 1e-2


@pytest.mark.parametrize("m", [100, 700])
def test_gemm_unaligned_output(cuda, m):
    """Outputs whose rows are not 16-byte aligned (a view at an odd column offset, odd row
    pitch) take the per-thread store path instead of the TMA-store epilogue; residual too."""
    g = torch.Generator(device=cuda).manual_seed(m)
    k, n = 512, 520
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = torch.randn(n, k, device=cuda, generator=g).bfloat16()
    buf = torch.zeros(m, n + 3, device=cuda, dtype=torch.bfloat16)
    out = buf[:, 1:1 + n]
    ops.linear(x, w, out=out)
    assert rel_err(out, x.float() @ w.float().T) < 1e-2
    assert torch.all(buf[:, 0] == 0) and torch.all(buf[:, 1 + n:] == 0)
    rbuf = torch.randn(m, n + 3, device=cuda, generator=g).bfloat16()
    r = rbuf[:, 1:1 + n]
    want = r.float() + x.float() @ w.float().T
    ops.linear(x, w, residual=r)
    assert rel_err(r, want) < 1e-2


def test_gemm_bias_residual(cuda):
    g = torch.Generator(device=cuda).manual_seed(1)
    m, n, k = 513, 768, 320
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = torch.randn(n, k, device=cuda, generator=g).bfloat16()
    b = torch.randn(n, device=cuda, generator=g).bfloat16()
    r = torch.randn(m, n, device=cuda, generator=g).bfloat16()
    want = r.float() + (x.float() @ w.float().T + b.float())
    ops.linear(x, w, bias=b, residual=r)  # in place into r
    assert rel_err(r, want) < 1e-2


def test_gemm_swiglu(cuda):
    g = torch.Generator(device=cuda).manual_seed(2)
    m, i, k = 333, 512, 256
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    wg = torch.randn(i, k, device=cuda, generator=g).bfloat16()
    wu = torch.randn(i, k, device=cuda, generator=g).bfloat16()
    y = ops.linear_swiglu(x, ops.interleave_gate_up(wg, wu))
    want = F.silu(x.float() @ wg.float().T) * (x.float() @ wu.float().T)
    assert rel_err(y, want) < 1e-2


@pytest.mark.parametrize("m,n,k", [(256, 512, 256), (130, 1280, 640)])
def test_gemm_e4m3(cuda, m, n, k):
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = (torch.randn(n, k, device=cuda, generator=g) * 0.05).bfloat16()
    xq, xs = ops.quantize_e4m3(x)
    wq, ws = ops.quantize_e4m3(w)
    y = ops.linear_e4m3(xq, xs, wq, ws)
    # the same quantisation on the CPU (oracle), then an exact product
    oxq, oxs = OF.quantize_rows(x.cpu())
    owq, ows = OF.quantize_rows(w.cpu())
    assert torch.equal(xq.float().cpu(), oxq) and torch.allclose(xs.cpu(), oxs.flatten())
    assert torch.equal(wq.float().cpu(), owq)
    want = OF.linear(x.cpu(), owq, ows.flatten())
    assert rel_err(y, want) < 1e-2


# Shapes whose last wave of 256 x 256 tiles would leave CTA pairs idle, with tiles at least
# 128 K iterations deep (K >= 8192 in bf16, 16384 in e4m3), take the stream-K path: the last
# tiles are split by K iteration across all CTA pairs and the partial sums are reduced in pair
# order. (7089, 4096, 14336) splits the last 78 of 448 tiles; (520, 2560, 9216) splits every
# tile over 2-3 pairs and (300, 1024, 8192) over about nine. The result must match fp32 and be
# bit-identical from one call to the next.
@pytest.mark.parametrize("m,n,k", [(7089, 4096, 14336), (520, 2560, 9216), (300, 1024, 8192)])
def test_gemm_stream_k(cuda, m, n, k):
    g = torch.Generator(device=cuda).manual_seed(m + k)
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = torch.randn(n, k, device=cuda, generator=g).bfloat16()
    y1 = ops.linear(x, w)
    y2 = ops.linear(x, w)
    assert torch.equal(y1, y2)
    assert rel_err(y1, x.float() @ w.float().T) < 1e-2


def _narrow_split(m, n, k, epilogue, hd=0):
    """Items per tile of the last, ragged wave of 256 x 256 tiles (the host rule of the pair
    kernel): 1 when every tile runs whole."""
    pairs = torch.cuda.get_device_properties(0).multi_processor_count // 2
    tiles = -(-m // 256) * -(-n // 256)
    if m < 256 or (k * 2 // 128 >= 128 and tiles % pairs and tiles * 100 < -(-tiles // pairs) * pairs * 95):
        return 1  # single-CTA kernel, or the stream-K tail
    s_max = 4 if epilogue == "swiglu" else (256 // hd if epilogue == "rope" else 8)
    rem, s = tiles % pairs, 1
    while 2 * s <= s_max and rem * 2 * s <= pairs:
        s *= 2
    return s if rem else 1


# A ragged last wave of whole tiles runs as narrow column slices (256 / s columns, s = 2, 4, 8)
# spread over the idle pairs. Shapes picked so each epilogue meets each slice width on a
# 148-SM part: (7089, 4096) is the Llama-3-8B o projection (448 tiles, 4 left over -> 8 slices
# of 32 columns), (7089, 6144) its q/k/v projection (6 left over, RoPE keeps 128-column heads),
# 6600 columns make slices past n. The result must match fp32 and repeat bit for bit.
@pytest.mark.parametrize("m,n,k,epilogue,split", [
    (7089, 4096, 4096, "residual", 8),
    (768, 6600, 512, "store", 8),
    (512, 11008, 256, "residual", 4),
    (7089, 6144, 1024, "rope", 2),
    (300, 960, 512, "rope64", 4),
    (256, 4096, 512, "swiglu", 4),
    (768, 2560, 512, "swiglu", 2),
    (7089, 4096, 2048, "e4m3", 8),
])
def test_gemm_narrow_tail(cuda, m, n, k, epilogue, split):
    hd = {"rope": 128, "rope64": 64}.get(epilogue, 0)
    kind = "rope" if hd else epilogue
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert _narrow_split(m, n, k, kind, hd) == split
    g = torch.Generator(device=cuda).manual_seed(m + n + k)
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = (torch.randn(n, k, device=cuda, generator=g) * 0.1).bfloat16()
    ref = x.float() @ w.float().T
    if kind == "residual":
        r = torch.randn(m, n, device=cuda, generator=g).bfloat16()
        want = r.float() + ref
        r2 = r.clone()
        ops.linear(x, w, residual=r)
        ops.linear(x, w, residual=r2)
        assert torch.equal(r, r2)
        assert rel_err(r, want) < 1e-2
    elif kind == "store":
        y = ops.linear(x, w)
        assert torch.equal(y, ops.linear(x, w))
        assert rel_err(y, ref) < 1e-2
    elif kind == "swiglu":
        wg, wu = w[:n // 2], w[n // 2:]
        y = ops.linear_swiglu(x, ops.interleave_gate_up(wg, wu))
        want = F.silu(x.float() @ wg.float().T) * (x.float() @ wu.float().T)
        assert rel_err(y, want) < 1e-2
    elif kind == "rope":
        pos = torch.randint(0, 3000, (m,), device=cuda, generator=g)
        inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, dtype=torch.float32, device=cuda) / hd))
        rot = n - 2 * hd if hd == 128 else n - 3 * hd  # v heads at the end stay unrotated
        y = ops.linear_rope(x, w, ops.rope_table(pos, inv), rot, hd)
        proj = ops.linear(x, w)
        want = proj.float().clone()
        want[:, :rot] = _rope_ref(proj[:, :rot].view(m, -1, hd), pos, inv, hd).reshape(m, -1)
        assert rel_err(y, want) < 1e-2
    else:
        xq, xs = ops.quantize_e4m3(x)
        wq, ws = ops.quantize_e4m3(w)
        r = torch.randn(m, n, device=cuda, generator=g).bfloat16()
        want = r.float() + (xq.float() * xs.view(-1, 1)) @ (wq.float() * ws.view(-1, 1)).T
        ops.linear_e4m3(xq, xs, wq, ws, residual=r)
        assert rel_err(r, want) < 1e-2


def test_gemm_stream_k_epilogues(cuda):
    g = torch.Generator(device=cuda).manual_seed(9)
    m, k = 300, 8192
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = torch.randn(4096, k, device=cuda, generator=g).bfloat16()
    r = torch.randn(m, 4096, device=cuda, generator=g).bfloat16()
    want = r.float() + x.float() @ w.float().T
    ops.linear(x, w, residual=r)
    assert rel_err(r, want) < 1e-2
    wg, wu = w[:2048], w[2048:]
    y = ops.linear_swiglu(x, ops.interleave_gate_up(wg, wu))
    assert rel_err(y, F.silu(x.float() @ wg.float().T) * (x.float() @ wu.float().T)) < 1e-2
    x8 = torch.randn(m, 2 * k, device=cuda, generator=g).bfloat16()
    w8 = (torch.randn(4096, 2 * k, device=cuda, generator=g) * 0.05).bfloat16()
    xq, xs = ops.quantize_e4m3(x8)
    wq, ws = ops.quantize_e4m3(w8)
    y8 = ops.linear_e4m3(xq, xs, wq, ws)
    want8 = (xq.float() * xs.view(-1, 1)) @ (wq.float() * ws.view(-1, 1)).T
    assert rel_err(y8, want8) < 1e-2


def test_rms_norm_modes(cuda):
    g = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(37, 4096, device=cuda, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(4096, device=cuda, generator=g)).bfloat16()
    xf = x.float()
    xh = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)
    assert rel_err(ops.rms_norm(x, w, 1e-5), w.float() * xh.bfloat16().float()) < 1e-2
    assert rel_err(ops.rms_norm(x, w, 1e-5, zero_centered=True), xh * (1 + w.float())) < 1e-2
    # per-head, in place on a strided view
    buf = torch.randn(10, 6 * 128, device=cuda, generator=g).bfloat16()
    view = buf[:, 128:5 * 128].view(10, 4, 128)
    ref = view.float()
    hw = (1 + 0.1 * torch.randn(128, device=cuda, generator=g)).bfloat16()
    want = hw.float() * (ref * torch.rsqrt(ref.pow(2).mean(-1, keepdim=True) + 1e-6)).bfloat16().float()
    before = buf.clone()
    ops.rms_norm(view, hw, 1e-6, out=view)
    assert rel_err(view, want) < 1e-2
    assert torch.equal(buf[:, :128], before[:, :128]) and torch.equal(buf[:, 5 * 128:], before[:, 5 * 128:])


def _e4m3_rows(cols, g):
    """Rows that stress per-row e4m3 quantisation: spread-out magnitudes, exact ties (a row
    max of 448 * 2^k makes the scale a power of two, so values at e4m3 midpoints divide
    exactly onto them), signed zeros and values that round to zero."""
    rows = [torch.randn(cols, generator=g) * 10.0 ** torch.empty(1).uniform_(-3, 3, generator=g)
            for _ in range(24)]
    mids = torch.tensor([1.0625, 1.1875, 0.0078125 * 1.5, 3.25, -1.0625, -13.0, 2.0 ** -10, 2.0 ** -9 * 1.5])
    for k in (0, -3, 4):
        r = mids[torch.randint(0, len(mids), (cols,), generator=g)] * 2.0 ** k
        r[0] = 448.0 * 2.0 ** k
        rows.append(r)
    z = torch.zeros(cols)
    z[1::2] = -0.0
    z[3] = 1e-5
    z[5] = -3e-6
    rows.append(z)
    return torch.stack(rows).bfloat16()


def _e4m3_codes(x):
    xf = x.float()
    scale = xf.abs().amax(dim=-1, keepdim=True).clamp(min=1e-12) / 448.0
    return (xf / scale).to(torch.float8_e4m3fn).view(torch.uint8), scale.flatten()


# Codes bit for bit (signed zeros included) against the reference's (x / scale).to(e4m3)
# on the CPU: the vector kernel (<= 8192 columns, 128 threads per row; <= 16384, 256), the
# one-block-per-row kernel beyond that, and the product-with-bracket quotient's division
# fallback on exact ties.
@pytest.mark.parametrize("cols", [528, 2560, 4096, 9216, 14336, 16400])
def test_quantize_e4m3_codes(cuda, cols):
    g = torch.Generator().manual_seed(cols)
    x = _e4m3_rows(cols, g)
    q, s = ops.quantize_e4m3(x.to(cuda))
    want_q, want_s = _e4m3_codes(x)
    assert torch.equal(s.cpu(), want_s)
    assert torch.equal(q.view(torch.uint8).cpu(), want_q)


@pytest.mark.parametrize("cols", [1024, 2560, 4096])
def test_rms_norm_fp8_codes(cuda, cols):
    g = torch.Generator().manual_seed(cols)
    x = _e4m3_rows(cols, g).to(cuda)
    w = (1 + 0.1 * torch.randn(cols, generator=g)).bfloat16().to(cuda)
    y = ops.rms_norm(x, w, 1e-6)
    _, q8, sc = ops.rms_norm(x, w, 1e-6, fp8=True)
    want_q, want_s = _e4m3_codes(y.cpu())
    assert torch.equal(sc.cpu(), want_s)
    assert torch.equal(q8.view(torch.uint8).cpu(), want_q)


def test_rms_norm_fp8_fused(cuda):
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(64, 2560, device=cuda, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(2560, device=cuda, generator=g)).bfloat16()
    y = ops.rms_norm(x, w, 1e-6)
    _, q8, sc = ops.rms_norm(x, w, 1e-6, fp8=True)
    oq, osc = OF.quantize_rows(y.cpu())
    assert torch.equal(q8.float().cpu(), oq) and torch.allclose(sc.cpu(), osc.flatten())


def _rope_ref(x, pos, inv, rot):
    from oracle.llama import rotate

    ang = pos.float()[:, None] * inv[None]
    ang = torch.cat([ang, ang], -1)
    cos, sin = ang.cos().bfloat16().float(), ang.sin().bfloat16().float()
    return torch.cat([rotate(x.float()[..., :rot], cos[:, None], sin[:, None]), x.float()[..., rot:]], -1)


@pytest.mark.parametrize("rot", [128, 64])
def test_rope(cuda, rot):
    g = torch.Generator(device=cuda).manual_seed(6)
    n, heads, d = 50, 6, 128
    x = torch.randn(n, heads, d, device=cuda, generator=g).bfloat16()
    pos = torch.randint(0, 5000, (n,), device=cuda, generator=g)
    inv = 1.0 / (500000.0 ** (torch.arange(0, rot, 2, dtype=torch.float32, device=cuda) / rot))
    want = _rope_ref(x, pos, inv, rot)
    ops.rope_(x, ops.rope_table(pos, inv), rot)
    assert rel_err(x, want) < 1e-2


@pytest.mark.parametrize("d,heads,kv", [(128, 4, 2), (64, 9, 3)])
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("k", [256, 8192])
def test_gemm_rope_epilogue(cuda, d, heads, kv, fp8, k):
    """q/k/v projection with RoPE on the q and k heads in the GEMM epilogue (k = 8192 in bf16
    takes the stream-K path with each tile split over about nine CTA pairs)."""
    g = torch.Generator(device=cuda).manual_seed(8)
    m = 300
    n = (heads + 2 * kv) * d
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = (torch.randn(n, k, device=cuda, generator=g) * 0.1).bfloat16()
    pos = torch.randint(0, 3000, (m,), device=cuda, generator=g)
    inv = 1.0 / (10000.0 ** (torch.arange(0, d, 2, dtype=torch.float32, device=cuda) / d))
    table = ops.rope_table(pos, inv)
    if fp8:
        xq, xs = ops.quantize_e4m3(x)
        wq, ws = ops.quantize_e4m3(w)
        y = ops.linear_e4m3_rope(xq, xs, wq, ws, table, (heads + kv) * d, d)
        proj = ops.linear_e4m3(xq, xs, wq, ws)
    else:
        y = ops.linear_rope(x, w, table, (heads + kv) * d, d)
        proj = ops.linear(x, w)
    want = proj.float().clone()
    want[:, :(heads + kv) * d] = _rope_ref(proj[:, :(heads + kv) * d].view(m, heads + kv, d), pos, inv,
                                           d).reshape(m, -1)
    assert rel_err(y, want) < 1e-2


# Hidden sizes of configurations 1, 4 and 3: the readout's label rows load 1024 elements per
# warp step, so 576 and 2560 also take its remainder path.
@pytest.mark.parametrize("hidden", [576, 2560, 4096])
def test_embed_and_readout(cuda, hidden):
    g = torch.Generator(device=cuda).manual_seed(7)
    vocab = 1000
    table = torch.randn(vocab, hidden, device=cuda, generator=g).bfloat16()
    ids = torch.randint(0, vocab, (40,), device=cuda, generator=g)
    x = ops.embed(ids, table)
    assert torch.equal(x, table[ids])
    nw = (1 + 0.1 * torch.randn(hidden, device=cuda, generator=g)).bfloat16()
    rows = torch.tensor([3, 17, 39], dtype=torch.int32, device=cuda)
    labels = [[5, 9], [1, 2, 3, 4, 999], list(range(100, 355))]
    flat = torch.tensor([i for l in labels for i in l], dtype=torch.int32, device=cuda)
    off = torch.tensor([0, 2, 7, 7 + 255], dtype=torch.int32, device=cuda)
    lg, pr = ops.label_readout(x, rows, nw, 1e-5, False, table, flat, off, 255)
    xf = x.float()[rows.long()]
    hn = nw.float() * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).bfloat16().float()
    hn = hn.bfloat16().float()
    for q, l in enumerate(labels):
        want = table.float()[torch.tensor(l, device=cuda)] @ hn[q]
        got = lg[off[q]:off[q + 1]]
        torch.testing.assert_close(got, want, atol=1e-3, rtol=1e-3)
        torch.testing.assert_close(pr[off[q]:off[q + 1]], torch.softmax(want, 0), atol=1e-5, rtol=1e-4)


def test_kv_store(cuda):
    k = torch.randn(20, 2, 64, device=cuda).bfloat16()
    v = torch.randn(20, 2, 64, device=cuda).bfloat16()
    pk = torch.zeros(256, 2, 64, device=cuda).bfloat16()
    pv = torch.zeros_like(pk)
    src = torch.tensor([3, 4, 5], dtype=torch.int32, device=cuda)
    dst = torch.tensor([130, 131, 132], dtype=torch.int32, device=cuda)
    ops.kv_store(k, v, pk, pv, src, dst)
    assert torch.equal(pk[130:133], k[3:6]) and torch.equal(pv[130:133], v[3:6])


@pytest.mark.parametrize("rows,cols,heads", [(4001, 4096, 1), (2900, 8192, 1), (3000, 2560, 1), (1200, 2048, 3),
                                             (5, 4096, 1)])
def test_rms_norm_hidden_rows(cuda, rows, cols, heads):
    """Hidden-size rows (128 threads per row): thousands of rows, a strided [n, heads, cols] view
    (rows r / heads, r % heads) and a handful of rows all give the reference's rounding."""
    g = torch.Generator(device=cuda).manual_seed(rows + cols)
    n = rows // heads
    base = torch.randn(n, heads + 1, cols, device=cuda, generator=g).bfloat16()
    x = base[:, :heads, :]  # rows of the view are not contiguous when heads > 1
    w = (1 + 0.1 * torch.randn(cols, device=cuda, generator=g)).bfloat16()
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)
    ref = (w.float() * (xf * inv).bfloat16().float()).bfloat16()
    y = ops.rms_norm(x, w, 1e-6)
    diff = (y.float() - ref.float()).abs()
    assert (diff <= ref.float().abs() * 2.0 ** -6 + 1e-30).all()
    assert (diff == 0).float().mean().item() > 0.99
    _lib.check_status(cuda)


@pytest.mark.parametrize("cols", [4096, 2560])
def test_rms_norm_wide_rounding(cuda, cols):
    """Hidden-size rows take the 128-threads-per-row kernel: outputs must follow the reference's
    rounding points (mode 0: bf16(w * bf16(x * inv)); mode 1: bf16(x * inv * (1 + w)) in fp32,
    fused.py:35-48) up to one-ulp flips where the sum-of-squares order moves x * inv across a
    rounding boundary; the fused e4m3 output matches the quantisation of that bf16 row."""
    g = torch.Generator(device=cuda).manual_seed(cols)
    x = torch.randn(301, cols, device=cuda, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(cols, device=cuda, generator=g)).bfloat16()
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)
    refs = {0: (w.float() * (xf * inv).bfloat16().float()).bfloat16(),
            1: (xf * inv * (1 + w.float())).bfloat16()}
    for mode, ref in refs.items():
        y = ops.rms_norm(x, w, 1e-5, zero_centered=bool(mode))
        diff = (y.float() - ref.float()).abs()
        ulp = ref.float().abs().clamp(min=1e-30) * 2.0 ** -6  # two bf16 ulps
        assert (diff <= ulp + 1e-30).all(), mode
        assert (diff == 0).float().mean().item() > 0.99, mode
    y = ops.rms_norm(x, w, 1e-5)
    _, q8, sc = ops.rms_norm(x, w, 1e-5, fp8=True)
    oq, osc = OF.quantize_rows(y.cpu())
    assert torch.equal(q8.float().cpu(), oq) and torch.allclose(sc.cpu(), osc.flatten())


@pytest.mark.parametrize("aligned", [True, False])
def test_sigmoid_gate(cuda, aligned):
    """o *= sigmoid(gate) in place (fused.py:64-66), the gate read from a per-head [q | gate] layout
    (strided rows and heads); the 16-byte path and, for an unaligned gate view, the scalar path."""
    g = torch.Generator(device=cuda).manual_seed(7)
    n, h, d = 777, 16, 256
    proj = torch.randn(n, h, 2 * d + (0 if aligned else 1), device=cuda, generator=g).bfloat16()
    gate = proj[:, :, d:2 * d] if aligned else proj[:, :, d + 1:2 * d + 1]
    o = torch.randn(n, h * d, device=cuda, generator=g).bfloat16()
    ref = (o.float() * torch.sigmoid(gate.reshape(n, h * d).float())).bfloat16()
    ops.sigmoid_gate_(o, gate, d)
    diff = (o.float() - ref.float()).abs()
    assert (diff <= ref.float().abs() * 2.0 ** -7 + 1e-30).all()
    assert (diff == 0).float().mean().item() > 0.99


@pytest.mark.parametrize("dv", [128, 256, 64])
def test_gated_rms_norm(cuda, dv):
    """y = bf16(bf16(w * bf16(x * rsqrt(mean(x^2) + eps))) * silu(z)) per (row, head) (fused.py:51-56):
    dv 128 / 256 take the vector kernel, 64 the per-element one; z is a strided view."""
    g = torch.Generator(device=cuda).manual_seed(dv)
    n, h = 1001, 8
    x = torch.randn(n, h * dv, device=cuda, generator=g).bfloat16()
    zbuf = torch.randn(n, 2 * h * dv, device=cuda, generator=g).bfloat16()
    z = zbuf[:, h * dv:]
    w = (1 + 0.1 * torch.randn(dv, device=cuda, generator=g)).bfloat16()
    y = torch.empty_like(x)
    _lib.call("dan_gated_rms_norm", _lib.ptr(x), x.stride(0), _lib.ptr(z), z.stride(0), _lib.ptr(w), 1e-6,
              _lib.ptr(y), y.stride(0), n, h, dv, _lib.stream())
    xf = x.float().view(n, h, dv)
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)
    t = (w.float() * (xf * inv).bfloat16().float()).bfloat16().float()
    zf = z.float().reshape(n, h, dv)
    ref = (t * zf * torch.sigmoid(zf)).bfloat16().view(n, h * dv)
    diff = (y.float() - ref.float()).abs()
    assert (diff <= ref.float().abs() * 2.0 ** -6 + 1e-30).all()
    assert (diff == 0).float().mean().item() > 0.98
