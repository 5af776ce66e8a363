"""Small standalone kernel cases for profiling (``ncu``) and quick timing.

    python bench_cases.py gemm|attention|deltanet|norm [--iters N]

Each case builds seeded inputs with the shapes of a benchmark configuration,
runs the kernel ``--iters`` times (4 by default) and prints one JSON line with
the mean CUDA-event time per launch (the first launch is a warm-up). Inputs
are larger than L2 where the configuration's are.

- gemm: the four Llama-3-8B decoder projections of one <=8192-token batch
  (M = 7089 tokens): q/k/v + RoPE epilogue, o + residual, gate/up + SwiGLU,
  down + residual.
- attention: tree attention of one configuration-2 batch (32/8 heads x 128).
- attention256: the same kernel family at 16/4 heads x 256 on a configuration-4 batch.
- deltanet: causal conv + gated delta scan of one configuration-4 batch
  (Qwen3.5-4B-style: 16 key / 32 value heads x 128); deltanet_whole: the same with the scan
  launched unsplit.
- norm: RMSNorm of [7089, 4096].
- gemm8: the four projections in e4m3 at M = 3400 (configuration 5).
- readout, gate, gnorm, conv, quant, kvstore: the HBM-bound kernels at benchmark sizes.
"""
import argparse
import json

import torch

from dan_b200 import _lib, ops, synthetic
from dan_b200.attention import TreeLayout, tree_attention
from dan_b200.plan import Branch, ReadPlan  # noqa: F401  (re-exported for callers building cases)


def _time(fn, iters):
    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters - 1):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / max(iters - 1, 1)


def _pack(cfg, seed):
    from dan_b200.runner import Runner

    r = Runner.__new__(Runner)
    r.device, r.cache = torch.device("cuda"), None
    return r.pack(synthetic.batch(cfg, seed=seed, vocab=1000), use_cache=False)


def gemm(iters):
    dev = torch.device("cuda")
    m = 7089
    g = torch.Generator(device=dev).manual_seed(0)
    out = {}
    pos = torch.arange(m, device=dev)
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, dtype=torch.float32, device=dev) / 128))
    table = ops.rope_table(pos, inv)
    for name, n, k in (("qkv_rope", 6144, 4096), ("o_residual", 4096, 4096), ("gate_up_swiglu", 28672, 4096),
                       ("down_residual", 4096, 14336)):
        x = torch.randn(m, k, device=dev, generator=g).bfloat16()
        w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
        r = torch.randn(m, n, device=dev, generator=g).bfloat16()
        fn = {"qkv_rope": lambda: ops.linear_rope(x, w, table, 5120, 128),
              "o_residual": lambda: ops.linear(x, w, residual=r),
              "gate_up_swiglu": lambda: ops.linear_swiglu(x, w),
              "down_residual": lambda: ops.linear(x, w, residual=r)}[name]
        ms = _time(fn, iters)
        out[name] = {"m": m, "n": n, "k": k, "ms": ms, "tflops": 2 * m * n * k / ms / 1e9}
    return out


def attention(iters):
    dev = torch.device("cuda")
    ids, pos, segs, reads, _ = _pack(2, 0)
    n = len(ids)
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(n, 32, 128, device=dev, generator=g).bfloat16()
    k = torch.randn(n, 8, 128, device=dev, generator=g).bfloat16()
    v = torch.randn(n, 8, 128, device=dev, generator=g).bfloat16()
    lay = TreeLayout.build(segs, n, dev)
    ms = _time(lambda: tree_attention(q, k, v, lay), iters)
    return {"tokens": n, "useful_pairs": lay.pairs, "tiles": lay.n_tiles, "ms": ms,
            "tflops": 4 * 32 * 128 * lay.pairs / ms / 1e9}


def attention256(iters):
    """Tree attention at the Qwen3.5-4B gated-attention heads (16 / 4 x 256, the single-head
    kernel) on one configuration-4 batch."""
    dev = torch.device("cuda")
    ids, pos, segs, reads, _ = _pack(4, 0)
    n = len(ids)
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(n, 16, 256, device=dev, generator=g).bfloat16()
    k = torch.randn(n, 4, 256, device=dev, generator=g).bfloat16()
    v = torch.randn(n, 4, 256, device=dev, generator=g).bfloat16()
    lay = TreeLayout.build(segs, n, dev)
    ms = _time(lambda: tree_attention(q, k, v, lay), iters)
    return {"tokens": n, "useful_pairs": lay.pairs, "tiles": lay.n_tiles, "ms": ms,
            "tflops": 4 * 16 * 256 * lay.pairs / ms / 1e9}


def deltanet(iters, split=True):
    from dan_b200.qwen3_5 import RecurrentLayout

    dev = torch.device("cuda")
    ids, pos, segs, reads, _ = _pack(4, 0)
    n = len(ids)
    hk, hv, dk, dv = 16, 32, 128, 128
    C = 2 * hk * dk + hv * dv
    g = torch.Generator(device=dev).manual_seed(0)
    pre = (torch.randn(n, C, device=dev, generator=g) * 0.5).bfloat16()
    ba = torch.randn(n, 2 * hv, device=dev, generator=g).bfloat16()
    w = (torch.randn(C, 4, device=dev, generator=g) * 0.5).bfloat16()
    a_log = torch.log(1 + 15 * torch.rand(hv, device=dev, generator=g))
    dt = 0.5 + 0.5 * torch.rand(hv, device=dev, generator=g)
    rl = RecurrentLayout.build(segs, n, 3, dev)
    lead = rl.choose_lead(hv) if split else (0, 0)
    conv = torch.empty(n, C, dtype=torch.bfloat16, device=dev)
    out = torch.empty(n, hv * dv, dtype=torch.bfloat16, device=dev)
    kd = hk * dk
    scratch = _lib.delta_scratch(rl.n_chunks, hk, hv, dev)

    def run():
        _lib.call("dan_causal_conv", _lib.ptr(pre), C, None, 0, _lib.ptr(w), _lib.ptr(rl.prev), _lib.ptr(conv), C, n,
                  C, _lib.stream())
        _lib.call("dan_gated_delta_scan", _lib.ptr(conv[:, :kd]), _lib.ptr(conv[:, kd:2 * kd]),
                  _lib.ptr(conv[:, 2 * kd:]), C, _lib.ptr(ba[:, :hv]), _lib.ptr(ba[:, hv:]), 2 * hv,
                  _lib.ptr(a_log), _lib.ptr(dt), _lib.ptr(rl.segs), rl.n_segs, _lib.ptr(rl.branches),
                  _lib.ptr(rl.chunks), rl.n_chunks, None, 0, _lib.ptr(out), hv * dv, hk, hv, dk, dv,
                  float(dk ** -0.5), _lib.ptr(scratch), scratch.numel(), *lead, _lib.ptr(_lib.status_word(dev)),
                  _lib.stream())

    ms = _time(run, iters)
    return {"tokens": n, "segments": rl.n_segs, "chunks": rl.n_chunks, "lead": list(lead), "ms": ms}


def deltanet_whole(iters):
    """The deltanet case with the scan launched unsplit (both kernels over everything)."""
    return deltanet(iters, split=False)


def fp8peak(iters):
    """Library FP8 reference point: torch._scaled_mm (cuBLASLt) e4m3 8192^3 with row-wise scales,
    best of ``iters`` back-to-back launches (burst) — the FP8 roofline denominator."""
    dev = torch.device("cuda")
    n = 8192
    a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    sa = torch.ones(n, 1, device=dev)
    sb = torch.ones(1, n, device=dev)
    best = min(_time(lambda: torch._scaled_mm(a, b.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16), 4)
               for _ in range(max(iters, 3)))
    xq, xs = ops.quantize_e4m3(torch.randn(n, n, device=dev).bfloat16())
    wq, ws = ops.quantize_e4m3(torch.randn(n, n, device=dev).bfloat16())
    ours = min(_time(lambda: ops.linear_e4m3(xq, xs, wq, ws), 4) for _ in range(max(iters, 3)))
    return {"scaled_mm_tflops": 2 * n ** 3 / best / 1e9, "ours_tflops": 2 * n ** 3 / ours / 1e9}


def norm(iters):
    """RMSNorm shapes of the benchmark configurations, graph-timed: the Llama-3-8B hidden norm
    (4096), the Qwen3.5-4B hidden norm (2560, zero-centred) and its per-head q / k norms (16 heads
    x 256 in place on a strided q/k/v buffer)."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    out = {}
    for name, n, cols, zc in (("hidden_4096", 7089, 4096, False), ("hidden_2560", 7189, 2560, True)):
        x = torch.randn(n, cols, device=dev, generator=g).bfloat16()
        w = (0.1 * torch.randn(cols, device=dev, generator=g)).bfloat16()
        y = torch.empty_like(x)
        ms = _graph_time(lambda x=x, w=w, y=y, zc=zc: ops.rms_norm(x, w, 1e-6, zero_centered=zc, out=y),
                         n=max(iters, 2) * 5)
        out[name] = {"us": 1000 * ms, "gbs": 2 * x.numel() * 2 / ms / 1e6}
    n, heads, d = 7189, 16, 256
    qkv = torch.randn(n, (heads + 2 * 4) * d * 2, device=dev, generator=g).bfloat16()
    q = qkv[:, :heads * d * 2].view(n, heads, 2 * d)[:, :, :d]  # q interleaved with its gate (head stride 2 D)
    w = (0.1 * torch.randn(d, device=dev, generator=g)).bfloat16()
    ms = _graph_time(lambda: ops.rms_norm(q, w, 1e-6, zero_centered=True, out=q), n=max(iters, 2) * 5)
    out["per_head_q_16x256"] = {"us": 1000 * ms, "gbs": 2 * n * heads * d * 2 / ms / 1e6}
    return out


def _graph_time(fn, n=20, reps=5):
    """Device time of one ``fn`` call in ms, from ``reps`` replays of a CUDA graph holding ``n``
    calls (for kernels shorter than the host's per-launch overhead; ``fn`` must not allocate)."""
    fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(n):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        graph.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / (n * reps)


def conv(iters):
    """Causal conv + SiLU of configuration-4 batches (8192 channels: q, k, v of 16 / 16 / 32
    heads x 128), graph-timed, three seeded batches."""
    from dan_b200.qwen3_5 import RecurrentLayout

    dev = torch.device("cuda")
    out = {}
    for seed in (0, 1, 2):
        ids, pos, segs, reads, _ = _pack(4, seed)
        n, c = len(ids), 8192
        g = torch.Generator(device=dev).manual_seed(0)
        pre = (torch.randn(n, c, device=dev, generator=g) * 0.5).bfloat16()
        w = (torch.randn(c, 4, device=dev, generator=g) * 0.5).bfloat16()
        rl = RecurrentLayout.build(segs, n, 3, dev)
        y = torch.empty(n, c, dtype=torch.bfloat16, device=dev)
        fn = (lambda pre=pre, w=w, rl=rl, y=y, n=n: _lib.call(
            "dan_causal_conv", _lib.ptr(pre), c, None, 0, _lib.ptr(w), _lib.ptr(rl.prev), _lib.ptr(y), c, n, c,
            _lib.stream()))
        ms = _graph_time(fn, n=max(iters, 2) * 5)
        out[f"batch{seed}"] = {"rows": n, "us": 1000 * ms, "gbs": 2 * n * c * 2 / ms / 1e6}
    return out


def gnorm(iters):
    """Gated RMSNorm of a configuration-4 batch (7189 rows x 32 value heads x 128), graph-timed."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    n, hv, dv = 7189, 32, 128
    x = torch.randn(n, hv * dv, device=dev, generator=g).bfloat16()
    zz = torch.randn(n, 2 * hv * dv, device=dev, generator=g).bfloat16()  # gate z strided inside a wider row
    z = zz[:, hv * dv:]
    w = (1 + 0.1 * torch.randn(dv, device=dev, generator=g)).bfloat16()
    y = torch.empty(n, hv * dv, dtype=torch.bfloat16, device=dev)
    fn = lambda: _lib.call("dan_gated_rms_norm", _lib.ptr(x), hv * dv, _lib.ptr(z), zz.stride(0), _lib.ptr(w), 1e-6,
                           _lib.ptr(y), hv * dv, n, hv, dv, _lib.stream())
    ms = _graph_time(fn, n=max(iters, 2) * 5)
    fn()
    torch.cuda.synchronize()
    return {"rows": n, "us": 1000 * ms, "gbs": 3 * n * hv * dv * 2 / ms / 1e6, "sum": float(y.float().sum())}


def readout(iters):
    """Fused label readout (final norm of each question's read row, label logits against a
    Llama-3-sized vocabulary, softmax), graph-timed: 48 questions with 2-26 labels (configuration
    3) and with 2-255 labels (configuration 5)."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    hidden, vocab, n = 4096, 128256, 7089
    h = torch.randn(n, hidden, device=dev, generator=g).bfloat16()
    nw = (1 + 0.1 * torch.randn(hidden, device=dev, generator=g)).bfloat16()
    wlm = (0.02 * torch.randn(vocab, hidden, device=dev, generator=g)).bfloat16()
    out = {}
    for name, kmax in (("labels_2_26", 26), ("labels_2_255", 255)):
        counts = torch.randint(2, kmax + 1, (48,), generator=torch.Generator().manual_seed(kmax))
        off = torch.zeros(49, dtype=torch.int32)
        off[1:] = torch.cumsum(counts, 0)
        ids = torch.randint(0, vocab, (int(off[-1]),), dtype=torch.int32, device=dev, generator=g)
        rows = torch.randint(0, n, (48,), dtype=torch.int32, device=dev, generator=g)
        offd = off.to(dev)
        ms = _graph_time(lambda rows=rows, ids=ids, offd=offd, kmax=kmax: ops.label_readout(
            h, rows, nw, 1e-5, False, wlm, ids, offd, kmax), n=max(iters, 2) * 5)
        out[name] = {"labels": int(off[-1]), "us": 1000 * ms, "label_gbs": int(off[-1]) * hidden * 2 / ms / 1e6}
    return out


def gate(iters):
    """Sigmoid output gate of the Qwen3.5-4B gated attention (7189 rows x 16 heads x 256, the
    gate interleaved in the q/k/v projection at head stride 512), graph-timed."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    n, heads, d = 7189, 16, 256
    o = torch.randn(n, heads * d, device=dev, generator=g).bfloat16()
    qg = torch.randn(n, heads * 2 * d, device=dev, generator=g).bfloat16()
    gate = qg[:, d:]  # head h's gate at columns [2 d h + d, 2 d h + 2 d)
    fn = lambda: _lib.call("dan_sigmoid_gate", _lib.ptr(o), o.stride(0), _lib.ptr(gate), qg.stride(0), 2 * d, d, n,
                           heads * d, _lib.stream())
    ms = _graph_time(fn, n=max(iters, 2) * 5)
    return {"us": 1000 * ms, "gbs": 3 * n * heads * d * 2 / ms / 1e6}


def quant(iters):
    """Per-row e4m3 quantisation at configuration-5 sizes (3400 rows: the attention output,
    4096 columns, and the SwiGLU output, 14336) and the e4m3-fused RMSNorm, graph-timed."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    cases = []
    for name, m, k in (("quant_4096", 3400, 4096), ("quant_14336", 3400, 14336), ("norm_e4m3_4096", 3400, 4096)):
        x = torch.randn(m, k, device=dev, generator=g).bfloat16()
        w = (1 + 0.1 * torch.randn(k, device=dev, generator=g)).bfloat16()
        q = torch.empty(m, k, dtype=torch.float8_e4m3fn, device=dev)
        sc = torch.empty(m, dtype=torch.float32, device=dev)
        if name.startswith("quant"):
            fn = (lambda x=x, q=q, sc=sc: ops.quantize_e4m3(x, out=q, scale=sc))
        else:
            fn = (lambda x=x, w=w, q=q, sc=sc, m=m, k=k: _lib.call(
                "dan_rms_norm", _lib.ptr(x), x.stride(0), x.stride(0), 1, _lib.ptr(w), 1e-5, 0, None, 0, 0,
                _lib.ptr(q), q.stride(0), _lib.ptr(sc), m, k, _lib.stream()))
        cases.append((name, m, k, fn))
    for _, _, _, fn in cases:  # one plain launch of each first (the launches a profiler picks up)
        fn()
    out = {}
    for name, m, k, fn in cases:
        ms = _graph_time(fn, n=max(iters, 2) * 5)
        hbm = m * k * 3 + m * 4  # bf16 in, e4m3 out, scales
        out[name] = {"rows": m, "cols": k, "us": 1000 * ms, "gbs": hbm / ms / 1e6}
    return out


def gemm8(iters):
    """The four Llama-3-8B decoder projections in e4m3 at configuration 5's batch size (M = 3400
    new tokens): q/k/v + RoPE, o + residual, gate/up + SwiGLU, down + residual, CUDA-event timed."""
    dev = torch.device("cuda")
    m = 3400
    g = torch.Generator(device=dev).manual_seed(0)
    pos = torch.arange(m, device=dev)
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, dtype=torch.float32, device=dev) / 128))
    table = ops.rope_table(pos, inv)
    out = {}
    for name, n, k in (("qkv_rope", 6144, 4096), ("o_residual", 4096, 4096), ("gate_up_swiglu", 28672, 4096),
                       ("down_residual", 4096, 14336)):
        xq, xs = ops.quantize_e4m3(torch.randn(m, k, device=dev, generator=g).bfloat16())
        wq, ws = ops.quantize_e4m3((torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16())
        r = torch.randn(m, n, device=dev, generator=g).bfloat16()
        fn = {"qkv_rope": lambda: ops.linear_e4m3_rope(xq, xs, wq, ws, table, 5120, 128),
              "o_residual": lambda: ops.linear_e4m3(xq, xs, wq, ws, residual=r),
              "gate_up_swiglu": lambda: ops.linear_e4m3(xq, xs, wq, ws, swiglu=True),
              "down_residual": lambda: ops.linear_e4m3(xq, xs, wq, ws, residual=r)}[name]
        ms = _time(fn, iters)
        out[name] = {"m": m, "n": n, "k": k, "ms": ms, "tflops": 2 * m * n * k / ms / 1e12 * 1e3}
    return out


def kvstore(iters):
    """Prefix K/V page stores of one configuration-5 save: 1024 rows of 8 kv heads x 128 (k and v,
    read in place from the fused q/k/v projection at row stride 6144) into pool pages, graph-timed."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    n, hkv, d = 1024, 8, 128
    qkv = torch.randn(n, 6144, device=dev, generator=g).bfloat16()
    k = qkv[:, 4096:5120].view(n, hkv, d)
    v = qkv[:, 5120:].view(n, hkv, d)
    pool_k = torch.zeros(64 * 128, hkv, d, dtype=torch.bfloat16, device=dev)
    pool_v = torch.zeros_like(pool_k)
    src = torch.arange(n, dtype=torch.int32, device=dev)
    dst = torch.randperm(64 * 128, device=dev, generator=g)[:n].to(torch.int32)
    ms = _graph_time(lambda: ops.kv_store(k, v, pool_k, pool_v, src, dst), n=max(iters, 2) * 5)
    return {"rows": n, "us": 1000 * ms, "gbs": 2 * 2 * n * hkv * d * 2 / ms / 1e6}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "gemm8", "attention", "attention256", "deltanet", "deltanet_whole", "conv", "gnorm", "norm", "quant", "readout",
                                     "gate", "kvstore", "fp8peak"])
    ap.add_argument("--iters", type=int, default=4)
    a = ap.parse_args()
    res = globals()[a.case](max(a.iters, 2))
    _lib.check_status(torch.device("cuda"))
    print(json.dumps({a.case: res}))


if __name__ == "__main__":
    main()
