"""Thin wrappers over the CUDA kernels, named after the reference operations
they replace (dan/fused.py:35-101, dan/quant.py:23-42, nn.Linear).

Every function takes torch tensors already on the GPU and launches on the
current stream; none has a CPU path.
"""
import torch

from . import _lib

STORE, RESIDUAL, SWIGLU, ROPE = 0, 1, 2, 3


def _st(t):
    return _lib.ptr(_lib.status_word(t.device))


def linear(x, w, bias=None, residual=None, out=None):
    """bf16 ``x @ w.T`` (+ bias) [(+ residual), in place when ``out is residual``] (nn.Linear)."""
    m, k = x.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device) if residual is None else residual
    ep = RESIDUAL if residual is not None else STORE
    _lib.call("dan_gemm_bf16", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(out), out.stride(0),
              _lib.ptr(residual), residual.stride(0) if residual is not None else 0, _lib.ptr(bias), m, n, k, ep,
              _st(x), _lib.stream(), work=2 * m * n * k, key=f"gemm_bf16 n={n} k={k} ep={ep}")
    return out


def linear_swiglu(x, w_gate_up, bias=None, out=None):
    """``silu(x @ Wg.T) * (x @ Wu.T)`` in one GEMM; ``w_gate_up`` rows interleave 128-row
    blocks of gate and up (``interleave_gate_up``) (fused.py:59-61 on llama.py:100-103)."""
    m, k = x.shape
    n = w_gate_up.shape[0]
    if out is None:
        out = torch.empty(m, n // 2, dtype=torch.bfloat16, device=x.device)
    _lib.call("dan_gemm_bf16", _lib.ptr(x), x.stride(0), _lib.ptr(w_gate_up), w_gate_up.stride(0), _lib.ptr(out),
              out.stride(0), None, 0, _lib.ptr(bias), m, n, k, SWIGLU, _st(x), _lib.stream(), work=2 * m * n * k,
              key=f"gemm_bf16 n={n} k={k} ep=swiglu")
    return out


def interleave_gate_up(gate, up, block=128):
    """[I, K] gate and up -> [2I, K] with rows [g_0:128, u_0:128, g_128:256, ...] (I % 128 == 0)."""
    i, k = gate.shape
    if i % block:
        raise ValueError(f"intermediate size {i} is not a multiple of {block}")
    return torch.stack([gate.reshape(i // block, block, k), up.reshape(i // block, block, k)], 1).reshape(2 * i, k)


def quantize_e4m3(x, out=None, scale=None):
    """Per-row e4m3 quantisation: scale = max(amax, 1e-12)/448, q = e4m3(x/scale) (fused.py:85-91)."""
    m, k = x.shape
    if out is None:
        out = torch.empty(m, k, dtype=torch.float8_e4m3fn, device=x.device)
    if scale is None:
        scale = torch.empty(m, dtype=torch.float32, device=x.device)
    _lib.call("dan_quantize_e4m3", _lib.ptr(x), x.stride(0), _lib.ptr(out), out.stride(0), _lib.ptr(scale), m, k,
              _lib.stream())
    return out, scale


def linear_e4m3(xq, x_scale, wq, w_scale, bias=None, residual=None, swiglu=False, out=None):
    """FP8 linear with per-token and per-output-channel scales, bf16 result (quant.py:37-42)."""
    m, k = xq.shape
    n = wq.shape[0]
    ep = SWIGLU if swiglu else (RESIDUAL if residual is not None else STORE)
    if out is None:
        if residual is not None:
            out = residual
        else:
            out = torch.empty(m, n // 2 if swiglu else n, dtype=torch.bfloat16, device=xq.device)
    _lib.call("dan_gemm_e4m3", _lib.ptr(xq), xq.stride(0), _lib.ptr(x_scale), _lib.ptr(wq), wq.stride(0),
              _lib.ptr(w_scale), _lib.ptr(out), out.stride(0), _lib.ptr(residual),
              residual.stride(0) if residual is not None else 0, _lib.ptr(bias), m, n, k, ep, _st(xq), _lib.stream(),
              work=2 * m * n * k, key=f"gemm_e4m3 n={n} k={k} ep={ep}")
    return out


def rms_norm(x, weight, eps, zero_centered=False, out=None, fp8=False):
    """Row RMSNorm over the last dim of a 2-D [rows, cols] or 3-D [n, heads, cols] view
    (Llama: fused.py:35-40; zero-centred: fused.py:43-48). With ``fp8`` also returns the
    e4m3 quantisation of the result and its per-row scales (only for 2-D)."""
    if x.dim() == 2:
        x3 = x[:, None, :]
    else:
        x3 = x
    n, inner, cols = x3.shape
    if out is None and not fp8:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    o3 = None if out is None else (out[:, None, :] if out.dim() == 2 else out)
    q8 = sc = None
    if fp8:
        q8 = torch.empty(n * inner, cols, dtype=torch.float8_e4m3fn, device=x.device)
        sc = torch.empty(n * inner, dtype=torch.float32, device=x.device)
    _lib.call("dan_rms_norm", _lib.ptr(x3), x3.stride(0), x3.stride(1), inner, _lib.ptr(weight), float(eps),
              1 if zero_centered else 0, _lib.ptr(o3), o3.stride(0) if o3 is not None else 0,
              o3.stride(1) if o3 is not None else 0, _lib.ptr(q8), cols, _lib.ptr(sc), n * inner, cols, _lib.stream(),
              work=n * inner * cols * (2 + (2 if o3 is not None else 0) + (1 if fp8 else 0)) + cols * 2)
    if fp8:
        return out, q8, sc
    return out


def rope_table(positions, inv_freq):
    """(cos, sin) fp32 [N, R/2]: angles from integer positions in fp32, rounded to bf16 as the
    reference casts them to the model dtype (llama.py:155-158). Built once per forward."""
    n, half = positions.shape[0], inv_freq.shape[0]
    cos = torch.empty(n, half, dtype=torch.float32, device=positions.device)
    sin = torch.empty_like(cos)
    _lib.call("dan_rope_table", _lib.ptr(positions), _lib.ptr(inv_freq), n, half, _lib.ptr(cos), _lib.ptr(sin),
              _lib.stream())
    return cos, sin


def rope_(x, table, rot=None):
    """In-place rotate-half RoPE on the first ``rot`` dims of each head; x: [N, heads, D]
    view, ``table`` from ``rope_table`` (llama.py:43-45 / fused.py:69-76)."""
    n, heads, d = x.shape
    rot = d if rot is None else rot
    cos, sin = table
    _lib.call("dan_rope", _lib.ptr(x), x.stride(0), x.stride(1), heads, d, rot, _lib.ptr(cos), _lib.ptr(sin), n,
              _lib.stream(), work=n * heads * rot * 4)
    return x


def linear_rope(x, w, table, rope_cols, head_dim, bias=None, out=None):
    """bf16 ``x @ w.T`` (+ bias) with RoPE applied in the epilogue to every ``head_dim`` head
    of the first ``rope_cols`` output columns (the fused q/k/v projection + rotary)."""
    m, k = x.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    cos, sin = table
    _lib.call("dan_gemm_bf16_rope", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(out), out.stride(0),
              None, 0, _lib.ptr(bias), m, n, k, ROPE, rope_cols, head_dim, _lib.ptr(cos), _lib.ptr(sin), _st(x),
              _lib.stream(), work=2 * m * n * k, key=f"gemm_bf16 n={n} k={k} ep=rope")
    return out


def linear_e4m3_rope(xq, x_scale, wq, w_scale, table, rope_cols, head_dim, bias=None, out=None):
    """FP8 ``linear_rope``: per-token / per-channel scaled e4m3 GEMM with RoPE in the epilogue."""
    m, k = xq.shape
    n = wq.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=xq.device)
    cos, sin = table
    _lib.call("dan_gemm_e4m3_rope", _lib.ptr(xq), xq.stride(0), _lib.ptr(x_scale), _lib.ptr(wq), wq.stride(0),
              _lib.ptr(w_scale), _lib.ptr(out), out.stride(0), None, 0, _lib.ptr(bias), m, n, k, ROPE, rope_cols,
              head_dim, _lib.ptr(cos), _lib.ptr(sin), _st(xq), _lib.stream(), work=2 * m * n * k,
              key=f"gemm_e4m3 n={n} k={k} ep=rope")
    return out


def embed(ids, table, out=None):
    n, (vocab, hidden) = ids.shape[0], table.shape
    if out is None:
        out = torch.empty(n, hidden, dtype=table.dtype, device=table.device)
    _lib.call("dan_embed", _lib.ptr(ids), _lib.ptr(table), table.stride(0), vocab, _lib.ptr(out), out.stride(0), n,
              hidden, _st(table), _lib.stream())
    return out


def sigmoid_gate_(o, gate, head_dim):
    """o *= sigmoid(gate) in place (fused.py:64-66); gate: [N, heads, head_dim] view."""
    n, cols = o.shape
    _lib.call("dan_sigmoid_gate", _lib.ptr(o), o.stride(0), _lib.ptr(gate), gate.stride(0), gate.stride(1), head_dim,
              n, cols, _lib.stream())
    return o


def kv_store(k, v, pool_k, pool_v, src_rows, dst_rows):
    """Copy rows ``src_rows`` of k/v [N, Hkv, D] into pool rows ``dst_rows`` (prefix saves)."""
    _lib.call("dan_kv_store", _lib.ptr(k), _lib.ptr(v), k.stride(0), k.stride(1), _lib.ptr(pool_k), _lib.ptr(pool_v),
              pool_k.stride(0), pool_k.stride(1), _lib.ptr(src_rows), _lib.ptr(dst_rows), src_rows.numel(),
              k.shape[1], k.shape[2], _lib.stream())


NORM_LLAMA, NORM_ZERO_CENTERED, NORM_NONE = 0, 1, 2


def label_readout(h, read_rows, norm_w, eps, norm_mode, w_lm, label_ids, offsets, max_labels):
    """Per question: final norm of its read row (``norm_mode``: Llama, zero-centred, or none for
    rows already normed), ``W_lm[labels] @ h`` in fp32 and the softmax (llama.py:161-165,
    runner.py:73-74, readout.py:13-17). Returns (logits, probs), flat fp32."""
    nq = read_rows.numel()
    total = label_ids.numel()
    logits = torch.empty(total, dtype=torch.float32, device=h.device)
    probs = torch.empty(total, dtype=torch.float32, device=h.device)
    _lib.call("dan_label_readout", _lib.ptr(h), h.stride(0), _lib.ptr(read_rows), _lib.ptr(norm_w), float(eps),
              int(norm_mode), _lib.ptr(w_lm), w_lm.stride(0), w_lm.shape[0], _lib.ptr(label_ids),
              _lib.ptr(offsets), nq, h.shape[1], max_labels, _lib.ptr(logits), _lib.ptr(probs), _st(h),
              _lib.stream())
    return logits, probs
