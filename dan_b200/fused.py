"""dan's element-wise functions (dan/fused.py:35-101) under their own names and signatures, on
the dan_b200 kernels.

dan's model code calls these on its activations; in dan they are torch.compile'd on CUDA and
eager elsewhere. Here each is one kernel launch on the current stream, with dan's rounding
points, for bf16 tensors on a B200 (``ValueError`` for anything else: there is no CPU path).
The model path in this package fuses most of them into neighbouring kernels (norms into the
FP8 quantiser, SwiGLU and RoPE into GEMM epilogues, the gates into the DeltaNet scan, and the
tree-attention kernel needs no LSE merge); these stand-alone forms are for callers of dan's
functions.
"""
import torch

from . import _lib, ops

E4M3 = torch.float8_e4m3fn


def _bf16_cuda(name, *ts):
    for t in ts:
        if not (t.is_cuda and t.dtype == torch.bfloat16):
            raise ValueError(f"{name}: dan_b200 runs bf16 CUDA tensors only (got {t.dtype} on {t.device})")


def _rows(x):
    """[..., C] -> a 2-D [R, C] view with unit column stride (copies only when needed)."""
    x2 = x.reshape(-1, x.shape[-1])
    return x2 if x2.stride(-1) == 1 else x2.contiguous()


def rms_norm(x, weight, eps):
    """Llama-style RMSNorm: normalise in fp32, cast, then scale (fused.py:35-40)."""
    _bf16_cuda("rms_norm", x, weight)
    return ops.rms_norm(_rows(x), weight, eps).reshape(x.shape)


def rms_norm_zero_centered(x, weight, eps):
    """Qwen3.5-style RMSNorm with the weight applied as (1 + w) in fp32 (fused.py:43-48)."""
    _bf16_cuda("rms_norm_zero_centered", x, weight)
    return ops.rms_norm(_rows(x), weight, eps, zero_centered=True).reshape(x.shape)


def gated_rms_norm(x, gate, weight, eps):
    """RMSNorm over the last dim of x, scaled by w, times silu(gate) (fused.py:51-56)."""
    _bf16_cuda("gated_rms_norm", x, gate, weight)
    x2, g2 = _rows(x), _rows(gate)
    y = torch.empty(x2.shape, dtype=torch.bfloat16, device=x.device)
    _lib.call("dan_gated_rms_norm", _lib.ptr(x2), x2.stride(0), _lib.ptr(g2), g2.stride(0), _lib.ptr(weight),
              float(eps), _lib.ptr(y), y.stride(0), x2.shape[0], 1, x2.shape[1], _lib.stream())
    return y.reshape(x.shape)


def swiglu(gate, up):
    """silu(gate) * up (fused.py:59-61)."""
    _bf16_cuda("swiglu", gate, up)
    g2, u2 = _rows(gate), _rows(up)
    y = torch.empty(g2.shape, dtype=torch.bfloat16, device=gate.device)
    _lib.call("dan_swiglu", _lib.ptr(g2), g2.stride(0), _lib.ptr(u2), u2.stride(0), _lib.ptr(y), y.stride(0),
              g2.shape[0], g2.shape[1], _lib.stream())
    return y.reshape(gate.shape)


def sigmoid_gate(x, gate):
    """x * sigmoid(gate) (fused.py:64-66)."""
    _bf16_cuda("sigmoid_gate", x, gate)
    y = _rows(x).clone()
    g2 = _rows(gate)
    ops.sigmoid_gate_(y, g2.view(g2.shape[0], 1, g2.shape[1]), g2.shape[1])
    return y.reshape(x.shape)


def rotate_partial(x, cos, sin):
    """Rotate-half RoPE on the first ``cos.shape[-1]`` dims of each head; x [N, H, D], cos/sin
    [N, R] in the model dtype with equal halves, as dan builds them (fused.py:69-76)."""
    _bf16_cuda("rotate_partial", x, cos, sin)
    n, h, d = x.shape
    r = cos.shape[-1]
    half = r // 2
    if not (torch.equal(cos[:, :half], cos[:, half:]) and torch.equal(sin[:, :half], sin[:, half:])):
        raise ValueError("rotate_partial: cos/sin halves differ (dan builds them as cat((ang, ang)))")
    y = x.contiguous().clone()
    table = (cos[:, :half].float().contiguous(), sin[:, :half].float().contiguous())
    return ops.rope_(y, table, rot=r)


def delta_gates(b, a, a_log, dt_bias):
    """Gated DeltaNet write strength beta = sigmoid(b) (b's dtype) and log decay
    g = -exp(A_log) * softplus(a + dt_bias) (fp32) (fused.py:79-82). b, a: [..., H]."""
    _bf16_cuda("delta_gates", b, a)
    b2, a2 = _rows(b), _rows(a)
    rows, heads = b2.shape
    beta = torch.empty(rows, heads, dtype=torch.bfloat16, device=b.device)
    g = torch.empty(rows, heads, dtype=torch.float32, device=b.device)
    al, dtb = a_log.float().contiguous(), dt_bias.float().contiguous()  # held until the launch
    _lib.call("dan_delta_gates", _lib.ptr(b2), b2.stride(0), _lib.ptr(a2), a2.stride(0), _lib.ptr(al),
              _lib.ptr(dtb), _lib.ptr(beta), beta.stride(0), _lib.ptr(g), g.stride(0), rows, heads, _lib.stream())
    return beta.reshape(b.shape), g.reshape(b.shape)


def fp8_quantize(x, fp8_max, rowwise: bool):
    """(e4m3 codes of x / scale, fp32 scale [R, 1] per row or [1, 1] for the tensor), scale =
    max(amax, 1e-12) / fp8_max (fused.py:85-91). fp8_max is e4m3's 448."""
    _bf16_cuda("fp8_quantize", x)
    if float(fp8_max) != 448.0:
        raise ValueError(f"fp8_quantize: e4m3 only (fp8_max 448, got {fp8_max})")
    x2 = _rows(x)
    if rowwise:
        q, s = ops.quantize_e4m3(x2)
        return q, s[:, None]
    rows, cols = x2.shape
    q = torch.empty(rows, cols, dtype=E4M3, device=x.device)
    s = torch.empty(1, 1, dtype=torch.float32, device=x.device)
    _lib.call("dan_quantize_e4m3_tensor", _lib.ptr(x2), x2.stride(0), _lib.ptr(q), q.stride(0), _lib.ptr(s), rows,
              cols, _lib.stream())
    return q, s


def lse_merge(o_a, lse_a, o_b, lse_b):
    """Attention over the union of two disjoint key sets from each part's output and
    log-sum-exp; o: [T, H, D], lse: [H, T] (fused.py:94-101)."""
    _bf16_cuda("lse_merge", o_a, o_b)
    t, h, d = o_a.shape
    oa, ob = o_a.contiguous(), o_b.contiguous()
    la, lb = lse_a.float().contiguous(), lse_b.float().contiguous()  # held until the launch
    out = torch.empty_like(oa)
    _lib.call("dan_lse_merge", _lib.ptr(oa), _lib.ptr(la), _lib.ptr(ob), _lib.ptr(lb), _lib.ptr(out), h * d, t, h,
              d, _lib.stream())
    return out
