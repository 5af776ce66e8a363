"""FP8 (e4m3) decoder linears, restated on the CPU (test infrastructure only).

Follows the reference's FP8 path:
- weight quantisation once per linear, one scale per output row:
  ``scale = max(amax(|W[j, :]|), 1e-12) / 448``, ``Wq = (W / scale).to(e4m3)``
  (dan/quant.py:26-33);
- activation quantisation per token (row): ``scale = max(amax(|x|), 1e-12) / 448``,
  ``xq = (x / scale).to(e4m3)`` (dan/fused.py:85-91);
- ``y = (xq @ Wq^T) * scale_x[:, None] * scale_w[None, :]`` (+ bias) in fp32, cast to
  the model dtype (``torch._scaled_mm`` with row-wise scales, dan/quant.py:37-42).

Pinning: the reference's FP8 path needs a CUDA GPU and its tests hold no FP8
case, so no CPU fixture exists; on the GPU box ``tests/test_gpu_model.py`` runs
the reference's own FP8 path (its offline install) and checks this restatement
against it at the 3e-2 probability bound.
"""
import torch

E4M3 = torch.float8_e4m3fn
E4M3_MAX = 448.0


def quantize_rows(x):
    """Per-row e4m3 quantisation -> (q as fp32 values of e4m3 codes, scale [rows, 1])."""
    xf = x.float()
    scale = xf.abs().amax(dim=-1, keepdim=True).clamp(min=1e-12) / E4M3_MAX
    return (xf / scale).to(E4M3).float(), scale


def linear(x, w_q, w_scale, bias=None):
    """FP8 linear with per-token and per-output-channel scales, fp32 result."""
    xq, xs = quantize_rows(x)
    y = (xq.double() @ w_q.double().T) * xs.double() * w_scale.double().reshape(1, -1)
    if bias is not None:
        y = y + bias.double()
    return y.float()
