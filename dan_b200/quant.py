"""FP8 (e4m3) decoder linears with dan's interface (dan/quant.py:23-42) on the dan_b200 kernels.

``FP8Linear(linear, rowwise=True)`` quantises ``linear.weight`` once on the GPU (scale per
output row, or one for the tensor) and its ``forward(x)`` quantises the activations on the fly
(per token, or per tensor) and runs the e4m3 GEMM with both scales applied in its epilogue,
bf16 out (dan: ``torch._scaled_mm``). Inside this package's models the activation quantisation
is fused into the preceding RMSNorm instead.
"""
import torch

from . import fused, ops

E4M3 = torch.float8_e4m3fn
E4M3_MAX = 448.0


class FP8Linear:
    def __init__(self, linear, rowwise=True):
        w = linear.weight.detach()
        if not (w.is_cuda and w.dtype == torch.bfloat16):
            raise ValueError("FP8Linear: dan_b200 quantises bf16 CUDA weights")
        self.out_features, self.in_features = w.shape
        self.weight, scale = fused.fp8_quantize(w.contiguous(), E4M3_MAX, rowwise)  # [out, in] e4m3
        self.weight_scale = scale.reshape(1, -1) if rowwise else scale  # [1, out] or [1, 1] (dan's layout)
        self._w_cols = scale.reshape(-1).expand(self.out_features).contiguous()  # per-column scales for the GEMM
        b = getattr(linear, "bias", None)
        self.bias = None if b is None else b.detach().to(torch.bfloat16).contiguous()
        self.rowwise = rowwise
        self.out_dtype = w.dtype

    def forward(self, x):
        shape = x.shape
        xq, scale = fused.fp8_quantize(x.reshape(-1, shape[-1]), E4M3_MAX, self.rowwise)
        a_rows = scale.reshape(-1).expand(xq.shape[0]).contiguous()
        y = ops.linear_e4m3(xq, a_rows, self.weight, self._w_cols, self.bias)
        return y.reshape(*shape[:-1], self.out_features)

    __call__ = forward
