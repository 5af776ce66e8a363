"""Llama-family decoder (Llama 2/3, Mistral, Qwen2/2.5/3, SmolLM), prefill only,
on the dan_b200 kernels.

Same interface and numerics as the reference's ``LlamaForReads``
(dan/models/llama.py:120-165): ``hidden(ids, positions, segments)`` and
``label_logits(h, label_ids)``, Hugging Face parameter names on load, RoPE with
default / linear / llama3 scaling (llama.py:18-40), pre-norm layers, merged
q/k/v and gate/up projections (llama.py:70-72, 95-96; common.py:6-22).

Per layer on the GPU: RMSNorm -> qkv GEMM -> [q/k RMSNorm] -> RoPE in place ->
prefix K/V page stores -> tree attention (reads q/k/v in place) -> o GEMM with
the residual add fused -> RMSNorm -> gate/up GEMM with SwiGLU fused -> down GEMM
with the residual add fused. With ``quantization="fp8"`` the four decoder
linears run as e4m3 GEMMs with per-token / per-channel scales; the norms emit
the e4m3 activations directly.
"""
import math

import torch

from . import _lib, ops
from .attention import layout_of, tree_attention

E4M3 = torch.float8_e4m3fn


def rope_settings(config):
    params = config.get("rope_parameters") or config.get("rope_scaling") or {}
    theta = params.get("rope_theta") or config.get("rope_theta") or 10000.0
    return float(theta), params


def inv_frequencies(config, head_dim):
    """llama.py:24-40."""
    theta, params = rope_settings(config)
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    kind = params.get("rope_type") or params.get("type") or "default"
    if kind == "default":
        return inv.float()
    if kind == "linear":
        return (inv / params["factor"]).float()
    if kind == "llama3":
        factor, lo, hi = params["factor"], params["low_freq_factor"], params["high_freq_factor"]
        old = params["original_max_position_embeddings"]
        wavelen = 2 * math.pi / inv
        smooth = (old / wavelen - lo) / (hi - lo)
        scaled = torch.where(wavelen > old / lo, inv / factor, inv)
        mid = (wavelen <= old / lo) & (wavelen >= old / hi)
        return torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled).float()
    raise NotImplementedError(f"rope type {kind!r} is not supported yet")


def quantize_weight(w):
    """Per-output-row e4m3 weights (quant.py:26-33) on the GPU: (wq [out, in], scale [out] fp32)."""
    return ops.quantize_e4m3(w.contiguous())


def _label_logits(model, h, label_ids):
    ids = torch.as_tensor(label_ids, dtype=torch.int32).reshape(-1).to(model.device)
    hr = h.reshape(1, -1).to(torch.bfloat16).contiguous()
    zero = torch.zeros(1, dtype=torch.int32, device=model.device)
    off = torch.tensor([0, ids.numel()], dtype=torch.int32, device=model.device)
    logits, _ = ops.label_readout(hr, zero, model.norm, model.eps, ops.NORM_NONE, model.lm_head, ids, off,
                                  max(ids.numel(), 1))
    return logits


class Linear:
    """A decoder projection: bf16 weight, or e4m3 weight + per-row scale."""

    def __init__(self, w, bias=None, fp8=False):
        self.fp8 = fp8
        self.bias = bias
        if fp8:
            self.wq, self.ws = quantize_weight(w)
            self.w = None
        else:
            self.w = w.contiguous()

    @property
    def out_features(self):
        return (self.wq if self.fp8 else self.w).shape[0]


class LlamaForReads:
    MODEL_TYPES = frozenset({"llama", "mistral", "qwen2", "qwen3"})

    def __init__(self, config, state, device="cuda", dtype=torch.bfloat16, quantization=None):
        if dtype != torch.bfloat16:
            raise ValueError("dan_b200 runs the decoder in bf16 (fp8 via quantization='fp8')")
        if quantization not in (None, "fp8"):
            raise ValueError(f"unknown quantization {quantization!r}; use 'fp8'")
        c = self.config = dict(config)
        self.device = torch.device(device)
        self.h, self.hkv = c["num_attention_heads"], c["num_key_value_heads"]
        self.d = c.get("head_dim") or c["hidden_size"] // self.h
        self.hidden_size = c["hidden_size"]
        self.eps = c["rms_norm_eps"]
        self.qk_norm = c["model_type"] == "qwen3"
        self.n_layers = c["num_hidden_layers"]
        self.fp8 = quantization == "fp8"
        qkv_bias = c.get("attention_bias", False) or c["model_type"] == "qwen2"
        o_bias = c.get("attention_bias", False)

        def g(name):
            return state[name].to(self.device, torch.bfloat16)

        self.embed_tokens = g("model.embed_tokens.weight").contiguous()
        self.lm_head = g("lm_head.weight").contiguous() if "lm_head.weight" in state else self.embed_tokens
        self.norm = g("model.norm.weight")
        self.layers = []
        for i in range(self.n_layers):
            p = f"model.layers.{i}."
            a = p + "self_attn."
            qkv = torch.cat([g(a + "q_proj.weight"), g(a + "k_proj.weight"), g(a + "v_proj.weight")])
            bias = None
            if qkv_bias:
                bias = torch.cat([g(a + n + "_proj.bias") if (a + n + "_proj.bias") in state else
                                  torch.zeros(w, dtype=torch.bfloat16, device=self.device)
                                  for n, w in (("q", self.h * self.d), ("k", self.hkv * self.d),
                                               ("v", self.hkv * self.d))])
            gate_up = ops.interleave_gate_up(g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight"))
            layer = {
                "in_norm": g(p + "input_layernorm.weight"),
                "post_norm": g(p + "post_attention_layernorm.weight"),
                "qkv": Linear(qkv, bias, self.fp8),
                "o": Linear(g(a + "o_proj.weight"), g(a + "o_proj.bias") if o_bias else None, self.fp8),
                "gate_up": Linear(gate_up, None, self.fp8),
                "down": Linear(g(p + "mlp.down_proj.weight"), None, self.fp8),
            }
            if self.qk_norm:
                layer["q_norm"], layer["k_norm"] = g(a + "q_norm.weight"), g(a + "k_norm.weight")
            self.layers.append(layer)
        self.inv_freq = inv_frequencies(c, self.d).to(self.device)
        self.pool = None  # the runner attaches a PrefixPool

    @staticmethod
    def frequencies(config):
        d = config.get("head_dim") or config["hidden_size"] // config["num_attention_heads"]
        return inv_frequencies(config, d)

    # ------------------------------------------------------------------ forward
    def _proj(self, lin, x, x8=None, residual=None, swiglu=False):
        if lin.fp8:
            if x8 is None:
                x8 = ops.quantize_e4m3(x)
            return ops.linear_e4m3(x8[0], x8[1], lin.wq, lin.ws, lin.bias, residual=residual, swiglu=swiglu)
        if swiglu:
            return ops.linear_swiglu(x, lin.w, lin.bias)
        return ops.linear(x, lin.w, lin.bias, residual=residual)

    def _proj_rope(self, lin, x, x8, table, rope_cols):
        if lin.fp8:
            return ops.linear_e4m3_rope(x8[0], x8[1], lin.wq, lin.ws, table, rope_cols, self.d, lin.bias)
        return ops.linear_rope(x, lin.w, table, rope_cols, self.d, lin.bias)

    def _norm(self, x, w):
        if self.fp8:
            _, q8, sc = ops.rms_norm(x, w, self.eps, fp8=True)
            return None, (q8, sc)
        return ops.rms_norm(x, w, self.eps), None

    def hidden(self, ids, positions, segments):
        """Final-normed hidden states [N, hidden] bf16 of a packed token sequence
        (llama.py:152-161). The runner reads only the read rows, so it uses ``residual`` and
        lets the readout kernel norm those rows."""
        return ops.rms_norm(self.residual(ids, positions, segments), self.norm, self.eps)

    def residual(self, ids, positions, segments, saves=None):
        """Residual-stream states [N, hidden] after the last layer, before the final norm.

        ``saves``: optional (src_rows, dst_rows) int32 device tensors: after each
        layer's RoPE, those rows' k/v are stored into the prefix pool."""
        n = ids.shape[0]
        x = ops.embed(ids, self.embed_tokens)
        lay = layout_of(segments, n, self.device)
        h, hkv, d = self.h, self.hkv, self.d
        table = ops.rope_table(positions, self.inv_freq)
        for i, L in enumerate(self.layers):
            hn, h8 = self._norm(x, L["in_norm"])
            if self.qk_norm:  # RoPE after the per-head q/k norms (llama.py:82-85)
                qkv = self._proj(L["qkv"], hn, h8)
            else:  # RoPE fused into the projection's epilogue
                qkv = self._proj_rope(L["qkv"], hn, h8, table, (h + hkv) * d)
            q = qkv[:, :h * d].view(n, h, d)
            k = qkv[:, h * d:(h + hkv) * d].view(n, hkv, d)
            v = qkv[:, (h + hkv) * d:].view(n, hkv, d)
            if self.qk_norm:
                ops.rms_norm(q, L["q_norm"], self.eps, out=q)
                ops.rms_norm(k, L["k_norm"], self.eps, out=k)
                ops.rope_(qkv[:, :(h + hkv) * d].view(n, h + hkv, d), table)
            if saves is not None and self.pool is not None:
                ops.kv_store(k, v, self.pool.k[i], self.pool.v[i], saves[0], saves[1])
            ao = torch.empty(n, h * d, dtype=torch.bfloat16, device=self.device)
            tree_attention(q, k, v, lay, out=ao.view(n, h, d), pool=self.pool, layer=i)
            self._proj(L["o"], ao, residual=x)
            hn, h8 = self._norm(x, L["post_norm"])
            act = self._proj(L["gate_up"], hn, h8, swiglu=True)
            self._proj(L["down"], act, residual=x)
        return x

    def readout(self, x, read_rows, label_ids, offsets, max_labels):
        """Final norm of the read rows, label logits in fp32 and per-question softmax."""
        return ops.label_readout(x, read_rows, self.norm, self.eps, ops.NORM_LLAMA, self.lm_head, label_ids, offsets,
                                 max_labels)

    def label_logits(self, h, label_ids):
        """fp32 logits of just ``label_ids`` for one final-normed hidden state h [hidden]
        (llama.py:163-165), by the readout kernel with its norm off."""
        return _label_logits(self, h, label_ids)

    def kv_layout(self):
        """(layers, kv heads, head dim) the prefix pool must hold for this model."""
        return self.n_layers, self.hkv, self.d

    def launches_per_forward(self):
        """Kernels one forward launches (embed, rope table, per layer, readout), excluding prefix saves."""
        per = 7 + (3 if self.qk_norm else 0) + (2 if self.fp8 else 0)
        return 2 + per * self.n_layers + 1

    def linear_params(self):
        """Parameters of the decoder linears (for FLOP accounting: 2 per token each)."""
        c = self.config
        hd, i = self.hidden_size, c["intermediate_size"]
        per = hd * (self.h + 2 * self.hkv) * self.d + self.h * self.d * hd + 3 * hd * i
        return per * self.n_layers
