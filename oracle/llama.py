"""Llama-family packed prefill, restated in fp32 on the CPU (test infrastructure only).

Follows dan/models/llama.py of the reference:
- RoPE inverse frequencies incl. "linear" and "llama3" scaling (llama.py:18-40),
  angles in fp32 from integer positions, rotate-half (llama.py:43-45, 155-158);
- pre-norm layer: x + attn(rms_norm(x)), then x + mlp(rms_norm(x)) (llama.py:115-117);
- RMSNorm: normalise in fp32, then scale by the weight (fused.py:35-40);
- attention: q/k/v projections, optional per-head q/k RMSNorm for qwen3
  (llama.py:75-87), tree attention (oracle.attention), o projection;
- MLP: down(silu(gate(x)) * up(x)) (llama.py:100-103, fused.py:59-61);
- final norm, then label logits ``W_lm[label_ids] @ h`` in fp32 (llama.py:161-165).

``state`` is a Hugging Face style fp32 state dict (oracle.weights).
"""
import math

import torch
import torch.nn.functional as F

from . import attention


def inv_frequencies(config, head_dim):
    """llama.py:18-40: default / linear / llama3 scaled inverse frequencies (fp32)."""
    params = config.get("rope_parameters") or config.get("rope_scaling") or {}
    theta = float(params.get("rope_theta") or config.get("rope_theta") or 10000.0)
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
    raise NotImplementedError(kind)


def rms_norm(x, w, eps):
    """fused.py:35-40 in fp32."""
    x = x.float()
    return w.float() * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def rotate(x, cos, sin):
    """Rotate-half RoPE (llama.py:43-45); x [..., D], cos/sin broadcastable [.., D]."""
    a, b = x.chunk(2, dim=-1)
    return x * cos + torch.cat((-b, a), dim=-1) * sin


def rope_tables(positions, inv_freq):
    """cos/sin [N, D] from integer positions (llama.py:155-158)."""
    ang = positions.float()[:, None] * inv_freq[None, :]
    ang = torch.cat((ang, ang), dim=-1)
    return ang.cos(), ang.sin()


def head_dim(config):
    return config.get("head_dim") or config["hidden_size"] // config["num_attention_heads"]


def rounding(bf16):
    """The model dtype's rounding of a tensor's values: to bf16 (kept in fp32 storage) when the
    reference runs in bf16 (``Runner(dtype=torch.bfloat16)``), none in fp32."""
    if bf16:
        return lambda t: t.bfloat16().float()
    return lambda t: t


def _linear(state, name, x, fp8, bf16=False):
    """x @ W^T in fp32, or the FP8 restatement (oracle.fp8) with per-output-row weight scales and
    per-token activation scales (dan/quant.py:26-42) when ``fp8``. With ``bf16`` the weight is
    the model's bf16 copy, x holds bf16 values and the result is rounded to bf16, as
    nn.Linear / torch._scaled_mm(out_dtype=bf16) return it (fp32 accumulation)."""
    rd = rounding(bf16)
    w = rd(state[name].float())
    bias = state.get(name[:-len("weight")] + "bias")  # qwen2's q/k/v, attention_bias (llama.py:62-66)
    b = 0.0 if bias is None else rd(bias.float())    # added in the fp32 accumulation, one rounding
    if not fp8:
        return rd(x @ w.T + b)
    from . import fp8 as F8

    wq, ws = F8.quantize_rows(w)
    return rd(F8.linear(x, wq, ws.flatten()) + b)


def norm(x, w, eps, bf16):
    """fused.py:35-40 at the model dtype's rounding points: normalise in fp32, cast to the model
    dtype, then the weight product in that dtype."""
    if not bf16:
        return rms_norm(x, w, eps)
    rd = rounding(True)
    y = x.float()
    y = rd(y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + eps))
    return rd(rd(w.float()) * y)


def rotate_rounded(x, cos, sin, bf16):
    """llama.py:43-45 at the model dtype's rounding points (each product and the sum rounded)."""
    if not bf16:
        return rotate(x, cos, sin)
    rd = rounding(True)
    a, b = x.chunk(2, dim=-1)
    return rd(rd(x * cos) + rd(torch.cat((-b, a), dim=-1) * sin))


def hidden(state, config, ids, positions, segments, fp8=False, bf16=False, p_bf16=False):
    """Final-normed hidden states [N, hidden] of a packed batch.

    ``segments``: list of dicts ``{"start", "end", "branch", "past": {layer: (k, v)} or None,
    "save": int}``; for segments with ``save`` the first ``save`` new tokens' (k, v) per
    layer are stored into ``s["saved"]`` (attention.py:202-204).

    ``bf16``: the reference's bf16 path (``Runner(dtype=torch.bfloat16)``, the dtype its GPU
    path and its FP8 linears run in): weights, cos / sin and every activation rounded to bf16
    where the reference's modules return them (embedding, norms, each linear, RoPE products and
    sums, attention output, SiLU and its product, residual sums); matmuls accumulate in fp32.
    ``p_bf16``: attention probabilities rounded to bf16 before the PV product
    (``attention.attend``)."""
    c = config
    eps = c["rms_norm_eps"]
    rd = rounding(bf16)
    d = head_dim(c)
    nh, nkv = c["num_attention_heads"], c["num_key_value_heads"]
    inv = inv_frequencies(c, d)
    cos, sin = rope_tables(torch.as_tensor(positions), inv)
    cos, sin = rd(cos), rd(sin)
    x = rd(state["model.embed_tokens.weight"][torch.as_tensor(ids)].float())
    n = x.shape[0]
    for s in segments:
        s["saved"] = {}
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}."
        h = norm(x, state[p + "input_layernorm.weight"], eps, bf16)
        q = _linear(state, p + "self_attn.q_proj.weight", h, fp8, bf16).reshape(n, nh, d)
        k = _linear(state, p + "self_attn.k_proj.weight", h, fp8, bf16).reshape(n, nkv, d)
        v = _linear(state, p + "self_attn.v_proj.weight", h, fp8, bf16).reshape(n, nkv, d)
        if c["model_type"] == "qwen3":
            q = norm(q, state[p + "self_attn.q_norm.weight"], eps, bf16)
            k = norm(k, state[p + "self_attn.k_norm.weight"], eps, bf16)
        q = rotate_rounded(q, cos[:, None], sin[:, None], bf16).transpose(0, 1)
        k = rotate_rounded(k, cos[:, None], sin[:, None], bf16).transpose(0, 1)
        v = v.transpose(0, 1)
        segs = []
        for s in segments:
            past = s["past"][i] if s.get("past") else None
            if s.get("save"):
                a = s["start"]
                s["saved"][i] = (k[:, a:a + s["save"]].clone(), v[:, a:a + s["save"]].clone())
            segs.append({"start": s["start"], "end": s["end"], "branch": s["branch"], "past": past})
        o = rd(attention.attend(q, k, v, segs, p_bf16=p_bf16))
        o = o.transpose(0, 1).reshape(n, nh * d)
        x = rd(x + _linear(state, p + "self_attn.o_proj.weight", o, fp8, bf16))
        h = norm(x, state[p + "post_attention_layernorm.weight"], eps, bf16)
        g = _linear(state, p + "mlp.gate_proj.weight", h, fp8, bf16)
        u = _linear(state, p + "mlp.up_proj.weight", h, fp8, bf16)
        x = rd(x + _linear(state, p + "mlp.down_proj.weight", rd(rd(F.silu(g)) * u), fp8, bf16))
    return norm(x, state["model.norm.weight"], eps, bf16)


def lm_head(state):
    return state.get("lm_head.weight", state["model.embed_tokens.weight"])


def label_logits(state, h_row, label_ids, bf16=False):
    """llama.py:163-165: fp32 logits of ``label_ids`` for one hidden row (the head in the model
    dtype, the product in fp32)."""
    return rounding(bf16)(lm_head(state)[torch.as_tensor(label_ids)].float()) @ h_row.float()
