"""Qwen3.5 hybrid (Gated DeltaNet + gated attention) packed prefill, restated in
fp32/fp64 on the CPU (test infrastructure only).

Follows dan/models/qwen3_5.py of the reference:
- zero-centred RMSNorm ``x_hat * (1 + w)`` (qwen3_5.py:77-86, fused.py:43-48);
- gated RMSNorm ``(w * x_hat) * silu(z)`` (fused.py:51-56);
- DeltaNet layer (qwen3_5.py:183-212): qkv/z/b/a projections, gates
  ``beta = sigmoid(b)``, ``g = -exp(A_log) * softplus(a + dt_bias)`` (fused.py:79-82),
  causal depthwise conv (kernel k) + SiLU over ``[history; run]``
  (qwen3_5.py:214-220), GQA head repeat (qwen3_5.py:225), gated delta rule
  with in-kernel q/k l2norm (eps 1e-6) and q scaled by Dk^-0.5
  (qwen3_5.py:99-133);
- tree runs (qwen3_5.py:231-298): each segment's trunk runs from its initial
  state (zeros, or the cached state) after ``k - 1`` history rows (zeros, or
  the cached conv tail); when a prefix is saved the trunk is cut at ``save``;
  every branch runs from the trunk's final state with the last ``k - 1`` rows
  of ``[history; trunk]`` as its conv history;
- gated attention (qwen3_5.py:301-329): q_proj gives per head ``[q | gate]``,
  zero-centred q/k norms, partial RoPE on the first ``D * partial`` dims
  (fused.py:69-76, qwen3_5.py:388-392), tree attention, ``o * sigmoid(gate)``.

The delta rule is computed token by token from its definition
``S_t = a_t S_{t-1} + k_t (beta_t (v_t - a_t S_{t-1}^T k_t))^T``, ``o_t = S_t^T q_t``
with ``a_t = exp(g_t)``, in fp64; the reference computes the same recurrence in
64-token chunks (qwen3_5.py:103-133).
"""
import torch
import torch.nn.functional as F

from . import attention
from .llama import rotate, rounding

PRE = "model.language_model."


def zc_rms_norm(x, w, eps, bf16=False):
    """fused.py:43-48 (the (1 + w) product in fp32, then the model dtype)."""
    x = x.float()
    return rounding(bf16)((x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)) * (1.0 + rounding(bf16)(w.float())))


def gated_rms_norm(x, gate, w, eps, bf16=False):
    """fused.py:51-56: w * x_hat in the model dtype, times silu(gate) in fp32, then the model dtype."""
    rd = rounding(bf16)
    x = x.float()
    y = rd(rd(w.float()) * rd(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)))
    return rd(y * F.silu(gate.float()))


def l2norm(x, eps=1e-6):
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def delta_rule(q, k, v, g, beta, state):
    """One run. q, k: [T, H, Dk]; v: [T, H, Dv]; g, beta: [T, H]; state [H, Dk, Dv].
    Returns (out [T, H, Dv] fp32, final state fp32)."""
    q = l2norm(q.double()) * q.shape[-1] ** -0.5
    k = l2norm(k.double())
    v, g, beta = v.double(), g.double(), beta.double()
    s = state.double().clone()
    out = torch.zeros(v.shape, dtype=torch.float64)
    for t in range(q.shape[0]):
        s = s * g[t].exp()[:, None, None]
        u = beta[t][:, None] * (v[t] - torch.einsum("hkv,hk->hv", s, k[t]))
        s = s + k[t][:, :, None] * u[:, None, :]
        out[t] = torch.einsum("hkv,hk->hv", s, q[t])
    return out.float(), s.float()


def causal_conv_silu(ext, weight, bf16=False):
    """ext: [hist + T, C] rows; weight [C, 1, k]. Row j of the result reads ext[j:j+k] (qwen3_5.py:218-220).
    With ``bf16`` the conv's result and the SiLU's are each rounded to bf16, as F.conv1d and
    F.silu return them in the model dtype."""
    rd = rounding(bf16)
    kk = weight.shape[-1]
    w = rd(weight[:, 0, :].float())
    t = ext.shape[0] - (kk - 1)
    y = torch.stack([(ext[j:j + kk].float() * w.T).sum(0) for j in range(t)]) if t > 0 else ext[:0].float()
    return rd(F.silu(rd(y)))


def inv_frequencies(config):
    rp = config["rope_parameters"]
    dim = int(config["head_dim"] * rp.get("partial_rotary_factor", 1.0))
    return 1.0 / (rp["rope_theta"] ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))


def deltanet(state, c, i, x, segments, bf16=False):
    rd = rounding(bf16)
    p = f"{PRE}layers.{i}.linear_attn."
    hk, hv, dk, dv = (c["linear_num_key_heads"], c["linear_num_value_heads"], c["linear_key_head_dim"],
                      c["linear_value_head_dim"])
    k1 = c["linear_conv_kernel_dim"] - 1
    n = x.shape[0]

    def lin(name):
        return rd(x @ rd(state[p + name].float()).T)

    qkv, z, b, a = lin("in_proj_qkv.weight"), lin("in_proj_z.weight"), lin("in_proj_b.weight"), lin("in_proj_a.weight")
    beta = rd(torch.sigmoid(b))
    g = -state[p + "A_log"].float().exp() * F.softplus(a + state[p + "dt_bias"].float())
    conv_w = state[p + "conv1d.weight"]
    key_dim = hk * dk
    out = torch.zeros(n, hv, dv)

    def run(hist, rows, init):
        ext = torch.cat([hist, qkv[rows]]) if len(rows) else hist
        y = causal_conv_silu(ext, conv_w, bf16)
        qq = y[:, :key_dim].reshape(-1, hk, dk).repeat_interleave(hv // hk, 1)
        kk = y[:, key_dim:2 * key_dim].reshape(-1, hk, dk).repeat_interleave(hv // hk, 1)
        vv = y[:, 2 * key_dim:].reshape(-1, hv, dv)
        o, fin = delta_rule(qq, kk, vv, g[rows], beta[rows], init)
        out[rows] = rd(o)
        return fin, ext

    for s in segments:
        past = s["past"][i] if s.get("past") else None
        hist = past[0].float() if past is not None else torch.zeros(k1, qkv.shape[1])
        init = past[1].float() if past is not None else torch.zeros(hv, dk, dv)
        trunk_rows = list(range(s["start"], s["start"] + s["trunk"]))
        virt = torch.cat([hist, qkv[trunk_rows]])  # [k1 + trunk, C]
        save = s.get("save", 0)
        cut = save if 0 < save < s["trunk"] else s["trunk"]
        fin1, _ = run(virt[:k1], trunk_rows[:cut], init)
        fin = fin1
        if cut < s["trunk"]:
            fin, _ = run(virt[cut:k1 + cut], trunk_rows[cut:], fin1)
        if save:
            s["saved"][i] = (virt[cut:k1 + cut].clone(), fin1.clone())
        for (ba, bb) in s["branches"]:
            run(virt[-k1:], list(range(ba, bb)), fin)
    y = gated_rms_norm(out.reshape(-1, dv), z.reshape(-1, dv), state[p + "norm.weight"], c["rms_norm_eps"], bf16)
    return rd(y.reshape(n, -1) @ rd(state[p + "out_proj.weight"].float()).T)


def gated_attention(state, c, i, x, cos, sin, segments, bf16=False):
    rd = rounding(bf16)
    p = f"{PRE}layers.{i}.self_attn."
    n = x.shape[0]
    h, hkv, d = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
    eps = c["rms_norm_eps"]

    def lin(name, y):
        return rd(y @ rd(state[p + name].float()).T)

    qg = lin("q_proj.weight", x).reshape(n, h, 2 * d)
    q, gate = qg[..., :d], qg[..., d:]
    k = lin("k_proj.weight", x).reshape(n, hkv, d)
    v = lin("v_proj.weight", x).reshape(n, hkv, d)
    q = zc_rms_norm(q, state[p + "q_norm.weight"], eps, bf16)
    k = zc_rms_norm(k, state[p + "k_norm.weight"], eps, bf16)
    r = cos.shape[-1]

    def rot(t):  # rotate_partial (fused.py:69-76): products and sums in the model dtype
        a, b = t[..., :r].chunk(2, dim=-1)
        turned = rd(rd(t[..., :r] * cos[:, None]) + rd(torch.cat((-b, a), dim=-1) * sin[:, None]))
        return torch.cat([turned, t[..., r:]], -1)

    q = rot(q).transpose(0, 1)
    k = rot(k).transpose(0, 1)
    v = v.transpose(0, 1)
    segs = []
    for s in segments:
        if s.get("save"):
            a = s["start"]
            s["saved"][i] = (k[:, a:a + s["save"]].clone(), v[:, a:a + s["save"]].clone())
        segs.append({"start": s["start"], "end": s["end"], "branch": s["branch"],
                     "past": s["past"][i] if s.get("past") else None})
    o = rd(attention.attend(q, k, v, segs)).transpose(0, 1).reshape(n, h * d)
    o = rd(o * rd(torch.sigmoid(gate.reshape(n, h * d))))
    return lin("o_proj.weight", o)


def hidden(state, c, ids, positions, segments, bf16=False):
    """Final-normed hidden states [N, hidden] (qwen3_5.py:410-417). ``bf16``: the reference's
    bf16 path, every module's result rounded to bf16 (see oracle.llama.hidden); the delta
    rule's state stays fp32 there and fp64 here."""
    rd = rounding(bf16)
    eps = c["rms_norm_eps"]
    inv = inv_frequencies(c)
    ang = torch.as_tensor(positions).float()[:, None] * inv[None, :]
    ang = torch.cat((ang, ang), -1)
    cos, sin = rd(ang.cos()), rd(ang.sin())
    x = rd(state[PRE + "embed_tokens.weight"][torch.as_tensor(ids)].float())
    for s in segments:
        s["saved"] = {}
    for i, kind in enumerate(c["layer_types"]):
        p = f"{PRE}layers.{i}."
        h = zc_rms_norm(x, state[p + "input_layernorm.weight"], eps, bf16)
        if kind == "linear_attention":
            h = deltanet(state, c, i, h, segments, bf16)
        else:
            h = gated_attention(state, c, i, h, cos, sin, segments, bf16)
        x = rd(x + h)
        h = zc_rms_norm(x, state[p + "post_attention_layernorm.weight"], eps, bf16)
        g = rd(h @ rd(state[p + "mlp.gate_proj.weight"].float()).T)
        u = rd(h @ rd(state[p + "mlp.up_proj.weight"].float()).T)
        x = rd(x + rd(rd(rd(F.silu(g)) * u) @ rd(state[p + "mlp.down_proj.weight"].float()).T))
    return zc_rms_norm(x, state[PRE + "norm.weight"], eps, bf16)


def lm_head(state):
    return state.get("lm_head.weight", state[PRE + "embed_tokens.weight"])


def label_logits(state, h_row, label_ids, bf16=False):
    return rounding(bf16)(lm_head(state)[torch.as_tensor(label_ids)].float()) @ h_row.float()
