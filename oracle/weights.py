"""Deterministic random checkpoints for parity tests (test infrastructure).

A checkpoint is a Hugging Face style state dict (parameter name -> fp32 CPU
tensor) plus a config dict. Each tensor is drawn from its own CPU generator,
seeded from the global seed and the tensor's index in a fixed name order, so
the same (config, seed) gives bit-identical weights on any machine with the
same torch build. Linear and embedding weights are N(0, std); Llama RMSNorm
weights are 1 + N(0, 0.1); Qwen3.5 zero-centred norm weights are N(0, 0.1).
"""
import json
import math
import os

import torch


ARCHITECTURES = {"llama": "LlamaForCausalLM", "mistral": "MistralForCausalLM", "qwen2": "Qwen2ForCausalLM",
                 "qwen3": "Qwen3ForCausalLM"}


def llama_config(vocab=49152, hidden=576, inter=1536, layers=30, heads=9, kv_heads=3, head_dim=64,
                 theta=10000.0, tie=True, rope_scaling=None, model_type="llama", eps=1e-5):
    """A Llama-family config dict in transformers' field names (``model_type`` llama, mistral,
    qwen2: q/k/v projections with bias, or qwen3: per-head q/k RMSNorm)."""
    c = {"model_type": model_type, "architectures": [ARCHITECTURES[model_type]], "vocab_size": vocab,
         "hidden_size": hidden, "intermediate_size": inter, "num_hidden_layers": layers,
         "num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": head_dim,
         "rope_theta": theta, "rms_norm_eps": eps, "tie_word_embeddings": tie, "max_position_embeddings": 131072,
         "hidden_act": "silu", "attention_bias": False, "mlp_bias": False, "torch_dtype": "float32"}
    if rope_scaling:
        c["rope_scaling"] = rope_scaling
    return c


def qwen35_config(vocab=1024, hidden=128, inter=256, layers=4, heads=4, kv_heads=2, head_dim=64,
                  lin_k_heads=2, lin_v_heads=4, lin_k_dim=32, lin_v_dim=32, conv=4, partial=0.25,
                  theta=10000.0, tie=False, eps=1e-6, full_every=4):
    """A Qwen3.5 text config dict: ``full_every - 1`` Gated DeltaNet layers, then one attention layer."""
    types = ["full_attention" if (i + 1) % full_every == 0 else "linear_attention" for i in range(layers)]
    return {"model_type": "qwen3_5_text", "architectures": ["Qwen3_5ForCausalLM"], "vocab_size": vocab,
            "hidden_size": hidden, "intermediate_size": inter, "num_hidden_layers": layers,
            "num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": head_dim,
            "linear_num_key_heads": lin_k_heads, "linear_num_value_heads": lin_v_heads,
            "linear_key_head_dim": lin_k_dim, "linear_value_head_dim": lin_v_dim,
            "linear_conv_kernel_dim": conv, "layer_types": types, "rms_norm_eps": eps,
            "rope_parameters": {"rope_theta": theta, "partial_rotary_factor": partial, "rope_type": "default"},
            "tie_word_embeddings": tie, "attention_bias": False, "hidden_act": "silu",
            "max_position_embeddings": 32768, "torch_dtype": "float32"}


def _shapes_llama(c):
    h, d = c["hidden_size"], c["head_dim"]
    out = [("model.embed_tokens.weight", (c["vocab_size"], h), "w")]
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}."
        out += [(p + "input_layernorm.weight", (h,), "n1"),
                (p + "self_attn.q_proj.weight", (c["num_attention_heads"] * d, h), "w"),
                (p + "self_attn.k_proj.weight", (c["num_key_value_heads"] * d, h), "w"),
                (p + "self_attn.v_proj.weight", (c["num_key_value_heads"] * d, h), "w"),
                (p + "self_attn.o_proj.weight", (h, c["num_attention_heads"] * d), "w"),
                (p + "post_attention_layernorm.weight", (h,), "n1"),
                (p + "mlp.gate_proj.weight", (c["intermediate_size"], h), "w"),
                (p + "mlp.up_proj.weight", (c["intermediate_size"], h), "w"),
                (p + "mlp.down_proj.weight", (h, c["intermediate_size"]), "w")]
        if c["model_type"] == "qwen3":
            out += [(p + "self_attn.q_norm.weight", (d,), "n1"), (p + "self_attn.k_norm.weight", (d,), "n1")]
        if c["model_type"] == "qwen2" or c.get("attention_bias"):  # q/k/v bias (llama.py:62-65)
            out += [(p + "self_attn.q_proj.bias", (c["num_attention_heads"] * d,), "n0"),
                    (p + "self_attn.k_proj.bias", (c["num_key_value_heads"] * d,), "n0"),
                    (p + "self_attn.v_proj.bias", (c["num_key_value_heads"] * d,), "n0")]
        if c.get("attention_bias"):
            out.append((p + "self_attn.o_proj.bias", (h,), "n0"))
    out.append(("model.norm.weight", (h,), "n1"))
    if not c.get("tie_word_embeddings"):
        out.append(("lm_head.weight", (c["vocab_size"], h), "w"))
    return out


def _shapes_qwen35(c):
    h, d = c["hidden_size"], c["head_dim"]
    hk, hv, dk, dv = (c["linear_num_key_heads"], c["linear_num_value_heads"], c["linear_key_head_dim"],
                      c["linear_value_head_dim"])
    conv_dim = 2 * hk * dk + hv * dv
    pre = "model.language_model."
    out = [(pre + "embed_tokens.weight", (c["vocab_size"], h), "w")]
    for i, kind in enumerate(c["layer_types"]):
        p = f"{pre}layers.{i}."
        out.append((p + "input_layernorm.weight", (h,), "n0"))
        if kind == "linear_attention":
            a = p + "linear_attn."
            out += [(a + "in_proj_qkv.weight", (conv_dim, h), "w"), (a + "in_proj_z.weight", (hv * dv, h), "w"),
                    (a + "in_proj_b.weight", (hv, h), "w"), (a + "in_proj_a.weight", (hv, h), "w"),
                    (a + "conv1d.weight", (conv_dim, 1, c["linear_conv_kernel_dim"]), "conv"),
                    (a + "dt_bias", (hv,), "dt"), (a + "A_log", (hv,), "alog"),
                    (a + "norm.weight", (dv,), "n1"), (a + "out_proj.weight", (h, hv * dv), "w")]
        else:
            a = p + "self_attn."
            out += [(a + "q_proj.weight", (c["num_attention_heads"] * d * 2, h), "w"),
                    (a + "k_proj.weight", (c["num_key_value_heads"] * d, h), "w"),
                    (a + "v_proj.weight", (c["num_key_value_heads"] * d, h), "w"),
                    (a + "o_proj.weight", (h, c["num_attention_heads"] * d), "w"),
                    (a + "q_norm.weight", (d,), "n0"), (a + "k_norm.weight", (d,), "n0")]
        out += [(p + "post_attention_layernorm.weight", (h,), "n0"),
                (p + "mlp.gate_proj.weight", (c["intermediate_size"], h), "w"),
                (p + "mlp.up_proj.weight", (c["intermediate_size"], h), "w"),
                (p + "mlp.down_proj.weight", (h, c["intermediate_size"]), "w")]
    out.append((pre + "norm.weight", (h,), "n0"))
    if not c.get("tie_word_embeddings"):
        out.append(("lm_head.weight", (c["vocab_size"], h), "w"))
    return out


def shapes(config):
    """(name, shape, kind) of every parameter, in the fixed generation order."""
    return _shapes_qwen35(config) if config["model_type"].startswith("qwen3_5") else _shapes_llama(config)


def draw(kind, shape, gen, std):
    if kind == "w":
        return torch.randn(shape, generator=gen) * std
    if kind == "n1":
        return 1.0 + 0.1 * torch.randn(shape, generator=gen)
    if kind == "n0":
        return 0.1 * torch.randn(shape, generator=gen)
    if kind == "conv":
        return torch.randn(shape, generator=gen) / math.sqrt(shape[-1])
    if kind == "dt":
        return 0.5 + 0.5 * torch.rand(shape, generator=gen)
    if kind == "alog":
        return torch.log(1.0 + 15.0 * torch.rand(shape, generator=gen))
    raise ValueError(kind)


def random_state(config, seed=0, std=0.02):
    """Seeded fp32 state dict for ``config`` (Hugging Face parameter names)."""
    state = {}
    for i, (name, shape, kind) in enumerate(shapes(config)):
        gen = torch.Generator().manual_seed(seed * 1_000_003 + i)
        state[name] = draw(kind, shape, gen, std).contiguous()
    return state


def save_checkpoint(path, config, state):
    """Write ``config.json`` + ``model.safetensors`` (a Hugging Face model directory)."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config, f, indent=1)
    save_file({k: v.contiguous() for k, v in state.items()}, os.path.join(path, "model.safetensors"))
