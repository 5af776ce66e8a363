"""Model registry and loading (dan/models/__init__.py:13-43).

``load(path)`` reads a Hugging Face model directory (``config.json`` +
``*.safetensors``), picks the architecture by ``model_type`` and builds it on
the GPU. ``random_model(config, seed)`` builds the same architecture from
seeded N(0, std) weights generated directly on the GPU (benchmarks; no
checkpoint download is possible offline).
"""
import glob
import json
import math
import os

import torch


def arch_for(config):
    from .llama import LlamaForReads
    from .qwen3_5 import Qwen35ForReads

    for cls in (LlamaForReads, Qwen35ForReads):
        if config["model_type"] in cls.MODEL_TYPES:
            return cls
    raise NotImplementedError(f"model type {config['model_type']!r} is not supported yet")


def read_config(path):
    with open(os.path.join(path, "config.json")) as f:
        c = json.load(f)
    return c.get("text_config", c) if c.get("model_type") == "qwen3_5" else c


def read_state(path):
    from safetensors.torch import load_file

    state = {}
    for f in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
        state.update(load_file(f))
    return state


def broadcast_state(state, device, src=0, group=None, bucket_bytes=256 << 20):
    """Send a state dict from rank ``src`` to every rank of ``group`` (NCCL over NVLink for
    CUDA devices, gloo for CPU): names, shapes and dtypes first, then the tensors packed into
    byte buckets of about ``bucket_bytes``, one broadcast per bucket. Ranks other than ``src``
    pass ``state=None``; every rank returns the full state on ``device``."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    meta = [[(k, tuple(v.shape), str(v.dtype).replace("torch.", "")) for k, v in state.items()]] if rank == src else [None]
    dist.broadcast_object_list(meta, src=src, group=group)
    out = {}
    bucket = []

    def flush():
        if not bucket:
            return
        nbytes = sum(n for _, _, _, n in bucket)
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        if rank == src:
            off = 0
            for k, _, _, n in bucket:
                buf[off:off + n].copy_(state[k].contiguous().view(-1).view(torch.uint8))
                off += n
        dist.broadcast(buf, src=src, group=group)
        off = 0
        for k, shape, dt, n in bucket:
            out[k] = buf[off:off + n].view(dt).view(shape).clone()
            off += n
        bucket.clear()

    total = 0
    for k, shape, dname in meta[0]:
        dt = getattr(torch, dname)
        n = math.prod(shape) * torch.empty(0, dtype=dt).element_size()
        bucket.append((k, shape, dt, n))
        total += n
        if total >= bucket_bytes:
            flush()
            total = 0
    flush()
    return out


def load(name, device="cuda", dtype=torch.bfloat16, quantization=None, group=None):
    """Build the model of a local Hugging Face directory on ``device``. With a process group of
    several ranks, only rank 0 reads the checkpoint; the others receive it by broadcast."""
    if not isinstance(name, str):
        return name  # an already-built model
    if group is not None:
        import torch.distributed as dist

        rank = dist.get_rank(group)
        config = [read_config(name) if rank == 0 else None]
        dist.broadcast_object_list(config, src=0, group=group)
        state = broadcast_state(read_state(name) if rank == 0 else None, device, group=group)
        return arch_for(config[0])(config[0], state, device, dtype, quantization)
    if not os.path.isdir(name):
        raise FileNotFoundError(f"{name!r} is not a local model directory (no network access)")
    config = read_config(name)
    return arch_for(config)(config, read_state(name), device, dtype, quantization)


def _shapes(config):
    # Parameter shapes by Hugging Face name, for random initialisation.
    c = config
    out = []
    if c["model_type"].startswith("qwen3_5"):
        pre = "model.language_model."
        h, d = c["hidden_size"], c["head_dim"]
        hk, hv, dk, dv = (c["linear_num_key_heads"], c["linear_num_value_heads"], c["linear_key_head_dim"],
                          c["linear_value_head_dim"])
        conv_dim = 2 * hk * dk + hv * dv
        out.append((pre + "embed_tokens.weight", (c["vocab_size"], h), "w"))
        for i, kind in enumerate(c["layer_types"]):
            p = f"{pre}layers.{i}."
            out.append((p + "input_layernorm.weight", (h,), "n0"))
            if kind == "linear_attention":
                a = p + "linear_attn."
                out += [(a + "in_proj_qkv.weight", (conv_dim, h), "w"), (a + "in_proj_z.weight", (hv * dv, h), "w"),
                        (a + "in_proj_b.weight", (hv, h), "w"), (a + "in_proj_a.weight", (hv, h), "w"),
                        (a + "conv1d.weight", (conv_dim, 1, c["linear_conv_kernel_dim"]), "conv"),
                        (a + "dt_bias", (hv,), "dt"), (a + "A_log", (hv,), "alog"), (a + "norm.weight", (dv,), "n1"),
                        (a + "out_proj.weight", (h, hv * dv), "w")]
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
    else:
        h = c["hidden_size"]
        d = c.get("head_dim") or h // c["num_attention_heads"]
        out.append(("model.embed_tokens.weight", (c["vocab_size"], h), "w"))
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
        out.append(("model.norm.weight", (h,), "n1"))
    if not c.get("tie_word_embeddings"):
        out.append(("lm_head.weight", (c["vocab_size"], c["hidden_size"]), "w"))
    return out


def random_weights(config, seed=0, std=0.02, device="cuda"):
    """Seeded random bf16 weights generated on ``device``: linears / embeddings N(0, std),
    norm weights near their identity value, DeltaNet gate parameters in their usual ranges."""
    gen = torch.Generator(device=device).manual_seed(seed)
    state = {}
    for name, shape, kind in _shapes(config):
        if kind == "w":
            t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std
        elif kind == "n1":
            t = 1.0 + 0.1 * torch.randn(shape, generator=gen, device=device)
        elif kind == "n0":
            t = 0.1 * torch.randn(shape, generator=gen, device=device)
        elif kind == "conv":
            t = torch.randn(shape, generator=gen, device=device) / math.sqrt(shape[-1])
        elif kind == "dt":
            t = 0.5 + 0.5 * torch.rand(shape, generator=gen, device=device)
        else:
            t = torch.log(1.0 + 15.0 * torch.rand(shape, generator=gen, device=device))
        state[name] = t.to(torch.bfloat16) if kind not in ("dt", "alog") else t
    return state


def random_model(config, seed=0, device="cuda", quantization=None, std=0.02):
    state = random_weights(config, seed, std, device)
    model = arch_for(config)(config, state, device, torch.bfloat16, quantization)
    del state
    return model


def llama3_8b_config():
    """Llama-3-8B architecture (benchmark configurations 3 and 5)."""
    return {"model_type": "llama", "vocab_size": 128256, "hidden_size": 4096, "intermediate_size": 14336,
            "num_hidden_layers": 32, "num_attention_heads": 32, "num_key_value_heads": 8, "head_dim": 128,
            "rope_theta": 500000.0, "rms_norm_eps": 1e-5, "tie_word_embeddings": False,
            "rope_scaling": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                             "original_max_position_embeddings": 8192}}


def qwen35_4b_config():
    """Qwen3.5-4B-style hybrid (benchmark configuration 4): 32 layers, 3 Gated DeltaNet : 1
    gated attention, hidden 2560. Unstated fields use Qwen3_5TextConfig defaults; the MLP
    intermediate size is chosen as 9216."""
    return {"model_type": "qwen3_5_text", "vocab_size": 151936, "hidden_size": 2560, "intermediate_size": 9216,
            "num_hidden_layers": 32, "num_attention_heads": 16, "num_key_value_heads": 4, "head_dim": 256,
            "linear_num_key_heads": 16, "linear_num_value_heads": 32, "linear_key_head_dim": 128,
            "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4,
            "layer_types": ["full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(32)],
            "rms_norm_eps": 1e-6, "tie_word_embeddings": False,
            "rope_parameters": {"rope_theta": 10000.0, "partial_rotary_factor": 0.25, "rope_type": "default"}}
