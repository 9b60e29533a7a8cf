"""Writes Hugging Face Qwen3.5 checkpoint folders for the loader tests (no GPU needed).

The tensor names, shapes and dtypes follow a Transformers Qwen3.5 language-model export
(`save_pretrained` of the backbone, as recipe/open_jev/export_merged.py of the reference
does): bf16 everywhere except linear_attn.A_log and linear_attn.norm.weight in fp32,
config.json (here nested under text_config, as in the full-model config), and the
Open-Jev export manifest open_jev_export.json with the scorer head.
"""
import json
import os

import numpy as np
from safetensors.numpy import save_file


def _bf16(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def hf_state(cfg, W, fp32_extra=True):
    """{hf name (no prefix): (numpy array, dtype)}; bf16 tensors as uint16 bit patterns.
    With fp32_extra, the fp32 A_log / norm values carry extra mantissa bits below half a
    bf16 unit, so rounding them to bf16 gives back exactly W's values."""
    out = {"embed_tokens.weight": W["embed"], "norm.weight": W["final_norm"]}
    for i, t in enumerate(cfg.layer_types):
        p, q = f"layers.{i}.", f"l{i}."
        out[p + "input_layernorm.weight"] = W[q + "input_norm"]
        out[p + "post_attention_layernorm.weight"] = W[q + "post_norm"]
        out[p + "mlp.gate_proj.weight"] = W[q + "gate"]
        out[p + "mlp.up_proj.weight"] = W[q + "up"]
        out[p + "mlp.down_proj.weight"] = W[q + "down"]
        if t == "gdn":
            la = p + "linear_attn."
            out[la + "in_proj_qkv.weight"] = W[q + "in_qkv"]
            out[la + "in_proj_z.weight"] = W[q + "in_z"]
            out[la + "in_proj_b.weight"] = W[q + "in_b"]
            out[la + "in_proj_a.weight"] = W[q + "in_a"]
            out[la + "conv1d.weight"] = W[q + "conv"][:, None, :]
            out[la + "A_log"] = W[q + "A_log"]
            out[la + "dt_bias"] = W[q + "dt_bias"]
            out[la + "norm.weight"] = W[q + "norm"]
            out[la + "out_proj.weight"] = W[q + "out"]
        else:
            sa = p + "self_attn."
            for n, m in (("q", "q_proj"), ("k", "k_proj"), ("v", "v_proj"), ("o", "o_proj")):
                out[sa + m + ".weight"] = W[q + n]
            out[sa + "q_norm.weight"] = W[q + "q_norm"]
            out[sa + "k_norm.weight"] = W[q + "k_norm"]
    typed = {}
    for k, v in out.items():
        if k.endswith("linear_attn.A_log") or k.endswith("linear_attn.norm.weight"):
            x = np.asarray(v, np.float32)
            if fp32_extra:
                x = x + x * np.float32(2.0 ** -10)
            typed[k] = (np.ascontiguousarray(x, np.float32), "F32")
        else:
            typed[k] = (_bf16(v), "BF16")
    return typed


def write_checkpoint(folder, cfg, W, prefix="model.language_model.", shards=2, fp32_extra=True):
    """A checkpoint folder: shards of safetensors + index (or one model.safetensors),
    config.json with text_config, and open_jev_export.json with the head."""
    os.makedirs(folder, exist_ok=True)
    state = hf_state(cfg, W, fp32_extra)
    names = sorted(state)
    parts = [names[i::shards] for i in range(shards)] if shards > 1 else [names]
    weight_map = {}
    for s, part in enumerate(parts):
        fname = f"model-{s + 1:05d}-of-{len(parts):05d}.safetensors" if shards > 1 else "model.safetensors"
        tensors = {}
        for n in part:
            arr = state[n][0]
            # safetensors.numpy writes uint16 as U16: the bf16 tag is set in the header below
            tensors[prefix + n] = arr
            weight_map[prefix + n] = fname
        path = os.path.join(folder, fname)
        save_file(tensors, path)
        _retag_bf16(path, {prefix + n for n in part if state[n][1] == "BF16"})
    if shards > 1:
        with open(os.path.join(folder, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {}, "weight_map": weight_map}, f)
    hf_types = ["linear_attention" if t == "gdn" else "full_attention" for t in cfg.layer_types]
    text = {"model_type": "qwen3_5_text", "hidden_size": cfg.hidden, "intermediate_size": cfg.intermediate,
            "num_hidden_layers": len(cfg.layer_types), "layer_types": hf_types,
            "linear_num_key_heads": cfg.lin_k_heads, "linear_num_value_heads": cfg.lin_v_heads,
            "linear_key_head_dim": cfg.lin_k_dim, "linear_value_head_dim": cfg.lin_v_dim,
            "linear_conv_kernel_dim": 4, "num_attention_heads": cfg.heads, "num_key_value_heads": cfg.kv_heads,
            "head_dim": cfg.head_dim, "vocab_size": cfg.vocab, "rms_norm_eps": cfg.eps,
            "rope_parameters": {"rope_type": "default", "rope_theta": cfg.theta, "partial_rotary_factor": 0.25}}
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump({"model_type": "qwen3_5", "text_config": text}, f, indent=1)
    with open(os.path.join(folder, "open_jev_export.json"), "w") as f:
        json.dump({"format": "open-jev-text-merged/1", "temperature": 1.0, "max_length": 16384,
                   "head_weight": np.asarray(W["head_w"], np.float64).tolist(),
                   "head_bias": np.asarray(W["head_b"], np.float64).tolist()}, f)
    return folder


def _retag_bf16(path, names):
    """safetensors.numpy has no bfloat16: rewrite the dtype tag of the uint16 payloads."""
    with open(path, "rb") as f:
        blob = f.read()
    n = int.from_bytes(blob[:8], "little")
    header = json.loads(blob[8:8 + n])
    for k in names:
        header[k]["dtype"] = "BF16"
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * (-len(text) % 8)  # data offsets are relative to the header's end
    with open(path, "wb") as f:
        f.write(len(text).to_bytes(8, "little") + text + blob[8 + n:])
