"""Checkpoint reading of the C++ host, without a GPU (src/models/qwen3_5/native/src/model.rs
:96-226 and :267-397 of the reference are the loader it replaces).

* config.json (nested text_config or flat; layer_types or full_attention_interval;
  rope_parameters) -> the model configuration;
* the safetensors tensor listing: HF names under each accepted prefix mapped to this
  host's parameter names, shapes and dtypes read from sharded and single-file folders;
* the checks made before any payload is read: every weight present, shapes, fp32 only
  for A_log / the GDN norm, payload sizes;
* a folder written by Transformers' own save_pretrained passes the same checks.
"""
import json
import os

import numpy as np
import pytest

from oracle import model as OM

from hf_checkpoint import hf_state, write_checkpoint


@pytest.fixture(scope="module")
def tiny_folder(tmp_path_factory):
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    folder = tmp_path_factory.mktemp("ckpt")
    write_checkpoint(str(folder), cfg, W)
    return cfg, W, str(folder)


def _s1cfg(cfg, labels=1):
    from s1omni import Config
    return Config(cfg.hidden, cfg.intermediate, list(cfg.layer_types), cfg.lin_k_heads, cfg.lin_v_heads, cfg.heads,
                  cfg.kv_heads, cfg.vocab, labels=labels)


def test_config_from_nested_text_config(tiny_folder):
    from s1omni import config_from_hf
    cfg, _, folder = tiny_folder
    c = config_from_hf(os.path.join(folder, "config.json"))
    assert (c.hidden, c.intermediate, c.vocab) == (cfg.hidden, cfg.intermediate, cfg.vocab)
    assert c.layer_types == cfg.layer_types
    assert (c.lin_k_heads, c.lin_v_heads, c.heads, c.kv_heads) == (cfg.lin_k_heads, cfg.lin_v_heads, cfg.heads,
                                                                   cfg.kv_heads)
    assert (c.lin_k_dim, c.lin_v_dim, c.head_dim) == (128, 128, 256)
    assert c.rotary_half == 32 and c.theta == cfg.theta and abs(c.eps - cfg.eps) < 1e-12
    assert c.labels == 1


def test_config_flat_interval_and_defaults(tmp_path):
    from s1omni import config_from_hf
    flat = {"hidden_size": 4096, "intermediate_size": 12288, "num_hidden_layers": 8, "linear_num_key_heads": 16,
            "linear_num_value_heads": 32, "num_attention_heads": 16, "num_key_value_heads": 4,
            "vocab_size": 151936, "full_attention_interval": 4, "rope_theta": 5e6, "partial_rotary_factor": 0.5}
    p = tmp_path / "config.json"
    p.write_text(json.dumps(flat))
    c = config_from_hf(str(p))
    assert c.layer_types == ["gdn", "gdn", "gdn", "attn"] * 2
    assert c.head_dim == 256 and c.rotary_half == 64 and c.theta == 5e6 and abs(c.eps - 1e-6) < 1e-12


@pytest.mark.parametrize("edit, message", [
    (lambda t: t.pop("hidden_size"), "hidden_size"),
    (lambda t: t.__setitem__("layer_types", ["linear_attention", "sliding"] * 2), "unknown layer type"),
    (lambda t: t.__setitem__("layer_types", ["linear_attention"] * 3), "num_hidden_layers"),
    (lambda t: t.__setitem__("linear_conv_kernel_dim", 3), "linear_conv_kernel_dim"),
])
def test_config_errors(tiny_folder, tmp_path, edit, message):
    from s1omni import config_from_hf
    root = json.load(open(os.path.join(tiny_folder[2], "config.json")))
    edit(root["text_config"])
    p = tmp_path / "config.json"
    p.write_text(json.dumps(root))
    with pytest.raises(ValueError, match=message):
        config_from_hf(str(p))
    p.write_text("{\"text_config\": {")
    with pytest.raises(ValueError, match="unreadable"):
        config_from_hf(str(p))


def test_listing_maps_every_tensor(tiny_folder):
    from s1omni import checkpoint_list
    cfg, W, folder = tiny_folder
    listing = checkpoint_list(folder)
    names = {n for n, _, _, _ in listing}
    want = {n for n, _, _ in OM.weight_shapes(cfg)} - {"head_w", "head_b"}
    assert names == want and len(listing) == len(want)
    state = hf_state(cfg, W)
    for name, hf, dtype, shape in listing:
        assert hf.startswith("model.language_model.")
        arr, kind = state[hf[len("model.language_model."):]]
        assert dtype == kind and shape == arr.shape, (name, dtype, shape)
        if name.endswith(".conv"):
            assert shape == (cfg.conv_dim, 1, 4)
        elif name in W:
            assert shape == W[name].shape


@pytest.mark.parametrize("prefix, shards", [("model.language_model.", 1), ("model.", 3), ("", 2)])
def test_prefixes_and_shards(tiny_folder, tmp_path, prefix, shards):
    from s1omni import checkpoint_check, checkpoint_list
    cfg, W, _ = tiny_folder
    folder = write_checkpoint(str(tmp_path / "c"), cfg, W, prefix=prefix, shards=shards)
    listing = checkpoint_list(folder)
    assert all(hf.startswith(prefix) for _, hf, _, _ in listing)
    assert len(listing) == len(OM.weight_shapes(cfg)) - 2
    checkpoint_check(folder, _s1cfg(cfg))


def test_other_prefixes_ignored(tiny_folder, tmp_path):
    """Vision and MTP tensors beside the language model are not mapped."""
    from safetensors.numpy import save_file
    from s1omni import checkpoint_check, checkpoint_list
    cfg, W, _ = tiny_folder
    folder = write_checkpoint(str(tmp_path / "c"), cfg, W, shards=2)
    save_file({"model.visual.blocks.0.attn.qkv.weight": np.zeros((4, 4), np.float32),
               "mtp.layers.0.mlp.up_proj.weight": np.zeros((4, 4), np.float32)},
              os.path.join(folder, "extra.safetensors"))
    idx = json.load(open(os.path.join(folder, "model.safetensors.index.json")))
    idx["weight_map"]["model.visual.blocks.0.attn.qkv.weight"] = "extra.safetensors"
    idx["weight_map"]["mtp.layers.0.mlp.up_proj.weight"] = "extra.safetensors"
    json.dump(idx, open(os.path.join(folder, "model.safetensors.index.json"), "w"))
    assert len(checkpoint_list(folder)) == len(OM.weight_shapes(cfg)) - 2
    checkpoint_check(folder, _s1cfg(cfg))


def _write_state(folder, state, prefix="model.language_model."):
    """One model.safetensors from an hf_state-like dict (bf16 entries as uint16)."""
    from safetensors.numpy import save_file
    from hf_checkpoint import _retag_bf16
    os.makedirs(folder, exist_ok=True)
    path = os.path.join(folder, "model.safetensors")
    save_file({prefix + k: v for k, (v, _) in state.items()}, path)
    _retag_bf16(path, {prefix + k for k, (_, d) in state.items() if d == "BF16"})
    return folder


def test_check_errors(tiny_folder, tmp_path):
    from s1omni import checkpoint_check, checkpoint_list
    cfg, W, _ = tiny_folder
    base = hf_state(cfg, W)
    good = _s1cfg(cfg)

    missing = dict(base)
    missing.pop("layers.3.self_attn.k_norm.weight")
    with pytest.raises(ValueError, match="lacks l3.k_norm"):
        checkpoint_check(_write_state(str(tmp_path / "missing"), missing), good)

    f32 = dict(base)
    f32["layers.0.mlp.up_proj.weight"] = (W["l0.up"].astype(np.float32), "F32")
    with pytest.raises(ValueError, match="up_proj.weight is F32, not bfloat16"):
        checkpoint_list(_write_state(str(tmp_path / "f32"), f32))

    folder = write_checkpoint(str(tmp_path / "shape"), cfg, W, shards=1)
    wrong = _s1cfg(cfg)
    wrong.intermediate = cfg.intermediate * 2
    with pytest.raises(ValueError, match="shape"):
        checkpoint_check(folder, wrong)
    deeper = _s1cfg(cfg)
    deeper.layer_types = deeper.layer_types + ["gdn"]
    with pytest.raises(ValueError, match="lacks l4."):
        checkpoint_check(folder, deeper)
    shallower = _s1cfg(cfg)
    shallower.layer_types = shallower.layer_types[:3]
    with pytest.raises(ValueError, match="no place"):
        checkpoint_check(folder, shallower)

    with pytest.raises(ValueError, match="embed_tokens"):
        noembed = dict(base)
        noembed.pop("embed_tokens.weight")
        checkpoint_list(_write_state(str(tmp_path / "noembed"), noembed))
    with pytest.raises(ValueError, match="cannot open"):
        checkpoint_list(str(tmp_path / "absent"))


def test_conv_weight_as_two_dims(tiny_folder, tmp_path):
    """A conv1d weight stored [C, 4] (squeezed) is accepted like [C, 1, 4]."""
    from s1omni import checkpoint_check
    cfg, W, _ = tiny_folder
    st = hf_state(cfg, W)
    st["layers.0.linear_attn.conv1d.weight"] = (st["layers.0.linear_attn.conv1d.weight"][0][:, 0, :], "BF16")
    checkpoint_check(_write_state(str(tmp_path / "c"), st), _s1cfg(cfg))


def test_transformers_save_pretrained_folder(tmp_path):
    """A folder written by Transformers' Qwen3_5TextModel.save_pretrained reads and checks."""
    torch = pytest.importorskip("torch")
    transformers = pytest.importorskip("transformers")
    if not hasattr(transformers, "Qwen3_5TextConfig"):
        pytest.skip("this transformers has no Qwen3.5")
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M
    from s1omni import checkpoint_check, checkpoint_list, config_from_hf
    cfg = OM.preset("tiny")
    hc = transformers.Qwen3_5TextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
        num_hidden_layers=len(cfg.layer_types), num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads,
        head_dim=256, linear_num_key_heads=cfg.lin_k_heads, linear_num_value_heads=cfg.lin_v_heads,
        linear_key_head_dim=128, linear_value_head_dim=128,
        rope_parameters={"rope_type": "default", "rope_theta": cfg.theta, "partial_rotary_factor": 0.25})
    torch.manual_seed(0)
    M.Qwen3_5TextModel._from_config(hc, dtype=torch.bfloat16).save_pretrained(str(tmp_path))
    c = config_from_hf(str(tmp_path / "config.json"))
    assert c.layer_types == cfg.layer_types and c.rotary_half == 32 and c.theta == cfg.theta
    assert len(checkpoint_list(str(tmp_path))) == len(OM.weight_shapes(cfg)) - 2
    checkpoint_check(str(tmp_path), c)
