"""A model loaded from a Hugging Face checkpoint folder by the C++ host (the reference's
loader: src/models/qwen3_5/native/src/model.rs:267-397; the head from the Open-Jev export
manifest, src/models/open_jev/native/src/engine.rs:125-177).

* sharded folder with fp32 A_log / GDN norm -> every parameter reads back equal to the
  bf16 weights, and the logits equal, bit for bit, those of the same weights set by name;
  within 2e-2 of the oracle;
* a folder written by Transformers' save_pretrained (random init) -> final-norm rows of the
  last tokens and head logits against Transformers' own forward of that folder.
"""
import os

import numpy as np
import pytest

from oracle import fixtures
from oracle import model as OM

from hf_checkpoint import write_checkpoint

pytestmark = pytest.mark.gpu


def test_checkpoint_folder_equals_named_weights(cs1, tmp_path):
    from s1omni import Model, config_from_hf, preset
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    folder = write_checkpoint(str(tmp_path / "ckpt"), cfg, W, shards=3)
    c = config_from_hf(os.path.join(folder, "config.json"), labels=cfg.labels)
    seqs = fixtures.tiny_prompts(cfg)
    a = Model(c, device=0, max_tokens=1024, max_seqs=8)
    try:
        a.load_checkpoint(folder)
        a.load_head(os.path.join(folder, "open_jev_export.json"))
        for name, shape, kind in OM.weight_shapes(cfg):
            got = a.get_weight(name, shape)
            assert np.array_equal(got, W[name].astype(np.float32)), name
        la = a.forward(seqs)
    finally:
        a.close()
    b = Model(preset("tiny"), device=0, max_tokens=1024, max_seqs=8)
    try:
        b.load(W)
        lb = b.forward(seqs)
    finally:
        b.close()
    assert np.array_equal(la, lb)
    ref = OM.forward_batch(cfg, W, seqs, gdn_mode="bf16")[1]
    assert np.abs(la - ref).max() <= 2e-2, np.abs(la - ref).max()


def test_load_head_errors(cs1, tmp_path):
    import json
    from s1omni import Model, preset
    m = Model(preset("tiny"), device=0, max_tokens=256, max_seqs=4)
    try:
        p = tmp_path / "open_jev_export.json"
        p.write_text(json.dumps({"head_weight": [[0.0] * 255] * 8, "head_bias": [0.0] * 8}))
        with pytest.raises(RuntimeError, match="head shape"):
            m.load_head(str(p))
        p.write_text(json.dumps({"head_weight": [[0.0] * 256] * 8}))
        with pytest.raises(RuntimeError, match="head_bias"):
            m.load_head(str(p))
    finally:
        m.close()


def test_transformers_folder_matches_transformers_forward(cs1, tmp_path):
    torch = pytest.importorskip("torch")
    transformers = pytest.importorskip("transformers")
    if not hasattr(transformers, "Qwen3_5TextConfig"):
        pytest.skip("this transformers has no Qwen3.5")
    import transformers.utils.import_utils as iu
    iu.is_flash_linear_attention_available = lambda *a, **k: False
    iu.is_causal_conv1d_available = lambda *a, **k: False
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M
    from s1omni import Model, config_from_hf
    cfg = OM.preset("tiny")
    hc = transformers.Qwen3_5TextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
        num_hidden_layers=len(cfg.layer_types), num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads,
        head_dim=256, linear_num_key_heads=cfg.lin_k_heads, linear_num_value_heads=cfg.lin_v_heads,
        linear_key_head_dim=128, linear_value_head_dim=128, max_position_embeddings=4096,
        rope_parameters={"rope_type": "default", "rope_theta": cfg.theta, "partial_rotary_factor": 0.25})
    hc._attn_implementation = "eager"
    torch.manual_seed(0)
    hf = M.Qwen3_5TextModel._from_config(hc, dtype=torch.bfloat16).eval()
    with torch.no_grad():  # the default init leaves norms at zero; give them values
        for n, p in hf.named_parameters():
            if p.dim() == 1:
                p.add_(torch.randn_like(p.float()).mul_(0.1).to(p.dtype))
    hf.save_pretrained(str(tmp_path))
    seqs = fixtures.tiny_prompts(cfg)
    with torch.inference_mode():
        rows = np.stack([hf(input_ids=torch.from_numpy(s.astype(np.int64))[None], use_cache=False)
                         .last_hidden_state[0, -1].float().numpy() for s in seqs])
    c = config_from_hf(str(tmp_path / "config.json"), labels=1)
    rng = np.random.default_rng(1)
    head_w = (rng.standard_normal((1, cfg.hidden)) * 0.05).astype(np.float32)
    (tmp_path / "open_jev_export.json").write_text(
        __import__("json").dumps({"head_weight": head_w[0].tolist(), "head_bias": 0.25}))
    m = Model(c, device=0, max_tokens=1024, max_seqs=8)
    try:
        m.load_checkpoint(str(tmp_path))
        m.load_head(str(tmp_path / "open_jev_export.json"))
        logits, hidden = m.forward(seqs, hidden=True)
    finally:
        m.close()
    rel = np.linalg.norm(hidden - rows) / np.linalg.norm(rows)
    assert rel <= 2e-2, rel
    ref = rows.astype(np.float64) @ head_w[0].astype(np.float64) + 0.25
    assert np.abs(logits[:, 0] - ref).max() <= 4e-2, np.abs(logits[:, 0] - ref).max()
