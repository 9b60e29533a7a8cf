"""Generate the golden vectors that pin the numpy oracle to Transformers.

Runs only where `transformers` with Qwen3.5 is importable on the CPU (the build
container). The reference's parity anchor is Transformers' no-FLA PyTorch code
(`tests/qwen3_5/test_gdn_fp32.py` and `recipe/open_jev/validation.md:22-31` of
InferMatrixLab/system1-omni, pinned there to transformers 5.17.0); this script
records the version it actually ran with inside every fixture.

    python tests/golden/make_golden.py

Writes:
  gdn_c0.npz     -- C0: torch_chunk_gated_delta_rule, fp32, T=512, 16/16 heads x 128,
                    seeded numpy inputs (oracle.fixtures.c0_inputs(0)); final state,
                    the first and last chunk of o, and per-token sums of o
  gdn_grouped.npz -- same operator, T=129, 4 value / 2 key heads, bf16-valued inputs
                    (the reference test's grouped case), full o and state
  tiny_model.npz -- Qwen3_5TextModel (bf16, eager attention, FLA off) with the oracle's
                    seeded "tiny" weights: final-norm hidden rows of three prompts
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import transformers.utils.import_utils as iu  # noqa: E402

# Force the pure-PyTorch GDN and conv paths, as the reference's HF baseline does.
iu.is_flash_linear_attention_available = lambda *a, **k: False
iu.is_causal_conv1d_available = lambda *a, **k: False
import transformers  # noqa: E402
from transformers import Qwen3_5TextConfig  # noqa: E402
from transformers.models.qwen3_5 import modeling_qwen3_5 as M  # noqa: E402

from oracle import fixtures  # noqa: E402
from oracle.model import make_weights, preset  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
VERSIONS = f"transformers {transformers.__version__}, torch {torch.__version__}"


def gdn_c0():
    q, k, v, g, beta = fixtures.c0_inputs(0)
    t = lambda x: torch.from_numpy(x)[None]
    o, s = M.torch_chunk_gated_delta_rule(t(q), t(k), t(v), t(g), t(beta), initial_state=None,
                                          output_final_state=True, use_qk_l2norm_in_kernel=True)
    o = o[0].numpy()
    np.savez_compressed(os.path.join(OUT, "gdn_c0.npz"), state=s[0].numpy(), o_head=o[:64], o_tail=o[-64:],
                        o_token_sum=o.astype(np.float64).sum((1, 2)), versions=VERSIONS)


def gdn_grouped():
    q, k, v, g, beta = fixtures.grouped_inputs(1, T=129, H=4, HK=2)
    t = lambda x: torch.from_numpy(x)[None]
    rep = 2
    o, s = M.torch_chunk_gated_delta_rule(t(np.repeat(q, rep, 1)), t(np.repeat(k, rep, 1)), t(v), t(g), t(beta),
                                          initial_state=None, output_final_state=True, use_qk_l2norm_in_kernel=True)
    np.savez_compressed(os.path.join(OUT, "gdn_grouped.npz"), o=o[0].numpy(), state=s[0].numpy(), versions=VERSIONS)


def tiny_model():
    cfg = preset("tiny")
    W = make_weights(cfg, seed=7)
    hf_types = ["linear_attention" if t == "gdn" else "full_attention" for t in cfg.layer_types]
    config = Qwen3_5TextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
        num_hidden_layers=len(cfg.layer_types), num_attention_heads=cfg.heads,
        num_key_value_heads=cfg.kv_heads, head_dim=cfg.head_dim, linear_num_key_heads=cfg.lin_k_heads,
        linear_num_value_heads=cfg.lin_v_heads, linear_key_head_dim=cfg.lin_k_dim,
        linear_value_head_dim=cfg.lin_v_dim, linear_conv_kernel_dim=4, layer_types=hf_types,
        rms_norm_eps=cfg.eps, max_position_embeddings=4096,
        rope_parameters={"rope_type": "default", "rope_theta": cfg.theta, "partial_rotary_factor": 0.25,
                         "mrope_section": [11, 11, 10], "mrope_interleaved": True},
    )
    config._attn_implementation = "eager"
    model = M.Qwen3_5TextModel(config).to(torch.bfloat16).eval()
    sd = {}
    b = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16)
    sd["embed_tokens.weight"] = b(W["embed"])
    sd["norm.weight"] = b(W["final_norm"])
    for i, t in enumerate(cfg.layer_types):
        p, q = f"layers.{i}.", f"l{i}."
        sd[p + "input_layernorm.weight"] = b(W[q + "input_norm"])
        sd[p + "post_attention_layernorm.weight"] = b(W[q + "post_norm"])
        sd[p + "mlp.gate_proj.weight"] = b(W[q + "gate"])
        sd[p + "mlp.up_proj.weight"] = b(W[q + "up"])
        sd[p + "mlp.down_proj.weight"] = b(W[q + "down"])
        if t == "gdn":
            la = p + "linear_attn."
            sd[la + "in_proj_qkv.weight"] = b(W[q + "in_qkv"])
            sd[la + "in_proj_z.weight"] = b(W[q + "in_z"])
            sd[la + "in_proj_b.weight"] = b(W[q + "in_b"])
            sd[la + "in_proj_a.weight"] = b(W[q + "in_a"])
            sd[la + "conv1d.weight"] = b(W[q + "conv"][:, None, :])
            sd[la + "A_log"] = b(W[q + "A_log"])
            sd[la + "dt_bias"] = b(W[q + "dt_bias"])
            sd[la + "norm.weight"] = b(W[q + "norm"])
            sd[la + "out_proj.weight"] = b(W[q + "out"])
        else:
            sa = p + "self_attn."
            for n, m in (("q", "q_proj"), ("k", "k_proj"), ("v", "v_proj"), ("o", "o_proj")):
                sd[sa + m + ".weight"] = b(W[q + n])
            sd[sa + "q_norm.weight"] = b(W[q + "q_norm"])
            sd[sa + "k_norm.weight"] = b(W[q + "k_norm"])
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [m for m in missing if "rotary" not in m]
    assert not missing and not unexpected, (missing, unexpected)
    seqs = fixtures.tiny_prompts(cfg)
    rows = []
    with torch.inference_mode():
        for ids in seqs:
            h = model(input_ids=torch.from_numpy(ids.astype(np.int64))[None], use_cache=False).last_hidden_state
            rows.append(h[0].float().numpy())
    np.savez_compressed(os.path.join(OUT, "tiny_model.npz"), last=np.stack([r[-1] for r in rows]),
                        full0=rows[1], versions=VERSIONS)


if __name__ == "__main__":
    torch.manual_seed(0)
    gdn_c0()
    gdn_grouped()
    tiny_model()
    print("wrote golden fixtures with", VERSIONS)
