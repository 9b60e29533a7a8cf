"""The numpy oracle, pinned against golden vectors produced by Transformers'
Qwen3.5 code (tests/golden/make_golden.py) and against its own invariants.

These run on the CPU and check the checker: GDN chunk forms vs
torch_chunk_gated_delta_rule (rel 1e-5), the float64 recurrence vs the same,
the whole tiny model vs Qwen3_5TextModel (logits within 2e-2), bf16 rounding,
the head's rounding order (tests/open_jev/head.rs:4-26), rotary tables and the
shared-prefix continuation."""
import os

import numpy as np
import pytest

from oracle import bf16, fixtures, ops
from oracle import gdn as G
from oracle import model as OM
from oracle.packing import layout, rotary_tables

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SCALE = np.float32(128 ** -0.5)


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, np.inf, -np.inf, 3.4e38, 1e-40], np.float32)
    got = bf16.rnd(x)
    assert got[0] == 1.0 and got[1] == 1.0 and got[2] == 1.0 + 2 ** -6 and got[3] == -2.5
    assert np.isinf(got[4]) and np.isinf(got[5]) and np.isinf(got[6])
    assert np.isnan(bf16.rnd(np.array([np.nan], np.float32)))[0]
    import torch
    r = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    assert np.array_equal(bf16.rnd(r), torch.from_numpy(r).bfloat16().float().numpy())


def test_gdn_c0_matches_transformers():
    g = np.load(os.path.join(GOLD, "gdn_c0.npz"))
    q, k, v, gg, beta = fixtures.c0_inputs(0)
    o, s = G.chunk_fp32(q, k, v, gg, beta, SCALE)
    assert rel(s, g["state"]) <= 1e-5
    assert rel(o[:64], g["o_head"]) <= 1e-5 and rel(o[-64:], g["o_tail"]) <= 1e-5
    assert np.abs(o.astype(np.float64).sum((1, 2)) - g["o_token_sum"]).max() <= 1e-4


def test_gdn_grouped_case_matches_transformers_and_float64():
    g = np.load(os.path.join(GOLD, "gdn_grouped.npz"))
    q, k, v, gg, beta = fixtures.grouped_inputs(1, T=129, H=4, HK=2)
    o, s = G.chunk_fp32(q, k, v, gg, beta, SCALE)
    assert rel(o, g["o"]) <= 1e-5 and rel(s, g["state"]) <= 1e-5
    o2, s2 = G.recurrent_f64(q, k, v, gg, beta, float(SCALE))
    assert rel(o2, g["o"]) <= 1e-5 and rel(s2, g["state"]) <= 1e-5
    o3, _ = G.chunk_bf16(q, k, v, gg, beta, SCALE)
    assert np.abs(o3 - o2).max() <= 2e-2 * np.abs(o2).max()


def test_gdn_chunk_state_continuation():
    q, k, v, g, beta = fixtures.grouped_inputs(2, T=200, H=4, HK=2)
    o, s = G.chunk_fp32(q, k, v, g, beta, SCALE)
    oa, sa = G.chunk_fp32(q[:128], k[:128], v[:128], g[:128], beta[:128], SCALE)
    ob, sb = G.chunk_fp32(q[128:], k[128:], v[128:], g[128:], beta[128:], SCALE, state=sa)
    assert rel(np.concatenate([oa, ob]), o) <= 1e-6 and rel(sb, s) <= 1e-6


def test_gdn_output_and_state_are_affine_in_the_initial_state():
    """The chunked recurrence is affine in its initial state: with f(S) = (o, S_end) from
    initial state S, f(a Sa + b Sb) - f(0) = a (f(Sa) - f(0)) + b (f(Sb) - f(0)). This is
    the property that lets a piece of a prompt run before its initial state is known
    (segments of one sequence corrected afterwards)."""
    # weak decay, so that the initial state still shapes the final one after 193 tokens
    q, k, v, g, beta = fixtures.grouped_inputs(9, T=193, H=4, HK=2, decay=0.02)
    rng = np.random.default_rng(10)
    sa, sb = (rng.standard_normal((4, 128, 128)).astype(np.float32) * np.float32(0.3) for _ in range(2))
    a, b = np.float32(0.7), np.float32(-1.3)
    f = {key: G.chunk_fp32(q, k, v, g, beta, SCALE, state=s) for key, s in
         (("0", None), ("a", sa), ("b", sb), ("ab", a * sa + b * sb))}
    for i in range(2):  # output rows, then the final state
        base = f["0"][i].astype(np.float64)
        lhs = f["ab"][i] - base
        rhs = a * (f["a"][i] - base) + b * (f["b"][i] - base)
        assert rel(lhs, rhs) <= 1e-5, (i, rel(lhs, rhs))


def test_tiny_model_matches_transformers():
    gold = np.load(os.path.join(GOLD, "tiny_model.npz"))
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    seqs = fixtures.tiny_prompts(cfg)
    for mode in ("hf", "bf16"):
        last, logits = OM.forward_batch(cfg, W, seqs, gdn_mode=mode)
        assert np.abs(logits - OM.head(cfg, W, gold["last"])).max() <= 2e-2
        assert rel(last, gold["last"]) <= 3e-2


def test_shared_prefix_oracle_equals_full_pass():
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    rng = np.random.default_rng(1)
    prefix = rng.integers(0, cfg.vocab, 128)
    sufs = [rng.integers(0, cfg.vocab, n) for n in (5, 64)]
    _, shared = OM.forward_shared_prefix(cfg, W, prefix, sufs, gdn_mode="fp32")
    _, full = OM.forward_batch(cfg, W, [np.concatenate([prefix, s]) for s in sufs], gdn_mode="fp32")
    assert np.abs(shared - full).max() <= 1e-3


def test_head_rounds_the_dot_product_before_the_bias():
    """tests/open_jev/head.rs:4-17: f64 accumulation, then f32, then the f32 bias."""
    cfg = OM.Config(3, 128, ["gdn"], 1, 1, 1, 1, 8, labels=1)
    W = {"head_w": np.array([[16777216.0, 1.0, -16777216.0]], np.float32), "head_b": np.array([0.25], np.float32)}
    assert OM.head(cfg, W, np.ones((1, 3), np.float32))[0, 0] == 1.25
    W = {"head_w": np.array([[16777216.0, 1.0]], np.float32), "head_b": np.array([-16777216.0], np.float32)}
    assert OM.head(cfg, W, np.ones((1, 2), np.float32))[0, 0] == 0.0


def test_rotary_tables_match_transformers_at_bf16():
    import torch
    pos = np.arange(0, 5000, 7)
    cos, sin = rotary_tables(pos, 32, 1e7)
    inv = 1.0 / (1e7 ** (torch.arange(0, 64, 2, dtype=torch.int64).float() / 64))
    ang = torch.from_numpy(pos).float()[:, None] * inv[None]
    assert np.abs(cos - ang.cos().bfloat16().float().numpy()).max() <= 2 ** -7
    assert np.abs(sin - ang.sin().bfloat16().float().numpy()).max() <= 2 ** -7


def test_layout_positions_restart_per_sequence():
    offs, pos, last = layout([3, 1, 4])
    assert offs.tolist() == [0, 3, 4]
    assert pos.tolist() == [0, 1, 2, 0, 0, 1, 2, 3]
    assert last.tolist() == [2, 3, 7]
    _, pos2, _ = layout([2, 2], prefix=2048)
    assert pos2.tolist() == [2048, 2049, 2048, 2049]


def test_conv_history_equals_concatenated_rows():
    rng = np.random.default_rng(3)
    x = bf16.rnd(rng.standard_normal((20, 48)).astype(np.float32))
    w = bf16.rnd(rng.uniform(-0.5, 0.5, (48, 4)).astype(np.float32))
    full = ops.gdn_conv(x, w, 16, 16)
    tail = ops.gdn_conv(x[10:], w, 16, 16, history=x[7:10])
    for a, b in zip(full, tail):
        assert np.array_equal(a[10:], b)


@pytest.mark.parametrize("name", ["4b", "9b", "27b"])
def test_presets_have_baseline_shapes(name):
    from s1omni import preset
    a, b = OM.preset(name), preset(name)
    assert (a.hidden, a.intermediate, a.lin_v_heads, a.heads) == (b.hidden, b.intermediate, b.lin_v_heads, b.heads)
    assert a.layer_types == b.layer_types
    assert a.layer_types.count("attn") * 4 == len(a.layer_types)


def test_precise_forward_is_the_float32_forward_to_bf16_noise():
    """The precise oracle (float64 ops, bf16 rounding at op outputs) and the float32 one
    on the tiny model: the same forward up to bf16 rounding flips, and the shared-prefix
    continuation of the precise form equals its full prompt up to the same noise."""
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    rng = np.random.default_rng(3)
    prefix = rng.integers(0, cfg.vocab, 128)
    sfx = rng.integers(0, cfg.vocab, 20)
    full = np.concatenate([prefix, sfx])
    a = OM.run_sequence(cfg, W, full, precise=True)[0][-1]
    b = OM.run_sequence(cfg, W, full)[0][-1]
    assert np.abs(a - b).max() <= 0.05 * np.abs(b).max()
    _, st = OM.run_sequence(cfg, W, prefix, capture=True, precise=True)
    c = OM.run_sequence(cfg, W, sfx, prefix=st, precise=True)[0][-1]
    assert np.abs(c - a).max() <= 0.05 * np.abs(a).max()
    # layer by layer from the embedding equals the whole forward's residual stream
    from oracle import ops
    res = OM.run_layers(cfg, W, full, 0, len(cfg.layer_types), ops.embed(full, W["embed"]))
    x = ops.rms_norm(res, W["final_norm"], cfg.eps)
    assert np.array_equal(x[-1], b)
