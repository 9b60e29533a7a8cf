"""Whole-forward oracle of the Qwen3.5 hybrid decision scorer (test infrastructure only).

Restates the reference's layer loop, `Model::run_with_attention`
(`src/models/qwen3_5/native/src/model.rs:3178-3727`), op by op with the
numerics of `oracle.ops` / `oracle.gdn`, the packed and shared-prefix layouts
(`model.rs:1548-1907`, `model.rs:3744`) and the final-token scorer head
(`src/models/open_jev/native/src/executor.rs:59-71`: float64 dot, rounded to
float32, plus a float32 bias; one row per label).

Weights are a dict of float32 arrays holding bfloat16 values (the head stays
float32), generated from a seed by `make_weights`.
"""
from dataclasses import dataclass, field

import numpy as np

from . import gdn as G
from . import ops
from .bf16 import rnd
from .packing import rotary_tables


@dataclass
class Config:
    hidden: int
    intermediate: int
    layer_types: list            # "gdn" / "attn" per layer
    lin_k_heads: int
    lin_v_heads: int
    heads: int
    kv_heads: int
    vocab: int
    labels: int = 8
    lin_k_dim: int = 128
    lin_v_dim: int = 128
    head_dim: int = 256
    rotary_half: int = 32
    theta: float = 1.0e7
    eps: float = 1e-6
    name: str = field(default="custom")

    @property
    def key_dim(self):
        return self.lin_k_heads * self.lin_k_dim

    @property
    def value_dim(self):
        return self.lin_v_heads * self.lin_v_dim

    @property
    def conv_dim(self):
        return 2 * self.key_dim + self.value_dim

    @property
    def gdn_in(self):
        """Row width of the stacked GDN input projection qkv|z|b|a (model.rs:481-491)."""
        return self.conv_dim + self.value_dim + 2 * self.lin_v_heads

    @property
    def attn_q(self):
        return self.heads * self.head_dim * 2

    @property
    def attn_in(self):
        """Row width of the stacked attention projection q(+gate)|k|v."""
        return self.attn_q + 2 * self.kv_heads * self.head_dim


def hybrid_layers(n, interval=4):
    return ["attn" if (i + 1) % interval == 0 else "gdn" for i in range(n)]


def preset(name):
    """Named shapes: the three benchmark model sizes (4B, 9B, 27B) and small test models."""
    if name == "4b":
        return Config(2560, 9216, hybrid_layers(32), 16, 32, 16, 4, 151936, name=name)
    if name == "9b":
        return Config(4096, 12288, hybrid_layers(32), 16, 32, 16, 4, 151936, name=name)
    if name == "27b":
        return Config(5120, 17408, hybrid_layers(64), 16, 48, 24, 4, 151936, name=name)
    if name == "tiny":
        return Config(256, 512, hybrid_layers(4), 2, 4, 4, 2, 512, name=name)
    if name == "tiny8":
        return Config(512, 1024, hybrid_layers(8), 2, 6, 6, 2, 1024, name=name)
    raise KeyError(name)


def weight_shapes(cfg):
    """Ordered (name, shape, kind) of every parameter; kind in {bf16, f32}."""
    H, I = cfg.hidden, cfg.intermediate
    out = [("embed", (cfg.vocab, H), "bf16")]
    for i, t in enumerate(cfg.layer_types):
        p = f"l{i}."
        out += [(p + "input_norm", (H,), "bf16"), (p + "post_norm", (H,), "bf16")]
        if t == "gdn":
            out += [
                (p + "in_qkv", (cfg.conv_dim, H), "bf16"),
                (p + "in_z", (cfg.value_dim, H), "bf16"),
                (p + "in_b", (cfg.lin_v_heads, H), "bf16"),
                (p + "in_a", (cfg.lin_v_heads, H), "bf16"),
                (p + "conv", (cfg.conv_dim, 4), "bf16"),
                (p + "A_log", (cfg.lin_v_heads,), "bf16"),
                (p + "dt_bias", (cfg.lin_v_heads,), "bf16"),
                (p + "norm", (cfg.lin_v_dim,), "bf16"),
                (p + "out", (H, cfg.value_dim), "bf16"),
            ]
        else:
            out += [
                (p + "q", (cfg.attn_q, H), "bf16"),
                (p + "k", (cfg.kv_heads * cfg.head_dim, H), "bf16"),
                (p + "v", (cfg.kv_heads * cfg.head_dim, H), "bf16"),
                (p + "q_norm", (cfg.head_dim,), "bf16"),
                (p + "k_norm", (cfg.head_dim,), "bf16"),
                (p + "o", (H, cfg.heads * cfg.head_dim), "bf16"),
            ]
        out += [(p + "gate", (I, H), "bf16"), (p + "up", (I, H), "bf16"), (p + "down", (H, I), "bf16")]
    out += [("final_norm", (H,), "bf16"), ("head_w", (cfg.labels, H), "f32"), ("head_b", (cfg.labels,), "f32")]
    return out


def make_weights(cfg, seed, std=0.02):
    """Seeded random-init weights (HF-style: normal(0, std) matrices; A_log = log U(1,16);
    dt_bias near 1; zero-centred norms near 0; gated-norm weight near 1)."""
    rng = np.random.default_rng(seed)
    W = {}
    for name, shape, kind in weight_shapes(cfg):
        leaf = name.split(".")[-1]
        if leaf in ("input_norm", "post_norm", "final_norm", "q_norm", "k_norm"):
            x = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.1)
        elif leaf == "norm":
            x = np.float32(1) + rng.standard_normal(shape, dtype=np.float32) * np.float32(0.1)
        elif leaf == "conv":
            x = rng.uniform(-0.5, 0.5, shape).astype(np.float32)
        elif leaf == "A_log":
            x = np.log(rng.uniform(1.0, 16.0, shape)).astype(np.float32)
        elif leaf == "dt_bias":
            x = np.float32(1) + rng.standard_normal(shape, dtype=np.float32) * np.float32(0.1)
        elif leaf == "head_b":
            x = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
        else:
            x = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
        W[name] = x.astype(np.float32) if kind == "f32" else rnd(x)
    return W


class PrefixState:
    """What a shared prefix hands to its suffixes (model.rs:691-713): per GDN layer
    the float32 state [HV,128,128] and the last 3 pre-conv rows; per attention
    layer the post-prep K and raw V of every prefix row."""

    def __init__(self):
        self.gdn_state = []
        self.conv_tail = []
        self.k = []
        self.v = []
        self.length = 0


def _attention_f64(q, k, v, gate, scale, prefix_k=None, prefix_v=None):
    """Causal GQA attention in float64 with unrounded probabilities (the op's exact value;
    only its output is rounded): the `precise` variant of `ops.attention_gated`."""
    S, Hq, Dh = q.shape
    if prefix_k is not None:
        k = np.concatenate([prefix_k, k], 0)
        v = np.concatenate([prefix_v, v], 0)
    P = k.shape[0] - S
    group = Hq // k.shape[1]
    mask = np.arange(P + S)[None, :] <= (P + np.arange(S))[:, None]
    out = np.zeros((S, Hq, Dh))
    for h in range(Hq):
        kh = h // group
        s = (q[:, h, :].astype(np.float64) @ k[:, kh, :].astype(np.float64).T) * float(scale)
        s = np.where(mask, s, -np.inf)
        e = np.exp(s - s.max(-1, keepdims=True))
        out[:, h, :] = (e / e.sum(-1, keepdims=True)) @ v[:, kh, :].astype(np.float64)
    att = rnd(out.astype(np.float32))
    return rnd(att * rnd(ops.sigmoid(gate.reshape(S, Hq, Dh))))


def _gemm64(x, w):
    """y = bf16(x @ w^T) accumulated in float64 (the `precise` variant of `ops.gemm`)."""
    return rnd((np.asarray(x, np.float64) @ np.asarray(w, np.float64).T).astype(np.float32))


def _layer(cfg, W, i, res, x, cos, sin, prefix, cap, gi, ai, gdn_mode, precise):
    """Layer i of `run_with_attention` (`model.rs:3308-3723`): the token mixer (GDN or
    gated attention), its residual add, the SwiGLU MLP and its residual add, each
    residual add followed by the next RMSNorm. Returns (res, x)."""
    T = res.shape[0]
    gemm = _gemm64 if precise else ops.gemm
    scale_gdn = np.float32(cfg.lin_k_dim ** -0.5)
    scale_attn = np.float32(cfg.head_dim ** -0.5)
    p = f"l{i}."
    if cfg.layer_types[i] == "gdn":
        w_in = np.concatenate([W[p + "in_qkv"], W[p + "in_z"], W[p + "in_b"], W[p + "in_a"]], 0)
        y = gemm(x, w_in)
        qkv = y[:, :cfg.conv_dim]
        z = y[:, cfg.conv_dim:cfg.conv_dim + cfg.value_dim]
        b = y[:, cfg.conv_dim + cfg.value_dim:cfg.conv_dim + cfg.value_dim + cfg.lin_v_heads]
        a = y[:, cfg.conv_dim + cfg.value_dim + cfg.lin_v_heads:]
        hist = prefix.conv_tail[gi] if prefix is not None else None
        q, k, v = ops.gdn_conv(qkv, W[p + "conv"], cfg.key_dim, cfg.value_dim, history=hist)
        beta, g = ops.gdn_gates(b, a, W[p + "A_log"], W[p + "dt_bias"])
        q = q.reshape(T, cfg.lin_k_heads, cfg.lin_k_dim)
        k = k.reshape(T, cfg.lin_k_heads, cfg.lin_k_dim)
        v = v.reshape(T, cfg.lin_v_heads, cfg.lin_v_dim)
        s_in = prefix.gdn_state[gi] if prefix is not None else None
        if precise:
            o, s_out = G.recurrent_f64(q, k, v, g, beta, float(scale_gdn), state=s_in)
            o = o.astype(np.float32)
        elif gdn_mode == "bf16":
            o, s_out = G.chunk_bf16(q, k, v, g, beta, scale_gdn, state=s_in)
        elif gdn_mode == "hf":
            o, s_out = G.chunk_fp32(G.l2norm_bf16(q), G.l2norm_bf16(k), v, g, beta, scale_gdn,
                                    state=s_in, l2norm=False)
        else:
            o, s_out = G.chunk_fp32(q, k, v, g, beta, scale_gdn, state=s_in)
        o = rnd(o)
        ln = ops.gated_rms_norm(o, z, W[p + "norm"], cfg.eps)
        delta = gemm(ln, W[p + "out"])
        if cap is not None:
            cap.gdn_state.append(s_out)
            full = qkv if hist is None else np.concatenate([hist, qkv], 0)
            tail = np.zeros((3, cfg.conv_dim), np.float32)
            n = min(3, full.shape[0])
            tail[3 - n:] = full[full.shape[0] - n:]
            cap.conv_tail.append(tail)
    else:
        w_in = np.concatenate([W[p + "q"], W[p + "k"], W[p + "v"]], 0)
        y = gemm(x, w_in)
        qg = y[:, :cfg.attn_q]
        kr = y[:, cfg.attn_q:cfg.attn_q + cfg.kv_heads * cfg.head_dim]
        vr = y[:, cfg.attn_q + cfg.kv_heads * cfg.head_dim:].reshape(T, cfg.kv_heads, cfg.head_dim)
        q, gate, k = ops.attn_prep(qg, kr, W[p + "q_norm"], W[p + "k_norm"], cos, sin,
                                   cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.rotary_half, cfg.eps)
        pk = prefix.k[ai] if prefix is not None else None
        pv = prefix.v[ai] if prefix is not None else None
        if precise:
            att = _attention_f64(q, k, vr, gate, scale_attn, pk, pv)
        else:
            att = ops.attention_gated(q, k, vr, gate, scale_attn, pk, pv)
        delta = gemm(att.reshape(T, -1), W[p + "o"])
        if cap is not None:
            cap.k.append(k if pk is None else np.concatenate([pk, k], 0))
            cap.v.append(vr if pv is None else np.concatenate([pv, vr], 0))
    res, x = ops.add_rms_norm(res, delta, W[p + "post_norm"], cfg.eps)
    gu = gemm(x, np.concatenate([W[p + "gate"], W[p + "up"]], 0))
    act = ops.silu_mul(gu, cfg.intermediate)
    delta = gemm(act, W[p + "down"])
    nxt = W[f"l{i + 1}.input_norm"] if i + 1 < len(cfg.layer_types) else W["final_norm"]
    return ops.add_rms_norm(res, delta, nxt, cfg.eps)


def run_sequence(cfg, W, ids, prefix=None, capture=False, gdn_mode="bf16", precise=False):
    """Forward one sequence (optionally continuing a PrefixState), in the layer order of
    `run_with_attention` (`src/models/qwen3_5/native/src/model.rs:3178-3727`).

    gdn_mode: "bf16" -- the reference kernel's bf16 intermediates (the CUDA path's
    arithmetic); "fp32" -- float32 chunk form with float32 L2 norms (the FP32
    operator); "hf" -- float32 chunk form after Transformers' bfloat16 L2 norm.
    precise: every projection accumulated in float64, the GDN as the float64 token
    recurrence and attention in float64 with unrounded probabilities; each op's output
    is rounded to bf16 at the same points as in the kernels (the exact value of every
    op, so the distance of a kernel from it is that kernel's own arithmetic error).

    Returns (final-norm hidden rows [T, H], PrefixState or None). Positions start
    at prefix.length (0 without a prefix)."""
    T = len(ids)
    P = prefix.length if prefix is not None else 0
    cos, sin = rotary_tables(np.arange(P, P + T), cfg.rotary_half, cfg.theta)
    cap = PrefixState() if capture else None
    res = ops.embed(ids, W["embed"])
    x = ops.rms_norm(res, W["l0.input_norm"], cfg.eps)
    gi = ai = 0
    for i, t in enumerate(cfg.layer_types):
        res, x = _layer(cfg, W, i, res, x, cos, sin, prefix, cap, gi, ai, gdn_mode, precise)
        gi, ai = (gi + 1, ai) if t == "gdn" else (gi, ai + 1)
    if cap is not None:
        cap.length = P + T
    return x, cap


def run_layers(cfg, W, ids, first, last, res, gdn_mode="bf16", precise=False):
    """Layers [first, last) of one sequence (positions from 0) from the residual stream
    `res` [T, H] entering layer `first`; returns the stream leaving layer last - 1 (the
    counterpart of the host's s1_model_run_layers, for layer-by-layer comparisons).
    W needs only the parameters of those layers (and the next input norm)."""
    cos, sin = rotary_tables(np.arange(len(ids)), cfg.rotary_half, cfg.theta)
    res = np.asarray(res, np.float32)
    x = ops.rms_norm(res, W[f"l{first}.input_norm"], cfg.eps)
    for i in range(first, last):
        res, x = _layer(cfg, W, i, res, x, cos, sin, None, None, 0, 0, gdn_mode, precise)
    return res


def head(cfg, W, h):
    """Scorer head on final-token rows h [n, H] (executor.rs:59-71, one row per
    label): f32(sum_d f64(W[l,d]) f64(h[d])) + b[l]."""
    h = np.asarray(h, np.float64)
    s = (h @ W["head_w"].astype(np.float64).T).astype(np.float32)
    return (s + W["head_b"][None, :]).astype(np.float32)


def forward_batch(cfg, W, seqs, gdn_mode="bf16"):
    """Packed independent candidates (`model.rs:1548-1632`, `forward_batch_layout`):
    each sequence's positions restart at 0 and its state starts at zero, so the packed
    result is the per-sequence result.
    Returns (last hidden rows [n, H], logits [n, labels])."""
    last = np.stack([run_sequence(cfg, W, s, gdn_mode=gdn_mode)[0][-1] for s in seqs])
    return last, head(cfg, W, last)


def forward_shared_prefix(cfg, W, prefix_ids, suffixes, gdn_mode="bf16"):
    """Shared prefix computed once, every suffix continued from its captured state
    (model.rs:1664-1907). Returns (last hidden rows, logits) per candidate."""
    _, state = run_sequence(cfg, W, prefix_ids, capture=True, gdn_mode=gdn_mode)
    last = np.stack([run_sequence(cfg, W, s, prefix=state, gdn_mode=gdn_mode)[0][-1] for s in suffixes])
    return last, head(cfg, W, last)
