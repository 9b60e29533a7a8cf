"""One numpy function per `cs1_*` operation (test infrastructure only).

Each function restates the arithmetic, and the bfloat16 rounding points, of
the reference kernel cited in its docstring (paths relative to the
InferMatrixLab/system1-omni tree). Inputs and outputs are float32 arrays that
hold bfloat16-representable values unless the docstring says otherwise.
"""
import numpy as np

from .bf16 import rnd


def silu(x):
    """PyTorch's float32 SiLU, x / (1 + e^-x) (`src/backends/cuda/qwen3_5/common.cuh:41`)."""
    x = np.asarray(x, dtype=np.float32)
    return (x / (np.float32(1) + np.exp(-x))).astype(np.float32)


def sigmoid(x):
    """PyTorch's float32 sigmoid, 1 / (1 + e^-x) (`common.cuh:42`)."""
    x = np.asarray(x, dtype=np.float32)
    return (np.float32(1) / (np.float32(1) + np.exp(-x))).astype(np.float32)


def embed(ids, table):
    """out[t] = table[ids[t]] (`elementwise.cu:11-17`, `cs1_embed`)."""
    return table[np.asarray(ids, dtype=np.int64)].astype(np.float32)


def rms_norm(x, w, eps):
    """Zero-centred RMSNorm, fp32, one rounding (`norm.cu:11-26`, `cs1_rms_norm`)."""
    x = np.asarray(x, dtype=np.float32)
    ms = (x.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(np.float32)
    inv = (np.float32(1) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return rnd(x * inv * (np.float32(1) + w.astype(np.float32)))


def add_rms_norm(res, delta, w, eps):
    """residual = bf16(res + delta); out = rms_norm(residual) (`norm.cu:30-48`)."""
    r = rnd(np.asarray(res, np.float32) + np.asarray(delta, np.float32))
    return r, rms_norm(r, w, eps)


def gated_rms_norm(x, z, w, eps):
    """GDN output norm over rows of 128 (`norm.cu:117-139`, `cs1_gated_rms_norm`).

    normed = bf16(x / rms(x)); scaled = bf16(w * normed); out = bf16(scaled * silu(z)).
    x: [T, H, 128]; z: [T, H*128]; w: [128].
    """
    T, H, D = x.shape
    x = x.astype(np.float32)
    ms = (x.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(np.float32)
    inv = (np.float32(1) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    normed = rnd(x * inv)
    scaled = rnd(w.astype(np.float32) * normed)
    return rnd(scaled * silu(z.reshape(T, H, D))).reshape(T, H * D)


def gdn_conv(qkv, w, key_dim, value_dim, history=None):
    """Causal depthwise conv1d (k=4) + SiLU, split q,k,v (`elementwise.cu:20-41`).

    qkv: [T, C] pre-conv rows (C = 2*key_dim + value_dim); w: [C, 4];
    history: optional [3, C] rows preceding row 0 (`elementwise.cu:44-65`).
    acc = sum_j w[c, j] * x[t - 3 + j, c] in fp32; y = bf16(silu(bf16(acc))).
    """
    T, C = qkv.shape
    pad = np.zeros((3, C), np.float32) if history is None else history.astype(np.float32)
    xp = np.concatenate([pad, qkv.astype(np.float32)], 0)
    acc = np.zeros((T, C), np.float32)
    for j in range(4):
        acc = (acc + w[:, j].astype(np.float32)[None, :] * xp[j:j + T]).astype(np.float32)
    y = rnd(silu(rnd(acc)))
    return y[:, :key_dim], y[:, key_dim:2 * key_dim], y[:, 2 * key_dim:]


def gdn_gates(b, a, A_log, dt_bias):
    """beta = bf16(sigmoid(b)); g = -exp(A_log) * softplus(a + dt_bias) in fp32,
    softplus threshold 20 (`elementwise.cu:102-113`, `cs1_gdn_gates`)."""
    beta = rnd(sigmoid(b))
    x = (a.astype(np.float32) + dt_bias.astype(np.float32)[None, :]).astype(np.float32)
    sp = np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(np.float32)
    g = (-np.exp(A_log.astype(np.float32))[None, :] * sp).astype(np.float32)
    return beta, g


def rotate_half_rope(x, cos, sin, half):
    """Partial rotary on the first 2*half dims, products and sum rounded
    (`attention.cu:53-66`). x: [T, heads, Dh]; cos, sin: [T, half]."""
    y = x.copy()
    c = cos[:, None, :].astype(np.float32)
    s = sin[:, None, :].astype(np.float32)
    x1 = x[..., :half]
    x2 = x[..., half:2 * half]
    y[..., :half] = rnd(rnd(x1 * c) + rnd(-x2 * s))
    y[..., half:2 * half] = rnd(rnd(x2 * c) + rnd(x1 * s))
    return y


def attn_prep(qg, kr, qw, kw, cos, sin, Hq, Hk, Dh, half, eps):
    """Per-head RMSNorm(1+w) and partial RoPE, gate split (`attention.cu:27-77`).

    qg: [T, Hq*2*Dh] (query|gate per head); kr: [T, Hk*Dh].
    Returns q [T, Hq, Dh], gate [T, Hq*Dh], k [T, Hk, Dh].
    """
    T = qg.shape[0]
    qg = qg.reshape(T, Hq, 2 * Dh)
    q = rms_norm(qg[..., :Dh], qw, eps)
    gate = qg[..., Dh:].reshape(T, Hq * Dh).copy()
    k = rms_norm(kr.reshape(T, Hk, Dh), kw, eps)
    return rotate_half_rope(q, cos, sin, half), gate, rotate_half_rope(k, cos, sin, half)


def attention_gated(q, k, v, gate, scale, prefix_k=None, prefix_v=None):
    """Causal GQA attention with the sigmoid-gate epilogue (`attention.cu:90-258`).

    q: [S, Hq, Dh] suffix queries at absolute positions P..P+S-1 where P is the
    prefix length (0 without prefix); k, v: [S, Hk, Dh]; prefix_k/v: [P, Hk, Dh].
    Scores in fp32, softmax in float64 then probabilities rounded to bf16 for the
    P*V product (flash attention's bf16 P), output rounded, then
    bf16(bf16(att) * bf16(sigmoid(gate))).
    """
    S, Hq, Dh = q.shape
    Hk = k.shape[1]
    if prefix_k is not None:
        k = np.concatenate([prefix_k, k], 0)
        v = np.concatenate([prefix_v, v], 0)
    P = k.shape[0] - S
    out = np.zeros((S, Hq, Dh), np.float32)
    group = Hq // Hk
    pos_q = P + np.arange(S)
    mask = np.arange(P + S)[None, :] <= pos_q[:, None]
    for h in range(Hq):
        kh = h // group
        s = (q[:, h, :].astype(np.float32) @ k[:, kh, :].astype(np.float32).T) * np.float32(scale)
        s = np.where(mask, s.astype(np.float64), -np.inf)
        m = s.max(-1, keepdims=True)
        e = np.exp(s - m)
        p = e / e.sum(-1, keepdims=True)
        out[:, h, :] = (rnd(p.astype(np.float32)) @ v[:, kh, :].astype(np.float32))
    att = rnd(out)
    g = rnd(sigmoid(gate.reshape(S, Hq, Dh)))
    return rnd(att * g)


def gemm(x, w):
    """y = bf16(x @ w^T) with fp32 accumulation (`gemm.cu:318-463`, cs1_gemm)."""
    return rnd(np.asarray(x, np.float32) @ np.asarray(w, np.float32).T)


def silu_mul(gate_up, I):
    """out = bf16(bf16(silu(gate)) * up) (`elementwise.cu:124-131`)."""
    g = gate_up[:, :I].astype(np.float32)
    u = gate_up[:, I:2 * I].astype(np.float32)
    return rnd(rnd(silu(g)) * u)


def sigmoid_gate(x, gate):
    """x = bf16(x * bf16(sigmoid(gate))) (`elementwise.cu:116-121`)."""
    return rnd(x.astype(np.float32) * rnd(sigmoid(gate)))


def bf16_nonfinite(bits_u16):
    """cs1_bf16_finite flag: 1 if any bf16 pattern has an all-ones exponent
    (`elementwise.cu:147-152`)."""
    b = np.asarray(bits_u16, dtype=np.uint16)
    return int(((b & 0x7F80) == 0x7F80).any())
