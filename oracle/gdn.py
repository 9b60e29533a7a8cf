"""Chunked Gated DeltaNet in numpy (test infrastructure only).

Three restatements of the same recurrence

    S_t = exp(g_t) S_{t-1} + k_t (beta_t (v_t - exp(g_t) S_{t-1}^T k_t))^T,
    o_t = S_t^T q_t,            q, k L2-normalised, q scaled by `scale`,

with S [K=128, V=128] per value head and value head h reading key head
h // (H / HK):

* `chunk_fp32`  -- Transformers' `torch_chunk_gated_delta_rule`
  (modeling_qwen3_5.py:234-311 in transformers 5.5.0) in float32, chunks of 64:
  the within-chunk UT transform, then the chunk-by-chunk state scan. This is the
  arithmetic the reference's FP32 operator matches (`gdn_fp32.cu:1-3`).
* `chunk_bf16`  -- the reference's bfloat16 kernel (`gdn_prefill.cu:1-15`):
  the same chunk form with u, w, q*exp(cum), k*exp(last-cum), the decayed q.k
  products, the per-chunk state copy and v_new rounded to bfloat16, fp32 state.
* `recurrent_f64` -- the token-by-token float64 recurrence the reference's GPU
  test uses as its ground truth (`tests/qwen3_5/kernels.rs:1056-1102`).

Shapes: q, k [T, HK, 128]; v [T, H, 128]; g [T, H] float; beta [T, H];
state [H, 128, 128] indexed [head, key, value]. Returns (o [T, H, 128], state).
"""
import numpy as np

from .bf16 import rnd

C = 64


def _l2n(x, eps=1e-6):
    x = x.astype(np.float32)
    ss = (x * x).sum(-1, keepdims=True, dtype=np.float32)
    return (x * (np.float32(1) / np.sqrt(ss + np.float32(eps)))).astype(np.float32)


def l2norm_bf16(x, eps=1e-6):
    """Transformers' `l2norm` applied to bfloat16 tensors (modeling_qwen3_5.py:228-231
    runs before the float32 cast): x*x, the sum, rsqrt and the product each
    rounded to bfloat16."""
    x = rnd(x)
    ss = rnd(rnd(x * x).sum(-1, keepdims=True, dtype=np.float32))
    return rnd(x * rnd(np.float32(1) / np.sqrt(ss + np.float32(eps))))


def _expand(q, k, H):
    HK = q.shape[1]
    rep = H // HK
    return np.repeat(q, rep, axis=1), np.repeat(k, rep, axis=1)


def chunk_fp32(q, k, v, g, beta, scale, state=None, l2norm=True):
    """torch_chunk_gated_delta_rule restated (float32), with an optional initial
    state [H,K,V]; returns float32 o and the final float32 state. Third-party source:
    transformers `models/qwen3_5/modeling_qwen3_5.py:234-311` (5.5.0 here; the reference
    pins 5.17.0, `tests/qwen3_5/test_gdn_fp32.py:3,24`)."""
    T, H, D = v.shape
    q, k = _expand(q, k, H)
    if l2norm:
        q, k = _l2n(q), _l2n(k)
    q = (q.astype(np.float32) * np.float32(scale)).astype(np.float32)
    k = k.astype(np.float32)
    v = v.astype(np.float32)
    g = g.astype(np.float32)
    beta = beta.astype(np.float32)
    pad = (C - T % C) % C
    NC = (T + pad) // C
    def padt(x):
        return np.concatenate([x, np.zeros((pad,) + x.shape[1:], np.float32)], 0)
    q, k, v, g, beta = map(padt, (q, k, v, g, beta))
    # [H, NC, C, D]
    q = q.transpose(1, 0, 2).reshape(H, NC, C, -1)
    k = k.transpose(1, 0, 2).reshape(H, NC, C, -1)
    v = v.transpose(1, 0, 2).reshape(H, NC, C, -1)
    g = g.T.reshape(H, NC, C)
    beta = beta.T.reshape(H, NC, C)
    k_beta = k * beta[..., None]
    v_beta = v * beta[..., None]
    g = np.cumsum(g, -1, dtype=np.float32)
    diff = g[..., :, None] - g[..., None, :]
    tril = np.tril(np.ones((C, C), bool))
    decay = np.where(tril, np.exp(np.where(tril, diff, 0)), 0).astype(np.float32)
    A = -(k_beta @ k.swapaxes(-1, -2)) * decay
    A = np.where(np.tril(np.ones((C, C), bool), -1), A, 0).astype(np.float32)
    for i in range(1, C):
        row = A[..., i, :i].copy()
        sub = A[..., :i, :i].copy()
        A[..., i, :i] = row + (row[..., :, None] * sub).sum(-2)
    A = A + np.eye(C, dtype=np.float32)
    value = A @ v_beta
    k_cumdecay = A @ (k_beta * np.exp(g)[..., None])
    S = np.zeros((H, D, D), np.float32) if state is None else state.astype(np.float32).copy()
    out = np.zeros_like(value)
    strict = np.triu(np.ones((C, C), bool), 1)
    for c in range(NC):
        qi, ki, vi = q[:, c], k[:, c], value[:, c]
        attn = np.where(strict, 0, (qi @ ki.swapaxes(-1, -2)) * decay[:, c]).astype(np.float32)
        v_new = vi - k_cumdecay[:, c] @ S
        inter = (qi * np.exp(g[:, c])[..., None]) @ S
        out[:, c] = inter + attn @ v_new
        last = g[:, c, -1]
        S = S * np.exp(last)[:, None, None] + (ki * np.exp(last[:, None] - g[:, c])[..., None]).swapaxes(-1, -2) @ v_new
    o = out.reshape(H, NC * C, D)[:, :T].transpose(1, 0, 2)
    return o.astype(np.float32), S.astype(np.float32)


def tf32(x):
    """Round float32 to TF32 (10-bit mantissa), nearest with ties away from zero: the
    operand rounding of the reference's pair products (gdn_prefill.cu:197-198)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u.astype(np.uint64) + 0x1000) & 0xFFFFE000).astype(np.uint32)
    return r.view(np.float32)


def _inverse_unit_lower(A):
    """(I + A)^-1 for strictly lower-triangular A [.., C, C], float32."""
    n = A.shape[-1]
    Tm = np.zeros_like(A)
    eye = np.eye(n, dtype=np.float32)
    for r in range(n):
        # row r of T: e_r - sum_{j<r} A[r, j] T[j, :]
        Tm[..., r, :] = eye[r] - np.einsum('...j,...jk->...k', A[..., r, :r], Tm[..., :r, :])
    return Tm.astype(np.float32)


def chunk_bf16(q, k, v, g, beta, scale, state=None):
    """The reference's bfloat16-intermediate chunk kernel (`gdn_prefill.cu:113-547`).

    Per chunk and head: cum = sequential fp32 cumsum of g; kn, qn = L2-normalised k, q
    (q also scaled); A[i,j] = beta_i kn_i.kn_j exp(cum_i - cum_j) for j < i, with the
    pair products on TF32-rounded operands as the reference computes them;
    T = (I + A)^-1; u = bf16(bf16(T diag(beta)) v); w = bf16(bf16(T diag(beta)) bf16(kn e^cum));
    qd = bf16(qn e^cum); kd = bf16(kn e^(last - cum)); P = bf16(qn.kn e^(cum_i - cum_j)), j <= i.
    Scan: S_b = bf16(S); v_new = bf16(u - w S_b); o = bf16(qd S_b + P v_new);
    S = e^last S + kd^T v_new (fp32 state).
    """
    T, H, D = v.shape
    HK = q.shape[1]
    NC = (T + C - 1) // C
    o = np.zeros((T, H, D), np.float32)
    S_all = np.zeros((H, D, D), np.float32) if state is None else state.astype(np.float32).copy()
    for h in range(H):
        hk = h // (H // HK)
        S = S_all[h]
        for c in range(NC):
            t0, t1 = c * C, min(T, (c + 1) * C)
            n = t1 - t0
            gg = np.zeros(C, np.float32)
            gg[:n] = g[t0:t1, h]
            bb = np.zeros(C, np.float32)
            bb[:n] = beta[t0:t1, h]
            cum = np.cumsum(gg, dtype=np.float32)
            ecum = np.exp(cum).astype(np.float32)
            erem = np.exp(cum[-1] - cum).astype(np.float32)
            kk = np.zeros((C, D), np.float32)
            qq = np.zeros((C, D), np.float32)
            kk[:n] = k[t0:t1, hk]
            qq[:n] = q[t0:t1, hk]
            kinv = (np.float32(1) / np.sqrt((kk * kk).sum(-1, dtype=np.float32) + np.float32(1e-6))).astype(np.float32)
            qinv = (np.float32(1) / np.sqrt((qq * qq).sum(-1, dtype=np.float32) + np.float32(1e-6)) * np.float32(scale)).astype(np.float32)
            kn = kk * kinv[:, None]
            qn = qq * qinv[:, None]
            dec = np.exp(np.minimum(cum[:, None] - cum[None, :], 0)).astype(np.float32)
            lower = np.tril(np.ones((C, C), bool), -1)
            kt, qt = tf32(kn), tf32(qn)  # pair products take TF32 operands
            A = np.where(lower, bb[:, None] * (kt @ kt.T) * dec, 0).astype(np.float32)
            Tm = _inverse_unit_lower(A)
            tb = rnd(Tm * bb[None, :])
            vb = np.zeros((C, D), np.float32)
            vb[:n] = v[t0:t1, h]
            u = rnd(tb @ vb)
            w = rnd(tb @ rnd(kn * ecum[:, None]))
            qd = rnd(qn * ecum[:, None])
            kd = rnd(kn * erem[:, None])
            P = rnd(np.where(np.tril(np.ones((C, C), bool)), (qt @ kt.T) * dec, 0))
            Sb = rnd(S)
            v_new = rnd(u - w @ Sb)
            oc = rnd(qd @ Sb + P @ v_new)
            o[t0:t1, h] = oc[:n]
            S = (S * np.exp(cum[-1]) + kd.T @ v_new).astype(np.float32)
        S_all[h] = S
    return o, S_all


def recurrent_f64(q, k, v, g, beta, scale, state=None):
    """Token-by-token float64 recurrence (`tests/qwen3_5/kernels.rs:1056-1102`)."""
    T, H, D = v.shape
    HK = q.shape[1]
    S = np.zeros((H, D, D)) if state is None else state.astype(np.float64).copy()
    o = np.zeros((T, H, D))
    for h in range(H):
        hk = h // (H // HK)
        Sh = S[h]
        for t in range(T):
            kt = k[t, hk].astype(np.float64)
            qt = q[t, hk].astype(np.float64)
            kt = kt / np.sqrt((kt * kt).sum() + 1e-6)
            qt = qt / np.sqrt((qt * qt).sum() + 1e-6) * scale
            Sh = Sh * np.exp(float(g[t, h]))
            delta = (v[t, h].astype(np.float64) - Sh.T @ kt) * float(beta[t, h])
            Sh = Sh + np.outer(kt, delta)
            o[t, h] = Sh.T @ qt
        S[h] = Sh
    return o, S
