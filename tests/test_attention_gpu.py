"""GPU parity of the gated GQA flash attention (head dim 256) against the oracle.

Gate: row-relative max error <= 1.6e-2 against the oracle's float64 softmax with
bf16 probabilities (the reference's attention test gate, tests/qwen3_5/kernels.rs:712-817).
Packed, windowed and shared-prefix variants must equal the single-sequence pass bit
for bit (same key tiles, same online-softmax order).
"""
import numpy as np
import pytest
import torch

from helpers import dev_bf16, empty_bf16, host
from oracle import ops
from oracle.bf16 import rnd

pytestmark = pytest.mark.gpu
SCALE = 256 ** -0.5


def _qkv(T, Hq, Hk, seed, ldv_extra=64):
    rng = np.random.default_rng(seed)
    q = rnd(rng.standard_normal((T, Hq, 256)).astype(np.float32))
    k = rnd(rng.standard_normal((T, Hk, 256)).astype(np.float32))
    ldv = Hk * 256 + ldv_extra
    vfull = rnd(rng.standard_normal((T, ldv)).astype(np.float32))
    gate = rnd(rng.standard_normal((T, Hq * 256)).astype(np.float32))
    return q, k, vfull, ldv, gate


def _row_rel(a, b):
    a = a.reshape(a.shape[0], -1).astype(np.float64)
    b = b.reshape(b.shape[0], -1).astype(np.float64)
    return float((np.abs(a - b).max(1) / np.maximum(np.abs(b).max(1), 1e-30)).max())


@pytest.mark.parametrize("T,Hq,Hk", [(1, 4, 2), (63, 4, 2), (65, 16, 4), (139, 4, 1), (700, 24, 4), (2048, 4, 2),
                                     (300, 6, 2), (130, 3, 3)])
def test_attention_gated_matches_oracle(cs1, stream, T, Hq, Hk):
    q, k, vfull, ldv, gate = _qkv(T, Hq, Hk, T)
    out = empty_bf16(T, Hq, 256)
    cs1.cs1_attention_gated(dev_bf16(q), dev_bf16(k), dev_bf16(vfull), ldv, dev_bf16(gate), out, T, Hq, Hk, 256, SCALE,
                            stream)
    v = vfull[:, :Hk * 256].reshape(T, Hk, 256)
    ref = ops.attention_gated(q, k, v, gate, SCALE)
    assert _row_rel(host(out), ref) <= 1.6e-2


def test_attention_ungated_and_bidirectional(cs1, stream):
    T, Hq, Hk = 100, 4, 2
    q, k, vfull, ldv, gate = _qkv(T, Hq, Hk, 3)
    v = vfull[:, :Hk * 256].reshape(T, Hk, 256)
    out = empty_bf16(T, Hq, 256)
    cs1.cs1_attention(dev_bf16(q), dev_bf16(k), dev_bf16(vfull), ldv, out, T, Hq, Hk, 256, SCALE, stream)
    one = np.full((T, Hq * 256), 1e4, np.float32)  # sigmoid == 1: the ungated result
    assert _row_rel(host(out), ops.attention_gated(q, k, v, rnd(one), SCALE)) <= 1.6e-2
    # bidirectional: every query reads every key
    cs1.cs1_attention_gated_bidirectional(dev_bf16(q), dev_bf16(k), dev_bf16(vfull), ldv, dev_bf16(gate), out, T, Hq,
                                          Hk, 256, SCALE, stream)
    S = np.einsum("thd,skd->htsk", q.astype(np.float64), k.astype(np.float64))
    ref = np.zeros((T, Hq, 256))
    for h in range(Hq):
        s = S[h, :, :, h // (Hq // Hk)] * SCALE
        p = np.exp(s - s.max(1, keepdims=True))
        p = rnd((p / p.sum(1, keepdims=True)).astype(np.float32))
        ref[:, h] = p @ v[:, h // (Hq // Hk)]
    ref = rnd(rnd(ref.astype(np.float32)) * rnd(ops.sigmoid(gate.reshape(T, Hq, 256))))
    assert _row_rel(host(out), ref) <= 1.6e-2


@pytest.mark.parametrize("lengths", [[1, 63, 64, 65, 129], [1] * 16, [300, 7]])
def test_attention_batch_equals_single(cs1, stream, lengths):
    Hq, Hk = 8, 2
    T = sum(lengths)
    q, k, vfull, ldv, gate = _qkv(T, Hq, Hk, 11)
    out = empty_bf16(T, Hq, 256)
    lens = np.asarray(lengths, dtype=np.uintp)
    Q, K_, V_, Gt = dev_bf16(q), dev_bf16(k), dev_bf16(vfull), dev_bf16(gate)
    cs1.cs1_attention_gated_batch(Q, K_, V_, ldv, Gt, out, lens.ctypes.data, len(lengths), Hq, Hk, 256, SCALE, stream)
    got = host(out)
    off = 0
    for n in lengths:
        one = empty_bf16(n, Hq, 256)
        cs1.cs1_attention_gated(Q[off:], K_[off:], V_[off:], ldv, Gt[off:], one, n, Hq, Hk, 256, SCALE, stream)
        assert np.array_equal(host(one), got[off:off + n])
        off += n


def test_attention_shared_prefix_equals_full_pass(cs1, stream):
    Hq, Hk, P = 4, 2, 192
    lengths = [1, 40, 130]
    T = P + max(lengths)
    q, k, vfull, ldv, gate = _qkv(T, Hq, Hk, 21)
    Q, K_, V_, Gt = dev_bf16(q), dev_bf16(k), dev_bf16(vfull), dev_bf16(gate)
    pk = dev_bf16(k[:P])
    pv = dev_bf16(vfull[:P, :Hk * 256])
    # suffixes packed: each continues the same prefix
    sq = np.concatenate([q[P:P + n] for n in lengths])
    sk = np.concatenate([k[P:P + n] for n in lengths])
    sv = np.concatenate([vfull[P:P + n] for n in lengths])
    sg = np.concatenate([gate[P:P + n] for n in lengths])
    out = empty_bf16(sum(lengths), Hq, 256)
    lens = np.asarray(lengths, dtype=np.uintp)
    cs1.cs1_attention_gated_shared_batch(dev_bf16(sq), dev_bf16(sk), dev_bf16(sv), ldv, dev_bf16(sg), out, pk, pv,
                                         lens.ctypes.data, len(lengths), P, Hq, Hk, 256, SCALE, stream)
    got = host(out)
    off = 0
    for n in lengths:
        full = empty_bf16(P + n, Hq, 256)
        cs1.cs1_attention_gated(Q, K_, V_, ldv, Gt, full, P + n, Hq, Hk, 256, SCALE, stream)
        assert np.array_equal(got[off:off + n], host(full)[P:P + n])
        one = empty_bf16(n, Hq, 256)
        cs1.cs1_attention_gated_shared(Q[P:], K_[P:], V_[P:], ldv, Gt[P:], one, pk, pv, n, P, Hq, Hk, 256, SCALE,
                                       stream)
        assert np.array_equal(host(one), got[off:off + n])
        off += n


def test_attention_window_equals_full_pass(cs1, stream):
    T, Hq, Hk, qb = 300, 4, 2, 128
    q, k, vfull, ldv, gate = _qkv(T, Hq, Hk, 31)
    Q, K_, V_, Gt = dev_bf16(q), dev_bf16(k), dev_bf16(vfull), dev_bf16(gate)
    full = empty_bf16(T, Hq, 256)
    cs1.cs1_attention_gated(Q, K_, V_, ldv, Gt, full, T, Hq, Hk, 256, SCALE, stream)
    win = torch.zeros(T, Hq, 256, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_attention_gated_prefix(Q, K_, V_, ldv, Gt, win, T, Hq, Hk, 256, SCALE, qb, stream)
    assert np.array_equal(host(win)[qb:], host(full)[qb:])
    assert not host(win)[:qb].any()
    assert cs1.raw.cs1_attention_gated_prefix(Q.data_ptr(), K_.data_ptr(), V_.data_ptr(), ldv, Gt.data_ptr(),
                                              win.data_ptr(), T, Hq, Hk, 256, SCALE, 100, stream) != 0


def test_attention_prefix_bidirectional(cs1, stream):
    T, Hq, Hk, state = 90, 4, 2, 33
    q, k, vfull, ldv, gate = _qkv(T, Hq, Hk, 41)
    Q, K_, V_, Gt = dev_bf16(q), dev_bf16(k), dev_bf16(vfull), dev_bf16(gate)
    out = empty_bf16(T, Hq, 256)
    cs1.cs1_attention_gated_prefix_bidirectional(Q, K_, V_, ldv, Gt, out, T, state, Hq, Hk, 256, SCALE, stream)
    bid = empty_bf16(T, Hq, 256)
    cs1.cs1_attention_gated_bidirectional(Q, K_, V_, ldv, Gt, bid, T, Hq, Hk, 256, SCALE, stream)
    st = empty_bf16(state, Hq, 256)
    cs1.cs1_attention_gated_bidirectional(Q, K_, V_, ldv, Gt, st, state, Hq, Hk, 256, SCALE, stream)
    got = host(out)
    assert np.array_equal(got[state:], host(bid)[state:])
    assert np.array_equal(got[:state], host(st))


def test_attention_growing_scores_rescale(cs1, stream):
    """Keys whose norm grows along the sequence: each row's running maximum keeps rising
    over the key tiles, so the deferred rescale of the output accumulator is exercised."""
    T, Hq, Hk = 700, 4, 2
    q, k, vfull, ldv, gate = _qkv(T, Hq, Hk, 51)
    k = rnd((k * np.linspace(0.1, 4.0, T, dtype=np.float32)[:, None, None]).astype(np.float32))
    out = empty_bf16(T, Hq, 256)
    cs1.cs1_attention_gated(dev_bf16(q), dev_bf16(k), dev_bf16(vfull), ldv, dev_bf16(gate), out, T, Hq, Hk, 256, SCALE,
                            stream)
    v = vfull[:, :Hk * 256].reshape(T, Hk, 256)
    assert _row_rel(host(out), ops.attention_gated(q, k, v, gate, SCALE)) <= 1.6e-2


def test_attention_long_gqa6(cs1, stream):
    """27B head grouping (6 query heads per key head) over 12 key tiles."""
    T, Hq, Hk = 1500, 6, 1
    q, k, vfull, ldv, gate = _qkv(T, Hq, Hk, 61)
    out = empty_bf16(T, Hq, 256)
    cs1.cs1_attention_gated(dev_bf16(q), dev_bf16(k), dev_bf16(vfull), ldv, dev_bf16(gate), out, T, Hq, Hk, 256, SCALE,
                            stream)
    v = vfull[:, :Hk * 256].reshape(T, Hk, 256)
    assert _row_rel(host(out), ops.attention_gated(q, k, v, gate, SCALE)) <= 1.6e-2
    assert cs1.cs1_fault_status(1) == 0
