"""GPU parity of the bandwidth-bound cs1_* operations against the numpy oracle.

Tolerance: the kernels and the oracle round at the same points but may sum in a
different order, so a bf16 result may differ by one unit in the last place:
max |gpu - oracle| <= 2^-7 * max|oracle| (one bf16 ulp at the largest magnitude),
except where the arithmetic is identical (embed, copies: bit-exact).
"""
import numpy as np
import pytest
import torch

from helpers import dev_bf16, dev_f32, empty_bf16, host, max_rel
from oracle import ops
from oracle.bf16 import rnd
from oracle.packing import rotary_tables

pytestmark = pytest.mark.gpu
ULP = 2.0 ** -7


def _r(shape, seed, scale=1.0):
    return rnd(np.random.default_rng(seed).standard_normal(shape).astype(np.float32) * np.float32(scale))


def test_embed(cs1, stream):
    table = _r((1000, 256), 1)
    ids = np.random.default_rng(2).integers(0, 1000, 77).astype(np.int32)
    out = empty_bf16(77, 256)
    cs1.cs1_embed(torch.from_numpy(ids).cuda(), dev_bf16(table), out, 77, 256, stream)
    assert np.array_equal(host(out), ops.embed(ids, table))


# D up to 5,120 takes the warp-per-row kernel with rows staged in shared memory (3,000 rows:
# several rows per warp, so every slot is refilled), 8,192 the CTA-per-row kernel, 100 and 72
# (not multiples of 8) the scalar one
@pytest.mark.parametrize("rows,D", [(33, 256), (33, 2560), (3000, 2560), (33, 4096), (33, 5120), (33, 8192),
                                    (33, 100)])
def test_rms_norm(cs1, stream, rows, D):
    x, w = _r((rows, D), 3), _r((D,), 4, 0.1)
    out = empty_bf16(rows, D)
    cs1.cs1_rms_norm(dev_bf16(x), dev_bf16(w), out, rows, D, 1e-6, stream)
    assert max_rel(host(out), ops.rms_norm(x, w, 1e-6)) <= ULP


@pytest.mark.parametrize("rows,D", [(20, 2560), (3000, 2560), (20, 5120), (20, 8192), (20, 72)])
def test_add_rms_norm(cs1, stream, rows, D):
    r, d, w = _r((rows, D), 5), _r((rows, D), 6), _r((D,), 7, 0.1)
    res = dev_bf16(r)
    out = empty_bf16(rows, D)
    cs1.cs1_add_rms_norm(res, dev_bf16(d), dev_bf16(w), out, rows, D, 1e-6, stream)
    er, eo = ops.add_rms_norm(r, d, w, 1e-6)
    assert np.array_equal(host(res), er)
    assert max_rel(host(out), eo) <= ULP


def test_gated_rms_norm(cs1, stream):
    T, H = 37, 6
    x, z, w = _r((T, H, 128), 8), _r((T, H * 128 + 40), 9), _r((128,), 10, 0.1) + 1
    out = empty_bf16(T, H * 128)
    cs1.cs1_gated_rms_norm(dev_bf16(x), dev_bf16(z), H * 128 + 40, dev_bf16(rnd(w)), out, T, H, 128, 1e-6, stream)
    assert max_rel(host(out), ops.gated_rms_norm(x, z[:, :H * 128], rnd(w), 1e-6)) <= ULP


@pytest.mark.parametrize("lengths", [[70], [1, 2, 3, 64, 65], [300, 5]])
@pytest.mark.parametrize("with_history", [False, True])
def test_gdn_conv_batch(cs1, stream, lengths, with_history):
    kd, vd, ld = 256, 512, 1544
    C = 2 * kd + vd
    T = sum(lengths)
    qkv = _r((T, ld), 11)
    w = rnd(np.random.default_rng(12).uniform(-0.5, 0.5, (C, 4)).astype(np.float32))
    hist = _r((3, ld), 13) if with_history else None
    q, k, v = empty_bf16(T, kd), empty_bf16(T, kd), empty_bf16(T, vd)
    lens = np.asarray(lengths, dtype=np.uintp)
    cs1.cs1_gdn_conv_batch(dev_bf16(qkv), dev_bf16(hist) if with_history else None, ld, dev_bf16(w), q, k, v,
                           lens.ctypes.data, len(lengths), kd, vd, stream)
    off = 0
    got = [host(q), host(k), host(v)]
    for n in lengths:
        eq, ek, ev = ops.gdn_conv(qkv[off:off + n, :C], w, kd, vd, history=hist[:, :C] if with_history else None)
        for g, e in zip(got, (eq, ek, ev)):
            assert max_rel(g[off:off + n], e) <= ULP
        off += n


# Channel layouts of the conv kernel: 128 packs of 4 channels per CTA, so (128, 192) leaves the
# last CTA part-filled (lanes past the last pack keep the staged ring's counts), (8, 16) is a
# single small CTA, and (4, 4) (channel counts not multiples of 8) takes the scalar kernel.
@pytest.mark.parametrize("kd,vd", [(128, 192), (8, 16), (4, 4)])
@pytest.mark.parametrize("with_history", [False, True])
def test_gdn_conv_channel_layouts(cs1, stream, kd, vd, with_history):
    lengths = [150, 1, 77]
    C = 2 * kd + vd
    ld = C + 8
    T = sum(lengths)
    qkv = _r((T, ld), 14)
    w = rnd(np.random.default_rng(15).uniform(-0.5, 0.5, (C, 4)).astype(np.float32))
    hist = _r((3, ld), 16) if with_history else None
    q, k, v = empty_bf16(T, kd), empty_bf16(T, kd), empty_bf16(T, vd)
    lens = np.asarray(lengths, dtype=np.uintp)
    assert cs1.cs1_gdn_conv_batch(dev_bf16(qkv), dev_bf16(hist) if with_history else None, ld, dev_bf16(w), q, k,
                                  v, lens.ctypes.data, len(lengths), kd, vd, stream) == 0
    off = 0
    got = [host(q), host(k), host(v)]
    for n in lengths:
        eq, ek, ev = ops.gdn_conv(qkv[off:off + n, :C], w, kd, vd, history=hist[:, :C] if with_history else None)
        for g, e in zip(got, (eq, ek, ev)):
            assert max_rel(g[off:off + n], e) <= ULP
        off += n
    assert cs1.cs1_fault_status(1) == 0


def test_gdn_conv_single_and_prefix_entry_points(cs1, stream):
    kd, vd, T = 128, 256, 90
    ld = 2 * kd + vd + 24
    qkv, hist = _r((T, ld), 14), _r((3, ld), 15)
    w = rnd(np.random.default_rng(16).uniform(-0.5, 0.5, (2 * kd + vd, 4)).astype(np.float32))
    for name, h in (("cs1_gdn_conv", None), ("cs1_gdn_conv_vector", None), ("cs1_gdn_conv_prefix", hist)):
        q, k, v = empty_bf16(T, kd), empty_bf16(T, kd), empty_bf16(T, vd)
        if h is None:
            getattr(cs1, name)(dev_bf16(qkv), ld, dev_bf16(w), q, k, v, T, kd, vd, stream)
        else:
            cs1.cs1_gdn_conv_prefix(dev_bf16(qkv), dev_bf16(h), ld, dev_bf16(w), q, k, v, T, kd, vd, stream)
        eq, ek, ev = ops.gdn_conv(qkv[:, :2 * kd + vd], w, kd, vd, history=None if h is None else h[:, :2 * kd + vd])
        assert max_rel(host(q), eq) <= ULP and max_rel(host(k), ek) <= ULP and max_rel(host(v), ev) <= ULP


def test_gdn_gates(cs1, stream):
    T, H, ld = 50, 48, 100
    ba = _r((T, ld), 17, 3.0)
    A_log = rnd(np.log(np.random.default_rng(18).uniform(1, 16, H)).astype(np.float32))
    dt = rnd(1 + 0.1 * np.random.default_rng(19).standard_normal(H).astype(np.float32))
    beta = empty_bf16(T, H)
    g = torch.empty(T, H, dtype=torch.float32, device="cuda")
    src = dev_bf16(ba)
    cs1.cs1_gdn_gates(src, src[:, H:], ld, dev_bf16(A_log), dev_bf16(dt), beta, g, T, H, stream)
    eb, eg = ops.gdn_gates(ba[:, :H], ba[:, H:2 * H], A_log, dt)
    assert max_rel(host(beta), eb) <= ULP
    assert np.allclose(host(g), eg, rtol=2e-6, atol=1e-7)


def test_silu_mul_and_sigmoid_gate(cs1, stream):
    T, I = 40, 1024
    gu = _r((T, 2 * I + 16), 20, 2.0)
    out = empty_bf16(T, I)
    cs1.cs1_silu_mul(dev_bf16(gu), 2 * I + 16, out, T, I, stream)
    assert max_rel(host(out), ops.silu_mul(gu, I)) <= ULP
    x, gate = _r((1000,), 21), _r((1000,), 22)
    xd = dev_bf16(x)
    cs1.cs1_sigmoid_gate(xd, dev_bf16(gate), 1000, stream)
    assert max_rel(host(xd), ops.sigmoid_gate(x, gate)) <= ULP


def _ordered(b):
    """bf16 bit patterns -> integers in value order (+0 and -0 both 0), so that the
    difference of two is their distance in bf16 ulps."""
    b = b.astype(np.int32)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def test_silu_every_bf16_value(cs1, stream):
    """cs1_silu_mul with up = 1 over every finite bf16 gate value, element by element,
    against PyTorch's float32 SiLU rounded to bf16. The kernels' SiLU, x * rcp(1 + 2^(-x
    log2 e)) on the hardware exp2 / reciprocal approximations, is within one bf16 ulp
    everywhere except below -87.34, where 1 + e^-x exceeds 2^126, the flush-to-zero
    reciprocal returns 0 and the result is a signed zero in place of a value of magnitude
    below 1.1e-36."""
    bits = np.arange(65536, dtype=np.uint32)
    g = (bits << 16).view(np.float32)
    g = g[np.isfinite(g)]
    I = 256
    T = (g.size + I - 1) // I
    gate = np.zeros(T * I, np.float32)
    gate[:g.size] = g
    gu = np.concatenate([gate.reshape(T, I), np.ones((T, I), np.float32)], axis=1)
    out = empty_bf16(T, I)
    cs1.cs1_silu_mul(dev_bf16(gu), 2 * I, out, T, I, stream)
    torch.cuda.synchronize()
    got = out.reshape(-1)[:g.size].cpu().view(torch.int16).numpy().view(np.uint16)
    want = torch.nn.functional.silu(torch.from_numpy(g)).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    dist = np.abs(_ordered(got) - _ordered(want))
    tail = g < -87.34
    assert dist[~tail].max() <= 1
    assert np.all((got[tail] & 0x7FFF) == 0)
    wv = (want[tail].astype(np.uint32) << 16).view(np.float32)
    assert np.abs(wv).max() < 1.1e-36
    assert np.mean(dist[~tail] == 0) > 0.99


@pytest.mark.parametrize("T,Hq,Hk", [(1, 4, 2), (70, 24, 4), (300, 16, 4)])
def test_attn_prep(cs1, stream, T, Hq, Hk):
    ld = Hq * 512 + 2 * Hk * 256
    qkv = _r((T, ld), 23, 2.0)
    qw, kw = _r((256,), 24, 0.1), _r((256,), 25, 0.1)
    cos, sin = rotary_tables(np.arange(5, 5 + T), 32, 1e7)
    q, gate, k = empty_bf16(T, Hq, 256), empty_bf16(T, Hq * 256), empty_bf16(T, Hk, 256)
    src = dev_bf16(qkv)
    cs1.cs1_attn_prep(src, src[:, Hq * 512:], ld, dev_bf16(qw), dev_bf16(kw), dev_bf16(cos), dev_bf16(sin), q, gate,
                      k, T, Hq, Hk, 256, 32, 1e-6, stream)
    eq, eg, ek = ops.attn_prep(qkv[:, :Hq * 512], qkv[:, Hq * 512:Hq * 512 + Hk * 256], qw, kw, cos, sin, Hq, Hk,
                               256, 32, 1e-6)
    assert max_rel(host(q), eq) <= 2 * ULP
    assert np.array_equal(host(gate), eg)
    assert max_rel(host(k), ek) <= 2 * ULP


def test_head_score(cs1, stream):
    H, L, n = 2560, 8, 5
    hidden = _r((40, H), 26)
    W = np.random.default_rng(27).standard_normal((L, H)).astype(np.float32) * 0.02
    b = np.random.default_rng(28).standard_normal(L).astype(np.float32) * 0.02
    rows = np.asarray([0, 7, 13, 30, 39], np.int32)
    logits = torch.empty(n, L, dtype=torch.float32, device="cuda")
    cs1.cs1_head_score(dev_bf16(hidden), H, torch.from_numpy(rows).cuda(), n, dev_f32(W), dev_f32(b), L, H, logits,
                       stream)
    s = (hidden[rows].astype(np.float64) @ W.astype(np.float64).T).astype(np.float32) + b[None]
    assert np.allclose(host(logits), s, rtol=1e-6, atol=1e-6)


def test_bf16_finite_flag(cs1, stream):
    x = torch.zeros(1000, dtype=torch.bfloat16, device="cuda")
    flag = torch.ones(1, dtype=torch.int32, device="cuda")
    cs1.cs1_bf16_finite(x, 1000, flag, stream)
    assert int(host(flag)[0]) == 0
    x[777] = float("inf")
    cs1.cs1_bf16_finite(x, 1000, flag, stream)
    assert int(host(flag)[0]) == 1


def test_invalid_shapes_are_rejected_before_launch(cs1, stream):
    p = torch.empty(1024, dtype=torch.bfloat16, device="cuda").data_ptr()
    assert cs1.raw.cs1_gated_rms_norm(p, p, 10, p, p, 4, 2, 64, 1e-6, stream) != 0
    assert cs1.raw.cs1_gdn_conv(p, 8, p, p, p, p, 4, 8, 8, stream) != 0
    assert cs1.raw.cs1_attn_prep(p, p, 512, p, p, p, p, p, p, p, 4, 1, 1, 128, 32, 1e-6, stream) != 0
    assert cs1.raw.cs1_embed(p, p, p, 4, 7, stream) != 0
    assert cs1.raw.cs1_silu_mul(p, 4, p, 2, 8, stream) != 0


def test_bounded_wait_gives_up_and_reports(cs1, stream):
    """The kernels' bounded mbarrier wait, cut to ~1 ms and made to run out on a barrier
    that nothing completes (no copy or MMA in flight): the kernel returns, the fault word
    reports bit 8, clearing it works, and the context stays usable."""
    import torch
    assert cs1.cs1_fault_status(1) == 0
    cs1.cs1_wait_selftest(2_000_000, stream)
    torch.cuda.synchronize()
    assert cs1.cs1_fault_status(0) == 8
    assert cs1.cs1_fault_status(1) == 8  # read and clear
    assert cs1.cs1_fault_status(0) == 0
    x = torch.arange(8, dtype=torch.float32, device="cuda")
    assert float((x * 2).sum()) == 56.0
    assert cs1.raw.cs1_wait_selftest(10, stream) != 0  # limits outside 1e3 .. 4e9 are refused
