"""The fused GDN front end (cs1_gdn_front_batch): the causal conv + SiLU of q, k, v, the
inverse L2 norms of q and k per (row, head) and the gates, in one launch.

q, k, v, beta and g equal cs1_gdn_conv_batch + cs1_gdn_gates bit for bit (the same
arithmetic, one launch); the inverse norms equal 1 / sqrt(sum y^2 + 1e-6) over the bf16
outputs of each head, computed in float64, within 2 float32 ulps (the reduction order
differs); and the prefill fed with those norms (cs1_gdn_prefill_batch_xn) stays within the
GDN gate of the float64 recurrence, as the prefill with its own norms does."""
import ctypes

import numpy as np
import pytest
import torch

from helpers import dev_bf16, dev_f32, empty_bf16, host
from oracle import fixtures
from oracle import gdn as G

pytestmark = pytest.mark.gpu


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("kd,vd,H,lens", [(2048, 6144, 48, [37, 100, 5, 64]), (256, 512, 4, [1, 63, 200]),
                                          (2048, 4096, 32, [771])])
def test_front_equals_conv_and_gates(cs1, stream, kd, vd, H, lens):
    T = sum(lens)
    ld = 2 * kd + vd + vd + 2 * H  # [q | k | v | z | b | a], as the GDN input projection
    qkv, w = _rand((T, ld), 1), _rand((2 * kd + vd, 4), 2, 0.3)
    A_log, dt = _rand((H,), 3, 0.5), _rand((H,), 4, 0.5)
    boff = (2 * kd + 2 * vd) * 2
    arr = np.asarray(lens, dtype=np.uintp)
    outs = []
    for fused in (False, True):
        q, k, v = empty_bf16(T, kd), empty_bf16(T, kd), empty_bf16(T, vd)
        beta, g = empty_bf16(T, H), torch.empty(T, H, device="cuda")
        rq, rk = torch.empty(T, kd // 128, device="cuda"), torch.empty(T, kd // 128, device="cuda")
        if fused:
            assert cs1.raw.cs1_gdn_front_batch(qkv.data_ptr(), None, ld, w.data_ptr(), q.data_ptr(), k.data_ptr(),
                                               v.data_ptr(), rq.data_ptr(), rk.data_ptr(), qkv.data_ptr() + boff,
                                               qkv.data_ptr() + boff + H * 2, A_log.data_ptr(), dt.data_ptr(),
                                               beta.data_ptr(), g.data_ptr(), H, arr.ctypes.data, len(lens), kd, vd,
                                               stream) == 0
        else:
            assert cs1.raw.cs1_gdn_conv_batch(qkv.data_ptr(), None, ld, w.data_ptr(), q.data_ptr(), k.data_ptr(),
                                              v.data_ptr(), arr.ctypes.data, len(lens), kd, vd, stream) == 0
            assert cs1.raw.cs1_gdn_gates(qkv.data_ptr() + boff, qkv.data_ptr() + boff + H * 2, ld, A_log.data_ptr(),
                                         dt.data_ptr(), beta.data_ptr(), g.data_ptr(), T, H, stream) == 0
        torch.cuda.synchronize()
        outs.append((q, k, v, beta, g, rq, rk))
    for a, b in zip(outs[0][:5], outs[1][:5]):
        assert torch.equal(a, b)
    q, k, rq, rk = outs[1][0], outs[1][1], outs[1][5], outs[1][6]
    for x, r in ((q, rq), (k, rk)):
        xf = host(x).astype(np.float64).reshape(T, -1, 128)
        want = 1.0 / np.sqrt((xf * xf).sum(-1) + 1e-6)
        got = host(r).astype(np.float64)
        assert np.abs(got - want).max() <= 2 * 2.0 ** -23 * want.max(), np.abs(got - want).max()
    assert cs1.cs1_fault_status(1) == 0


@pytest.mark.parametrize("T,H,HK", [(700, 48, 16), (65, 4, 2)])
def test_prefill_with_front_norms_meets_the_gdn_gate(cs1, stream, T, H, HK):
    q, k, v, g, beta = fixtures.grouped_inputs(T, T, H, HK)
    scale = 128 ** -0.5
    ref, _ = G.recurrent_f64(q, k, v, g, beta, scale)
    dq, dk, dv, dg, db = dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta)
    kf = torch.from_numpy(np.asarray(k, np.float64)).reshape(T, HK, 128)
    qf = torch.from_numpy(np.asarray(q, np.float64)).reshape(T, HK, 128)
    rnk = (1.0 / torch.sqrt((kf ** 2).sum(-1) + 1e-6)).float().cuda().contiguous()
    rnq = (1.0 / torch.sqrt((qf ** 2).sum(-1) + 1e-6)).float().cuda().contiguous()
    o = empty_bf16(T, H, 128)
    arr = np.asarray([T], dtype=np.uintp)
    assert cs1.raw.cs1_gdn_prefill_batch_xn(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                            rnq.data_ptr(), rnk.data_ptr(), o.data_ptr(), arr.ctypes.data, 1, H, HK,
                                            ctypes.c_float(scale), None, 0, None, stream) == 0
    got = host(o)
    assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()
    assert cs1.cs1_fault_status(1) == 0
