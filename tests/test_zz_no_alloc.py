"""cs1_gdn_prefill_noalloc: the chunked GDN prefill with its workspace in the library's
own fixed device array, for callers that cannot allocate device memory on the path where
they run the prefill.

Called through the C ABI twice in a row (a different input each time, so the second
call runs over the first call's leftover scratch) and checked against cs1_gdn_prefill
with a caller-owned workspace within the GDN gate of test_gdn_gpu.py (max |err| <= 2e-2 *
max |ref|): the no-alloc entry point runs the two-kernel form of the prefill (preparation,
then scan, through the fixed scratch), cs1_gdn_prefill the fused kernel, so their bits
differ. Repeating the first input after the second gives the first output bit for bit
(nothing of an earlier call leaks through the shared scratch). Also: the largest size the
fixed scratch holds (48 heads x 1,152 tokens) runs and matches, one token more is rejected
before any launch. This file is collected last so that a failure here stops a `-x` run
only after every other test has run; it also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

from helpers import dev_bf16, dev_f32, empty_bf16, host
from oracle import fixtures

pytestmark = pytest.mark.gpu
SCALE = 128 ** -0.5


def _inputs(T, H, HK, seed):
    return fixtures.grouped_inputs(seed, T, H, HK)


def _with_workspace(cs1, stream, q, k, v, g, beta, H, HK):
    T = v.shape[0]
    ws = torch.empty(cs1.cs1_gdn_workspace_floats(T, H), dtype=torch.float32, device="cuda")
    o = empty_bf16(T, H, 128)
    cs1.cs1_gdn_prefill(dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta), o, ws, T, H, HK, SCALE,
                        stream)
    return host(o)


def _noalloc(cs1, stream, q, k, v, g, beta, H, HK):
    T = v.shape[0]
    o = empty_bf16(T, H, 128)
    # keep the device inputs alive until the call has run on the stream
    dq, dk, dv, dg, db = dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta)
    rc = cs1.raw.cs1_gdn_prefill_noalloc(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                         o.data_ptr(), T, H, HK, SCALE, stream)
    assert rc == 0
    got = host(o)
    assert cs1.cs1_fault_status(1) == 0
    return got


def test_noalloc_matches_caller_workspace_twice(cs1, stream):
    H, HK = 48, 16
    outs = []
    for T, seed in ((700, 1), (333, 2)):
        q, k, v, g, beta = _inputs(T, H, HK, seed)
        ref = _with_workspace(cs1, stream, q, k, v, g, beta, H, HK)
        got = _noalloc(cs1, stream, q, k, v, g, beta, H, HK)
        assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max(), (T, np.abs(got - ref).max())
        outs.append(got)
    again = _noalloc(cs1, stream, *_inputs(700, H, HK, 1), H, HK)
    assert np.array_equal(again, outs[0])


def test_noalloc_largest_size_runs_and_one_token_more_is_rejected(cs1, stream):
    """ceil(T / 64) * H <= 910 fits the 64 MiB scratch: T = 1,152 at 48 heads (18 chunks)
    runs and matches cs1_gdn_prefill; T = 1,153 (19 chunks) is refused before any launch."""
    H, HK, T = 48, 16, 1152
    q, k, v, g, beta = _inputs(T, H, HK, 3)
    ref = _with_workspace(cs1, stream, q, k, v, g, beta, H, HK)
    dq, dk, dv, dg, db = dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta)
    o = empty_bf16(T, H, 128)
    assert cs1.raw.cs1_gdn_prefill_noalloc(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                           o.data_ptr(), T, H, HK, SCALE, stream) == 0
    got = host(o)
    assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()
    sentinel = torch.full((T + 1, H, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    big = [torch.zeros((T + 1) * n, dtype=dt, device="cuda") for n, dt in
           ((HK * 128, torch.bfloat16), (HK * 128, torch.bfloat16), (H * 128, torch.bfloat16), (H, torch.float32),
            (H, torch.bfloat16))]
    rc = cs1.raw.cs1_gdn_prefill_noalloc(*[b.data_ptr() for b in big], sentinel.data_ptr(), T + 1, H, HK, SCALE,
                                         stream)
    assert rc != 0
    torch.cuda.synchronize()
    assert bool((sentinel == 7.0).all())  # nothing was launched
    assert cs1.cs1_fault_status(1) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch(cs1, stream):
    p = torch.empty(16, dtype=torch.bfloat16, device="cuda").data_ptr()
    # 48 heads x 64 chunks needs about 226 MB of workspace, above the 64 MiB scratch
    assert cs1.raw.cs1_gdn_prefill_noalloc(p, p, p, p, p, p, 4096, 48, 16, SCALE, stream) != 0
    assert cs1.raw.cs1_gdn_prefill_noalloc(p, p, p, p, p, p, 64, 48, 5, SCALE, stream) != 0
