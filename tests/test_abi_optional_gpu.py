"""The reference's optional ABI symbols that the C++ host does not call itself, against the
entry points they stand beside (ops.h:123, 196-215 of the reference):

* `cs1_gemm_create_matched`, `cs1_gemm_compatible`, `cs1_gemm_enable_equivalent_tiles`,
  `cs1_gemm_reuse_check`, `cs1_gemm_reuse`: the reference's "recompute these rows exactly as
  an M = original_M call would" path. This build's GEMMs give every row the same bits for
  any M (the K reduction order does not depend on M or on the kernel chosen), so every handle
  is compatible, every reuse is supported, and `cs1_gemm_reuse` rows equal, bit for bit, the
  same rows of a plain `cs1_gemm` over original_M rows.
* `cs1_gdn_prefill_wide`: the same operator as `cs1_gdn_prefill`, identical bits.
"""
import numpy as np
import pytest
import torch

from oracle import fixtures
from oracle.bf16 import rnd

from helpers import dev_bf16, dev_f32, empty_bf16, host

pytestmark = pytest.mark.gpu


def test_gemm_reuse_family_matches_plain_gemm(cs1, stream):
    M0, M, N, K = 2048, 300, 16480, 1024
    g = torch.Generator(device="cpu").manual_seed(41)
    x = (torch.randn(M0, K, generator=g) * 0.5).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    plain = cs1.cs1_gemm_create(0)
    matched = cs1.cs1_gemm_create_matched(0, M0)
    assert plain and matched
    assert cs1.cs1_gemm_compatible(plain, matched, M, N, K) == 1
    assert cs1.cs1_gemm_enable_equivalent_tiles(matched) == 1
    rows = np.arange(M, dtype=np.uintp)
    assert cs1.cs1_gemm_reuse_check(matched, rows.ctypes.data, M0, rows.ctypes.data, M, N, K) == 0
    full = torch.empty(M0, N, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_gemm(plain, x, w, full, M0, N, K, N, stream)
    part = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_gemm_reuse(matched, x, w, part, M, N, K, M0, stream)
    torch.cuda.synchronize()
    cs1.cs1_gemm_destroy(plain)
    cs1.cs1_gemm_destroy(matched)
    assert cs1.cs1_fault_status(1) == 0
    assert torch.equal(part, full[:M])


@pytest.mark.parametrize("T,H,HK", [(65, 4, 2), (300, 48, 16)])
def test_gdn_prefill_wide_equals_prefill(cs1, stream, T, H, HK):
    q, k, v, g, beta = fixtures.grouped_inputs(43, T, H, HK, decay=0.25)
    q, k = rnd(q), rnd(k)
    args = (dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta))
    out = []
    for fn in (cs1.cs1_gdn_prefill, cs1.cs1_gdn_prefill_wide):
        ws = torch.empty(cs1.cs1_gdn_workspace_floats(T, H), dtype=torch.float32, device="cuda")
        o = empty_bf16(T, H, 128)
        fn(*args, o, ws, T, H, HK, 128 ** -0.5, stream)
        out.append(host(o))
    assert cs1.cs1_fault_status(1) == 0
    assert np.array_equal(out[0], out[1])
