"""GPU parity of the tcgen05 projection GEMM (cs1_gemm and its fused epilogues).

Reference: a PyTorch float32 matmul of the same bf16 operands (the GEMM is a
floating-point kernel). Tolerance: bf16 output of an fp32-accumulated dot product,
max |y - ref| <= 1e-2 * max|ref| and relative L2 <= 4e-3. Row invariance
(cs1_gemm_create_fixed's promise in the reference's ops.h:190-195) is bit-exact.
"""
import numpy as np
import pytest
import torch

from helpers import max_rel, rel_l2

pytestmark = pytest.mark.gpu


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).cuda()


@pytest.fixture(scope="module")
def gemm(cs1):
    h = cs1.cs1_gemm_create(32 << 20)
    assert h
    yield h
    cs1.cs1_gemm_destroy(h)


@pytest.mark.parametrize("M,N,K", [(1, 8, 64), (37, 200, 72), (129, 1544, 256), (300, 3072, 256),
                                   (777, 5120, 6144), (2048, 16480, 5120), (5, 7, 9), (130, 12, 20)])
def test_gemm_matches_fp32_reference(cs1, gemm, stream, M, N, K):
    x, w = _rand((M, K), 1), _rand((N, K), 2, 0.05)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_gemm(gemm, x, w, y, M, N, K, N, stream)
    ref = (x.float() @ w.float().T)
    torch.cuda.synchronize()
    assert cs1.cs1_fault_status(1) == 0
    yn, rn = y.float().cpu().numpy(), ref.cpu().numpy()
    assert max_rel(yn, rn) <= 1e-2 and rel_l2(yn, rn) <= 4e-3, (max_rel(yn, rn), rel_l2(yn, rn))


def test_gemm_strided_output(cs1, gemm, stream):
    M, N, K, ld = 200, 264, 128, 1000
    x, w = _rand((M, K), 3), _rand((N, K), 4, 0.05)
    y = torch.zeros(M, ld, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_gemm(gemm, x, w, y, M, N, K, ld, stream)
    ref = (x.float() @ w.float().T).cpu().numpy()
    yn = y.float().cpu().numpy()
    assert max_rel(yn[:, :N], ref) <= 1e-2
    assert np.all(yn[:, N:] == 0), "wrote outside the N columns"


def test_gemm_rows_do_not_depend_on_m(cs1, gemm, stream):
    """A row's bits are the same whatever M (and tile width) the call used."""
    N, K = 5120, 1024
    x, w = _rand((4096, K), 5), _rand((N, K), 6, 0.05)
    big = torch.empty(4096, N, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_gemm(gemm, x, w, big, 4096, N, K, N, stream)
    for m0, m in [(0, 1), (100, 37), (4000, 96), (129, 64)]:
        small = torch.empty(m, N, dtype=torch.bfloat16, device="cuda")
        cs1.cs1_gemm(gemm, x[m0:m0 + m], w, small, m, N, K, N, stream)
        torch.cuda.synchronize()
        assert torch.equal(small, big[m0:m0 + m]), (m0, m)


def test_gemm_packed_equals_per_sequence(cs1, gemm, stream):
    N, K = 1544, 256
    lengths = [1, 63, 64, 65, 129]
    M = sum(lengths)
    x, w = _rand((M, K), 7), _rand((N, K), 8, 0.05)
    packed = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    arr = (torch.tensor(lengths, dtype=torch.int64)).numpy().astype(np.uintp)
    cs1.cs1_gemm_packed(gemm, x, w, packed, arr.ctypes.data, len(lengths), N, K, stream)
    off = 0
    for n in lengths:
        one = torch.empty(n, N, dtype=torch.bfloat16, device="cuda")
        cs1.cs1_gemm(gemm, x[off:off + n], w, one, n, N, K, N, stream)
        torch.cuda.synchronize()
        assert torch.equal(one, packed[off:off + n])
        off += n


def test_cta_pair_kernel_equals_single_cta_kernel(cs1, stream, monkeypatch):
    """The 256x256 CTA-pair kernel and the 128-row single-CTA kernels give identical bits."""
    M, N, K = 1100, 16480, 1024
    x, w = _rand((M, K), 15), _rand((N, K), 16, 0.05)
    out = []
    for pairs in ("1", "0"):
        monkeypatch.setenv("S1_GEMM_PAIRS", pairs)
        h = cs1.cs1_gemm_create(0)
        y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        cs1.cs1_gemm(h, x, w, y, M, N, K, N, stream)
        torch.cuda.synchronize()
        cs1.cs1_gemm_destroy(h)
        out.append(y)
    assert cs1.cs1_fault_status(1) == 0
    ref = (x.float() @ w.float().T).cpu().numpy()
    assert max_rel(out[0].float().cpu().numpy(), ref) <= 1e-2
    assert torch.equal(out[0], out[1])


@pytest.mark.parametrize("M,N", [(1, 2560), (200, 2560), (1500, 2560), (4000, 5120)])
def test_gemm_residual_epilogue(cs1, gemm, stream, M, N):
    K = 512
    x, w = _rand((M, K), 9), _rand((N, K), 10, 0.05)
    res = _rand((M, N), 11)
    expect = (res.float() + (x.float() @ w.float().T).to(torch.bfloat16).float()).to(torch.bfloat16)
    out = res.clone()
    cs1.cs1_gemm_residual(gemm, x, w, out, M, N, K, N, stream)
    torch.cuda.synchronize()
    assert max_rel(out.float().cpu().numpy(), expect.float().cpu().numpy()) <= 1.6e-2
    # same bits as the unfused GEMM followed by the bf16 residual add
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_gemm(gemm, x, w, y, M, N, K, N, stream)
    torch.cuda.synchronize()
    assert torch.equal(out, (res.float() + y.float()).to(torch.bfloat16))


@pytest.mark.parametrize("M,I", [(1, 128), (77, 512), (1000, 1024), (2048, 2560)])
def test_gemm_swiglu_epilogue(cs1, gemm, stream, M, I):
    K = 384
    x = _rand((M, K), 12)
    gate, up = _rand((I, K), 13, 0.05), _rand((I, K), 14, 0.05)
    inter = torch.empty(2 * I, K, dtype=torch.bfloat16, device="cuda")
    for b in range(I // 128):
        inter[256 * b:256 * b + 128] = gate[128 * b:128 * b + 128]
        inter[256 * b + 128:256 * b + 256] = up[128 * b:128 * b + 128]
    out = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_gemm_swiglu(gemm, x, inter, out, M, I, K, I, stream)
    # unfused: stacked gate|up GEMM then cs1_silu_mul -- identical bits
    stacked = torch.cat([gate, up], 0)
    gu = torch.empty(M, 2 * I, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_gemm(gemm, x, stacked, gu, M, 2 * I, K, 2 * I, stream)
    ref = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_silu_mul(gu, 2 * I, ref, M, I, stream)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_gemm_invalid_arguments(cs1, gemm, stream):
    x = torch.empty(4, 64, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(4, 64, dtype=torch.bfloat16, device="cuda")
    assert cs1.raw.cs1_gemm(gemm, x.data_ptr(), x.data_ptr(), y.data_ptr(), 4, 64, 64, 32, stream) != 0
    assert cs1.raw.cs1_gemm(gemm, x.data_ptr(), x.data_ptr(), y.data_ptr(), -1, 64, 64, 64, stream) != 0
    assert cs1.raw.cs1_gemm(gemm, x.data_ptr(), x.data_ptr(), y.data_ptr(), 0, 64, 64, 64, stream) == 0


@pytest.mark.parametrize("M,N,epi", [(771, 16480, "store"), (300, 5120, "residual"), (771, 2560, "swiglu"),
                                     (17, 1544, "store"), (1, 5120, "residual")])
def test_swapped_operand_kernel_equals_row_kernels(cs1, stream, monkeypatch, M, N, epi):
    """Short inputs go through the swapped-operand kernel (rows of w as the MMA's M side,
    rows of x as its N side); its bits equal those of the 128-row kernels."""
    K = 1024
    x = _rand((M, K), 17)
    w = _rand((2 * N if epi == "swiglu" else N, K), 18, 0.05)
    res = _rand((M, N), 19)
    out = []
    for swap in ("1", "0"):
        monkeypatch.setenv("S1_GEMM_SWAP", swap)
        h = cs1.cs1_gemm_create(0)
        if epi == "swiglu":
            y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            cs1.cs1_gemm_swiglu(h, x, w, y, M, N, K, N, stream)
        elif epi == "residual":
            y = res.clone()
            cs1.cs1_gemm_residual(h, x, w, y, M, N, K, N, stream)
        else:
            y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            cs1.cs1_gemm(h, x, w, y, M, N, K, N, stream)
        torch.cuda.synchronize()
        cs1.cs1_gemm_destroy(h)
        out.append(y)
    assert cs1.cs1_fault_status(1) == 0
    if epi == "store":
        ref = (x.float() @ w.float().T).cpu().numpy()
        assert max_rel(out[0].float().cpu().numpy(), ref) <= 1e-2
    assert torch.equal(out[0], out[1])


@pytest.mark.parametrize("M,N", [(700, 16480), (1500, 14336), (400, 34816)])
def test_swapped_kernel_split_tail_equals_row_kernels(cs1, stream, monkeypatch, M, N):
    """Tile counts whose last wave is split along x (parts of the last tiles on idle SMs)."""
    K = 512
    x, w = _rand((M, K), 20), _rand((N, K), 21, 0.05)
    out = []
    for swap in ("1", "0"):
        monkeypatch.setenv("S1_GEMM_SWAP", swap)
        h = cs1.cs1_gemm_create(0)
        y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        cs1.cs1_gemm(h, x, w, y, M, N, K, N, stream)
        torch.cuda.synchronize()
        cs1.cs1_gemm_destroy(h)
        out.append(y)
    assert cs1.cs1_fault_status(1) == 0
    assert torch.equal(out[0], out[1])


@pytest.mark.parametrize("M,N,epi,nt", [(771, 16480, "store", 208), (771, 17408, "swiglu", 208),
                                        (771, 5120, "residual", 256), (17, 1544, "store", 32),
                                        (1, 5120, "residual", 32), (300, 2560, "swiglu", 96),
                                        (1500, 14336, "store", 256), (700, 16480, "store", 208),
                                        (130, 1000, "residual", 144)])
def test_swapped_pair_kernel_equals_row_kernels(cs1, stream, monkeypatch, M, N, epi, nt):
    """The CTA-pair swapped kernel (256 rows of w over two SMs as the MMA's M side, nt rows
    of x as its N side, split in halves between the CTAs), forced, against the 128 x 256
    kernel: identical bits for every epilogue, partial tiles of w and x, and the split last
    wave (700 x 16480 at nt = 208: 260 pair tiles over 74 pairs)."""
    K = 640
    x = _rand((M, K), 22)
    w = _rand((2 * N if epi == "swiglu" else N, K), 23, 0.05)
    res = _rand((M, N), 24)
    out = []
    for kernel in ("swap2", "row256"):
        monkeypatch.setenv("S1_GEMM_KERNEL", kernel)
        monkeypatch.setenv("S1_GEMM_NT", str(nt))
        h = cs1.cs1_gemm_create(0)
        if epi == "swiglu":
            y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            cs1.cs1_gemm_swiglu(h, x, w, y, M, N, K, N, stream)
        elif epi == "residual":
            y = res.clone()
            cs1.cs1_gemm_residual(h, x, w, y, M, N, K, N, stream)
        else:
            y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            cs1.cs1_gemm(h, x, w, y, M, N, K, N, stream)
        torch.cuda.synchronize()
        cs1.cs1_gemm_destroy(h)
        out.append(y)
    assert cs1.cs1_fault_status(1) == 0
    if epi == "store":
        ref = (x.float() @ w.float().T).cpu().numpy()
        assert max_rel(out[0].float().cpu().numpy(), ref) <= 1e-2
    assert torch.equal(out[0], out[1])
