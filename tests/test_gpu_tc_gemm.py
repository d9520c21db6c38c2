"""The tensor-core fp32 GEMM (tcgen05, 3 x tf32 split) against float64 on the
host: K-major and MN-major operands, ragged M / N / K, split-K reductions and
the feedthrough epilogue.

Tolerance (stated): max|gpu - ref| / max|ref| <= 1e-5 (one-pass tf32 would
miss it by two orders of magnitude; the test checks that too).
"""
import pytest
import torch

from momentummamba_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = 1e-5
DEV = "cuda:0"


def gemm(A, B, M, N, K, a_mn, b_mn, C=None, E=None, evec=None, accumulate=0, splits=1,
         B_lo=None):
    lib = _lib.load()
    if C is None:
        C = torch.zeros(M, N, device=DEV)
    P = _lib.ptr
    st = lib.mmb_gemm_f32(int(a_mn), int(b_mn), M, N, K, P(A), A.stride(0), P(B),
                          P(B_lo) if B_lo is not None else None, B.stride(0),
                          P(C), C.stride(0), P(E) if E is not None else None,
                          E.stride(0) if E is not None else 0, P(evec) if evec is not None else None,
                          accumulate, splits, _lib.stream_of(A))
    _lib.check(st, "mmb_gemm_f32")
    torch.cuda.synchronize()
    return C


def rel(a, b):
    return float((a.double() - b).abs().max() / b.abs().max())


SHAPES = [(128, 128, 32), (300, 200, 130), (65, 512, 128), (1000, 128, 512), (4096, 256, 96)]


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("shape", SHAPES, ids=[str(s) for s in SHAPES])
def test_gemm_layouts_vs_float64(shape, a_mn, b_mn):
    M, N, K = shape
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N + K)
    # MN-major operands are stored (K, M): pad the row pitch to a multiple of 4
    pad = lambda n: (n + 3) // 4 * 4
    Af = torch.randn(M, K, device=DEV, generator=g)
    Bf = torch.randn(N, K, device=DEV, generator=g)
    if a_mn:
        A = torch.zeros(K, pad(M), device=DEV)
        A[:, :M] = Af.t()
    else:
        A = torch.zeros(M, pad(K), device=DEV)
        A[:, :K] = Af
    if b_mn:
        B = torch.zeros(K, pad(N), device=DEV)
        B[:, :N] = Bf.t()
    else:
        B = torch.zeros(N, pad(K), device=DEV)
        B[:, :K] = Bf
    C = gemm(A, B, M, N, K, a_mn, b_mn)
    ref = Af.double().cpu() @ Bf.double().cpu().t()
    err = rel(C.cpu(), ref)
    assert err <= TOL, f"rel err {err:.3e}"


def test_split_k_accumulates_into_c():
    M, N, K = 512, 128, 65536 // 16
    g = torch.Generator(device=DEV).manual_seed(3)
    # both operands MN-major: C = A^T B, the shape of a weight gradient
    At = torch.randn(K, M, device=DEV, generator=g)
    Bt = torch.randn(K, N, device=DEV, generator=g)
    C0 = torch.randn(M, N, device=DEV, generator=g)
    C = gemm(At, Bt, M, N, K, 1, 1, C=C0.clone(), accumulate=1, splits=37)
    ref = C0.double().cpu() + At.double().cpu().t() @ Bt.double().cpu()
    assert rel(C.cpu(), ref) <= TOL


def test_feedthrough_epilogue():
    M, N, K = 777, 128, 256
    g = torch.Generator(device=DEV).manual_seed(5)
    A = torch.randn(M, K, device=DEV, generator=g)
    B = torch.randn(N, K, device=DEV, generator=g)
    E = torch.randn(M, N, device=DEV, generator=g)
    ev = torch.randn(N, device=DEV, generator=g)
    C = gemm(A, B, M, N, K, 0, 0, E=E, evec=ev)
    ref = A.double().cpu() @ B.double().cpu().t() + E.double().cpu() * ev.double().cpu()
    assert rel(C.cpu(), ref) <= TOL


def test_accuracy_beats_one_pass_tf32():
    """The split keeps fp32-grade accuracy where tf32 alone loses ~3 digits."""
    M, N, K = 256, 256, 1024
    g = torch.Generator(device=DEV).manual_seed(9)
    A = torch.randn(M, K, device=DEV, generator=g)
    B = torch.randn(N, K, device=DEV, generator=g)
    C = gemm(A, B, M, N, K, 0, 0)
    ref = A.double().cpu() @ B.double().cpu().t()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        t = (A @ B.t()).cpu()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert rel(C.cpu(), ref) <= TOL
    assert rel(t, ref) > 10 * rel(C.cpu(), ref)


def test_rejects_bad_arguments():
    lib = _lib.load()
    A = torch.zeros(8, 8, device=DEV)
    P = _lib.ptr
    s = _lib.stream_of(A)
    assert lib.mmb_gemm_f32(0, 0, 8, 8, 8, None, 8, P(A), None, 8, P(A), 8, None, 0, None, 0, 1, s) == 1
    assert lib.mmb_gemm_f32(0, 0, 0, 8, 8, P(A), 8, P(A), None, 8, P(A), 8, None, 0, None, 0, 1, s) == 2
    assert lib.mmb_gemm_f32(0, 0, 8, 8, 8, P(A), 6, P(A), None, 8, P(A), 8, None, 0, None, 0, 1, s) == 2
    # split-K must accumulate
    assert lib.mmb_gemm_f32(0, 0, 8, 8, 8, P(A), 8, P(A), None, 8, P(A), 8, None, 0, None, 0, 2, s) == 2
    # pre-split B must be K-major
    assert lib.mmb_gemm_f32(0, 1, 8, 8, 8, P(A), 8, P(A), P(A), 8, P(A), 8, None, 0, None, 0, 1, s) == 4


@pytest.mark.parametrize("a_mn", [0, 1])
def test_presplit_b_matches_float64(a_mn):
    """B given as (hi, lo) from mmb_split_tf32: only A is split per tile."""
    M, N, K = 1000, 512, 128
    g = torch.Generator(device=DEV).manual_seed(21)
    Af = torch.randn(M, K, device=DEV, generator=g)
    Bf = torch.randn(N, K, device=DEV, generator=g)
    A = Af.t().contiguous() if a_mn else Af
    hi, lo = torch.empty_like(Bf), torch.empty_like(Bf)
    lib = _lib.load()
    _lib.check(lib.mmb_split_tf32(_lib.ptr(Bf), _lib.ptr(hi), _lib.ptr(lo), Bf.numel(),
                                  _lib.stream_of(Bf)), "mmb_split_tf32")
    assert torch.equal(hi + lo, Bf)
    C = gemm(A, hi, M, N, K, a_mn, 0, B_lo=lo)
    ref = Af.double().cpu() @ Bf.double().cpu().t()
    assert rel(C.cpu(), ref) <= TOL


@pytest.mark.parametrize("M,N", [(65536, 128), (1000, 36), (3, 260)])
def test_col_dot_vs_float64(M, N):
    from momentummamba_b200.tc_gemm import col_dot
    g = torch.Generator(device=DEV).manual_seed(M + N)
    X = torch.randn(M, N, device=DEV, generator=g)
    Y = torch.randn(M, N, device=DEV, generator=g)
    out = col_dot(X, Y)
    ref = (X.double() * Y.double()).sum(0).cpu()
    assert rel(out.cpu(), ref) <= TOL


@pytest.mark.parametrize("b_mn", [0, 1])
def test_unaligned_c_takes_the_per_tile_kernel(b_mn):
    """C rows of 130 floats cannot be stored by TMA boxes: the one-CTA-per-tile
    kernel with direct stores runs instead, with the same result."""
    M, N, K = 300, 130, 64
    g = torch.Generator(device=DEV).manual_seed(31)
    Af = torch.randn(M, K, device=DEV, generator=g)
    Bf = torch.randn(N, K, device=DEV, generator=g)
    if b_mn:
        B = torch.zeros(K, 132, device=DEV)
        B[:, :N] = Bf.t()
    else:
        B = Bf
    C = gemm(Af, B, M, N, K, 0, b_mn)
    ref = Af.double().cpu() @ Bf.double().cpu().t()
    assert C.stride(0) == 130
    assert rel(C.cpu(), ref) <= TOL
    # and as a K-sliced reduction into an unaligned C
    Bt = torch.zeros(K, 132, device=DEV)  # MN-major rows keep a 16-byte pitch
    Bt[:, :N] = Bf.t()
    C2 = torch.zeros(M, N, device=DEV)
    gemm(Af.t().contiguous(), Bt, M, N, K, 1, 1, C=C2, accumulate=1, splits=3)
    assert rel(C2.cpu(), ref) <= TOL


def test_col_dot_accumulates_into_unaligned_output():
    """An output that is not 16-byte aligned takes scalar atomics; accumulate=1
    adds to what is there."""
    lib = _lib.load()
    M, N = 4097, 132
    g = torch.Generator(device=DEV).manual_seed(41)
    X = torch.randn(M, N, device=DEV, generator=g)
    Y = torch.randn(M, N, device=DEV, generator=g)
    buf = torch.randn(N + 1, device=DEV, generator=g)
    out = buf[1:]  # 4 bytes past a 16-byte boundary
    assert out.data_ptr() % 16 == 4
    before = out.clone()
    P = _lib.ptr
    _lib.check(lib.mmb_col_dot_f32(M, N, P(X), N, P(Y), N, P(out), 1, _lib.stream_of(X)),
               "mmb_col_dot_f32")
    torch.cuda.synchronize()
    ref = before.double().cpu() + (X.double() * Y.double()).sum(0).cpu()
    assert rel(out.cpu(), ref) <= TOL
