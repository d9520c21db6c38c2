"""fp32-accurate GEMMs on the sm_100a tensor cores (mmb_gemm_f32: tcgen05 with a
3 x tf32 split), for the dense contractions around the LinOSS layer scan.

``gemm_nt(A, B)``: A (M, K) @ B (N, K)^T, both K-contiguous, with an optional
feedthrough epilogue ``+ E * evec`` (E (M, N), evec (N,)).
``gemm_tn(A, B)``: A (K, M)^T @ B (K, N), both row-major over K, accumulated
over K slices (split-K): the weight-gradient shape.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def _k_major(t: torch.Tensor) -> torch.Tensor:
    """fp32, unit stride along the last dim, rows 16-byte aligned (pitch % 4 == 0)."""
    t = t.float()
    if t.stride(-1) != 1 or t.stride(0) % 4 or t.data_ptr() % 16:
        t = t.contiguous()
    if t.stride(0) % 4:
        pad = torch.zeros(t.shape[0], (t.shape[1] + 3) // 4 * 4, device=t.device)
        pad[:, : t.shape[1]] = t
        t = pad
    return t


def split_tf32(x: torch.Tensor):
    """(hi, lo): hi = x with the low 13 mantissa bits cleared (exact in tf32),
    lo = x - hi (exact in fp32): a weight split once for gemm_nt's B."""
    x = x.float().contiguous()
    hi = (x.view(torch.int32) & -8192).view(torch.float32)
    return hi, x - hi


def gemm_nt(A: torch.Tensor, B, E: Optional[torch.Tensor] = None,
            evec: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C = A @ B^T (+ E * evec): A (M, K), B (N, K) -> C (M, N) fp32.  B may be a
    (hi, lo) pair from split_tf32 (then only A is split per tile)."""
    B_lo = None
    if isinstance(B, tuple):
        B, B_lo = B
    _lib.require_cuda(A, B, B_lo, E, evec)
    M, K = A.shape
    N = B.shape[0]
    if B.shape[1] != K:
        raise ValueError("gemm_nt: A (M, K) and B (N, K) must share K")
    A, B = _k_major(A), _k_major(B)
    if B_lo is not None:
        B_lo = _k_major(B_lo)
        if B_lo.stride(0) != B.stride(0):
            raise ValueError("gemm_nt: B and its low parts must share the row pitch")
    C = torch.empty(M, N, device=A.device)
    if E is not None:
        E = E.float().contiguous()
        evec = evec.float().contiguous()
    lib = _lib.load()
    P = _lib.ptr
    with torch.cuda.device(A.device):
        st = lib.mmb_gemm_f32(0, 0, M, N, K, P(A), A.stride(0), P(B),
                              P(B_lo) if B_lo is not None else None, B.stride(0), P(C), N,
                              P(E) if E is not None else None, N if E is not None else 0,
                              P(evec) if evec is not None else None, 0, 1, _lib.stream_of(A))
    _lib.check(st, "mmb_gemm_f32")
    return C


def gemm_tn(A: torch.Tensor, B: torch.Tensor, splits: int = 0) -> torch.Tensor:
    """C = A^T @ B: A (K, M), B (K, N) -> C (M, N) fp32, K cut into slices that
    separate CTAs reduce into C."""
    _lib.require_cuda(A, B)
    K, M = A.shape
    N = B.shape[1]
    if B.shape[0] != K:
        raise ValueError("gemm_tn: A (K, M) and B (K, N) must share K")
    A, B = _k_major(A), _k_major(B)
    C = torch.zeros(M, N, device=A.device)
    if splits <= 0:
        tiles = -(-M // 128) * -(-N // (256 if N > 128 else 128))
        splits = max(1, min(-(-K // 32), 2 * 148 // tiles))
    lib = _lib.load()
    P = _lib.ptr
    with torch.cuda.device(A.device):
        st = lib.mmb_gemm_f32(1, 1, M, N, K, P(A), A.stride(0), P(B), None, B.stride(0), P(C), N,
                              None,
                              0, None, 1, splits, _lib.stream_of(A))
    _lib.check(st, "mmb_gemm_f32")
    return C


def col_dot(X: torch.Tensor, Y: torch.Tensor) -> torch.Tensor:
    """out[n] = sum_m X[m, n] Y[m, n] for X, Y (M, N) fp32 (N a multiple of 4)."""
    _lib.require_cuda(X, Y)
    M, N = X.shape
    X, Y = _k_major(X), _k_major(Y)
    out = torch.empty(N, device=X.device)
    lib = _lib.load()
    with torch.cuda.device(X.device):
        st = lib.mmb_col_dot_f32(M, N, _lib.ptr(X), X.stride(0), _lib.ptr(Y), Y.stride(0),
                                 _lib.ptr(out), 0, _lib.stream_of(X))
    _lib.check(st, "mmb_col_dot_f32")
    return out
