"""2x2 (LinOSS) scans on the sm_100a kernels, with autograd.

``scan2(M, F)``: x_t = M_t x_{t-1} + F_t per (b, p) chain, M (B, L, 4P) real in
[M11 | M12 | M21 | M22] blocks, F (B, L, 2P) real or complex in [F1 | F2]
blocks.  Returns (Mscan, X) like the reference's scans (mamba_linoss.py:336-415):
Mscan_t = M_t ... M_0 and X = the scanned states.  Gradients flow to M and F
from both outputs.

``linoss_scan(disc, A_diag, step, Bu)``: the LinOSS layer's scan with a
time-invariant transition per oscillator (IM 'IM' or IMEX 'IMEX',
LinOSS_pytorch.py:153-239); Bu (B, L, P) complex; returns x2 (B, L, P) complex.
Gradients flow to A_diag, step and Bu.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def _real_view(t: torch.Tensor) -> torch.Tensor:
    """fp32 storage with interleaved (re, im) for complex tensors."""
    if t.is_complex():
        return torch.view_as_real(t.to(torch.complex64).contiguous())
    return t.float().contiguous()


class Scan2Fn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, M, F, want_mscan):
        _lib.require_cuda(M, F)
        if M.dim() != 3 or F.dim() != 3 or M.shape[-1] % 4 or F.shape[-1] * 2 != M.shape[-1]:
            raise ValueError("expected M (B, L, 4P) and F (B, L, 2P)")
        if M.shape[:2] != F.shape[:2]:
            raise ValueError("M and F must share (B, L)")
        lib = _lib.load()
        Bsz, L, P4 = M.shape
        P = P4 // 4
        cplx = F.is_complex()
        Mf = M.float().contiguous()
        Fr = _real_view(F)
        X = torch.empty_like(Fr)
        Ms = torch.empty_like(Mf) if want_mscan else None
        work = torch.empty(lib.mmb_scan2_work_floats(Bsz, L, P, int(cplx)), device=M.device)
        with torch.cuda.device(M.device):
            st = lib.mmb_scan2_fwd(Bsz, L, P, int(cplx), _lib.ptr(Mf), _lib.ptr(Fr), _lib.ptr(Ms),
                                   _lib.ptr(X), _lib.ptr(work), _lib.stream_of(M))
        _lib.check(st, "mmb_scan2_fwd")
        ctx.save_for_backward(Mf, X, Ms)
        ctx.cplx = cplx
        Xo = torch.view_as_complex(X) if cplx else X
        return Ms, Xo

    @staticmethod
    def backward(ctx, gMs, gX):
        Mf, X, Ms = ctx.saved_tensors
        cplx = ctx.cplx
        lib = _lib.load()
        Bsz, L, P4 = Mf.shape
        P = P4 // 4
        gXr = None if gX is None else _real_view(gX)
        gMr = None if gMs is None else gMs.float().contiguous()
        dM = torch.empty_like(Mf)
        dF = torch.empty_like(X)
        work = torch.empty(lib.mmb_scan2_work_floats(Bsz, L, P, int(cplx)), device=Mf.device)
        with torch.cuda.device(Mf.device):
            st = lib.mmb_scan2_bwd(Bsz, L, P, int(cplx), _lib.ptr(Mf), _lib.ptr(X), _lib.ptr(gXr),
                                   _lib.ptr(Ms), _lib.ptr(gMr), _lib.ptr(dM), _lib.ptr(dF),
                                   _lib.ptr(work), _lib.stream_of(Mf))
        _lib.check(st, "mmb_scan2_bwd")
        dFo = torch.view_as_complex(dF) if cplx else dF
        return dM, dFo, None


def scan2(M: torch.Tensor, F: torch.Tensor, want_mscan: bool = True):
    """(Mscan, X) of x_t = M_t x_{t-1} + F_t; Mscan is None when not wanted."""
    return Scan2Fn.apply(M, F, bool(want_mscan))


_DISC = {"IM": 0, "IMEX": 1}


class LinossScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, disc, A_diag, step, Bu):
        _lib.require_cuda(A_diag, step, Bu)
        if disc not in _DISC:
            raise ValueError(f"Discretization type {disc} not implemented")
        if Bu.dim() != 3:
            raise ValueError("expected Bu of shape (B, L, P)")
        lib = _lib.load()
        Bsz, L, P = Bu.shape
        if A_diag.shape != (P,) or step.shape != (P,):
            raise ValueError("A_diag and step must have shape (P,)")
        A = A_diag.float().contiguous()
        s = step.float().contiguous()
        Bur = _real_view(Bu if Bu.is_complex() else Bu.to(torch.complex64))
        x2 = torch.empty_like(Bur)
        work = torch.empty(lib.mmb_linoss_work_floats(Bsz, L, P), device=Bu.device)
        with torch.cuda.device(Bu.device):
            st = lib.mmb_linoss_fwd(_DISC[disc], Bsz, L, P, _lib.ptr(A), _lib.ptr(s),
                                    _lib.ptr(Bur), _lib.ptr(x2), _lib.ptr(work),
                                    _lib.stream_of(Bu))
        _lib.check(st, "mmb_linoss_fwd")
        ctx.save_for_backward(A, s, Bur, work)
        ctx.disc = disc
        return torch.view_as_complex(x2)

    @staticmethod
    def backward(ctx, dx2):
        A, s, Bur, work = ctx.saved_tensors
        lib = _lib.load()
        Bsz, L, P, _ = Bur.shape
        g = _real_view(dx2)
        dBu = torch.empty_like(Bur)
        dA = torch.empty_like(A)
        ds = torch.empty_like(s)
        with torch.cuda.device(A.device):
            st = lib.mmb_linoss_bwd(_DISC[ctx.disc], Bsz, L, P, _lib.ptr(A), _lib.ptr(s),
                                    _lib.ptr(Bur), _lib.ptr(g), _lib.ptr(dBu), _lib.ptr(dA),
                                    _lib.ptr(ds), _lib.ptr(work), _lib.stream_of(A))
        _lib.check(st, "mmb_linoss_bwd")
        return None, dA, ds, torch.view_as_complex(dBu)


def linoss_scan(disc: str, A_diag, step, Bu):
    """x2 of the LinOSS layer scan (complex (B, L, P)) for Bu (B, L, P) complex."""
    return LinossScanFn.apply(disc, A_diag, step, Bu)


# ---------------------------------------------------------------------------
# selective LinOSS scan of the Mamba-LinOSS block (fused transitions and output)
# ---------------------------------------------------------------------------
def _pair(re: torch.Tensor, im: torch.Tensor):
    """fp32 (B, L, P) re/im views with unit stride along P and one shared
    (batch, seq) stride pair (column slices of one projection keep theirs)."""
    re, im = re.float(), im.float()
    if re.stride(-1) != 1 or im.stride(-1) != 1 or re.stride() != im.stride():
        re, im = re.contiguous(), im.contiguous()
    return re, im, (ctypes.c_int64 * 2)(re.stride(0), re.stride(1))


class LinossSelFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, disc, A_diag, s, B_re, B_im, C_re, C_im):
        _lib.require_cuda(A_diag, s, B_re, B_im, C_re, C_im)
        if disc not in _DISC:
            raise ValueError(f"Discretization type {disc} not implemented")
        lib = _lib.load()
        Bsz, L, P = B_re.shape
        A = A_diag.float().contiguous()
        sv = s.float().contiguous()
        br, bi, bst = _pair(B_re, B_im)
        cr, ci, cst = _pair(C_re, C_im)
        y = torch.empty((Bsz, L), device=sv.device, dtype=torch.float32)
        work = torch.empty(lib.mmb_linoss_sel_work_floats(Bsz, L, P), device=sv.device)
        with torch.cuda.device(sv.device):
            st = lib.mmb_linoss_sel_fwd(_DISC[disc], Bsz, L, P, _lib.ptr(A), _lib.ptr(sv),
                                        _lib.ptr(br), _lib.ptr(bi), bst, _lib.ptr(cr),
                                        _lib.ptr(ci), cst, _lib.ptr(y), _lib.ptr(work),
                                        _lib.stream_of(sv))
        _lib.check(st, "mmb_linoss_sel_fwd")
        ctx.save_for_backward(A, sv, br, bi, cr, ci, work)
        ctx.disc = disc
        ctx.dtypes = (A_diag.dtype, s.dtype, B_re.dtype, B_im.dtype, C_re.dtype, C_im.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        A, sv, br, bi, cr, ci, work = ctx.saved_tensors
        lib = _lib.load()
        Bsz, L, P = br.shape
        dy = dy.float().contiguous()
        bst = (ctypes.c_int64 * 2)(br.stride(0), br.stride(1))
        cst = (ctypes.c_int64 * 2)(cr.stride(0), cr.stride(1))
        dev = sv.device
        dbr, dbi = (torch.empty((Bsz, L, P), device=dev) for _ in range(2))
        dcr, dci = (torch.empty((Bsz, L, P), device=dev) for _ in range(2))
        dA = torch.empty((P,), device=dev)
        ds = torch.empty((Bsz, L), device=dev)
        with torch.cuda.device(dev):
            st = lib.mmb_linoss_sel_bwd(_DISC[ctx.disc], Bsz, L, P, _lib.ptr(A), _lib.ptr(sv),
                                        _lib.ptr(br), _lib.ptr(bi), bst, _lib.ptr(cr),
                                        _lib.ptr(ci), cst, _lib.ptr(dy), _lib.ptr(dbr),
                                        _lib.ptr(dbi), _lib.ptr(dcr), _lib.ptr(dci), _lib.ptr(dA),
                                        _lib.ptr(ds), _lib.ptr(work), _lib.stream_of(sv))
        _lib.check(st, "mmb_linoss_sel_bwd")
        grads = (dA, ds, dbr, dbi, dcr, dci)
        return (None,) + tuple(g.to(dt) for g, dt in zip(grads, ctx.dtypes))


def linoss_selective(disc: str, A_diag, s, B_re, B_im, C_re, C_im):
    """y[b, t] = Re sum_p C x2 of the selective LinOSS scan (IM or IMEX) with
    per-step step size s (B, L), A_diag (P), B and C (B, L, P) as re/im pairs."""
    return LinossSelFn.apply(disc, A_diag, s, B_re, B_im, C_re, C_im)
