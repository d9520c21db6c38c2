"""Worker for test_gpu_two_copies.py: loads the library and a second copy of
the same file under another name into this one process, and runs the row
scan, the fused momentum scan (forward + backward: TMA tiles, shared-memory
attributes set per copy) and the tensor-core GEMM (TMEM) through both copies,
interleaved.  Each copy links its own CUDA runtime; both must launch on the
process's device context and agree with each other.

Exit status 0 when every call returns MMB_OK and the copies agree (bitwise for
deterministic outputs, max|a - b| / max|b| <= 1e-5 for the atomically summed
parameter gradients).
"""
import ctypes
import os
import shutil
import sys
import tempfile

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from momentummamba_b200 import _lib  # noqa: E402

P = _lib.ptr


def load_copy(tmpdir):
    path = os.path.join(tmpdir, "libmomentum_scan_b200_copy.so")
    shutil.copy(_lib.lib_path(), path)
    lib = ctypes.CDLL(path)
    for name, (res, args) in _lib._SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def check(lib, st, what):
    if st != 0:
        raise SystemExit(f"{what}: status {st} {lib.mmb_status_string(st).decode()} "
                         f"{lib.mmb_last_error().decode()}")


def rows(lib, a, u):
    h = torch.empty_like(a)
    check(lib, lib.mmb_rows_fwd(a.shape[0], a.shape[1], P(a), 0.6, P(u), P(h), None,
                                _lib.stream_of(a)), "rows")
    return h


def scan(lib, t, Bsz, L, D, N):
    d = _lib.MMScanDesc()
    d.batch, d.seqlen, d.dim, d.dstate = Bsz, L, D, N
    d.x_stride[:] = (L * D, D); d.delta_stride[:] = (L * D, D); d.z_stride[:] = (L * D, D)
    d.B_stride[:] = (L * N, N); d.C_stride[:] = (L * N, N)
    d.beta, d.alpha, d.delta_softplus = 0.6, 1.0, 1
    dev = t["x"].device
    o = {k: torch.empty(Bsz, L, D, device=dev) for k in ("out", "dx", "ddelta", "dz")}
    o["ckpt"] = torch.empty(lib.mmb_mmscan_workspace_floats(ctypes.byref(d)), device=dev)
    o["dB"] = torch.empty(Bsz, L, N, device=dev)
    o["dC"] = torch.empty(Bsz, L, N, device=dev)
    o["dA"] = torch.empty(D, N, device=dev)
    o["dD"] = torch.empty(D, device=dev)
    o["dbias"] = torch.empty(D, device=dev)
    s = _lib.stream_of(t["x"])
    check(lib, lib.mmb_mmscan_fwd(ctypes.byref(d), P(t["x"]), P(t["delta"]), P(t["A"]), P(t["B"]),
                                  P(t["C"]), P(t["D"]), P(t["z"]), P(t["bias"]), P(o["out"]),
                                  P(o["ckpt"]), s), "mmscan_fwd")
    check(lib, lib.mmb_mmscan_bwd(ctypes.byref(d), P(t["x"]), P(t["delta"]), P(t["A"]), P(t["B"]),
                                  P(t["C"]), P(t["D"]), P(t["z"]), P(t["bias"]), P(o["ckpt"]),
                                  P(t["dout"]), P(o["dx"]), P(o["ddelta"]), P(o["dA"]), P(o["dB"]),
                                  P(o["dC"]), P(o["dD"]), P(o["dz"]), P(o["dbias"]), s), "mmscan_bwd")
    del o["ckpt"]
    return o


def gemm(lib, A, B):
    M, K = A.shape
    N = B.shape[0]
    C = torch.empty(M, N, device=A.device)
    check(lib, lib.mmb_gemm_f32(0, 0, M, N, K, P(A), K, P(B), None, K, P(C), N, None, 0, None, 0,
                                1, _lib.stream_of(A)), "gemm")
    return C


def rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max().clamp_min(1e-30))


def main():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(3)
    r = lambda *s: torch.randn(*s, device=dev, generator=g)
    Bsz, L, D, N = 64, 40, 512, 16  # wide enough for the two-channel backward
    t = dict(x=r(Bsz, L, D), delta=0.5 * r(Bsz, L, D) - 2.0, z=r(Bsz, L, D), B=r(Bsz, L, N),
             C=r(Bsz, L, N), D=r(D), bias=0.1 * r(D), dout=r(Bsz, L, D),
             A=-torch.arange(1, N + 1, device=dev, dtype=torch.float32).repeat(D, 1))
    a, u = torch.rand(128, 300, device=dev, generator=g), r(128, 300)
    GA, GB = r(1000, 128), r(512, 128)
    lib1 = _lib.load()
    with tempfile.TemporaryDirectory() as tmp:
        lib2 = load_copy(tmp)
        res = []
        for lib in (lib1, lib2, lib1, lib2):
            res.append((rows(lib, a, u), scan(lib, t, Bsz, L, D, N), gemm(lib, GA, GB)))
            torch.cuda.synchronize()
        for lib in (lib1, lib2):
            check(lib, lib.mmb_device_status(_lib.stream_of(a)), "device_status")
    h0, s0, c0 = res[0]
    ok = True
    for k, (h, s, c) in enumerate(res[1:], 1):
        same = torch.equal(h, h0) and torch.equal(c, c0)
        for key in ("out", "dx", "ddelta", "dz"):
            same = same and torch.equal(s[key], s0[key])
        sums = max(rel(s[key], s0[key]) for key in ("dA", "dB", "dC", "dD", "dbias"))
        print(f"call {k} (copy {1 + k % 2}): outputs equal {same}, summed gradients rel {sums:.1e}",
              flush=True)
        ok = ok and same and sums <= 1e-5
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
