"""The C-ABI library loads here (no GPU needed), exports every symbol that
include/*.h declares, and validates its arguments before touching the device."""
import ctypes
import glob
import json
import os
import re

import pytest
import torch

from momentummamba_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(mmb_\w+)\s*\(", src):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("mmb_mmscan_fwd", "mmb_mmscan_bwd", "mmb_rows_fwd", "mmb_rows_bwd",
                     "mmb_pscan_fwd", "mmb_pscan_bwd", "mmb_status_string", "mmb_abi_version"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.load()._name)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.mmb_abi_version() >= 3
    assert lib.mmb_status_string(0) == b"ok"
    for code in range(1, 8):
        assert lib.mmb_status_string(code) != b"unknown status"
    assert lib.mmb_status_string(99) == b"unknown status"


def test_ckpt_size_formula():
    lib = _lib.load()
    # batch * ceil(L / 8) * dim * dstate * 2 when the call does not split along time
    assert lib.mmb_mmscan_ckpt_floats(2, 256, 64, 16) == 2 * 32 * 64 * 16 * 2
    assert lib.mmb_mmscan_ckpt_floats(32, 1024, 256, 16) == 32 * 128 * 256 * 16 * 2
    assert lib.mmb_mmscan_ckpt_floats(0, 10, 10, 16) == 0
    # one sequence of 16 channels gives the GPU one warp: the library splits 300
    # steps into chunks of 256 and adds chunks * batch * dim * dstate * 6 floats
    assert lib.mmb_mmscan_ckpt_floats(1, 300, 16, 8) == 1 * 38 * 16 * 8 * 2 + 2 * 16 * 8 * 6


def test_workspace_follows_the_time_chunk():
    lib = _lib.load()
    d = _desc(shape=(2, 1000, 64, 16))
    ck = 2 * 125 * 64 * 16 * 2
    d.time_chunk = -1                      # never split
    assert lib.mmb_mmscan_workspace_floats(ctypes.byref(d)) == ck
    d.time_chunk = 100                     # rounded up to 128 steps: 8 chunks
    assert lib.mmb_mmscan_workspace_floats(ctypes.byref(d)) == ck + 8 * 2 * 64 * 16 * 6
    d.time_chunk = 1000                    # one chunk
    assert lib.mmb_mmscan_workspace_floats(ctypes.byref(d)) == ck
    d.time_chunk = 0                       # automatic: 16 warps -> chunks of 256 steps
    assert lib.mmb_mmscan_workspace_floats(ctypes.byref(d)) == ck + 4 * 2 * 64 * 16 * 6
    assert lib.mmb_mmscan_workspace_floats(ctypes.byref(d)) == lib.mmb_mmscan_ckpt_floats(
        2, 1000, 64, 16)
    assert lib.mmb_mmscan_workspace_floats(None) == 0
    assert ctypes.sizeof(_lib.MMScanDesc) == 136


def _desc(**kw):
    d = _lib.MMScanDesc()
    d.batch, d.seqlen, d.dim, d.dstate = kw.get("shape", (2, 16, 8, 16))
    d.beta, d.alpha = 0.5, 1.0
    return d


def test_argument_validation_without_device():
    lib = _lib.load()
    p = ctypes.c_void_p(256)  # never dereferenced: validation fails first
    nul = None
    # missing desc / inputs
    assert lib.mmb_mmscan_fwd(None, p, p, p, p, p, nul, nul, nul, p, nul, nul) == 1
    assert lib.mmb_mmscan_fwd(_desc(), nul, p, p, p, p, nul, nul, nul, p, nul, nul) == 1
    # bad sizes
    assert lib.mmb_mmscan_fwd(_desc(shape=(0, 16, 8, 16)), p, p, p, p, p, nul, nul, nul, p, nul,
                              nul) == 2
    # d_state outside the compiled set
    assert lib.mmb_mmscan_fwd(_desc(shape=(2, 16, 8, 12)), p, p, p, p, p, nul, nul, nul, p, nul,
                              nul) == 4
    # backward without checkpoints
    args = [p] * 5 + [nul] * 3
    assert lib.mmb_mmscan_bwd(_desc(), *args, nul, p, p, p, p, p, p, nul, nul, nul, nul) == 5
    assert lib.mmb_rows_fwd(0, 16, p, 0.5, p, p, nul, nul) == 2
    assert lib.mmb_rows_fwd(4, 16, nul, 0.5, p, p, nul, nul) == 1
    assert lib.mmb_pscan_fwd(1, 0, 4, p, p, p, nul) == 2
    assert lib.mmb_pscan_bwd(1, 4, 4, p, p, nul, p, p, nul) == 1


def test_product_path_has_no_cpu_fallback():
    from momentummamba_b200 import selective_scan_momentum_fn
    from momentummamba_b200.pscan import pscan
    x = torch.randn(1, 8, 8)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        selective_scan_momentum_fn(x, x.abs(), -torch.ones(8, 16), torch.randn(1, 8, 16),
                                   torch.randn(1, 8, 16))
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        pscan(torch.rand(1, 8, 4), torch.randn(1, 8, 4))


def test_module_tree_matches_reference_state_dict(golden_dir):
    from momentummamba_b200.mamba_momentum import MambaMomentum, MambaMomentumConfig
    want = json.load(open(os.path.join(golden_dir, "mm_state_dict.json")))
    m = MambaMomentum(MambaMomentumConfig(d_model=128, n_layers=2, dt_rank=8))
    got = {k: list(v.shape) for k, v in m.state_dict().items()}
    assert got == want


def test_selftest_wait_rejects_out_of_range_poll_counts():
    # checked before any device work: no GPU needed
    lib = _lib.load()
    assert lib.mmb_selftest_device_wait(0, None) == 2       # MMB_ERR_SHAPE
    assert lib.mmb_selftest_device_wait(4097, None) == 2
