"""The fused momentum scan inside the reference's mixed-precision training step
(training_UESTC.py:100-118): forward under torch.amp.autocast('cuda'), loss
scaled by torch.amp.GradScaler, backward, unscale_, clip_grad_norm_,
scaler.step / scaler.update.

Under fp16 autocast the projections run in fp16 and the conv and scan kernels
take their activations up to fp32, as the reference's CUDA path does
(momentum_scan_cuda.py:215-216); under bf16 autocast the scan runs its
bf16-activation kernels (fp32 state and sums).  Each mixed-precision step is
checked against the same model stepped in fp32 without autocast.

Tolerances (mixed-precision GEMMs around the scan set them, not the scan):
    loss                      |l_amp - l_32| / |l_32|            <= 2e-2
    unscaled gradients        ||g_amp - g_32|| / ||g_32||          <= 3e-2 (fp16), 6e-2 (bf16)
    per-parameter direction   cos(g_amp, g_32)                    >= 0.99
    clipped total norm        |n_amp - n_32| / n_32               <= 3e-2 (fp16), 6e-2 (bf16)
and every parameter is finite after the optimizer step, with no step skipped
by the scaler.
"""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _model(seed=0):
    from momentummamba_b200.mamba_momentum import MambaMomentum, MambaMomentumConfig
    torch.manual_seed(seed)
    cfg = MambaMomentumConfig(d_model=64, n_layers=2, d_state=16, momentum_beta=0.6,
                              pscan_mode="cuda_sequential")
    return MambaMomentum(cfg).to(DEV)


def _step(model, x, dtype, max_norm=1.0):
    """One training step as training_UESTC.py:100-118; dtype None = plain fp32."""
    opt = torch.optim.SGD(model.parameters(), lr=1e-3)
    scaler = torch.amp.GradScaler("cuda", init_scale=2.0 ** 12,
                                  enabled=dtype == torch.float16)
    opt.zero_grad()
    with torch.amp.autocast("cuda", dtype=dtype or torch.float16, enabled=dtype is not None):
        out = model(x)
        loss = (out.float() ** 2).mean()
    scaler.scale(loss).backward()
    scaler.unscale_(opt)
    grads = [p.grad.detach().float().clone() for p in model.parameters()]
    norm = float(torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm))
    scale_before = scaler.get_scale() if scaler.is_enabled() else None
    scaler.step(opt)
    scaler.update()
    torch.cuda.synchronize()
    skipped = scaler.is_enabled() and scaler.get_scale() < scale_before
    return float(loss.detach()), grads, norm, skipped


@pytest.mark.parametrize("dtype,tol", [(torch.float16, 3e-2), (torch.bfloat16, 6e-2)],
                         ids=["fp16", "bf16"])
def test_amp_training_step_matches_fp32(dtype, tol):
    base = _model()
    ref_model, amp_model = copy.deepcopy(base), copy.deepcopy(base)
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(4, 256, 64, device=DEV, generator=g)

    l32, g32, n32, _ = _step(ref_model, x, None)
    lamp, gamp, namp, skipped = _step(amp_model, x, dtype)

    assert not skipped, "the scaler skipped the step (inf/nan in the scaled gradients)"
    assert abs(lamp - l32) / abs(l32) <= 2e-2
    flat32 = torch.cat([t.flatten() for t in g32])
    flatamp = torch.cat([t.flatten() for t in gamp])
    assert torch.isfinite(flatamp).all()
    assert float((flatamp - flat32).norm() / flat32.norm()) <= tol
    for (name, _), a, b in zip(base.named_parameters(), gamp, g32):
        if b.norm() > 0:
            cos = float(torch.dot(a.flatten(), b.flatten()) / (a.norm() * b.norm()))
            assert cos >= 0.99, f"{name}: cosine {cos:.4f}"
    assert abs(namp - n32) / n32 <= tol
    for p in amp_model.parameters():
        assert torch.isfinite(p).all()


def test_scan_dtype_under_autocast():
    """fp16 activations are computed in fp32 (output fp32); bf16 activations stay
    bf16 through the bf16 kernels; gradients come back in the inputs' dtypes."""
    from momentummamba_b200 import selective_scan_momentum_fn
    g = torch.Generator(device=DEV).manual_seed(2)
    Bsz, L, D, N = 2, 64, 32, 16
    for dt, out_dt in ((torch.float16, torch.float32), (torch.bfloat16, torch.bfloat16)):
        x = torch.randn(Bsz, L, D, device=DEV, generator=g).to(dt).requires_grad_()
        delta = (0.5 * torch.randn(Bsz, L, D, device=DEV, generator=g) - 2).to(dt)
        A = -torch.arange(1, N + 1, device=DEV, dtype=torch.float32).repeat(D, 1)
        B = torch.randn(Bsz, L, N, device=DEV, generator=g).to(dt)
        C = torch.randn(Bsz, L, N, device=DEV, generator=g).to(dt)
        with torch.amp.autocast("cuda", dtype=dt):
            y = selective_scan_momentum_fn(x, delta, A, B, C, None, delta_softplus=True,
                                           beta=0.6, alpha=1.0)
        assert y.dtype == out_dt
        (gx,) = torch.autograd.grad(y.float().sum(), [x])
        assert gx.dtype == dt and torch.isfinite(gx.float()).all()
