"""The dense layers of the Dream-shaped forward (``dense.py``): the tcgen05
GEMM with its fused epilogues and the RMSNorm kernel, against torch on the
same bf16 operands (fp32 accumulation on both sides; outputs within bf16
rounding)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(got, want, rel=1e-2):
    got, want = got.float(), want.float()
    err = (got - want).norm() / want.norm()
    assert torch.isfinite(got).all() and err <= rel, err.item()


@pytest.mark.parametrize("m,n,k", [(300, 512, 192), (128, 256, 64), (1000, 768, 3584)])
def test_linear_with_bias(mrsa, cuda_device, m, n, k):
    from mrsa_b200 import dense

    g = torch.Generator(device=cuda_device).manual_seed(m + n + k)
    x = torch.randn(m, k, device=cuda_device, generator=g).bfloat16()
    w = (torch.randn(n, k, device=cuda_device, generator=g) * 0.05).bfloat16()
    b = torch.randn(n, device=cuda_device, generator=g).bfloat16()
    got = dense.linear(x, w, b)
    want = (x.float() @ w.float().t() + b.float()).bfloat16()
    _close(got, want, 4e-3)
    # no element further than a few bf16 ulps
    d = (got.float() - want.float()).abs() / want.float().abs().clamp_min(1e-2)
    assert (d > 0.02).float().mean() < 1e-3


def test_swiglu_and_residual(mrsa, cuda_device):
    from mrsa_b200 import dense

    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(5)
    m, h, f = 520, 512, 768
    x = torch.randn(m, h, device=dev, generator=g).bfloat16()
    wg = (torch.randn(f, h, device=dev, generator=g) * 0.05).bfloat16()
    wu = (torch.randn(f, h, device=dev, generator=g) * 0.05).bfloat16()
    got = dense.swiglu(x, dense.interleave_gate_up(wg, wu))
    gate = (x.float() @ wg.float().t()).bfloat16()
    up = (x.float() @ wu.float().t()).bfloat16()
    want = torch.nn.functional.silu(gate) * up
    _close(got, want, 1e-2)
    wd = (torch.randn(h, f, device=dev, generator=g) * 0.05).bfloat16()
    r = torch.randn(m, h, device=dev, generator=g).bfloat16()
    got2 = dense.linear_residual(got, wd, r)
    want2 = r + (got.float() @ wd.float().t()).bfloat16()
    _close(got2, want2, 4e-3)


def test_rms_norm(mrsa, cuda_device):
    from mrsa_b200 import dense

    g = torch.Generator(device=cuda_device).manual_seed(6)
    x = torch.randn(77, 3584, device=cuda_device, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(3584, device=cuda_device, generator=g)).bfloat16()
    got = dense.rms_norm(x, w, 1e-6)
    xf = x.float()
    want = w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).bfloat16()
    _close(got, want, 4e-3)


def test_gemm_rejects_bad_shapes(mrsa, cuda_device):
    from mrsa_b200 import dense

    x = torch.zeros(8, 100, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        dense.linear(x, torch.zeros(256, 100, device=cuda_device, dtype=torch.bfloat16))   # K % 64
    assert mrsa._lib.load().mrsa_device_error_flags(1) == 0
