"""RMSNorm and silu(gate) * up kernels for half-precision models (model.py:29-36, 78-86)
against PyTorch: outputs within one bf16 rounding of the float32 computation (the kernels
round once, PyTorch's silu-then-multiply twice), gradients against torch autograd."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,dim", [(64, 4096), (3, 520), (1000, 128)])
def test_rms_norm_matches_torch(rows, dim):
    from kvstreams.model import _RMSNormFn

    g = torch.Generator(device="cuda").manual_seed(dim)
    x = (torch.randn(rows, dim, generator=g, device="cuda") * 3).bfloat16().requires_grad_()
    w = (torch.rand(dim, generator=g, device="cuda") + 0.5).bfloat16().requires_grad_()
    y = _RMSNormFn.apply(x, w, 1e-5)
    ref = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5) * w.float())
    assert ((y.float() - ref).abs() / ref.abs().clamp_min(1e-3)).max().item() <= 2 ** -8
    gy = torch.randn(rows, dim, generator=g, device="cuda").bfloat16()
    y.backward(gy)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    F.rms_norm(xr, (dim,), wr, 1e-5).backward(gy.float())
    assert (x.grad.float() - xr.grad).abs().max().item() <= 2e-2 * xr.grad.abs().max().item()
    assert (w.grad.float() - wr.grad).abs().max().item() <= 2e-2 * wr.grad.abs().max().item()


@pytest.mark.parametrize("rows,dim", [(16384, 4096), (1, 8192), (777, 64)])
def test_rms_norm_backward_kernel_matches_float64(rows, dim):
    """kvs_rms_norm_backward against the float64 formula on the same bf16 inputs (gx within bf16
    rounding, gw float32 to 1e-4 relative), and the same bits on a second call (gw is summed
    per CTA and then in CTA order, without float atomics)."""
    from kvstreams import ops

    g = torch.Generator(device="cuda").manual_seed(rows + dim)
    x = (torch.randn(rows, dim, generator=g, device="cuda") * 2).bfloat16()
    w = (torch.rand(dim, generator=g, device="cuda") + 0.5).bfloat16()
    gy = torch.randn(rows, dim, generator=g, device="cuda").bfloat16()
    _, rstd = ops.rms_norm(x, w, 1e-5)
    gx, gw = ops.rms_norm_backward(x, w, rstd, gy)
    xd, wd, gd, rd = x.double(), w.double(), gy.double(), rstd.double()[:, None]
    xn, gxn = xd * rd, gd * wd
    want_gx = rd * (gxn - xn * (gxn * xn).mean(-1, keepdim=True))
    want_gw = (gd * xn).sum(0)
    assert ((gx.double() - want_gx).abs() / want_gx.abs().clamp_min(1e-2)).max().item() <= 2 ** -7
    assert ((gw.double() - want_gw).abs().max() / want_gw.abs().max()).item() <= 1e-4
    gx2, gw2 = ops.rms_norm_backward(x, w, rstd, gy)
    assert torch.equal(gx, gx2) and torch.equal(gw, gw2)


@pytest.mark.parametrize("rows,f", [(64, 14336), (5, 24), (300, 512)])
def test_silu_mul_matches_torch(rows, f):
    from kvstreams.model import _SiluMulFn

    g = torch.Generator(device="cuda").manual_seed(f)
    gu = (torch.randn(rows, 2 * f, generator=g, device="cuda") * 2).bfloat16().requires_grad_()
    out = _SiluMulFn.apply(gu)
    gf, uf = gu.detach().float().chunk(2, dim=-1)
    ref = F.silu(gf) * uf
    assert (out.float() - ref).abs().max().item() <= 2 ** -7 * ref.abs().max().item()
    go = torch.randn(rows, f, generator=g, device="cuda").bfloat16()
    out.backward(go)
    gur = gu.detach().float().requires_grad_()
    a, b = gur.chunk(2, dim=-1)
    (F.silu(a) * b).backward(go.float())
    assert (gu.grad.float() - gur.grad).abs().max().item() <= 2e-2 * gur.grad.abs().max().item()


def test_model_uses_the_kernels_for_bf16_only():
    """fp32 models keep PyTorch's ops (bit-identical to the reference's composition)."""
    from kvstreams.model import RMSNorm

    n = RMSNorm(256).cuda()
    x = torch.randn(4, 256, device="cuda")
    assert torch.equal(n(x), F.rms_norm(x, (256,), n.weight, n.eps))
