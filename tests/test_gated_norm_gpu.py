"""Fused gated RMSNorm (``gated_norm.gated_rmsnorm``, the tree GDN output
norm) against transformers' own Qwen3_5MoeRMSNormGated run in float32:
output and the gradients of x, the gate z and the weight.  Bars: fp32 1e-5,
bf16 2e-2 (one rounding of the fused path against the module's fp32 result)."""
import pytest
import torch

from tree_training_b200 import _lib
from tree_training_b200.gated_norm import fusable, gated_rmsnorm

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def rel(a, b):
    a, b = a.detach().double(), b.detach().double()
    return float((a - b).abs().max() / (b.abs().max() + 1e-30))


def _module(D, w, eps):
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeRMSNormGated
    m = Qwen3_5MoeRMSNormGated(D, eps=eps).to(DEV)
    with torch.no_grad():
        m.weight.copy_(w)
    return m


@pytest.mark.parametrize("dtype,D,rows,tol", [
    (torch.float32, 32, 1000, 1e-5), (torch.float32, 64, 333, 1e-5),
    (torch.float32, 128, 4099, 1e-5), (torch.float32, 256, 77, 1e-5),
    (torch.bfloat16, 128, 4099, 2e-2), (torch.float16, 64, 1000, 2e-2)])
def test_gated_rmsnorm_matches_transformers(dtype, D, rows, tol):
    g = torch.Generator(device=DEV).manual_seed(D + rows)
    x = (torch.randn(rows, D, device=DEV, generator=g) * 2).to(dtype).requires_grad_(True)
    z = (torch.randn(rows, D, device=DEV, generator=g) * 2).to(dtype).requires_grad_(True)
    w32 = 1 + 0.1 * torch.randn(D, device=DEV, generator=g)
    w = w32.to(dtype).requires_grad_(True)
    dy = torch.randn(rows, D, device=DEV, generator=g)
    y = gated_rmsnorm(x, z, w, 1e-6)
    assert y.dtype == dtype and y.shape == x.shape
    (y.float() * dy).sum().backward()
    m = _module(D, w.detach().float(), 1e-6)
    assert fusable(m)
    rx = x.detach().float().requires_grad_(True)
    rz = z.detach().float().requires_grad_(True)
    ry = m(rx, rz)
    (ry * dy).sum().backward()
    torch.cuda.synchronize()
    assert rel(y, ry) < tol
    assert rel(x.grad, rx.grad) < tol
    assert rel(z.grad, rz.grad) < tol
    assert rel(w.grad, m.weight.grad) < tol


def test_gated_rmsnorm_edges():
    # zero rows: nothing launched, empty result
    e = torch.empty(0, 64, device=DEV)
    assert gated_rmsnorm(e, e, torch.ones(64, device=DEV), 1e-6).shape == (0, 64)
    # unsupported widths and CPU tensors raise; the kernel entry refuses them too
    x = torch.randn(8, 48, device=DEV)
    with pytest.raises(ValueError):
        gated_rmsnorm(x, x, torch.ones(48, device=DEV), 1e-6)
    with pytest.raises(RuntimeError):
        gated_rmsnorm(x.cpu(), x.cpu(), torch.ones(48), 1e-6)
    rc = _lib.lib().tt_gated_rmsnorm_fwd(0, 8, 48, x.data_ptr(), x.data_ptr(),
                                          x.data_ptr(), 1e-6, x.data_ptr(), None)
    assert rc == _lib.TT_ERR_UNSUPPORTED
    assert not fusable(torch.nn.LayerNorm(64))
