"""Fused LM-head cross-entropy (``ce.fused_linear_cross_entropy``, kernel
``tt_ce_fwd_grad``) against the plain torch computation it replaces:
logits = h W^T, per-token cross_entropy (ignored labels 0), weighted sum, and
autograd for dH and dW.

* fp32, several chunks and ignored tokens: 1e-5 relative;
* bf16 at the Qwen3 vocabulary (151,936) vs a float32 reference on the same
  bf16 inputs: 2e-2 relative.
"""
import pytest
import torch
import torch.nn.functional as F

from tree_training_b200.ce import fused_linear_cross_entropy

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _ref(h, W, labels, w, ignore_index):
    h = h.detach().float().requires_grad_(True)
    W = W.detach().float().requires_grad_(True)
    logits = h @ W.t()
    ce = F.cross_entropy(logits, labels, ignore_index=ignore_index, reduction="none")
    loss = (ce * w).sum()
    loss.backward()
    return loss.detach(), h.grad, W.grad


def rel(a, b):
    return float((a.double() - b.double()).abs().max() / (b.double().abs().max() + 1e-30))


@pytest.mark.parametrize("dtype,T,H,V,chunk,tol", [
    (torch.float32, 700, 64, 1000, 128, 1e-5),
    (torch.float32, 37, 32, 5, 4096, 1e-5),
    (torch.bfloat16, 1024, 256, 151936, 512, 2e-2),
])
def test_fused_ce_matches_torch(dtype, T, H, V, chunk, tol):
    g = torch.Generator(device=DEV).manual_seed(0)
    h = (torch.randn(T, H, device=DEV, generator=g) * 2).to(dtype).requires_grad_(True)
    W = (torch.randn(V, H, device=DEV, generator=g) * 0.1).to(dtype).requires_grad_(True)
    labels = torch.randint(0, V, (T,), device=DEV, generator=g)
    labels[::7] = -100                                     # ignored tokens
    w = torch.rand(T, device=DEV, generator=g)
    loss = fused_linear_cross_entropy(h, W, labels, w, ignore_index=-100, chunk=chunk)
    (loss * 1.5).backward()
    rl, rh, rW = _ref(h, W, labels, w, -100)
    assert rel(loss, rl) < tol
    assert rel(h.grad, rh * 1.5) < tol
    assert rel(W.grad, rW * 1.5) < tol
    assert h.grad[::7].abs().sum() >= 0                   # ignored rows: finite
    assert torch.isfinite(h.grad).all() and torch.isfinite(W.grad).all()
