"""Fused q/k RMSNorm + rotary prologue (``prologue.qk_norm_rope``) against
transformers' own Qwen3RMSNorm + apply_rotary_pos_emb run in float32, forward
and gradients (x and the norm weight); and a Qwen3 model with the fused
prologue through the tree drivers against the flat per-path gradients.
Bars: fp32 1e-5, bf16 2e-2, drivers 1e-4."""
import pytest
import torch

from tests.test_hybrid_gpu import _forest47, _grads, _model, flat_per_path_grads, max_rel

import tree_training_b200 as tt
from tree_training_b200.hybrid import make_tree_loss_fn, tree_grad_hybrid
from tree_training_b200.prologue import fuse_attention_prologue, qk_norm_rope

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _torch_ref(x, w, cos, sin, eps):
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb
    norm = Qwen3RMSNorm(x.shape[-1], eps=eps).to(DEV)
    with torch.no_grad():
        norm.weight.copy_(w)
    xx = x.detach().float().requires_grad_(True)
    n = norm(xx)                                            # [T, H, D]
    q, _ = apply_rotary_pos_emb(n.transpose(0, 1)[None], n.transpose(0, 1)[None],
                                cos.float()[None], sin.float()[None])
    return q[0].transpose(0, 1), xx, norm.weight


def rel(a, b):
    return float((a.double() - b.double()).abs().max() / (b.double().abs().max() + 1e-30))


@pytest.mark.parametrize("dtype,D,tol", [(torch.float32, 128, 1e-5), (torch.float32, 64, 1e-5),
                                         (torch.bfloat16, 128, 2e-2), (torch.float32, 256, 1e-5)])
def test_qk_norm_rope_matches_transformers(dtype, D, tol):
    g = torch.Generator(device=DEV).manual_seed(0)
    T, H = 517, 6
    x = (torch.randn(T, H, D, device=DEV, generator=g) * 3).to(dtype).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(D, device=DEV, generator=g)).to(dtype).requires_grad_(True)
    pos = torch.randint(0, 4000, (T,), device=DEV, generator=g).float()
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=DEV).float() / D))
    emb = torch.cat([pos[:, None] * inv[None], pos[:, None] * inv[None]], -1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    y = qk_norm_rope(x, w, cos, sin, 1e-6)
    dy = torch.randn(T, H, D, device=DEV, generator=g)
    (y.float() * dy).sum().backward()
    ry, rx, rw = _torch_ref(x, w.detach().float(), cos, sin, 1e-6)
    (ry * dy).sum().backward()
    assert rel(y, ry) < tol
    assert rel(x.grad, rx.grad) < tol
    assert rel(w.grad, rw.grad) < tol


def test_drivers_with_fused_prologue_match_flat_per_path():
    torch.backends.cuda.matmul.allow_tf32 = False
    model = _model()
    roots = _forest47()
    ref, leaves, labels = flat_per_path_grads(model, roots)
    assert fuse_attention_prologue(model) == len(model.model.layers)
    fn = make_tree_loss_fn(labels, leaves, len(leaves))
    for max_tokens in (1000, 10):
        model.zero_grad(set_to_none=True)
        tree_grad_hybrid(model, roots, fn, max_tokens)
        torch.cuda.synchronize()
        tt.check_device_status(DEV)
        assert max_rel(ref, _grads(model)) < 1e-4
