"""Fused gated RMSNorm for the tree GDN output: ``norm(core, z)`` of the
Qwen3.5 / Qwen3-Next gated delta-net layers (transformers' ``*RMSNormGated``:
x * rsqrt(mean(x^2) + eps) * weight * silu(z)), which the reference's tree
forward applies per node after the delta rule (dfs_tree_forward.py:420-433).
One kernel each way (``tt_gated_rmsnorm_fwd/bwd``) over all rows of the DFS
sequence, in place of the module's chain of elementwise ops.
"""
from __future__ import annotations

import torch

from . import _lib
from .attention import _stream_ptr

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
_DIMS = (32, 64, 128, 256)


class _GatedRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, z, weight, eps: float):
        rows, D = x.shape
        w32 = weight.float().contiguous()
        y = torch.empty_like(x)
        _lib.call("tt_gated_rmsnorm_fwd", _DTYPES[x.dtype], rows, D, x.data_ptr(), z.data_ptr(),
                  w32.data_ptr(), float(eps), y.data_ptr(), _stream_ptr(x.device))
        ctx.save_for_backward(x, z, w32)
        ctx.eps, ctx.w_dtype = eps, weight.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, z, w32 = ctx.saved_tensors
        rows, D = x.shape
        blocks = int(_lib.lib().tt_gated_rmsnorm_bwd_blocks(rows))
        dx = torch.empty_like(x)
        dz = torch.empty_like(z)
        part = torch.empty((blocks, D), dtype=torch.float32, device=x.device)
        _lib.call("tt_gated_rmsnorm_bwd", _DTYPES[x.dtype], rows, D, x.data_ptr(), z.data_ptr(),
                  w32.data_ptr(), float(ctx.eps), dy.contiguous().data_ptr(), dx.data_ptr(),
                  dz.data_ptr(), part.data_ptr(), blocks, _stream_ptr(x.device))
        return dx, dz, part.sum(0).to(ctx.w_dtype), None


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor,
                  eps: float) -> torch.Tensor:
    """x, z [rows, D] (fp32/bf16/fp16, same dtype; D in 32/64/128/256), weight
    [D] -> x * rsqrt(mean(x^2) + eps) * weight * silu(z), shape and dtype of x.
    CUDA tensors only (no CPU path)."""
    if not x.is_cuda:
        raise RuntimeError("gated_rmsnorm: CUDA tensors required (no CPU path)")
    if x.dtype not in _DTYPES or z.dtype != x.dtype:
        raise TypeError("gated_rmsnorm: x and z must share one of float32/bfloat16/float16")
    if x.dim() != 2 or z.shape != x.shape or x.shape[1] not in _DIMS:
        raise ValueError(f"gated_rmsnorm: x, z [rows, D] with D in {_DIMS}")
    return _GatedRMSNorm.apply(x.contiguous(), z.contiguous(), weight, float(eps))


def fusable(norm) -> bool:
    """True for transformers' torch gated RMSNorm modules (``*RMSNormGated``
    with ``weight`` and ``variance_epsilon``), whose arithmetic the kernel
    implements; other norm modules keep their own forward."""
    return (type(norm).__name__.endswith("RMSNormGated") and hasattr(norm, "variance_epsilon")
            and isinstance(getattr(norm, "weight", None), torch.Tensor)
            and norm.weight.dim() == 1 and norm.weight.shape[0] in _DIMS)
