"""Fused attention prologue: q/k per-head RMSNorm + rotary embedding in one
kernel pass each way (``tt_qk_norm_rope_fwd/bwd``), in place of the separate
q_norm / k_norm / apply_rotary_pos_emb ops of transformers' Qwen3 attention
(models/qwen3/modeling_qwen3.py lines 263-268).  The rotary cos / sin rows
are the ones the model computed from the tree's depth-based position ids, so
the packed tree's positions reach the kernel unchanged.

``fuse_attention_prologue(model)`` swaps the forward of every Qwen3 attention
module for one that calls the fused op; everything after the rotation
(cache update, attention interface, o_proj) is the module's own code path.
"""
from __future__ import annotations

import types

import torch

from . import _lib
from .attention import _stream_ptr

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, cos, sin, eps: float):
        n, H, D = x.shape
        w32 = weight.float().contiguous()
        y = torch.empty_like(x)
        _lib.call("tt_qk_norm_rope_fwd", _DTYPES[x.dtype], n, H, D, x.data_ptr(), w32.data_ptr(),
                  cos.data_ptr(), sin.data_ptr(), float(eps), y.data_ptr(), _stream_ptr(x.device))
        ctx.save_for_backward(x, w32, cos, sin)
        ctx.eps, ctx.w_dtype = eps, weight.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w32, cos, sin = ctx.saved_tensors
        n, H, D = x.shape
        blocks = int(_lib.lib().tt_qk_norm_rope_bwd_blocks(n * H))
        dx = torch.empty_like(x)
        part = torch.empty((blocks, D), dtype=torch.float32, device=x.device)
        _lib.call("tt_qk_norm_rope_bwd", _DTYPES[x.dtype], n, H, D, x.data_ptr(), w32.data_ptr(),
                  cos.data_ptr(), sin.data_ptr(), float(ctx.eps), dy.contiguous().data_ptr(),
                  dx.data_ptr(), part.data_ptr(), blocks, _stream_ptr(x.device))
        return dx, part.sum(0).to(ctx.w_dtype), None, None, None


def qk_norm_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 eps: float) -> torch.Tensor:
    """x [tokens, heads, D] (fp32/bf16/fp16, D in 64/128/256), weight [D],
    cos/sin [tokens, D] -> rotary(rmsnorm(x) * weight), same shape and dtype.
    CUDA tensors only (no CPU path)."""
    if not x.is_cuda:
        raise RuntimeError("qk_norm_rope: CUDA tensors required (no CPU path)")
    if x.dtype not in _DTYPES:
        raise TypeError("qk_norm_rope: float32/bfloat16/float16 input required")
    c = cos.to(x.dtype).reshape(x.shape[0], x.shape[2]).contiguous()
    s = sin.to(x.dtype).reshape(x.shape[0], x.shape[2]).contiguous()
    return _QKNormRope.apply(x.contiguous(), weight, c, s, float(eps))


def _fused_qwen3_attention_forward(self, hidden_states, position_embeddings, attention_mask,
                                   past_key_values=None, **kwargs):
    from transformers.models.qwen3.modeling_qwen3 import (ALL_ATTENTION_FUNCTIONS,
                                                          eager_attention_forward)
    B, N = hidden_states.shape[:2]
    D = self.head_dim
    cos, sin = position_embeddings
    q = qk_norm_rope(self.q_proj(hidden_states).view(B * N, -1, D), self.q_norm.weight, cos, sin,
                     self.q_norm.variance_epsilon)
    k = qk_norm_rope(self.k_proj(hidden_states).view(B * N, -1, D), self.k_norm.weight, cos, sin,
                     self.k_norm.variance_epsilon)
    query_states = q.view(B, N, -1, D).transpose(1, 2)
    key_states = k.view(B, N, -1, D).transpose(1, 2)
    value_states = self.v_proj(hidden_states).view(B, N, -1, D).transpose(1, 2)
    if past_key_values is not None:
        key_states, value_states = past_key_values.update(key_states, value_states,
                                                          self.layer_idx)
    attention_interface = ALL_ATTENTION_FUNCTIONS.get_interface(
        self.config._attn_implementation, eager_attention_forward)
    attn_output, attn_weights = attention_interface(
        self, query_states, key_states, value_states, attention_mask,
        dropout=0.0 if not self.training else self.attention_dropout, scaling=self.scaling,
        sliding_window=self.sliding_window, **kwargs)
    attn_output = attn_output.reshape(B, N, -1).contiguous()
    return self.o_proj(attn_output), attn_weights


def fuse_attention_prologue(model) -> int:
    """Route every transformers Qwen3 attention module of ``model`` through the
    fused q/k norm + rotary op.  Returns how many modules were patched."""
    from transformers.models.qwen3.modeling_qwen3 import Qwen3Attention
    n = 0
    for mod in model.modules():
        if type(mod) is Qwen3Attention and mod.head_dim in (64, 128, 256):
            mod.forward = types.MethodType(_fused_qwen3_attention_forward, mod)
            n += 1
    return n
