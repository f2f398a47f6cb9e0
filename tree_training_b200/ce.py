"""Leaf-token LM head + cross-entropy without the [tokens, vocab] logits.

The reference's loss (make_tree_loss_fn, tree_grad_hybrid.py:546-558) is, per
loss leaf, ``F.cross_entropy(logits[leaf tokens], labels) / n_leaves`` on the
full-vocabulary logits of the partition (151,936 columns for Qwen3 models), and
autograd keeps those logits alive until the backward.  Here the same sum of
per-token losses,  sum_t w_t * CE(h_t W^T, y_t)  with  w_t = 1 / (len(leaf) *
n_leaves),  is computed over chunks of tokens:

  forward   logits_c = h_c W^T (cuBLAS, model dtype); loss_c (``tt_ce_fwd_grad``,
            loss only); the logits are dropped
  backward  logits_c recomputed; dlogits_c = w (softmax - onehot) in place
            (``tt_ce_fwd_grad``); dH_c = dlogits_c W; dW += dlogits_c^T h_c
            (fp32 accumulation)

so at most one chunk of logits exists at a time and the forward keeps only
the hidden states it was given.  The recompute costs one more LM-head GEMM
per chunk, which is small next to a decoder step.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .attention import _stream_ptr

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _ce_chunk(logits: torch.Tensor, labels: torch.Tensor, weights: torch.Tensor,
              ignore_index: int, loss: torch.Tensor, write_grad: bool) -> None:
    n, V = logits.shape
    _lib.call("tt_ce_fwd_grad", _DTYPES[logits.dtype], n, V, logits.data_ptr(),
              logits.stride(0), labels.data_ptr(), weights.data_ptr(), int(ignore_index),
              loss.data_ptr(), int(write_grad), _stream_ptr(logits.device))


class _FusedLinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, weight, labels, weights, chunk: int, ignore_index: int):
        T = h.shape[0]
        loss = torch.empty(T, dtype=torch.float32, device=h.device)
        wt = weight.t()
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            logits = torch.mm(h[c0:c1], wt)
            _ce_chunk(logits, labels[c0:c1], weights[c0:c1], ignore_index, loss[c0:c1], False)
            del logits
        ctx.save_for_backward(h, weight, labels, weights)
        ctx.chunk, ctx.ignore_index = chunk, ignore_index
        return loss.sum()

    @staticmethod
    def backward(ctx, go):
        h, weight, labels, weights = ctx.saved_tensors
        T = h.shape[0]
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dh = torch.empty_like(h) if need_h else None
        dw = torch.zeros(weight.shape, dtype=torch.float32, device=h.device) if need_w else None
        scratch = torch.empty(T, dtype=torch.float32, device=h.device)
        wt = weight.t()
        # the incoming gradient scales every token's weight
        ws = weights * go.float()
        for c0 in range(0, T, ctx.chunk):
            c1 = min(T, c0 + ctx.chunk)
            hc = h[c0:c1]
            logits = torch.mm(hc, wt)
            _ce_chunk(logits, labels[c0:c1], ws[c0:c1], ctx.ignore_index, scratch[c0:c1], True)
            if need_h:
                torch.mm(logits, weight, out=dh[c0:c1])
            if need_w:
                if logits.dtype == torch.float32:
                    dw.addmm_(logits.t(), hc)
                else:
                    dw += torch.mm(logits.t(), hc, out_dtype=torch.float32)
            del logits
        return dh, (dw.to(weight.dtype) if need_w else None), None, None, None, None


def fused_linear_cross_entropy(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                               token_weights: Optional[torch.Tensor] = None,
                               ignore_index: int = -100, chunk: int = 4096) -> torch.Tensor:
    """sum_t w_t * cross_entropy(hidden_t @ weight^T, labels_t) with gradients
    for ``hidden`` [T, H] and ``weight`` [V, H] (an LM head's weight); labels
    [T] int64; token_weights [T] (default 1).  Ignored labels contribute 0.
    CUDA tensors only (no CPU path)."""
    if not hidden.is_cuda:
        raise RuntimeError("fused cross-entropy: CUDA tensors required (no CPU path)")
    if hidden.dtype not in _DTYPES or weight.dtype != hidden.dtype:
        raise TypeError("fused cross-entropy: hidden and weight must share fp32/bf16/fp16")
    T = hidden.shape[0]
    lab = labels.to(device=hidden.device, dtype=torch.int64).contiguous()
    w = (torch.ones(T, dtype=torch.float32, device=hidden.device) if token_weights is None
         else token_weights.to(device=hidden.device, dtype=torch.float32).contiguous())
    return _FusedLinearCE.apply(hidden.contiguous(), weight, lab, w, int(chunk), int(ignore_index))
