"""Tree gated delta rule and tree-correct conv as torch custom ops.

Drop-ins (same signatures and return conventions as the reference):

* ``torch_chunk_gated_delta_rule_tree_varlen`` (tree_dfs_ssm.py:38-156)
* ``_tree_correct_conv_varlen`` (tree_dfs_ssm.py:285-348)

Both run in the C-ABI library (``tt_gdn_tree_fwd/_bwd``, ``tt_tree_conv_fwd/
_bwd``) with fp32 arithmetic inside; there is no PyTorch fallback.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from .attention import _DTYPES, _stream_ptr


GDN_QK_L2NORM = 1        # TT_GDN_QK_L2NORM
GDN_EXACT_INVERSE = 2    # TT_GDN_EXACT_INVERSE
GDN_SAVED_FORWARD = 4    # TT_GDN_SAVED_FORWARD
_NO_CAPTURE = torch.zeros(0, dtype=torch.int32)


def _tree_arrays(chunk_boundaries, chunk_parent_map) -> Tuple[torch.Tensor, torch.Tensor]:
    """bounds [n, 2] / parents [n] as int32 CPU tensors (lists, arrays or tensors)."""
    if isinstance(chunk_boundaries, torch.Tensor):
        b = chunk_boundaries.detach().to("cpu", torch.int32).reshape(-1, 2).contiguous()
    else:
        b = torch.as_tensor(np.asarray(chunk_boundaries, dtype=np.int32).reshape(-1, 2))
    if isinstance(chunk_parent_map, torch.Tensor):
        p = chunk_parent_map.detach().to("cpu", torch.int32).reshape(-1).contiguous()
    else:
        p = torch.as_tensor(np.asarray(chunk_parent_map, dtype=np.int32).reshape(-1))
    return b, p


# -----------------------------------------------------------------------------
# GDN
# -----------------------------------------------------------------------------

def _ws(S, H, Dk, Dv, bounds: torch.Tensor, backward: bool, device) -> Tuple[torch.Tensor, int]:
    n = int(bounds.shape[0])
    nbytes = int(_lib.lib().tt_gdn_tree_workspace_size(S, H, Dk, Dv, n, bounds.data_ptr(),
                                                       int(backward)))
    if nbytes < 0:
        raise ValueError("tree GDN: invalid chunk boundaries")
    return torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device), nbytes


def _rows_in_place(t: torch.Tensor) -> bool:
    """t [S, heads, dim] whose token rows the kernels can read in place: each
    row [heads, dim] contiguous, rows at a fixed stride of at least a row."""
    S, nh, d = t.shape
    return t.stride(2) == 1 and t.stride(1) == d and (S <= 1 or t.stride(0) >= nh * d)


def _token_strides(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> Tuple[int, int, int]:
    """The token strides the C ABI takes (0 = packed rows)."""
    st = lambda t: 0 if t.is_contiguous() else int(t.stride(0))
    return st(q), st(k), st(v)


@torch.library.custom_op("tt_b200::gdn_tree_fwd", mutates_args=())
def _gdn_fwd_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                beta: torch.Tensor, bounds: torch.Tensor, parents: torch.Tensor,
                init: torch.Tensor, has_init: bool, flags: int, want_last: bool,
                capture: torch.Tensor, keep: bool
                ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """q/k [S, Hk, Dk], v [S, H, Dv] (one dtype), g/beta fp32 [S, H],
    bounds int32 [n, 2], parents int32 [n] (CPU), flags (GDN_QK_L2NORM |
    GDN_EXACT_INVERSE), capture int32 [m] (CPU, distinct node indices) ->
    out [S, H, Dv], last fp32 [H, Dk, Dv] (zeros-shaped when not requested),
    captured fp32 [m, H, Dk, Dv] = the state after each captured node, and
    with ``keep`` the workspace holding the forward pass (sized for the
    backward, which then skips recomputing it), else an empty tensor."""
    S, Hk, Dk = q.shape
    H, Dv = v.shape[1], v.shape[2]
    m = int(capture.numel())
    out = torch.empty((S, H, Dv), dtype=q.dtype, device=q.device)
    last = torch.empty((H, Dk, Dv) if want_last else (0,), dtype=torch.float32, device=q.device)
    cap = torch.empty((m, H, Dk, Dv), dtype=torch.float32, device=q.device)
    ws, nbytes = _ws(S, H, Dk, Dv, bounds, keep, q.device)
    _lib.call("tt_gdn_tree_fwd_ex", _DTYPES[q.dtype], S, Hk, H, Dk, Dv, q.data_ptr(),
              k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), int(bounds.shape[0]),
              bounds.data_ptr(), parents.data_ptr(), init.data_ptr() if has_init else None,
              int(flags), out.data_ptr(), last.data_ptr() if want_last else None, m,
              capture.data_ptr() if m else None, cap.data_ptr() if m else None,
              *_token_strides(q, k, v), ws.data_ptr(), nbytes, _stream_ptr(q.device))
    return out, last, cap, (ws if keep else ws.new_empty(0))


@_gdn_fwd_op.register_fake
def _(q, k, v, g, beta, bounds, parents, init, has_init, flags, want_last, capture, keep):
    S, Hk, Dk = q.shape
    H, Dv = v.shape[1], v.shape[2]
    return (q.new_empty((S, H, Dv)),
            q.new_empty((H, Dk, Dv) if want_last else (0,), dtype=torch.float32),
            q.new_empty((capture.numel(), H, Dk, Dv), dtype=torch.float32),
            q.new_empty(0, dtype=torch.uint8))


@torch.library.custom_op("tt_b200::gdn_tree_bwd", mutates_args=("kept",))
def _gdn_bwd_op(dout: torch.Tensor, dlast: torch.Tensor, has_dlast: bool, q: torch.Tensor,
                k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                bounds: torch.Tensor, parents: torch.Tensor, init: torch.Tensor, has_init: bool,
                flags: int, capture: torch.Tensor, dcap: torch.Tensor,
                has_dcap: bool, kept: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                       torch.Tensor, torch.Tensor]:
    S, Hk, Dk = q.shape
    H, Dv = v.shape[1], v.shape[2]
    packed = lambda t: torch.empty(t.shape, dtype=t.dtype, device=t.device)
    dq, dk, dv = packed(q), packed(k), packed(v)
    dg = torch.empty((S, H), dtype=torch.float32, device=q.device)
    db = torch.empty((S, H), dtype=torch.float32, device=q.device)
    dinit = torch.zeros((H, Dk, Dv) if has_init else (0,), dtype=torch.float32, device=q.device)
    if kept.numel():                     # the forward's workspace, still holding its pass
        ws, nbytes = kept, int(kept.numel())
        flags = int(flags) | GDN_SAVED_FORWARD
    else:
        ws, nbytes = _ws(S, H, Dk, Dv, bounds, True, q.device)
    m = int(capture.numel())
    _lib.call("tt_gdn_tree_bwd_ex", _DTYPES[q.dtype], S, Hk, H, Dk, Dv, q.data_ptr(),
              k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), int(bounds.shape[0]),
              bounds.data_ptr(), parents.data_ptr(), init.data_ptr() if has_init else None,
              int(flags), dout.contiguous().data_ptr(),
              dlast.contiguous().data_ptr() if has_dlast else None, m,
              capture.data_ptr() if m else None,
              dcap.contiguous().data_ptr() if (m and has_dcap) else None, dq.data_ptr(),
              dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), db.data_ptr(),
              dinit.data_ptr() if has_init else None, *_token_strides(q, k, v), ws.data_ptr(),
              nbytes, _stream_ptr(q.device))
    return dq, dk, dv, dg, db, dinit


@_gdn_bwd_op.register_fake
def _(dout, dlast, has_dlast, q, k, v, g, beta, bounds, parents, init, has_init, flags, capture,
      dcap, has_dcap, kept):
    S, Hk, Dk = q.shape
    H, Dv = v.shape[1], v.shape[2]
    f = lambda *s: q.new_empty(s, dtype=torch.float32)
    packed = lambda t: t.new_empty(t.shape)
    return (packed(q), packed(k), packed(v), f(S, H), f(S, H),
            f(H, Dk, Dv) if has_init else f(0))


def _gdn_setup(ctx, inputs, output):
    q, k, v, g, beta, bounds, parents, init, has_init, flags, want_last, capture, keep = inputs
    ctx.save_for_backward(q, k, v, g, beta, bounds, parents, init, capture)
    # the kept workspace: its forward part is read, its backward part written
    # by every backward call, so it is held outside autograd's version checks;
    # it has no gradient, and no zero gradient is built for it (or for any
    # other output the loss does not reach: the backward takes None for those)
    ctx.kept = output[3]
    ctx.mark_non_differentiable(output[3])
    ctx.set_materialize_grads(False)
    ctx.has_init, ctx.flags, ctx.want_last = has_init, flags, want_last


def _gdn_backward(ctx, dout, dlast, dcap, _dkept):
    q, k, v, g, beta, bounds, parents, init, capture = ctx.saved_tensors
    kept = ctx.kept
    has_dlast = ctx.want_last and dlast is not None and dlast.numel() > 0
    has_dcap = dcap is not None and dcap.numel() > 0
    if dout is None:
        dout = torch.zeros((q.shape[0], v.shape[1], v.shape[2]), dtype=q.dtype, device=q.device)
    empty = dout.new_empty(0, dtype=torch.float32)
    dq, dk, dv, dg, db, dinit = _gdn_bwd_op(
        dout, dlast if has_dlast else empty, bool(has_dlast),
        q, k, v, g, beta, bounds, parents, init, ctx.has_init, ctx.flags, capture,
        dcap if has_dcap else empty, bool(has_dcap), kept)
    return (dq, dk, dv, dg, db, None, None, dinit if ctx.has_init else None, None, None, None,
            None, None)


_gdn_fwd_op.register_autograd(_gdn_backward, setup_context=_gdn_setup)


def torch_chunk_gated_delta_rule_tree_varlen(query, key, value, g, beta, chunk_boundaries,
                                             chunk_parent_map, initial_state=None,
                                             output_final_state=False,
                                             use_qk_l2norm_in_kernel=False,
                                             exact_inverse=False, keep_forward=None):
    """Drop-in for tree_dfs_ssm.py:38-156.

    query/key [B, S, Hk, Dk] (Hk == H, or a divisor of H: v-head h then uses
    k-head h // (H // Hk)), value [B, S, H, Dv], g/beta [B, S, H];
    chunk_boundaries / chunk_parent_map as lists or tensors.  Returns
    (core_out [B, S, H, Dv] in query's dtype, last_state [B, H, Dk, Dv] fp32 or
    None) with gradients for every tensor input.

    ``exact_inverse=False`` reproduces the reference, whose intra-node
    correction is the truncated T = I + A + A^2 (tree_dfs_ssm.py:119-126).
    ``exact_inverse=True`` (an addition, not in the reference's signature) uses
    T = (I - A)^-1, i.e. the gated delta rule's token-by-token recurrence along
    each root-to-node path, independent of where node boundaries fall.
    ``keep_forward=True`` keeps the forward's fp32 intermediates on the device
    until the backward (a workspace of ``tt_gdn_tree_workspace_size(...,
    backward=1)`` bytes), which then skips recomputing the forward; ``False``
    holds only the output and recomputes in the backward (about half the
    device memory, a slower backward).  The default (None) keeps them whenever
    autograd will run the backward (grad enabled and an input requires grad),
    as torch autograd keeps the reference loop's intermediates."""
    if keep_forward is None:
        keep_forward = torch.is_grad_enabled() and any(
            isinstance(t, torch.Tensor) and t.requires_grad
            for t in (query, key, value, g, beta, initial_state))
    if query.dtype not in _DTYPES or key.dtype != query.dtype or value.dtype != query.dtype:
        raise TypeError("tree GDN: query, key, value must share one of float32/bfloat16/float16")
    if not query.is_cuda:
        raise RuntimeError("tree GDN: CUDA tensors required (no CPU path)")
    bounds, parents = _tree_arrays(chunk_boundaries, chunk_parent_map)
    B = query.shape[0]
    outs, lasts = [], []
    for b in range(B):
        # rows read in place where the layout allows (the q / k / v views the
        # layer splits off a token-major conv output), else packed copies
        q, k, v = (t[b] if _rows_in_place(t[b]) else t[b].contiguous()
                   for t in (query, key, value))
        gg = g[b].float().contiguous()
        bt = beta[b].float().contiguous()
        has_init = initial_state is not None
        init = (initial_state[b].float().contiguous() if has_init
                else q.new_empty(0, dtype=torch.float32))
        flags = ((GDN_QK_L2NORM if use_qk_l2norm_in_kernel else 0)
                 | (GDN_EXACT_INVERSE if exact_inverse else 0))
        o, last, _, _ = _gdn_fwd_op(q, k, v, gg, bt, bounds, parents, init, has_init, flags,
                                    bool(output_final_state), _NO_CAPTURE, bool(keep_forward))
        outs.append(o)
        lasts.append(last)
    # batch 1 (every tree of the reference): a view, not a copy
    core = outs[0].unsqueeze(0) if B == 1 else torch.stack(outs, 0)
    last_state = None
    if output_final_state:
        last_state = lasts[0].unsqueeze(0) if B == 1 else torch.stack(lasts, 0)
    return core, last_state


# -----------------------------------------------------------------------------
# tree conv
# -----------------------------------------------------------------------------

class TreeConvPlan:
    """Predecessor / successor tables of one tree for a width-K conv (device).

    The four tables travel in one pinned host buffer by one asynchronous copy:
    a copy from pageable memory would synchronise the stream, so the host
    would wait for every kernel queued before it."""

    def __init__(self, bounds: torch.Tensor, parents: torch.Tensor, K: int, device):
        n = int(bounds.shape[0])
        S = int(bounds[-1, 1]) if n else 0
        self.S, self.K = S, K
        pred = np.zeros((max(S, 1), max(K - 1, 1)), np.int32)
        _lib.call("tt_conv_predecessors", n, bounds.data_ptr(), parents.data_ptr(), K,
                  pred.ctypes.data)
        cap = max(S * max(K - 1, 1), 1)
        sp = np.zeros(S + 1, np.int32)
        stok = np.zeros(cap, np.int32)
        slag = np.zeros(cap, np.int32)
        _lib.call("tt_conv_successors", S, K, pred.ctypes.data, sp.ctypes.data, stok.ctypes.data,
                  slag.ctypes.data, cap)
        # each table starts on a 16-byte boundary (the 4-token kernels read
        # the predecessor rows of 4 tokens at once)
        parts = [pred.reshape(-1), sp, stok, slag]
        offs, total = [], 0
        for a in parts:
            offs.append(total)
            total += (a.size + 3) // 4 * 4
        pinned = torch.device(device).type == "cuda"
        host = torch.zeros(total, dtype=torch.int32, pin_memory=pinned)
        hv = host.numpy()
        for o, a in zip(offs, parts):
            hv[o:o + a.size] = a
        dev = host.to(device, non_blocking=pinned)
        self._host = host
        self.pred = dev[offs[0]:offs[0] + pred.size].view(pred.shape)
        self.succ_ptr = dev[offs[1]:offs[1] + sp.size]
        self.succ_tok = dev[offs[2]:offs[2] + cap]
        self.succ_lag = dev[offs[3]:offs[3] + cap]


_conv_plans: "dict" = {}
_CONV_PLAN_CACHE = 16


def _conv_plan(bounds: torch.Tensor, parents: torch.Tensor, K: int, device) -> TreeConvPlan:
    """The plan of a tree, reused while the same tree (same node bounds and
    parents) comes back: a training step calls the conv on one tree once per
    layer."""
    key = (bounds.numpy().tobytes(), parents.numpy().tobytes(), int(K), str(torch.device(device)))
    plan = _conv_plans.pop(key, None)
    if plan is None:
        plan = TreeConvPlan(bounds, parents, K, device)
        while len(_conv_plans) >= _CONV_PLAN_CACHE:
            _conv_plans.pop(next(iter(_conv_plans)))
    _conv_plans[key] = plan      # most recently used last
    return plan


def _tm_sizes_ok(C: int, S: int, dtype: torch.dtype) -> bool:
    """Sizes the token-major conv kernels take: C % 8 == 0 and whole 16-byte
    chunks of tokens per channel row (S * element size % 16 == 0)."""
    el = torch.empty((), dtype=dtype).element_size()
    return C % 8 == 0 and (S * el) % 16 == 0


def _token_major_ok(t: torch.Tensor) -> bool:
    """t [C, S] held token-major (strides (1, C)) with the sizes and 16-byte
    base the token-major conv kernels need."""
    C, S = t.shape
    return t.stride() == (1, C) and _tm_sizes_ok(C, S, t.dtype) and t.data_ptr() % 16 == 0


def _conv_out(x: torch.Tensor, token_major: bool) -> torch.Tensor:
    """The conv output [C, S]: token-major memory (strides (1, C)) or plain."""
    C, S = x.shape
    return x.new_empty((S, C)).t() if token_major else torch.empty_like(x)


@torch.library.custom_op("tt_b200::tree_conv_fwd", mutates_args=())
def _conv_fwd_op(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, has_b: bool,
                 pred: torch.Tensor, sp: torch.Tensor, stok: torch.Tensor,
                 slag: torch.Tensor, token_major: bool) -> torch.Tensor:
    C, S = x.shape
    K = w.shape[1]
    out = _conv_out(x, token_major)
    _lib.call("tt_tree_conv_fwd_ex", _DTYPES[x.dtype], C, S, K, x.data_ptr(), w.data_ptr(),
              b.data_ptr() if has_b else None, pred.data_ptr(), out.data_ptr(),
              int(token_major), _stream_ptr(x.device))
    return out


@_conv_fwd_op.register_fake
def _(x, w, b, has_b, pred, sp, stok, slag, token_major):
    return _conv_out(x, token_major)


@torch.library.custom_op("tt_b200::tree_conv_bwd", mutates_args=())
def _conv_bwd_op(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor,
                 has_b: bool, pred: torch.Tensor, sp: torch.Tensor, stok: torch.Tensor,
                 slag: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    C, S = x.shape
    K = w.shape[1]
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    db = torch.empty((C,) if has_b else (0,), dtype=torch.float32, device=x.device)
    ws_bytes = int(_lib.lib().tt_tree_conv_bwd_workspace_size(C, S, K))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=x.device)
    # a gradient in token-major memory (what autograd hands back through the
    # layer's transpose + split of a token-major output) is read in place
    tm = _token_major_ok(dy) and x.data_ptr() % 16 == 0
    if not tm:
        dy = dy.contiguous()
    _lib.call("tt_tree_conv_bwd_ex", _DTYPES[x.dtype], C, S, K, x.data_ptr(), w.data_ptr(),
              b.data_ptr() if has_b else None, pred.data_ptr(), sp.data_ptr(), stok.data_ptr(),
              slag.data_ptr(), dy.data_ptr(), int(tm), dx.data_ptr(), dw.data_ptr(),
              db.data_ptr() if has_b else None, ws.data_ptr(), ws_bytes, _stream_ptr(x.device))
    return dx, dw, db


@_conv_bwd_op.register_fake
def _(dy, x, w, b, has_b, pred, sp, stok, slag):
    return (torch.empty_like(x), torch.empty_like(w),
            x.new_empty((x.shape[0],) if has_b else (0,), dtype=torch.float32))


def _conv_setup(ctx, inputs, output):
    x, w, b, has_b, pred, sp, stok, slag, _token_major = inputs
    ctx.save_for_backward(x, w, b, pred, sp, stok, slag)
    ctx.has_b = has_b


def _conv_backward(ctx, dy):
    x, w, b, pred, sp, stok, slag = ctx.saved_tensors
    dx, dw, db = _conv_bwd_op(dy, x, w, b, ctx.has_b, pred, sp, stok, slag)
    return dx, dw, (db if ctx.has_b else None), None, None, None, None, None, None


_conv_fwd_op.register_autograd(_conv_backward, setup_context=_conv_setup)


def tree_conv(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
              chunk_boundaries, chunk_parent_map) -> torch.Tensor:
    """silu(depthwise causal conv over each token's tree path).  x [B, C, S],
    weight [C, K] (or [C, 1, K] as stored by nn.Conv1d), bias [C] or None."""
    if not x.is_cuda:
        raise RuntimeError("tree conv: CUDA tensors required (no CPU path)")
    if x.dtype not in _DTYPES:
        raise TypeError("tree conv: float32/bfloat16/float16 input required")
    w = weight.reshape(weight.shape[0], -1).float().contiguous()
    bounds, parents = _tree_arrays(chunk_boundaries, chunk_parent_map)
    plan = _conv_plan(bounds, parents, int(w.shape[1]), x.device)
    has_b = bias is not None
    b = bias.float().contiguous() if has_b else w.new_empty(0)
    # batch 1 (every tree of the reference): the output in token-major memory
    # when the kernels allow it, so the layer's transpose + split into q / k / v
    # (dfs_tree_forward.py:403-410) are views with no transposing copy
    outs = []
    for i in range(x.shape[0]):
        xi = x[i].contiguous()
        tm = (x.shape[0] == 1 and _tm_sizes_ok(xi.shape[0], xi.shape[1], xi.dtype)
              and xi.data_ptr() % 16 == 0)
        outs.append(_conv_fwd_op(xi, w, b, has_b, plan.pred, plan.succ_ptr, plan.succ_tok,
                                 plan.succ_lag, tm))
    return outs[0].unsqueeze(0) if len(outs) == 1 else torch.stack(outs, 0)


def _tree_correct_conv_varlen(ssm, mixed_qkv_raw, chunk_boundaries, chunk_parent_map):
    """Drop-in for tree_dfs_ssm.py:285-348: uses ``ssm.conv1d`` (weight
    [C, 1, K], optional bias) with SiLU, on [B, C, S]."""
    act = getattr(ssm, "activation", "silu")
    if act not in ("silu", "swish"):
        raise ValueError(f"tree conv implements SiLU only, got activation={act!r}")
    return tree_conv(mixed_qkv_raw, ssm.conv1d.weight, ssm.conv1d.bias, chunk_boundaries,
                     chunk_parent_map)
