"""Tree attention as a torch custom op with autograd, and its HF registration.

The op replaces what the reference gets from HF's SDPA call with a dense
additive mask (dfs_tree_forward.py:548-560, tree_grad_hybrid.py:312-317 ->
TF/integrations/sdpa_attention.py:40-104): O = softmax(Q K^T * scale + M) V
with GQA, M given as one visible-row interval per key.  Forward and backward
run in the C-ABI library (tcgen05 kernels for bf16/fp16 head_dim 128, exact
CUDA-core kernels otherwise).  There is no PyTorch or CPU fallback: a CPU
tensor or a missing library raises.
"""
from __future__ import annotations

import os
from typing import Optional, Tuple

import numpy as np
import torch

from . import _lib
from .packer import TreeAttnMeta

_DTYPES = {torch.float32: _lib.TT_F32, torch.bfloat16: _lib.TT_BF16, torch.float16: _lib.TT_F16}

_status: dict = {}


def _status_word(device: torch.device) -> torch.Tensor:
    s = _status.get(device)
    if s is None:
        s = torch.zeros(1, dtype=torch.int32, device=device)
        _status[device] = s
    return s


def check_device_status(device: Optional[torch.device] = None) -> None:
    """Raise if a kernel on ``device`` recorded an error (e.g. a bounded wait
    that timed out).  Synchronises with the device; call between steps."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    s = _status.get(dev)
    if s is not None:
        code = int(s.item())
        if code:
            s.zero_()
            raise _lib.TTError("device kernel", code)
    # the tree GDN's tensor-core kernels record into a word of their own
    word = np.zeros(1, np.int32)
    with torch.cuda.device(dev):
        _lib.call("tt_gdn_take_device_status", word.ctypes.data)
    if int(word[0]):
        raise _lib.TTError("tree GDN kernel", int(word[0]))


def lse_ld(n_q: int) -> int:
    """Row stride of the LSE / delta buffers: n_q rounded up to 128."""
    return (n_q + 127) // 128 * 128


_tile_cache: dict = {}


def tile_shape(dtype: torch.dtype, head_dim: int, kind: int) -> Tuple[int, int]:
    """Tile shape the library's kernels expect (cached per kernel-path setting)."""
    key = (_lib.path_generation(), dtype, head_dim, kind)
    t = _tile_cache.get(key)
    if t is None:
        tq = np.zeros(1, np.int32)
        tk = np.zeros(1, np.int32)
        _lib.call("tt_attn_tile_shape", _DTYPES[dtype], head_dim, kind, tq.ctypes.data,
                  tk.ctypes.data)
        t = (int(tq[0]), int(tk[0]))
        _tile_cache[key] = t
    return t


def _check_tensor(name, t, ndim=3):
    if not t.is_cuda:
        raise RuntimeError(f"tree attention: {name} must be a CUDA tensor (no CPU path)")
    if t.dim() != ndim or t.stride(-1) != 1:
        raise RuntimeError(f"tree attention: {name} must be [tokens, heads, dim] with unit last stride")


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# -----------------------------------------------------------------------------
# raw launches (no autograd)
# -----------------------------------------------------------------------------

def attn_fwd_raw(q, k, v, meta_dev, scale: float):
    """q [n_q, hq, D], k/v [n_kv, hkv, D] -> out [n_q, hq, D] (q.dtype), lse [hq, n_q]."""
    for n, t in (("q", q), ("k", k), ("v", v)):
        _check_tensor(n, t)
    n_q, hq, D = q.shape
    n_kv, hkv, _ = k.shape
    out = torch.empty((n_q, hq, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((hq, lse_ld(n_q)), dtype=torch.float32, device=q.device)
    _lib.call("tt_tree_attn_fwd", _DTYPES[q.dtype], n_q, n_kv, hq, hkv, D,
              q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
              v.data_ptr(), v.stride(0), v.stride(1), meta_dev["kv_lo"].data_ptr(),
              meta_dev["kv_hi"].data_ptr(), meta_dev["fwd_ptr"].data_ptr(),
              meta_dev["fwd_list"].data_ptr(), float(scale), out.data_ptr(), lse.data_ptr(),
              _status_word(q.device).data_ptr(), _stream_ptr(q.device))
    return out, lse


# Backward schedule on the tcgen05 path: "stored" (default) keeps every dS tile
# the dK/dV kernel forms in a workspace and sums dQ from it; "recompute" runs
# the dQ kernel that recomputes S and dP beside dK/dV on a second stream.
_BWD_SCHEDULE = os.environ.get("TT_ATTN_BWD_SCHEDULE", "stored")
# Most workspace bytes the stored schedule's dS slots may take; larger problems
# run in passes over the kv heads (one pass needs rep * n_tile_pairs * 32 KB).
_DS_WORKSPACE_CAP = int(float(os.environ.get("TT_ATTN_DS_WORKSPACE_GB", "16")) * (1 << 30))


def set_backward_schedule(schedule: str) -> str:
    """Select the tcgen05 backward schedule ("stored" or "recompute");
    returns the previous one.  Both are deterministic and give dK/dV bit for
    bit equal; dQ differs only by the rounding of its recomputed dS."""
    global _BWD_SCHEDULE
    if schedule not in ("stored", "recompute"):
        raise ValueError(f"unknown backward schedule {schedule!r}")
    prev, _BWD_SCHEDULE = _BWD_SCHEDULE, schedule
    return prev


def _stored_plan(dt, n_q, n_kv, hq, hkv, D, n_pairs):
    """(kv heads per pass, workspace bytes) of the stored schedule: the most kv
    heads whose dS slots fit the cap.  None when the schedule is off, the
    problem is off the tcgen05 path, or one pass alone exceeds the cap (the
    recompute schedule then runs)."""
    if _BWD_SCHEDULE != "stored" or n_q == 0 or n_kv == 0:
        return None
    L = _lib.lib()
    regular = int(L.tt_tree_attn_bwd_workspace_size(dt, n_q, n_kv, hq, hkv, D))
    for p in range(hkv, 0, -1):
        b = int(L.tt_tree_attn_bwd_stored_workspace_size(dt, n_q, n_kv, hq, hkv, D, n_pairs, p))
        if b <= regular:
            return None            # off the tcgen05 path: nothing is stored
        if b - regular <= _DS_WORKSPACE_CAP:
            return p, b
    return None


def attn_bwd_raw(dout, q, k, v, out, lse, meta_dev, scale: float):
    for n, t in (("dout", dout), ("q", q), ("k", k), ("v", v)):
        _check_tensor(n, t)
    n_q, hq, D = q.shape
    n_kv, hkv, _ = k.shape
    dt = _DTYPES[q.dtype]
    dq = torch.empty((n_q, hq, D), dtype=q.dtype, device=q.device)
    dk = torch.empty((n_kv, hkv, D), dtype=k.dtype, device=k.device)
    dv = torch.empty((n_kv, hkv, D), dtype=v.dtype, device=v.device)
    n_pairs = int(meta_dev["fwd_list"].numel())
    plan = _stored_plan(dt, n_q, n_kv, hq, hkv, D, n_pairs)
    if plan is not None:
        ws_bytes = plan[1]
    else:
        ws_bytes = int(_lib.lib().tt_tree_attn_bwd_workspace_size(dt, n_q, n_kv, hq, hkv, D))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)
    out = out.contiguous()
    args = [dt, n_q, n_kv, hq, hkv, D,
            q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
            v.data_ptr(), v.stride(0), v.stride(1), out.data_ptr(), dout.data_ptr(),
            dout.stride(0), dout.stride(1), lse.data_ptr(), meta_dev["kv_lo"].data_ptr(),
            meta_dev["kv_hi"].data_ptr(), meta_dev["fwd_ptr"].data_ptr(),
            meta_dev["fwd_list"].data_ptr(), meta_dev["bwd_ptr"].data_ptr(),
            meta_dev["bwd_list"].data_ptr(), float(scale),
            dq.data_ptr(), dq.stride(0), dq.stride(1), dk.data_ptr(), dk.stride(0),
            dk.stride(1), dv.data_ptr(), dv.stride(0), dv.stride(1)]
    status = _status_word(q.device).data_ptr()
    main = torch.cuda.current_stream(q.device)
    timer = _PHASE_TIMER
    if plan is not None:
        sargs = args + [n_pairs, plan[0], ws.data_ptr(), ws_bytes]
        if plan[0] == hkv and timer is not None:
            # one pass: the phases as separate calls, with events between them
            timer.mark(main, "bwd_start")
            _lib.call("tt_tree_attn_bwd_stored", *sargs, _lib.TT_BWD_PREP, status,
                      main.cuda_stream)
            timer.mark(main, "prep_done")
            _lib.call("tt_tree_attn_bwd_stored", *sargs, _lib.TT_BWD_DKDV, status,
                      main.cuda_stream)
            timer.mark(main, "dkdv_done")
            timer.mark(main, "dq_start")
            _lib.call("tt_tree_attn_bwd_stored", *sargs, _lib.TT_BWD_DQ, status,
                      main.cuda_stream)
            timer.mark(main, "dq_done")
        else:
            if timer is not None:
                timer.mark(main, "bwd_start")
            _lib.call("tt_tree_attn_bwd_stored", *sargs, _lib.TT_BWD_ALL, status,
                      main.cuda_stream)
            if timer is not None:
                timer.mark(main, "bwd_all_done")
        return dq, dk, dv
    args += [ws.data_ptr(), ws_bytes]
    if timer is not None:
        timer.mark(main, "bwd_start")
    _lib.call("tt_tree_attn_bwd", *args, _lib.TT_BWD_PREP, status, main.cuda_stream)
    if timer is not None:
        timer.mark(main, "prep_done")
    # dK/dV and dQ only share read-only inputs: run them side by side
    side = _side_stream(q.device)
    side.wait_stream(main)
    _lib.call("tt_tree_attn_bwd", *args, _lib.TT_BWD_DKDV, status, main.cuda_stream)
    if timer is not None:
        timer.mark(main, "dkdv_done")
    with torch.cuda.stream(side):
        _lib.call("tt_tree_attn_bwd", *args, _lib.TT_BWD_DQ, status, side.cuda_stream)
        if timer is not None:
            timer.mark(side, "dq_done")
    # Every tensor the side stream touched was allocated on `main`, and `main`
    # waits for the side stream here, so any later reuse of their memory (which
    # the caching allocator orders on `main`) is ordered after the dQ kernel.
    main.wait_stream(side)
    return dq, dk, dv


_side_streams: dict = {}
_PHASE_TIMER = None


def _side_stream(device) -> torch.cuda.Stream:
    s = _side_streams.get(device)
    if s is None:
        s = torch.cuda.Stream(device=device)
        _side_streams[device] = s
    return s


def set_phase_timer(timer) -> None:
    """Install an object with ``mark(stream, name)`` that records CUDA events
    between the backward's kernels (used by bench.py to time each kernel
    live); ``None`` removes it."""
    global _PHASE_TIMER
    _PHASE_TIMER = timer


# -----------------------------------------------------------------------------
# custom op + autograd
# -----------------------------------------------------------------------------

@torch.library.custom_op("tt_b200::tree_attn_fwd", mutates_args=())
def _tree_attn_fwd_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_lo: torch.Tensor,
                      kv_hi: torch.Tensor, fwd_ptr: torch.Tensor, fwd_list: torch.Tensor,
                      b_fwd_ptr: torch.Tensor, b_fwd_list: torch.Tensor, b_bwd_ptr: torch.Tensor,
                      b_bwd_list: torch.Tensor,
                      scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """Forward launch.  ``fwd_*`` are the work lists for the forward tile
    shape; ``b_*`` the lists for the backward tile shape (kept for autograd)."""
    md = dict(kv_lo=kv_lo, kv_hi=kv_hi, fwd_ptr=fwd_ptr, fwd_list=fwd_list)
    return attn_fwd_raw(q, k, v, md, scale)


@_tree_attn_fwd_op.register_fake
def _(q, k, v, kv_lo, kv_hi, fwd_ptr, fwd_list, b_fwd_ptr, b_fwd_list, b_bwd_ptr, b_bwd_list,
      scale):
    n_q, hq, D = q.shape
    return q.new_empty((n_q, hq, D)), q.new_empty((hq, lse_ld(n_q)), dtype=torch.float32)


@torch.library.custom_op("tt_b200::tree_attn_bwd", mutates_args=())
def _tree_attn_bwd_op(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      out: torch.Tensor, lse: torch.Tensor, kv_lo: torch.Tensor,
                      kv_hi: torch.Tensor, fwd_ptr: torch.Tensor, fwd_list: torch.Tensor,
                      bwd_ptr: torch.Tensor, bwd_list: torch.Tensor,
                      scale: float) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    md = dict(kv_lo=kv_lo, kv_hi=kv_hi, fwd_ptr=fwd_ptr, fwd_list=fwd_list, bwd_ptr=bwd_ptr,
              bwd_list=bwd_list)
    return attn_bwd_raw(dout, q, k, v, out, lse, md, scale)


@_tree_attn_bwd_op.register_fake
def _(dout, q, k, v, out, lse, kv_lo, kv_hi, fwd_ptr, fwd_list, bwd_ptr, bwd_list, scale):
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)


def _setup_context(ctx, inputs, output):
    (q, k, v, kv_lo, kv_hi, _fp, _fl, b_fp, b_fl, b_bp, b_bl, scale) = inputs
    out, lse = output
    ctx.save_for_backward(q, k, v, out, lse, kv_lo, kv_hi, b_fp, b_fl, b_bp, b_bl)
    ctx.scale = scale


def _backward(ctx, dout, dlse):
    q, k, v, out, lse, kv_lo, kv_hi, b_fp, b_fl, b_bp, b_bl = ctx.saved_tensors
    if dout.stride(-1) != 1:
        dout = dout.contiguous()
    dq, dk, dv = _tree_attn_bwd_op(dout, q, k, v, out, lse, kv_lo, kv_hi, b_fp, b_fl, b_bp,
                                   b_bl, ctx.scale)
    return dq, dk, dv, None, None, None, None, None, None, None, None, None


_tree_attn_fwd_op.register_autograd(_backward, setup_context=_setup_context)


def tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, meta: TreeAttnMeta,
                   scale: Optional[float] = None) -> torch.Tensor:
    """Differentiable tree attention.  q [n_q, hq, D], k/v [n_kv, hkv, D]
    (last dim contiguous, any token/head strides) -> out [n_q, hq, D]."""
    if q.shape[0] != meta.n_q or k.shape[0] != meta.n_kv:
        raise ValueError(f"tree attention: q/k lengths {q.shape[0]}/{k.shape[0]} do not match "
                         f"the tree metadata {meta.n_q}/{meta.n_kv}")
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("tree attention: q, k, v must share one of float32/bfloat16/float16")
    D = q.shape[-1]
    if scale is None:
        scale = D ** -0.5
    q, k, v = (_aligned(t) for t in (q, k, v))
    md = meta.device(q.device, *tile_shape(q.dtype, D, 0))
    mb = meta.device(q.device, *tile_shape(q.dtype, D, 1))
    if meta.prefetched:
        # uploaded on another stream (prefetch_tree_meta): keep the caching
        # allocator from reusing the memory while this stream's kernels read it
        cur = torch.cuda.current_stream(q.device)
        for x in (md["kv_lo"], md["fwd_ptr"], mb["fwd_ptr"]):
            x.record_stream(cur)
    out, _ = _tree_attn_fwd_op(q, k, v, md["kv_lo"], md["kv_hi"], md["fwd_ptr"], md["fwd_list"],
                               mb["fwd_ptr"], mb["fwd_list"], mb["bwd_ptr"], mb["bwd_list"],
                               float(scale))
    return out


def prefetch_tree_meta(meta: TreeAttnMeta, device: torch.device, dtype: torch.dtype,
                       head_dim: int) -> TreeAttnMeta:
    """Upload the tree's kernel metadata for ``tree_attention`` on ``device``
    on the CURRENT stream, ahead of the call: a training loop's prefetch stage
    calls it on its upload stream beside the step's q/k/v copies (and orders
    the compute stream after that stream, as for the inputs), so the compute
    stream never waits for a copy queued behind a large upload.  Returns
    ``meta``."""
    for kind in (0, 1):
        meta.device(device, *tile_shape(dtype, head_dim, kind))
    meta.prefetched = True
    return meta


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """TMA wants 16-byte aligned bases and strides; copy otherwise."""
    es = t.element_size()
    if (t.stride(-1) != 1 or t.data_ptr() % 16 or (t.stride(0) * es) % 16
            or (t.stride(1) * es) % 16):
        return t.contiguous()
    return t


# -----------------------------------------------------------------------------
# dense mask -> intervals (lets the reference's own drivers run unchanged)
# -----------------------------------------------------------------------------

def meta_from_dense_mask(mask: torch.Tensor) -> TreeAttnMeta:
    """Key intervals of a [.., n_q, n_kv] additive (0 / -inf) or boolean mask,
    computed on the GPU.  Raises if the mask is not a tree mask (some column's
    visible rows are not one contiguous run)."""
    m = mask
    while m.dim() > 2:
        if m.shape[0] != 1:
            raise ValueError("tree attention supports batch 1 (one packed sequence)")
        m = m[0]
    n_q, n_kv = m.shape
    if m.dtype == torch.bool:
        m = m.view(torch.uint8)
        dt = _lib.TT_U8
    else:
        dt = _DTYPES[m.dtype]
    dev = m.device
    lo = torch.empty(n_kv, dtype=torch.int32, device=dev)
    hi = torch.empty(n_kv, dtype=torch.int32, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call("tt_mask_to_intervals", dt, n_q, n_kv, m.data_ptr(), m.stride(0), m.stride(1),
              lo.data_ptr(), hi.data_ptr(), st.data_ptr(), _stream_ptr(dev))
    code = int(st.item())
    if code:
        raise _lib.TTError("tt_mask_to_intervals", code)
    return TreeAttnMeta(n_q, lo.cpu().numpy(), hi.cpu().numpy())


def tree_attention_forward(module, query, key, value, attention_mask, dropout: float = 0.0,
                           scaling: Optional[float] = None, sliding_window=None, **kwargs):
    """HF attention-interface function (drop-in for sdpa_attention_forward,
    TF/integrations/sdpa_attention.py:40-104).

    query [1, Hq, n_q, D], key/value [1, Hkv, n_kv, D] -> ([1, n_q, Hq, D], None).
    Tree metadata comes from ``kwargs['tree_meta']``, else from a
    ``tree_meta`` attribute on ``attention_mask``, else the dense mask itself
    is converted to key intervals on the GPU (cached on the mask tensor)."""
    if dropout:
        raise ValueError("tree attention does not implement dropout")
    if sliding_window is not None:
        raise ValueError("tree attention does not implement sliding windows")
    if query.shape[0] != 1:
        raise ValueError("tree attention supports batch 1 (one packed sequence)")
    meta = kwargs.get("tree_meta")
    if meta is None and attention_mask is not None:
        meta = getattr(attention_mask, "tree_meta", None)
        if meta is None:
            meta = meta_from_dense_mask(attention_mask)
            try:
                attention_mask.tree_meta = meta
            except Exception:
                pass
    if meta is None:
        raise ValueError("tree attention needs tree metadata (tree_meta=...) or a tree mask")
    q = query[0].transpose(0, 1)
    k = key[0].transpose(0, 1)
    v = value[0].transpose(0, 1)
    out = tree_attention(q, k, v, meta, scaling)
    return out.unsqueeze(0), None


ATTN_IMPL_NAME = "tree_sm100"


def register_hf_attention(name: str = ATTN_IMPL_NAME) -> str:
    """Register :func:`tree_attention_forward` with transformers'
    AttentionInterface so ``config._attn_implementation = name`` selects it."""
    from transformers import AttentionInterface
    AttentionInterface.register(name, tree_attention_forward)
    return name


def tree_mask_placeholder(meta: TreeAttnMeta, dtype=torch.float32, device=None) -> torch.Tensor:
    """A stride-0 [1, 1, n_q, n_kv] tensor that carries ``meta`` through HF's
    mask plumbing (a 4-D mask is passed on unchanged, TF/masking_utils.py:827-829)."""
    t = torch.zeros(1, 1, 1, 1, dtype=dtype, device=device).expand(1, 1, meta.n_q, meta.n_kv)
    t.tree_meta = meta
    return t
