"""Tree-aware Gated DeltaNet layers for hybrid (linear + full attention) models,
with the SSM gateway that partitioned training passes between partitions.

The reference does this in three places with one algorithm: the tree SSM
forward of dfs_tree_forward.py (lines 253-353 and 420-433), the capture /
inject functions of tree_grad_hybrid_ssm.py (lines 48-353) and their use in
tree_grad_hybrid.py (lines 232-250, 325-362).  Per linear-attention layer and
partition:

* the token projections, gated RMSNorm and output projection are per token,
  so they run once over the whole DFS sequence (the gated RMSNorm as one fused
  kernel each way, ``gated_norm.gated_rmsnorm``, for transformers' torch
  ``*RMSNormGated`` modules);
* the depthwise conv reads each token's K-1 predecessors on its
  root-to-node path (``gdn.tree_conv``); the partition's root chunks continue
  the gateway's conv context (the last K-1 pre-conv inputs on the path to the
  cut node in the parent partition);
* the gated delta rule routes each node from its parent node's state
  (``gdn`` ops); the partition's root chunks start from the gateway's
  recurrent state (the state after the cut node);
* at each of the partition's own cut nodes the same two things are captured
  for the child partition, with their autograd history.

Unlike the reference, a partition that both received an SSM gateway and has
cuts of its own both injects and captures (the reference's parent-capture
branch never injects, so such a partition restarts from a zero state).
"""
from __future__ import annotations

from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from .gated_norm import fusable, gated_rmsnorm
from .gdn import (GDN_EXACT_INVERSE, GDN_QK_L2NORM, _gdn_fwd_op, _tree_arrays, tree_conv)


def has_ssm_layers(model) -> bool:
    """True when the model has Qwen3.5-style linear-attention layers
    (``layer.linear_attn``), the test tree_grad_hybrid_ssm.py:384 uses."""
    layers = getattr(getattr(model, "model", model), "layers", [])
    return any(hasattr(l, "linear_attn") for l in layers)


def ssm_layers(model) -> List[Tuple[int, torch.nn.Module]]:
    layers = getattr(getattr(model, "model", model), "layers", [])
    return [(i, l.linear_attn) for i, l in enumerate(layers) if hasattr(l, "linear_attn")]


# -----------------------------------------------------------------------------
# the two stateful operators with capture / inject
# -----------------------------------------------------------------------------

def ssm_varlen_capture(query, key, value, g, beta, chunk_boundaries, chunk_parent_map,
                       initial_state: Optional[torch.Tensor] = None,
                       capture_states_at: Optional[Iterable[int]] = None,
                       use_qk_l2norm: bool = True, exact_inverse: bool = False
                       ) -> Tuple[torch.Tensor, Dict[int, torch.Tensor]]:
    """Tree GDN that also returns the state after each node in
    ``capture_states_at`` (tree_grad_hybrid_ssm.py:48-135).

    query/key [B, S, Hk, Dk] (Hk divides H; no repeat needed), value
    [B, S, H, Dv], g/beta [B, S, H]; initial_state [B, H, Dk, Dv] feeds the
    root chunks.  Returns (core_out [B, S, H, Dv] in query's dtype,
    {chunk index: state [B, H, Dk, Dv] fp32}); the states carry gradients."""
    if not query.is_cuda:
        raise RuntimeError("tree GDN: CUDA tensors required (no CPU path)")
    bounds, parents = _tree_arrays(chunk_boundaries, chunk_parent_map)
    cap_list = sorted(set(int(c) for c in (capture_states_at or ())))
    cap = torch.tensor(cap_list, dtype=torch.int32)
    flags = (GDN_QK_L2NORM if use_qk_l2norm else 0) | (GDN_EXACT_INVERSE if exact_inverse else 0)
    outs, caps = [], []
    for b in range(query.shape[0]):
        has_init = initial_state is not None
        init = (initial_state[b].float().contiguous() if has_init
                else query.new_empty(0, dtype=torch.float32))
        o, _, c, _ = _gdn_fwd_op(query[b].contiguous(), key[b].contiguous(),
                                 value[b].contiguous(), g[b].float().contiguous(),
                                 beta[b].float().contiguous(), bounds, parents, init, has_init,
                                 flags, False, cap, False)
        outs.append(o)
        caps.append(c)
    core = torch.stack(outs, 0)
    captured = {c: torch.stack([cb[i] for cb in caps], 0) for i, c in enumerate(cap_list)}
    return core, captured


def _path_tail(bounds: Sequence[Tuple[int, int]], parents: Sequence[int], c: int,
               n: int) -> List[int]:
    """Token indices of the last ``n`` tokens on the root-to-node path ending
    with node c, oldest first; -1 where the path is shorter."""
    out: List[int] = []
    node = c
    while node >= 0 and len(out) < n:
        s, e = bounds[node]
        t = e - 1
        while t >= s and len(out) < n:
            out.append(t)
            t -= 1
        node = parents[node]
    out += [-1] * (n - len(out))
    return out[::-1]


def conv_varlen_capture(ssm, mixed_qkv_raw: torch.Tensor, chunk_boundaries, chunk_parent_map,
                        init_context: Optional[torch.Tensor] = None,
                        capture_states_at: Optional[Iterable[int]] = None
                        ) -> Tuple[torch.Tensor, Dict[int, torch.Tensor]]:
    """Tree conv + SiLU that continues ``init_context`` in the root chunks and
    returns each captured node's conv context (tree_grad_hybrid_ssm.py:142-205).

    mixed_qkv_raw [B, C, S]; init_context [B, C, K-1] (the K-1 inputs before
    the root chunks, oldest first) or None (zeros).  Returns (out [B, C, S],
    {chunk index: context [B, C, K-1]}) where a node's context is the last K-1
    inputs on the path ending with it, continuing into init_context."""
    act = getattr(ssm, "activation", "silu")
    if act not in ("silu", "swish"):
        raise ValueError(f"tree conv implements SiLU only, got activation={act!r}")
    K = int(ssm.conv1d.weight.shape[-1])
    bounds = [tuple(int(x) for x in b) for b in chunk_boundaries]
    parents = [int(p) for p in chunk_parent_map]
    x = mixed_qkv_raw
    off = 0
    if init_context is not None and K > 1:
        # the context as a (K-1)-token node in front, parent of every root chunk
        x = torch.cat([init_context.to(x.dtype), x], dim=-1)
        off = K - 1
        bounds = [(0, off)] + [(s + off, e + off) for s, e in bounds]
        parents = [-1] + [p + 1 if p >= 0 else 0 for p in parents]
    out = tree_conv(x, ssm.conv1d.weight, ssm.conv1d.bias, bounds, parents)[..., off:]
    captured: Dict[int, torch.Tensor] = {}
    cap_list = sorted(set(int(c) for c in (capture_states_at or ())))
    if cap_list and K > 1:
        xz = torch.cat([x, x.new_zeros(x.shape[0], x.shape[1], 1)], dim=-1)
        zero = x.shape[-1]
        for c in cap_list:
            idx = [t if t >= 0 else zero
                   for t in _path_tail(bounds, parents, c + (1 if off else 0), K - 1)]
            captured[c] = xz[:, :, torch.as_tensor(idx, device=x.device)]
    return out, captured


# -----------------------------------------------------------------------------
# the layer forward
# -----------------------------------------------------------------------------

class SSMPartitionState:
    """What one partition's forward gives the patched linear-attention layers:
    the DFS chunks, the gateway to inject (per layer index: recurrent state,
    conv context) and the chunks whose states to capture; it collects the
    captured tensors per layer."""

    def __init__(self, chunk_boundaries, chunk_parent_map,
                 inject: Optional[Dict[int, Tuple[torch.Tensor, torch.Tensor]]] = None,
                 capture_at: Sequence[int] = (), exact_inverse: bool = False,
                 fused_norm: bool = True):
        self.bounds = [tuple(int(x) for x in b) for b in chunk_boundaries]
        self.parents = [int(p) for p in chunk_parent_map]
        self.inject = inject or {}
        self.capture_at = sorted(set(int(c) for c in capture_at))
        self.exact_inverse = exact_inverse
        self.fused_norm = fused_norm      # gated RMSNorm by tt_gated_rmsnorm_fwd/bwd
        self.rec: Dict[int, Dict[int, torch.Tensor]] = {}    # layer -> {chunk: state}
        self.conv: Dict[int, Dict[int, torch.Tensor]] = {}   # layer -> {chunk: context}


def tree_ssm_forward(layer, hidden_states: torch.Tensor, st: SSMPartitionState) -> torch.Tensor:
    """Qwen3.5 GatedDeltaNet forward over a DFS-packed tree (the layer's own
    projections, conv weights, gates and norm; batch 1 per tree)."""
    B, S, _ = hidden_states.shape
    li = int(layer.layer_idx)
    mixed = layer.in_proj_qkv(hidden_states).transpose(1, 2)
    z = layer.in_proj_z(hidden_states).reshape(B, S, -1, layer.head_v_dim)
    b = layer.in_proj_b(hidden_states)
    a = layer.in_proj_a(hidden_states)
    rec0, conv0 = st.inject.get(li, (None, None))
    mixed, conv_cap = conv_varlen_capture(layer, mixed, st.bounds, st.parents,
                                          init_context=conv0, capture_states_at=st.capture_at)
    mixed = mixed.transpose(1, 2)
    q, k, v = torch.split(mixed, [layer.key_dim, layer.key_dim, layer.value_dim], dim=-1)
    q = q.reshape(B, S, -1, layer.head_k_dim)
    k = k.reshape(B, S, -1, layer.head_k_dim)
    v = v.reshape(B, S, -1, layer.head_v_dim)
    beta = b.sigmoid()
    g = -layer.A_log.float().exp() * F.softplus(a.float() + layer.dt_bias)
    core, rec_cap = ssm_varlen_capture(q, k, v, g, beta, st.bounds, st.parents,
                                       initial_state=rec0, capture_states_at=st.capture_at,
                                       use_qk_l2norm=True, exact_inverse=st.exact_inverse)
    if st.capture_at:
        st.rec[li] = rec_cap
        st.conv[li] = conv_cap
    core2, z2 = core.reshape(-1, layer.head_v_dim), z.reshape(-1, layer.head_v_dim)
    if st.fused_norm and fusable(layer.norm) and core2.dtype == z2.dtype:
        core = gated_rmsnorm(core2, z2, layer.norm.weight, layer.norm.variance_epsilon)
    else:
        core = layer.norm(core2, z2)
    return layer.out_proj(core.reshape(B, S, -1))


class patch_ssm_layers:
    """Context manager: every ``linear_attn`` of the model runs
    :func:`tree_ssm_forward` with ``state`` (tree_grad_hybrid_ssm.py:360-381),
    restoring the original forwards on exit."""

    def __init__(self, model, state: SSMPartitionState):
        self.model, self.state = model, state
        self.saved: List[Tuple[torch.nn.Module, object]] = []

    def __enter__(self):
        for _, layer in ssm_layers(self.model):
            self.saved.append((layer, layer.__dict__.get("forward")))

            def fwd(hidden_states, cache_params=None, attention_mask=None, _l=layer, **_kw):
                return tree_ssm_forward(_l, hidden_states, self.state)

            layer.forward = fwd
        return self.state

    def __exit__(self, *exc):
        for layer, f in self.saved:
            if f is None:
                del layer.forward          # back to the class's forward
            else:
                layer.forward = f
        self.saved = []
        return False
