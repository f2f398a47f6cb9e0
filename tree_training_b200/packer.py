"""Forest packing: the drop-in for ``build_dfs_tree_info`` plus the metadata the
tree-attention kernels consume.

Reference: dfs_tree_forward.py:46-65 (TreeNode), :72-89 (DFSTreeInfo),
:91-184 (build_dfs_tree_info).  The Python side walks the forest once in
pre-order (parent before children, children left to right, :95-97) and hands
(len, parent) arrays to the native packer ``tt_pack_forest``, which returns
the position ids, chunk boundaries, leaves and one visible-row interval per
key.  The dense [N,N] mask of :157-172 is never built unless a caller reads
``attn_mask_bool`` (kept for API compatibility).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib


@dataclass
class TreeNode:
    """One node of the generation tree (dfs_tree_forward.py:46-65)."""
    token_ids: List[int]
    children: List["TreeNode"] = field(default_factory=list)

    def add_child(self, token_ids: List[int]) -> "TreeNode":
        child = TreeNode(token_ids)
        self.children.append(child)
        return child

    @property
    def is_leaf(self) -> bool:
        return len(self.children) == 0


def preorder_arrays(roots: Sequence) -> Tuple[np.ndarray, np.ndarray, np.ndarray, list]:
    """Walk a forest in pre-order.  Returns (node_len int32, node_parent int32,
    token ids int64, node objects in pre-order).  Any object with
    ``token_ids`` and ``children`` works (the reference's TreeNode included)."""
    lens: List[int] = []
    par: List[int] = []
    toks: List[int] = []
    nodes: list = []
    stack = [(r, -1) for r in reversed(list(roots))]
    while stack:
        n, p = stack.pop()
        me = len(lens)
        tid = n.token_ids
        lens.append(len(tid))
        par.append(p)
        toks.extend(tid)
        nodes.append(n)
        ch = n.children
        for i in range(len(ch) - 1, -1, -1):
            stack.append((ch[i], me))
    return (np.asarray(lens, dtype=np.int32), np.asarray(par, dtype=np.int32),
            np.asarray(toks, dtype=np.int64), nodes)


def pack_arrays(node_len: np.ndarray, node_parent: np.ndarray, pos_offset: int = 0):
    """Native packer on (len, parent) arrays in pre-order.  Returns a dict of
    int32 numpy arrays: pos_ids, chunk_bounds [n,2], subtree_end, leaf_ids,
    token_node, kv_lo, kv_hi."""
    node_len = np.ascontiguousarray(node_len, dtype=np.int32)
    node_parent = np.ascontiguousarray(node_parent, dtype=np.int32)
    n = int(node_len.shape[0])
    N = int(node_len.sum())
    pos = np.empty(N, np.int32)
    bounds = np.empty((n, 2), np.int32)
    sub_end = np.empty(n, np.int32)
    leaves = np.empty(max(n, 1), np.int32)
    n_leaves = np.zeros(1, np.int32)
    tok_node = np.empty(N, np.int32)
    lo = np.empty(N, np.int32)
    hi = np.empty(N, np.int32)
    _lib.call("tt_pack_forest", n, node_len.ctypes.data, node_parent.ctypes.data,
              int(pos_offset), pos.ctypes.data, bounds.ctypes.data, sub_end.ctypes.data,
              leaves.ctypes.data, n_leaves.ctypes.data, tok_node.ctypes.data, lo.ctypes.data,
              hi.ctypes.data)
    return dict(pos_ids=pos, chunk_bounds=bounds, subtree_end=sub_end,
                leaf_ids=leaves[: int(n_leaves[0])].copy(), token_node=tok_node,
                kv_lo=lo, kv_hi=hi)


class DFSTreeInfo:
    """Drop-in for the reference DFSTreeInfo (dfs_tree_forward.py:72-89).

    Same attribute names and types as the reference (lists of Python ints,
    list of (start, end) tuples, a BoolTensor mask); the list views are built
    on first access from numpy arrays.  Extra attributes: ``*_np`` arrays,
    ``subtree_end``, ``kv_lo``/``kv_hi`` and :meth:`attn_meta`.
    """

    def __init__(self, token_ids: np.ndarray, packed: dict, nodes: list, pos_offset: int = 0):
        self.dfs_token_ids_np = token_ids
        self.dfs_pos_ids_np = packed["pos_ids"]
        self.chunk_bounds_np = packed["chunk_bounds"]
        self.subtree_end = packed["subtree_end"]
        self.leaf_chunk_ids_np = packed["leaf_ids"]
        self.token_node = packed["token_node"]
        self.kv_lo = packed["kv_lo"]
        self.kv_hi = packed["kv_hi"]
        self.nodes = nodes
        self.N = int(token_ids.shape[0])
        self.n_chunks = len(nodes)
        self.pos_offset = pos_offset
        self._parents: Optional[np.ndarray] = None
        self._cache: Dict[str, object] = {}

    # --- reference-compatible views ------------------------------------------
    @property
    def dfs_token_ids(self) -> List[int]:
        return self._cached("ids", lambda: self.dfs_token_ids_np.tolist())

    @property
    def dfs_pos_ids(self) -> List[int]:
        return self._cached("pos", lambda: self.dfs_pos_ids_np.tolist())

    @property
    def chunk_boundaries(self) -> List[Tuple[int, int]]:
        return self._cached("bounds", lambda: [tuple(b) for b in self.chunk_bounds_np.tolist()])

    @property
    def chunk_parent_map(self) -> List[int]:
        return self._cached("parents", lambda: self.parents_np.tolist())

    @property
    def parents_np(self) -> np.ndarray:
        return self._parents

    @property
    def leaf_chunk_ids(self) -> List[int]:
        return self._cached("leaves", lambda: self.leaf_chunk_ids_np.tolist())

    @property
    def leaf_nodes(self) -> list:
        return self._cached("leaf_nodes", lambda: [self.nodes[i] for i in self.leaf_chunk_ids_np])

    @property
    def attn_mask_bool(self) -> torch.Tensor:
        """Dense [N,N] mask, materialised only on request (reference API)."""
        def make():
            rows = torch.arange(self.N).unsqueeze(1)
            lo = torch.from_numpy(self.kv_lo.astype(np.int64)).unsqueeze(0)
            hi = torch.from_numpy(self.kv_hi.astype(np.int64)).unsqueeze(0)
            return (rows >= lo) & (rows < hi)
        return self._cached("mask", make)

    def _cached(self, key, fn):
        if key not in self._cache:
            self._cache[key] = fn()
        return self._cache[key]

    # --- kernel metadata --------------------------------------------------------
    def attn_meta(self, gateway_lo: Optional[np.ndarray] = None,
                  gateway_hi: Optional[np.ndarray] = None) -> "TreeAttnMeta":
        """Key intervals for attention over [gateway keys, own keys]."""
        if gateway_lo is None:
            return TreeAttnMeta(self.N, self.kv_lo, self.kv_hi)
        lo = np.concatenate([np.asarray(gateway_lo, np.int32), self.kv_lo])
        hi = np.concatenate([np.asarray(gateway_hi, np.int32), self.kv_hi])
        return TreeAttnMeta(self.N, lo, hi)


def build_dfs_tree_info(roots: Sequence, pos_offset: int = 0) -> DFSTreeInfo:
    """Drop-in for build_dfs_tree_info (dfs_tree_forward.py:91-184).

    ``pos_offset`` is added to every position id (the partition offset the
    reference adds at tree_grad_hybrid.py:308-310)."""
    lens, par, toks, nodes = preorder_arrays(roots)
    packed = pack_arrays(lens, par, pos_offset)
    info = DFSTreeInfo(toks, packed, nodes, pos_offset)
    info._parents = par
    return info


def _upload(a: np.ndarray, device: torch.device) -> torch.Tensor:
    """Host array -> device tensor on the current stream, staged through
    pinned memory so the copy is asynchronous (a pageable source can make the
    call wait for the stream; torch's pinned-buffer cache keeps the staging
    buffer until the copy has run)."""
    h = torch.from_numpy(a)
    if torch.device(device).type == "cuda":
        h = h.pin_memory()
    return h.to(device, non_blocking=True)


class TreeAttnMeta:
    """Per-key visible-row intervals of one attention call plus the tile work
    lists and device copies the kernels need (cached per device and tile
    shape).  Rows are [0, n_q); keys are [0, n_kv) with gateway keys first."""

    def __init__(self, n_q: int, kv_lo: np.ndarray, kv_hi: np.ndarray):
        self.n_q = int(n_q)
        self.kv_lo = np.ascontiguousarray(kv_lo, dtype=np.int32)
        self.kv_hi = np.ascontiguousarray(kv_hi, dtype=np.int32)
        self.n_kv = int(self.kv_lo.shape[0])
        self._dev: Dict[object, object] = {}
        self._tiles: Dict[Tuple[int, int], dict] = {}
        self.prefetched = False     # device copies made on a caller's upload stream

    def tiles(self, tile_q: int, tile_kv: int) -> dict:
        key = (tile_q, tile_kv)
        t = self._tiles.get(key)
        if t is None:
            nqt = (self.n_q + tile_q - 1) // tile_q
            nkt = (self.n_kv + tile_kv - 1) // tile_kv
            cap = max(nqt * nkt, 1)
            fp = np.zeros(nqt + 1, np.int32)
            bp = np.zeros(nkt + 1, np.int32)
            fl = np.zeros(cap, np.int32)
            bl = np.zeros(cap, np.int32)
            vp = np.zeros(1, np.int64)
            _lib.call("tt_build_tiles", self.n_q, self.n_kv, self.kv_lo.ctypes.data,
                      self.kv_hi.ctypes.data, tile_q, tile_kv, fp.ctypes.data, fl.ctypes.data,
                      bp.ctypes.data, bl.ctypes.data, cap, vp.ctypes.data)
            t = dict(fwd_ptr=fp, fwd_list=fl[: max(int(fp[-1]), 1)],
                     bwd_ptr=bp, bwd_list=bl[: max(int(bp[-1]), 1)],
                     visible_pairs=int(vp[0]))
            self._tiles[key] = t
        return t

    @property
    def visible_pairs(self) -> int:
        return self.tiles(128, 128)["visible_pairs"]

    def device(self, device: torch.device, tile_q: int, tile_kv: int) -> dict:
        """Device tensors for one tile shape (copied once, on the current
        stream, then cached)."""
        key = (device, tile_q, tile_kv)
        d = self._dev.get(key)
        if d is None:
            ivk = (device, "iv")
            iv = self._dev.get(ivk)
            if iv is None:
                # one buffer, padded so vectorised kernel reads stay inside it
                pad = (-self.n_kv) % 128
                lohi = np.zeros((2, self.n_kv + pad), np.int32)
                lohi[0, : self.n_kv] = self.kv_lo
                lohi[1, : self.n_kv] = self.kv_hi
                g = _upload(lohi, device)
                iv = (g[0], g[1])
                self._dev[ivk] = iv
            t = self.tiles(tile_q, tile_kv)
            cat = np.concatenate([t["fwd_ptr"], t["fwd_list"], t["bwd_ptr"], t["bwd_list"]])
            g = _upload(cat, device)
            o1 = t["fwd_ptr"].size
            o2 = o1 + t["fwd_list"].size
            o3 = o2 + t["bwd_ptr"].size
            d = dict(kv_lo=iv[0], kv_hi=iv[1], fwd_ptr=g[:o1], fwd_list=g[o1:o2],
                     bwd_ptr=g[o2:o3], bwd_list=g[o3:])
            self._dev[key] = d
        return d

    def h2d_bytes(self) -> int:
        """Bytes copied host->device per device for the kernel metadata."""
        n = 0
        for k, v in self._dev.items():
            if isinstance(v, tuple):
                n += 2 * v[0].numel() * 4
            else:
                n += sum(x.numel() * 4 for kk, x in v.items() if kk not in ("kv_lo", "kv_hi"))
        return n

    def dense_mask(self) -> np.ndarray:
        rows = np.arange(self.n_q)[:, None]
        return (rows >= self.kv_lo[None, :]) & (rows < self.kv_hi[None, :])


def gateway_intervals_from_bias(bias, n_q: int) -> Tuple[np.ndarray, np.ndarray]:
    """Key intervals of the reference's additive gateway bias
    (tree_grad_hybrid.py:206-209): 0 -> all rows, -inf -> none."""
    b = np.ascontiguousarray(np.asarray(bias, dtype=np.float32))
    P = int(b.shape[0])
    lo = np.zeros(P, np.int32)
    hi = np.zeros(P, np.int32)
    _lib.call("tt_gateway_intervals_from_bias", P, b.ctypes.data, int(n_q), lo.ctypes.data,
              hi.ctypes.data)
    return lo, hi
