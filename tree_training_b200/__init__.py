"""B200-native (sm_100a) hot path of Tree Training.

Drop-in replacements for the reference's packed-tree attention path:
``build_dfs_tree_info`` (native packer, no dense mask), tree attention forward
and backward as a torch custom op backed by tcgen05 kernels, registered as an
HF attention implementation (``"tree_sm100"``).
"""
from .packer import (TreeNode, DFSTreeInfo, TreeAttnMeta, build_dfs_tree_info,  # noqa: F401
                     gateway_intervals_from_bias, pack_arrays, preorder_arrays)
from .attention import (tree_attention, tree_attention_forward, register_hf_attention,  # noqa: F401
                        tree_mask_placeholder, meta_from_dense_mask, check_device_status,
                        prefetch_tree_meta, ATTN_IMPL_NAME)
from ._lib import LIB_PATH, TTError  # noqa: F401

__all__ = [
    "TreeNode", "DFSTreeInfo", "TreeAttnMeta", "build_dfs_tree_info",
    "gateway_intervals_from_bias", "tree_attention", "tree_attention_forward",
    "register_hf_attention", "tree_mask_placeholder", "meta_from_dense_mask",
    "check_device_status", "prefetch_tree_meta", "ATTN_IMPL_NAME", "LIB_PATH", "TTError",
]
