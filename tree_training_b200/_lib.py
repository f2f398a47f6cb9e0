"""ctypes binding of the C ABI declared in include/tree_training_b200.h.

The shared library is built in-tree (``python -m tree_training_b200.build``).
There is no fallback: if the library is missing or fails to load, every entry
point raises, so a GPU run can never silently take a CPU path.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtt_sm100.so")

TT_OK = 0
TT_ERR_INVALID_ARG = 1
TT_ERR_UNSUPPORTED = 2
TT_ERR_CUDA = 3
TT_ERR_DEVICE_TIMEOUT = 4
TT_ERR_NOT_INTERVAL = 5
TT_ERR_WORKSPACE = 6
TT_ERR_CAPACITY = 7

TT_F32, TT_BF16, TT_F16, TT_U8 = 0, 1, 2, 3
TT_BWD_PREP, TT_BWD_DKDV, TT_BWD_DQ, TT_BWD_ALL = 1, 2, 4, 7

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float
_INT = ctypes.c_int

# name -> (restype, argtypes); must match include/tree_training_b200.h
SIGNATURES = {
    "tt_status_string": (ctypes.c_char_p, [_INT]),
    "tt_abi_version": (_INT, []),
    "tt_set_kernel_path": (_INT, [_INT]),
    "tt_kernel_launches": (_I64, []),
    "tt_gdn_gemm_flops": (_I64, []),
    "tt_gdn_gemm_tc_flops": (_I64, []),
    "tt_gdn_set_gemm_mode": (_INT, [_INT]),
    "tt_gdn_take_device_status": (_INT, [_P]),
    "tt_gdn_segmented_gemm_workspace_size": (_I64, [_I32, _P]),
    "tt_gdn_segmented_gemm": (_INT, [_INT, _I32, _P, _I32, _P, _I64, _P, _I64, _P, _I64, _F32,
                                     _F32, _P, _I64, _P]),
    "tt_diag_bounded_wait": (_INT, [_P, _P]),
    "tt_pack_forest": (_INT, [_I32, _P, _P, _I32, _P, _P, _P, _P, _P, _P, _P, _P]),
    "tt_gateway_intervals_from_bias": (_INT, [_I32, _P, _I32, _P, _P]),
    "tt_build_tiles": (_INT, [_I32, _I32, _P, _P, _I32, _I32, _P, _P, _P, _P, _I64, _P]),
    "tt_attn_tile_shape": (_INT, [_INT, _I32, _INT, _P, _P]),
    "tt_mask_to_intervals": (_INT, [_INT, _I32, _I32, _P, _I64, _I64, _P, _P, _P, _P]),
    "tt_tree_attn_fwd": (_INT, [_INT, _I32, _I32, _I32, _I32, _I32,
                                _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                                _P, _P, _P, _P, _F32, _P, _P, _P, _P]),
    "tt_tree_attn_bwd_workspace_size": (_I64, [_INT, _I32, _I32, _I32, _I32, _I32]),
    "tt_tree_attn_bwd": (_INT, [_INT, _I32, _I32, _I32, _I32, _I32,
                                _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                                _P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _F32,
                                _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                                _P, _I64, _INT, _P, _P]),
    "tt_tree_attn_bwd_stored_workspace_size": (_I64, [_INT, _I32, _I32, _I32, _I32, _I32,
                                                      _I64, _I32]),
    "tt_tree_attn_bwd_stored": (_INT, [_INT, _I32, _I32, _I32, _I32, _I32,
                                       _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                                       _P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _F32,
                                       _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                                       _I64, _I32, _P, _I64, _INT, _P, _P]),
    "tt_tree_attn_bwd_noalloc": (_INT, [_INT, _I32, _I32, _I32, _I32, _I32,
                                        _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                                        _P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _F32,
                                        _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                                        _P, _P]),
    "tt_tree_attn_bwd_noalloc_max_row_terms": (_I64, []),
    "tt_gdn_tree_workspace_size": (_I64, [_I32, _I32, _I32, _I32, _I32, _P, _INT]),
    "tt_gdn_tree_fwd": (_INT, [_INT, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P,
                               _I32, _P, _P, _P, _INT, _P, _P, _P, _I64, _P]),
    "tt_gdn_tree_bwd": (_INT, [_INT, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P,
                               _I32, _P, _P, _P, _INT, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                               _I64, _P]),
    "tt_gdn_tree_fwd_ex": (_INT, [_INT, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P,
                                  _I32, _P, _P, _P, _INT, _P, _P, _I32, _P, _P, _I64, _I64,
                                  _I64, _P, _I64, _P]),
    "tt_gdn_tree_bwd_ex": (_INT, [_INT, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P,
                                  _I32, _P, _P, _P, _INT, _P, _P, _I32, _P, _P, _P, _P, _P,
                                  _P, _P, _P, _I64, _I64, _I64, _P, _I64, _P]),
    "tt_ce_fwd_grad": (_INT, [_INT, _I32, _I32, _P, _I64, _P, _P, _I64, _P, _INT, _P]),
    "tt_qk_norm_rope_fwd": (_INT, [_INT, _I64, _I32, _I32, _P, _P, _P, _P, _F32, _P, _P]),
    "tt_qk_norm_rope_bwd_blocks": (_INT, [_I64]),
    "tt_qk_norm_rope_bwd": (_INT, [_INT, _I64, _I32, _I32, _P, _P, _P, _P, _F32, _P, _P, _P,
                                   _I32, _P]),
    "tt_gated_rmsnorm_fwd": (_INT, [_INT, _I64, _I32, _P, _P, _P, _F32, _P, _P]),
    "tt_gated_rmsnorm_bwd_blocks": (_INT, [_I64]),
    "tt_gated_rmsnorm_bwd": (_INT, [_INT, _I64, _I32, _P, _P, _P, _F32, _P, _P, _P, _P, _I32,
                                    _P]),
    "tt_conv_predecessors": (_INT, [_I32, _P, _P, _I32, _P]),
    "tt_conv_successors": (_INT, [_I32, _I32, _P, _P, _P, _P, _I64]),
    "tt_tree_conv_fwd": (_INT, [_INT, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P]),
    "tt_tree_conv_fwd_ex": (_INT, [_INT, _I32, _I32, _I32, _P, _P, _P, _P, _P, _I32, _P]),
    "tt_tree_conv_bwd_workspace_size": (_I64, [_I32, _I32, _I32]),
    "tt_tree_conv_bwd": (_INT, [_INT, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                _P, _P, _P, _I64, _P]),
    "tt_tree_conv_bwd_ex": (_INT, [_INT, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P,
                                   _I32, _P, _P, _P, _P, _I64, _P]),
}

_lib = None
_lock = threading.Lock()


class TTError(RuntimeError):
    """Raised with the library's status text when a C-ABI call fails."""

    def __init__(self, fn: str, code: int):
        self.code = code
        super().__init__(f"{fn} failed: {status_string(code)} (status {code})")


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m tree_training_b200.build`"
                        " (there is no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    f = getattr(L, name)
                    f.restype = res
                    f.argtypes = args
                _lib = L
    return _lib


def status_string(code: int) -> str:
    return lib().tt_status_string(int(code)).decode()


def check(fn: str, code: int) -> None:
    if code != TT_OK:
        raise TTError(fn, code)


def call(name: str, *args) -> int:
    rc = getattr(lib(), name)(*args)
    check(name, rc)
    return rc


_path_generation = [0]


def set_kernel_path(path: int) -> int:
    """Select the attention kernel path (0 automatic, 1 exact CUDA-core) and
    invalidate cached tile shapes.  Returns the previous setting."""
    prev = lib().tt_set_kernel_path(int(path))
    _path_generation[0] += 1
    return prev


def path_generation() -> int:
    return _path_generation[0]
