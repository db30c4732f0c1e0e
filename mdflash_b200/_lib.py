"""ctypes binding of libddtree_b200.so (the C ABI declared in include/ddtree_b200.h).

There is no fallback: if the library is missing or cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

_lib = None

DDT_OK = 0
DDT_ERR_TIMEOUT = -6
DDT_F32 = 0
DDT_BF16 = 1
DDT_MASK_TREE = 0
DDT_MASK_CAUSAL = 1
DDT_MASK_NONE = 2
DDT_MAX_BUDGET = 1024
DDT_MAX_DEPTH = 20
DDT_MAX_NODES = DDT_MAX_BUDGET + 1

_P = ctypes.c_void_p
_I = ctypes.c_int64
_i = ctypes.c_int
_F = ctypes.c_float
_S = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/ddtree_b200.h
SIGNATURES = {
    "ddt_error_string": (ctypes.c_char_p, [_i]),
    "ddt_version": (_i, []),
    "ddt_topk_tree_workspace_bytes": (_S, [_I, _I, _I]),
    "ddt_topk_tree": (_i, [_P, _i, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _P, _I, _P, _P,
                           _P, _S, _P]),
    "ddt_topk_tree_batched_workspace_bytes": (_S, [_I, _I, _I, _I]),
    "ddt_topk_tree_batched": (_i, [_P, _i, _I, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P, _P, _I, _P,
                                   _P, _P, _P, _P, _S, _P]),
    "ddt_topk_tree_noalloc": (_i, [_P, _i, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _P, _I,
                                   _P, _P, _P]),
    "ddt_sample_chains": (_i, [_P, _i, _I, _I, _I, _I, _F, ctypes.c_uint64, ctypes.c_uint64, _P,
                               _P]),
    "ddt_chain_tree": (_i, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _I, _P, _P, _P]),
    "ddt_argmax": (_i, [_P, _i, _I, _I, _I, _P, _P]),
    "ddt_lm_head_argmax_workspace_bytes": (_S, [_I]),
    "ddt_lm_head_argmax": (_i, [_P, _I, _P, _I, _I, _I, _I, _P, _P, _I, _P, _S, _P, _P]),
    "ddt_accept_compact": (_i, [_P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "ddt_accept_compact_batched": (_i, [_I, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I, _I, _I, _P, _I,
                                        _I, _P, _P, _I, _P, _P, _P, _P]),
    "ddt_compact_kv": (_i, [_P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "ddt_tree_attn_workspace_bytes": (_S, [_I, _I, _I, _I]),
    "ddt_tree_attn": (_i, [_P, _I, _I, _P, _P, _I, _I, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _i,
                           _F, _I, _P, _S, _P, _P]),
    "ddt_gather_rows": (_i, [_P, _I, _I, _P, _P, _I, _P, _I, _I, _P]),
    "ddt_advance_round": (_i, [_I, _P, _P, _P, _P, _I, _P, _I, _I, _P, _P, _P, _I, _I, _P, _I, _I,
                               _P, _P]),
    "ddt_tree_attn_device_past": (_i, [_P, _I, _I, _P, _P, _I, _I, _P, _I, _I, _I, _I, _P, _I, _I,
                                       _I, _P, _I, _i, _F, _I, _P, _S, _P, _P]),
    "ddt_tree_attn_partial_splits": (_I, [_I, _I, _I, _I]),
    "ddt_tree_attn_plan": (_i, [_I, _I, _I, _I, _I, _I, _I, _P]),
    "ddt_tree_attn_partial": (_i, [_P, _I, _I, _P, _P, _I, _I, _I, _I, _P, _P, _P, _I, _I, _I, _I,
                                   _I, _P, _I, _i, _F, _I, _P, _P]),
    "ddt_tree_attn_partial_merged_workspace_bytes": (_S, [_I, _I, _I]),
    "ddt_tree_attn_partial_merged": (_i, [_P, _I, _I, _P, _P, _I, _I, _I, _I, _P, _P, _P, _I, _I,
                                          _I, _I, _I, _P, _I, _i, _F, _P, _S, _P, _P]),
    "ddt_tree_attn_wait_check": (_i, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _I, ctypes.c_uint64, _P,
                                      _P]),
    "ddt_attn_merge": (_i, [_P, _P, _P, _I, _I, _I, _I, _P, _I, _I, _P]),
    "ddt_peer_buffer_bytes": (_S, [_I, _I, _I, _I]),
    "ddt_tree_attn_partial_push_workspace_bytes": (_S, [_I, _I, _I]),
    "ddt_tree_attn_partial_push": (_i, [_P, _I, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I,
                                        _P, _I, _i, _F, _P, _I, _I, ctypes.c_uint32, _P, _P, _S,
                                        _P, _P]),
    "ddt_peer_alloc": (_i, [_S, _P, _P]),
    "ddt_peer_open": (_i, [_P, _P]),
    "ddt_peer_close": (_i, [_P]),
    "ddt_peer_free": (_i, [_P]),
    "ddt_peer_push": (_i, [_P, _P, _P, _I, _I, _I, _P, _I, _I, ctypes.c_uint32, _P, _P]),
    "ddt_peer_merge": (_i, [_P, _I, _I, _I, _I, ctypes.c_uint32, _P, _I, _I, _P, ctypes.c_uint64,
                            _P]),
    "ddt_mask_to_bits": (_i, [_P, _i, _I, _I, _P, _I, _P]),
    "ddt_add_rmsnorm": (_i, [_P, _P, _P, _I, _I, _F, _P, _P, _P]),
    "ddt_qk_norm_rope_cache": (_i, [_P, _I, _I, _I, _I, _P, _P, _F, _P, _P, _F, _P, _P, _P, _I, _I,
                                    _I, _P]),
    "ddt_rope_table": (_i, [_P, _I, _P, _I, _F, _P, _P]),
    "ddt_qk_norm_rope_cache_table": (_i, [_P, _I, _I, _I, _I, _P, _P, _F, _P, _P, _P, _P, _I, _I,
                                          _I, _P]),
    "ddt_qk_norm_rope_cache_table_device_past": (_i, [_P, _I, _I, _I, _I, _P, _P, _F, _P, _P, _P,
                                                      _P, _I, _I, _I, _P, _P]),
    "ddt_silu_mul": (_i, [_P, _I, _I, _P, _P]),
}


class DDTreeError(RuntimeError):
    pass


def library_path() -> str:
    return _build.library_path()


def load(build_if_missing: bool = True):
    """Loads the C-ABI library (building it first when it is missing or stale and nvcc
    is available).  Raises if it cannot be loaded."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if build_if_missing and (not os.path.exists(path) or _build.needs_build()):
        try:
            _build.build()
        except Exception:
            if not os.path.exists(path):
                raise
    if not os.path.exists(path):
        raise DDTreeError(f"ddtree_b200 CUDA library not found at {path}; run "
                          "`python -m mdflash_b200.build`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != DDT_OK:
        msg = load().ddt_error_string(rc).decode()
        raise DDTreeError(f"{what} failed: {msg} (code {rc})")
