"""ctypes binding of the C-ABI kernel library (``include/retree_b200.h``).

The library is built in-tree (``python -m retree_b200.build``) as
``retree_b200/lib/libretree_b200.so``.  There is no fallback: if the library
is missing or cannot be loaded, every kernel entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libretree_b200.so"

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_D = ctypes.c_double
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/retree_b200.h
SIGNATURES = {
    "rt_abi_version": (_I, []),
    "rt_last_cuda_error": (_I, []),
    "rt_status_string": (ctypes.c_char_p, [_I]),
    "rt_set_pdl": (None, [_I]),
    "rt_pdl_enabled": (_I, []),
    "rt_kv_compact": (_I, [_P, _P, _I, _I64, _I, _I64, _I64, _I, _I64, _P, _I64, _P, _I, _P, _P, _P]),
    "rt_kv_append": (_I, [_P, _P, _I64, _I64, _P, _P, _I64, _I64, _I, _I, _I, _I64, _I64, _P, _P, _P]),
    "rt_tree_attn_workspace_size": (_SZ, [_I, _I, _I, _I, _I64, _I]),
    "rt_tree_attn": (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I64, _P, _I64, _I64, _P, _I, _I, _I64, _P,
                          _I, _I, _I, _F, _I, _I, _P, _SZ, _P, _P]),
    "rt_tree_attn_default_splits": (_I, [_I, _I, _I, _I64]),
    "rt_tree_attn_plan": (_I, [_I, _I, _I, _I64, _I, _I, _P, _P, _P]),
    "rt_ipc_alloc": (_I, [_SZ, _P, _P]),
    "rt_ipc_free": (_I, [_P]),
    "rt_ipc_open": (_I, [_P, _P]),
    "rt_ipc_close": (_I, [_P]),
    "rt_peer_epoch_step": (_I, [_P, _I64, _P]),
    "rt_peer_signal": (_I, [_P, _I, _I, _P, _I64, _P]),
    "rt_peer_gather": (_I, [_P, _I, _I, _I64, _I64, _P, _I64, _P, _P, _I64, _P, _P]),
    "rt_linear_gather": (_I, [_P, _I, _I, _I64, _I, _P, _I, _I, _P, _I64, _P, _P, _I64, _P, _P]),
    "rt_linear_argmax": (_I, [_P, _I64, _I, _I, _P, _I, _P, _I64, _P, _P, _P, _P]),
    "rt_tree_attn_noalloc_max_bytes": (_SZ, []),
    "rt_tree_attn_noalloc": (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I64, _P, _I64, _I64, _P, _I, _I, _I64, _P,
                                  _I, _I, _I, _F, _I, _I, _P, _P]),
    "rt_mask_from_dense": (_I, [_P, _I, _I64, _I64, _I, _P, _I, _P]),
    "rt_draft_topk_workspace_size": (_SZ, [_I, _I, _I]),
    "rt_draft_topk": (_I, [_P, _I, _I64, _I, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    "rt_tree_build": (_I, [_P, _P, _I, _I, _I, _I, _P, _I64, _P, _I, _I, _D, _I, _I, _I, _P, _D, _P, _I,
                           _P, _P, _P, _P, _I, _P, _P, _P, _I64, _P, _I64, _P, _P, _P]),
    "rt_tree_walk": (_I, [_P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _P]),
    "rt_recovery_walk": (_I, [_P, _P, _I, _P, _P, _P, _I64, _I, _I64, _D, _I64, _I, _I, _I, _P, _I, _P, _P, _P,
                              _I64, _P, _P, _I, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _P]),
    "rt_embed_rmsnorm": (_I, [_P, _P, _I64, _P, _P, _P, _I, _I, _F, _P, _P]),
    "rt_add_rmsnorm": (_I, [_P, _P, _P, _P, _I, _I, _F, _P]),
    "rt_qk_norm_rope_append": (_I, [_P, _I, _I, _I, _I, _P, _P, _F, _P, _P, _I64, _P, _P, _P, _P, _I64, _I64,
                                    _I64, _I64, _P, _P, _P]),
    "rt_silu_mul": (_I, [_P, _P, _I, _I, _P]),
    "rt_linear_check": (_I, [_I, _I, _I, _I]),
    "rt_linear_plan": (_I, [_I, _I, _I, _I, _P, _P, _P]),
    "rt_linear": (_I, [_P, _I64, _I, _I, _P, _I, _I, _P, _I64, _P, _P, _P]),
}

RT_EPI_STORE = 0
RT_EPI_SILU_MUL = 1
RT_EPI_QKV_ROPE = 2


class QkvEpilogue(ctypes.Structure):
    """``rt_qkv_epilogue`` (include/retree_b200.h), field for field."""

    _fields_ = [("num_q_heads", ctypes.c_int), ("num_kv_heads", ctypes.c_int), ("q_norm_weight", _P),
                ("k_norm_weight", _P), ("eps", ctypes.c_float), ("cos_table", _P), ("sin_table", _P),
                ("table_len", ctypes.c_int64), ("positions", _P), ("q_out", _P), ("k_cache", _P), ("v_cache", _P),
                ("cache_head_stride", ctypes.c_int64), ("cache_row_stride", ctypes.c_int64),
                ("capacity", ctypes.c_int64), ("offset", ctypes.c_int64), ("offset_dev", _P)]

# Host return codes / device status codes (include/retree_b200.h)
RT_OK = 0
RT_ERR_INVALID_ARGUMENT = 1
RT_ERR_UNSUPPORTED = 2
RT_ERR_WORKSPACE = 3
RT_ERR_CUDA = 4
RT_DEV_WAIT_TIMEOUT = 100
RT_DEV_BAD_INDEX = 101
RT_DEV_OVERFLOW = 102

_lib = None


class KernelLibraryError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load (once) and return the kernel library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("RETREE_B200_LIB", LIB_PATH))
    if not path.exists():
        raise KernelLibraryError(
            f"retree_b200 kernel library not found at {path}; build it with `python -m retree_b200.build`")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def status_string(code: int) -> str:
    return load().rt_status_string(int(code)).decode()


def check(rc: int, what: str) -> None:
    """Raise RuntimeError for a non-zero host return code (the reference's TORCH_CHECK role)."""
    if rc != RT_OK:
        msg = status_string(rc)
        if rc == RT_ERR_CUDA:
            msg += f" (cudaError {load().rt_last_cuda_error()})"
        raise RuntimeError(f"{what}: {msg}")
