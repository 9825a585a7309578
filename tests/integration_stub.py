"""The ctypes binding a maintainer would add to the reference for KV compaction.

It replaces the reference's inline C++ extension call (ddtree.py:38 signature,
``compact_tail_inplace(cache_tensor, past_length, keep_current_indices)``) with
the C ABI of this library.  tests/test_abi.py checks it against the header.
"""

import ctypes
import os

import torch

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "retree_b200", "lib",
                   "libretree_b200.so")

lib = ctypes.CDLL(LIB)
lib.rt_kv_compact.restype = ctypes.c_int
lib.rt_kv_compact.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int,
                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p,
                              ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                              ctypes.c_void_p]
lib.rt_status_string.restype = ctypes.c_char_p
lib.rt_status_string.argtypes = [ctypes.c_int]


def compact_tail_inplace(cache_tensor, past_length, keep_current_indices):
    """Move the kept rows of the current block to ``past_length..`` in place (ddtree.py:37-65)."""
    t = cache_tensor.view(-1, cache_tensor.shape[-2], cache_tensor.shape[-1])
    es = t.element_size()
    rc = lib.rt_kv_compact(None, t.data_ptr(), 1, 0, t.shape[0], t.stride(0) * es, t.stride(1) * es,
                           t.shape[2] * es, past_length, None, t.shape[1] - past_length,
                           keep_current_indices.data_ptr(), keep_current_indices.numel(), None, None,
                           torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(lib.rt_status_string(rc).decode())  # the reference's TORCH_CHECK role
    return cache_tensor
