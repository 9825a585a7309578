"""The allocation-free tree-attention entry point (rt_tree_attn_noalloc).

It exists for callers that cannot allocate device memory when they call the
kernel -- code running during CUDA stream capture, serving runtimes whose
memory is all held by their own pool, C hosts without an allocator -- and keeps
the split partials in a fixed device array inside the library instead of a
caller-supplied workspace.  This checks, through the C ABI, that it returns
what the workspace entry point (rt_tree_attn) returns, on two calls in a row
(the second call sees the first call's leftovers in the shared array).

The file is named to be collected last, so a run that stops at its first
failure has run every other test already.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import tree as ot
from retree_b200 import _lib, kernels, synthetic

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2   # the attention tolerance of the parity tests
MEAN_ABS = 1e-3


def _case(seed, n, prefix, dev):
    parents = synthetic.random_tree_parents(seed, n - 1).tolist()
    bits = torch.from_numpy(ot.pack_bits(ot.visibility(parents)).view(np.int32)).to(dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn((n, 32, 128), device=dev, generator=g).to(torch.bfloat16)
    kv = torch.randn((2, 8, prefix + n + 64, 128), device=dev, generator=g).to(torch.bfloat16)
    return q, kv[0], kv[1], bits


def _noalloc(q, k, v, bits, prefix, splits, status, stream):
    lib = _lib.load()
    n = q.shape[0]
    out = torch.full_like(q, float("nan"))
    rc = lib.rt_tree_attn_noalloc(q.data_ptr(), q.stride(0) * 2, q.stride(1) * 2, k.data_ptr(), v.data_ptr(),
                                  k.stride(0) * 2, k.stride(1) * 2, k.shape[1], out.data_ptr(), out.stride(0) * 2,
                                  out.stride(1) * 2, bits.data_ptr(), bits.shape[1], n, prefix, None, 32, 8, 128,
                                  ctypes.c_float(128 ** -0.5), splits, 0, status.data_ptr(), stream)
    assert rc == _lib.RT_OK, _lib.status_string(rc)
    return out


def test_noalloc_matches_workspace_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _lib.load()
    assert lib.rt_tree_attn_noalloc_max_bytes() == 16 << 20
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    # two calls in a row, each with more key splits than one cluster merges (so the
    # partials go through the fixed array): a budget-16 tree over 4096 keys in 20
    # splits, then a 29-node tree over 2048 keys in 18 -- the second reuses the
    # array the first left behind
    for seed, n, prefix, splits in ((1, 17, 4096, 20), (2, 29, 2048, 18)):
        q, k, v, bits = _case(seed, n, prefix, dev)
        assert 0 < lib.rt_tree_attn_workspace_size(n, 32, 8, 128, prefix, splits) <= \
            lib.rt_tree_attn_noalloc_max_bytes()
        got = _noalloc(q, k, v, bits, prefix, splits, status, stream)
        want = kernels.tree_attention(q, k, v, bits, prefix, num_splits=splits)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        err = (got.float() - want.float()).abs()
        assert float(err.max()) <= MAX_ABS and float(err.mean()) <= MEAN_ABS
    # a shape whose partials exceed the fixed array is refused before any launch:
    # RT_ERR_WORKSPACE, the output left as it was and no device status raised
    n_big, prefix_big, splits_big = 257, 4096, 64
    assert lib.rt_tree_attn_workspace_size(n_big, 32, 8, 128, prefix_big, splits_big) > \
        lib.rt_tree_attn_noalloc_max_bytes()
    q, k, v, bits = _case(3, n_big, prefix_big, dev)
    out = torch.full_like(q, float("nan"))
    torch.cuda.synchronize()
    rc = lib.rt_tree_attn_noalloc(q.data_ptr(), q.stride(0) * 2, q.stride(1) * 2, k.data_ptr(), v.data_ptr(),
                                  k.stride(0) * 2, k.stride(1) * 2, k.shape[1], out.data_ptr(), out.stride(0) * 2,
                                  out.stride(1) * 2, bits.data_ptr(), bits.shape[1], n_big, prefix_big, None, 32, 8,
                                  128, ctypes.c_float(128 ** -0.5), splits_big, 0, status.data_ptr(), stream)
    assert rc == _lib.RT_ERR_WORKSPACE, _lib.status_string(rc)
    torch.cuda.synchronize()
    assert bool(torch.isnan(out.float()).all())
    assert int(status.item()) == 0
