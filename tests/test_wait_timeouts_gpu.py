"""Failure detection without a GPU fault: a cross-GPU wait that nothing satisfies gives up.

The peer-memory gather and the gathered projection wait for a flag that
another rank stores.  Here nothing stores it (one GPU, one process, a flag
left at zero), so each wait runs out its bound (4M polls: half a second to
a few seconds), the kernel records RT_DEV_WAIT_TIMEOUT in the device status
word, skips its copies, and exits; the host raises on the status, and the
same context keeps working -- the calls succeed once the flag is set.
"""

import ctypes

import pytest
import torch

from retree_b200 import _lib, kernels
from tests.gpu_util import cuda

pytestmark = [pytest.mark.gpu, pytest.mark.late]


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


@torch.inference_mode()
def test_peer_gather_gives_up_on_a_flag_nobody_sets():
    dev = cuda()
    lib = _lib.load()
    src = torch.full((8, 64), 3.0, dtype=torch.bfloat16, device=dev)
    out = torch.zeros((8, 64), dtype=torch.bfloat16, device=dev)
    flags = torch.zeros(1, dtype=torch.int64, device=dev)
    epoch = torch.tensor([5], dtype=torch.int64, device=dev)
    bufs = (ctypes.c_void_p * 1)(src.data_ptr())
    status = kernels.status_tensor(dev)

    def gather():
        return lib.rt_peer_gather(bufs, 1, 8, 128, 128, out.data_ptr(), 128, flags.data_ptr(), epoch.data_ptr(), 0,
                                  status.data_ptr(), _stream(dev))

    assert gather() == _lib.RT_OK
    torch.cuda.synchronize(dev)
    with pytest.raises(RuntimeError, match="wait"):
        kernels.check_device_status(dev)
    assert float(out.float().abs().sum()) == 0.0  # nothing copied
    flags.fill_(5)  # the announcement arrives: the same call now copies
    assert gather() == _lib.RT_OK
    torch.cuda.synchronize(dev)
    kernels.check_device_status(dev)
    assert torch.equal(out, src)


@torch.inference_mode()
def test_gathered_projection_gives_up_on_a_flag_nobody_sets():
    dev = cuda()
    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(0)
    m, k, n_out = 17, 256, 256
    x = torch.randn((m, k), device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn((n_out, k), device=dev, generator=g) * k ** -0.5).to(torch.bfloat16)
    out = torch.zeros((m, n_out), dtype=torch.bfloat16, device=dev)
    flags = torch.zeros(1, dtype=torch.int64, device=dev)
    epoch = torch.tensor([5], dtype=torch.int64, device=dev)
    xr = (ctypes.c_void_p * 1)(x.data_ptr())
    status = kernels.status_tensor(dev)

    def gathered():
        return lib.rt_linear_gather(xr, 1, k, k, m, w.data_ptr(), n_out, k, out.data_ptr(), n_out, flags.data_ptr(),
                                    epoch.data_ptr(), 0, status.data_ptr(), _stream(dev))

    assert gathered() == _lib.RT_OK
    torch.cuda.synchronize(dev)
    with pytest.raises(RuntimeError, match="wait"):
        kernels.check_device_status(dev)
    want = kernels.linear(x, w)  # the context is fine: a plain projection runs
    torch.cuda.synchronize(dev)
    kernels.check_device_status(dev)
    flags.fill_(5)
    assert gathered() == _lib.RT_OK
    torch.cuda.synchronize(dev)
    kernels.check_device_status(dev)
    assert torch.equal(out, want)  # same kernel, same plan: the gathered X is X
