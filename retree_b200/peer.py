"""Attention-output all-gather of a KV-head split over NVLink peer memory.

Under ``headsplit`` every rank attends over its own KV heads and o_proj needs
all ranks' outputs in head order.  ``headsplit.gather_heads`` does that with
an NCCL all-gather per layer; ``PeerExchange`` does it with this package's
kernels over buffers the ranks map from each other (CUDA IPC handles swapped
once through the process group; plain peer mappings, no multicast object):

  rank r's attention writes its rows straight into its exchange slot;
  ``signal(layer)``  stores the layer's epoch into slot r of every rank's flag
                     array (rt_peer_signal);
  ``gather(layer)``  waits (bounded, per source rank) for the flags and copies
                     every rank's rows into the ``[n, world * cols]`` o_proj
                     input (rt_peer_gather);
  ``linear(layer)``  or, instead of gather + o_proj, the o_proj itself pulls
                     each rank's columns as its K loop reaches them, after the
                     same wait (rt_linear_gather), so the transfers overlap the
                     weight stream.

Two slots alternate by layer, which is safe without a consumed-handshake: rank
r writes a slot again two layers later, after its own o_proj of the layer in
between, which needed every peer's attention of that layer, which the peers
ran after their o_proj of the layer whose slot is being overwritten.  Epochs
come from a device counter advanced once per forward (``step``), so CUDA-graph
replays see fresh epochs; the flags only grow.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, kernels

MAX_PEERS = 8


class _Raw:
    """A raw device allocation seen as a torch tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


def _tensor(ptr: int, nbytes: int, device) -> torch.Tensor:
    return torch.as_tensor(_Raw(ptr, nbytes), device=device)


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


class PeerExchange:
    def __init__(self, group, rank: int, world: int, max_rows: int, cols: int, num_layers: int, device):
        if not 1 <= world <= MAX_PEERS:
            raise ValueError(f"the peer exchange takes 1..{MAX_PEERS} ranks")
        if (cols * 2) % 16:
            raise ValueError("exchange rows must be a multiple of 16 bytes")
        self.group, self.rank, self.world = group, int(rank), int(world)
        self.max_rows, self.cols, self.layers = int(max_rows), int(cols), int(num_layers)
        self.device = torch.device(device)
        lib = _lib.load()
        self.slot_bytes = _align(self.max_rows * self.cols * 2)
        nbytes = 2 * self.slot_bytes + _align(8 * MAX_PEERS)
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        with torch.cuda.device(self.device):
            _lib.check(lib.rt_ipc_alloc(nbytes, ctypes.byref(ptr), handle), "rt_ipc_alloc")
        self._own = ptr.value
        self._opened: list[int] = []
        # every rank's handle, once, through the process group
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(self._own)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            with torch.cuda.device(self.device):
                _lib.check(lib.rt_ipc_open(hb, ctypes.byref(p)), "rt_ipc_open")
            self._opened.append(p.value)
            bases.append(p.value)
        self.bases = bases
        self.flags_off = 2 * self.slot_bytes
        self._mem = _tensor(self._own, nbytes, self.device)
        self.flags_local = self._mem[self.flags_off: self.flags_off + 8 * self.world].view(torch.int64)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        self._flag_ptrs = (ctypes.c_void_p * self.world)(*[b + self.flags_off for b in bases])
        self._slot_ptrs = [(ctypes.c_void_p * self.world)(*[b + s * self.slot_bytes for b in bases]) for s in (0, 1)]
        dist.barrier(group=group)

    # ------------------------------------------------------------------ views
    def slot(self, layer: int, rows: int) -> torch.Tensor:
        """This rank's exchange rows for ``layer``: ``[rows, cols]`` bf16 (the attention's output buffer)."""
        s = layer % 2
        b = self._mem[s * self.slot_bytes: s * self.slot_bytes + rows * self.cols * 2]
        return b.view(torch.bfloat16).view(rows, self.cols)

    def _epoch_add(self, layer: int) -> int:
        # epoch of layer l in the forward that advanced the counter to E: E - layers + l + 1
        return layer + 1 - self.layers

    # ------------------------------------------------------------------ steps
    def step(self) -> None:
        """Once per forward, before its first layer."""
        _lib.check(_lib.load().rt_peer_epoch_step(self.epoch.data_ptr(), self.layers,
                                                    kernels._stream(self.device)), "rt_peer_epoch_step")
        kernels._count()

    def signal(self, layer: int) -> None:
        """Announce this rank's rows of ``layer`` (after the kernel that wrote them, on the same stream)."""
        _lib.check(_lib.load().rt_peer_signal(self._flag_ptrs, self.world, self.rank, self.epoch.data_ptr(),
                                                self._epoch_add(layer), kernels._stream(self.device)),
                   "rt_peer_signal")
        kernels._count()

    def gather(self, layer: int, rows: int, out: torch.Tensor) -> torch.Tensor:
        """Every rank's rows of ``layer`` into ``out [rows, world * cols]`` (bf16, head order)."""
        if out.dtype != torch.bfloat16 or out.shape[-1] != self.world * self.cols or out.stride(-1) != 1:
            raise RuntimeError("gather output must be bf16 [rows, world * cols] with unit inner stride")
        if rows > self.max_rows:
            raise RuntimeError("more rows than the exchange holds")
        _lib.check(_lib.load().rt_peer_gather(
            self._slot_ptrs[layer % 2], self.world, rows, self.cols * 2, self.cols * 2, out.data_ptr(),
            out.stride(0) * 2, self.flags_local.data_ptr(), self.epoch.data_ptr(), self._epoch_add(layer),
            kernels.status_tensor(self.device).data_ptr(), kernels._stream(self.device)), "rt_peer_gather")
        kernels._count()
        return out

    def linear(self, layer: int, rows: int, w: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """``out [rows, n_out] = X @ w^T`` with X gathered from every rank's slot inside the projection
        (rt_linear_gather: each CTA waits for a rank's announcement before its first load of that rank's
        columns; no separate gather launch)."""
        n_out, k = w.shape
        if k != self.world * self.cols or w.dtype != torch.bfloat16 or not w.is_contiguous():
            raise RuntimeError("weights must be contiguous bf16 [n_out, world * cols]")
        if out.dtype != torch.bfloat16 or out.stride(-1) != 1 or out.shape[-1] != n_out:
            raise RuntimeError("out must be bf16 [rows, n_out] with unit inner stride")
        _lib.check(_lib.load().rt_linear_gather(
            self._slot_ptrs[layer % 2], self.world, self.cols, self.cols, rows, w.data_ptr(), n_out, k,
            out.data_ptr(), out.stride(0), self.flags_local.data_ptr(), self.epoch.data_ptr(),
            self._epoch_add(layer), kernels.status_tensor(self.device).data_ptr(), kernels._stream(self.device)),
            "rt_linear_gather")
        kernels._count()
        return out

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (every rank calls it; it synchronises the group)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _lib.load()
        for p in self._opened:
            lib.rt_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        dist.barrier(group=self.group)
        lib.rt_ipc_free(ctypes.c_void_p(self._own))
        self._own = None
