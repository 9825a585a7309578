"""Multi-process plumbing: the reference's ``distributed.py`` API plus fixed-shape
recovery-delta exchange.

One process per GPU (``torchrun``); ``init`` opens an NCCL process group (gloo
when no GPU is visible, e.g. in CPU tests).  The helpers keep the reference's
single-process behaviour when ``RANK`` is unset (distributed.py:21-79).

``all_gather_recovery_delta`` replaces the pickled ``all_gather_object`` of
each rank's online delta (benchmark.py:134-143) with one fixed-shape
``all_gather_into_tensor`` of ``int32[capacity, 3]`` (draft token, target
token, count) per rank -- 48 KiB at the benchmark's 4096 pairs -- and
``synchronize_online_memory`` applies the other ranks' deltas exactly as the
reference does.
"""

from __future__ import annotations

import datetime
import os
import warnings
from typing import Any

import torch
import torch.distributed as dist

__all__ = ["init", "is_initialized", "size", "rank", "local_size", "local_rank", "is_main", "barrier",
           "gather", "all_gather", "encode_delta", "decode_deltas", "all_gather_recovery_delta",
           "synchronize_online_memory"]


def init(timeout_s: float = 600.0, backend: str | None = None) -> None:
    """Open the process group from ``env://`` (distributed.py:21-29); no-op without ``RANK``."""
    if "RANK" not in os.environ:
        warnings.warn("Environment variable `RANK` is not set. Skipping distributed initialization.")
        return
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local_rank())
    dist.init_process_group(backend=backend, init_method="env://", timeout=datetime.timedelta(seconds=timeout_s))
    if backend == "nccl":
        # NCCL collectives on the same streams: no programmatic dependent launch (rt_set_pdl)
        from . import kernels
        kernels.set_pdl(False)


def is_initialized() -> bool:
    return dist.is_available() and dist.is_initialized()


def size() -> int:
    return int(os.environ.get("WORLD_SIZE", 1))


def rank() -> int:
    return int(os.environ.get("RANK", 0))


def local_size() -> int:
    return int(os.environ.get("LOCAL_WORLD_SIZE", 1))


def local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", 0))


def is_main() -> bool:
    return rank() == 0


def barrier() -> None:
    if is_initialized():
        dist.barrier()


def gather(obj: Any, dst: int = 0):
    """Python objects to rank ``dst`` (distributed.py:62-71)."""
    if not is_initialized():
        return [obj]
    if rank() == dst:
        out = [None] * size()
        dist.gather_object(obj, out, dst=dst)
        return out
    dist.gather_object(obj, dst=dst)
    return None


def all_gather(obj: Any) -> list:
    """Python objects from every rank (distributed.py:74-79)."""
    if not is_initialized():
        return [obj]
    out = [None] * size()
    dist.all_gather_object(out, obj)
    return out


# ---------------------------------------------------------------------------
# Fixed-shape recovery-delta exchange
# ---------------------------------------------------------------------------
def encode_delta(delta: dict, capacity: int, device=None) -> torch.Tensor:
    """``{(draft, target): count}`` -> ``int32[capacity, 3]``, zero-count rows as padding."""
    if len(delta) > capacity:
        raise ValueError(f"recovery delta has {len(delta)} pairs, more than the exchange capacity {capacity}")
    buf = torch.zeros((capacity, 3), dtype=torch.int32)
    if delta:
        rows = sorted(((int(d), int(t), int(c)) for (d, t), c in delta.items()))
        for d, t, c in rows:
            if not (0 <= d < 2 ** 31 and 0 <= t < 2 ** 31 and 0 < c < 2 ** 31):
                raise ValueError("recovery delta entries must be non-negative int32 token ids and positive counts")
        buf[: len(rows)] = torch.tensor(rows, dtype=torch.int32)
    return buf.to(device) if device is not None else buf


def decode_deltas(gathered: torch.Tensor) -> list[dict]:
    """``int32[world, capacity, 3]`` -> one ``{(draft, target): count}`` per rank."""
    out = []
    for rows in gathered.cpu().tolist():
        out.append({(d, t): c for d, t, c in rows if c > 0})
    return out


def all_gather_recovery_delta(delta: dict, capacity: int = 4096, group=None) -> list[dict]:
    """Every rank's online delta, via one ``all_gather_into_tensor`` of ``int32[capacity, 3]``."""
    if not is_initialized():
        return [dict(delta)]
    backend = dist.get_backend(group)
    device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    send = encode_delta(delta, capacity, device)
    world = dist.get_world_size(group)
    recv = torch.empty((world * capacity, 3), dtype=torch.int32, device=device)
    dist.all_gather_into_tensor(recv, send, group=group)
    return decode_deltas(recv.view(world, capacity, 3))


def synchronize_online_memory(recovery_memory, online_counts_before_request: dict, capacity: int = 4096,
                              group=None) -> None:
    """Apply every other rank's completed online events (benchmark.py:134-143)."""
    local = recovery_memory.online_delta_since(online_counts_before_request)
    deltas = all_gather_recovery_delta(local, capacity, group)
    me = dist.get_rank(group) if is_initialized() else 0
    for src, delta in enumerate(deltas):
        if src != me:
            recovery_memory.apply_online_delta(delta)
