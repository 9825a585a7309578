"""Recovery memory as a device hash table for the on-device recovery walk.

Layout shared with ``csrc/recovery_walk.cuh``: open addressing with linear
probing over a power-of-two capacity, key ``draft << 32 | target`` (uint64,
all ones = empty), slot = splitmix64-mix(key) & (capacity - 1), and separate
int32 prior / online count arrays (the two tables of RecoveryMemory,
model/recovery.py:35-266).  ``RecoveryTable`` builds and reads the table on
the host (numpy); ``to_device`` hands the three arrays to torch.
"""

from __future__ import annotations

import math

import numpy as np

from .recovery import RecoveryMemory

EMPTY = np.uint64(0xFFFFFFFFFFFFFFFF)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def mix64(x) -> np.uint64:
    """splitmix64's output mix (Steele, Lea, Flood 2014), wrapping uint64 arithmetic."""
    x = np.uint64(x)
    with np.errstate(over="ignore"):
        x ^= x >> np.uint64(30)
        x = np.uint64(x * _M1)
        x ^= x >> np.uint64(27)
        x = np.uint64(x * _M2)
        x ^= x >> np.uint64(31)
    return x


def pair_key(draft: int, target: int) -> np.uint64:
    return np.uint64(((int(draft) & 0xFFFFFFFF) << 32) | (int(target) & 0xFFFFFFFF))


class RecoveryTable:
    def __init__(self, capacity: int):
        if capacity <= 0 or capacity & (capacity - 1):
            raise ValueError("capacity must be a power of two")
        self.capacity = int(capacity)
        self.keys = np.full(self.capacity, EMPTY, dtype=np.uint64)
        self.prior = np.zeros(self.capacity, dtype=np.int32)
        self.online = np.zeros(self.capacity, dtype=np.int32)

    @staticmethod
    def capacity_for(pairs: int, load: float = 0.5, minimum: int = 1 << 12) -> int:
        need = max(minimum, int(math.ceil(max(pairs, 1) / load)))
        return 1 << (need - 1).bit_length()

    @classmethod
    def from_memory(cls, memory: RecoveryMemory, capacity: int | None = None, extra_pairs: int = 1 << 16):
        """The table of ``memory``'s pair rows (both counts of a pair in one slot)."""
        t = cls(capacity or cls.capacity_for(memory.total_pairs() + extra_pairs))
        for d, g, prior, online in memory.rows():
            s = t.insert(d, g)
            t.prior[s] += prior
            t.online[s] += online
        return t

    def _slot(self, key: np.uint64, insert: bool) -> int:
        mask = self.capacity - 1
        s = int(mix64(key)) & mask
        for _ in range(self.capacity):
            k = self.keys[s]
            if k == key:
                return s
            if k == EMPTY:
                if not insert:
                    return -1
                self.keys[s] = key
                return s
            s = (s + 1) & mask
        if insert:
            raise RuntimeError("recovery table full")
        return -1

    def insert(self, draft: int, target: int) -> int:
        return self._slot(pair_key(draft, target), True)

    def frequency(self, draft: int, target: int) -> int:
        s = self._slot(pair_key(draft, target), False)
        return 0 if s < 0 else int(self.prior[s]) + int(self.online[s])

    def online_counts(self) -> dict:
        used = (self.keys != EMPTY) & (self.online > 0)
        out = {}
        for k, c in zip(self.keys[used].tolist(), self.online[used].tolist()):
            d, g = k >> 32, k & 0xFFFFFFFF
            out[(d - (1 << 32) if d >= 1 << 31 else d, g - (1 << 32) if g >= 1 << 31 else g)] = c
        return out

    def to_device(self, device):
        import torch
        return (torch.from_numpy(self.keys.view(np.int64)).to(device), torch.from_numpy(self.prior).to(device),
                torch.from_numpy(self.online).to(device))


class DeviceRecoveryMemory:
    """A RecoveryMemory whose counts live in a device table that the recovery walk updates in place.

    ``memory`` (the host RecoveryMemory) stays the record for files and the
    cross-rank delta exchange: ``sync()`` applies the walk's logged online
    increments to it.  The log holds ``log_capacity`` increments between syncs.
    """

    def __init__(self, memory: RecoveryMemory, device, capacity: int | None = None, log_capacity: int = 1 << 16,
                 stop_ids=None):
        import torch
        self.memory = memory
        self.device = torch.device(device)
        host = RecoveryTable.from_memory(memory, capacity)
        self.capacity = host.capacity
        self.table = host.to_device(self.device)
        self.log_pairs = torch.zeros((log_capacity, 2), dtype=torch.int32, device=self.device)
        self.log_count = torch.zeros(1, dtype=torch.int32, device=self.device)
        # an empty stop set behaves as none (no pair is a stop pair)
        stops = sorted({int(t) for t in stop_ids}) if stop_ids is not None else []
        self.stop_ids = torch.tensor(stops, dtype=torch.int64, device=self.device) if stops else None

    @property
    def freq_threshold(self) -> int:
        return self.memory.freq_threshold

    def log(self):
        return self.log_pairs, self.log_count

    def sync(self) -> int:
        """Apply the logged online increments to the host memory; returns how many."""
        n = int(self.log_count.item())
        if n:
            for d, t in self.log_pairs[:n].cpu().tolist():
                self.memory.record_online(d, t)
            self.log_count.zero_()
        return n

    def apply_online_delta(self, delta: dict) -> None:
        """Other ranks' online counts (distributed.synchronize_online_memory), on both copies."""
        if not delta:
            return
        self.memory.apply_online_delta(delta)
        keys, prior, online = self.table
        host = RecoveryTable(self.capacity)
        host.keys[:] = keys.cpu().numpy().view(np.uint64)
        host.prior[:] = prior.cpu().numpy()
        host.online[:] = online.cpu().numpy()
        for (d, t), c in delta.items():
            host.online[host.insert(d, t)] += int(c)
        # in place: CUDA graphs captured over the walk keep the same buffers
        for dst, src in zip(self.table, host.to_device(self.device)):
            dst.copy_(src)
