"""Round-robin layer eigendecompositions shared through peer memory.

With N ranks solving the row shards of a stream of layers (one process per GPU), layer k's floored fp64
eigendecomposition (mpq/adapters/quip_sharp.py:33-67) is computed on rank k mod N only -- ahead of time, on that
rank's set-up pipeline -- and written into one of that rank's exported peer buffers.  The other ranks copy it from
there with the copy engines over NVLink when they reach layer k.  Readiness and buffer reuse go through the process
group's key-value store: the owner sets a ready key once its copy into the buffer is complete, each reader sets an
acknowledgement once its copy out is complete, and the owner reuses a buffer slot only after every reader
acknowledged the layer held there.  No collective runs per layer, so a rank busy with an eigendecomposition delays
only the ranks that need that very layer, not every step of every rank.

The store is used from two threads (the owner publishes from its set-up thread, readers fetch from the solving
thread): every store operation is short and taken under one lock, and waiting is polling, so neither thread holds
the store while it waits.
"""
from __future__ import annotations

import ctypes
import itertools
import threading
import time
from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist

from ._lib import call

_INSTANCES = itertools.count()
IPC_HANDLE_BYTES = 64

Eigen = Tuple[torch.Tensor, torch.Tensor, float]


class _DeviceMemory:
    """A raw device allocation seen by torch.as_tensor (zero copy) as a 1-D float32 array."""

    def __init__(self, ptr: int, nfloats: int):
        self.__cuda_array_interface__ = {"shape": (nfloats,), "typestr": "<f4", "data": (ptr, False), "version": 3}


class EigenExchange:
    """Per-rank exported buffer of `slots` eigendecompositions of size n, and mappings of every other rank's."""

    def __init__(self, n: int, device: torch.device, *, slots: int = 2, timeout_s: float = 300.0, group=None):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("EigenExchange needs an initialised process group")
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.dev = torch.device(device)
        self.n, self.slots = int(n), max(int(slots), 1)
        self.unit = self.n + self.n * self.n + 1  # lam, V (row-major), floor
        self.timeout_s = float(timeout_s)
        self.prefix = f"mpq-eig/{next(_INSTANCES)}"
        self._store = dist.distributed_c10d._get_default_store()
        self._lock = threading.Lock()
        self.recv = torch.empty(self.unit, device=self.dev, dtype=torch.float32)
        self._open_transport()

    # ---- transport: one exported buffer per rank, mapped by every other rank ----
    def _open_transport(self) -> None:
        nbytes = self.slots * self.unit * 4
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        call("mpq_peer_alloc", nbytes, ctypes.addressof(ptr), ctypes.addressof(handle))
        self._ptr = int(ptr.value)
        self.local = torch.as_tensor(_DeviceMemory(self._ptr, self.slots * self.unit), device=self.dev)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=self.group)
        self._peers: Dict[int, int] = {}
        for r, h in enumerate(handles):
            if r == self.rank:
                continue
            hb = ctypes.create_string_buffer(h, IPC_HANDLE_BYTES)
            p = ctypes.c_void_p()
            call("mpq_peer_open", ctypes.addressof(hb), ctypes.addressof(p))
            self._peers[r] = int(p.value)

    def _write_slot(self, slot: int, eig: Eigen) -> None:
        lam, V, floor = eig
        dst = self.local[slot * self.unit:(slot + 1) * self.unit]
        n = self.n
        dst[:n].copy_(lam)
        dst[n:n + n * n].view(n, n).copy_(V)
        dst[-1:].fill_(float(floor))

    def _read_slot(self, owner: int, slot: int) -> None:
        src = self._peers[owner] + slot * self.unit * 4
        call("mpq_copy_bytes", self.recv.data_ptr(), src, self.unit * 4)

    def _close_transport(self) -> None:
        dist.barrier(group=self.group)  # every reader has finished its copies
        for p in self._peers.values():
            call("mpq_peer_close", p)
        self._peers = {}
        dist.barrier(group=self.group)  # every mapping of this rank's buffer is gone
        self.local = None
        call("mpq_peer_free", self._ptr)
        self._ptr = 0

    # ---- store access (two threads) ----
    def _set(self, key: str, value: bytes = b"1") -> None:
        with self._lock:
            self._store.set(key, value)

    def _get(self, key: str) -> bytes:
        with self._lock:
            return self._store.get(key)

    def _wait(self, keys) -> None:
        deadline = time.monotonic() + self.timeout_s
        while True:
            with self._lock:
                if self._store.check(keys):
                    return
            if time.monotonic() > deadline:
                raise TimeoutError(f"EigenExchange: rank {self.rank} gave up waiting for {keys}")
            time.sleep(2e-4)

    # ---- protocol ----
    def owner(self, k: int) -> int:
        return k % self.world

    def _slot(self, k: int) -> int:
        return (k // self.world) % self.slots

    def _key(self, kind: str, k: int, r: Optional[int] = None) -> str:
        return f"{self.prefix}/{kind}/{k}" + ("" if r is None else f"/{r}")

    def publish(self, k: int, eig: Eigen) -> None:
        """On layer k's owner, from the set-up thread with the set-up's stream current: write the result into
        this layer's slot once the layer that used it before was acknowledged by every reader."""
        if self.owner(k) != self.rank:
            raise ValueError(f"rank {self.rank} does not own layer {k}")
        prev = k - self.slots * self.world
        if prev >= 0 and self.world > 1:
            self._wait([self._key("ack", prev, r) for r in range(self.world) if r != self.rank])
        self._write_slot(self._slot(k), eig)
        if self.dev.type == "cuda":
            torch.cuda.current_stream(self.dev).synchronize()
        self._set(self._key("ready", k))

    def fetch(self, k: int) -> Eigen:
        """On a reader, on the calling stream: layer k's (lam, V, floor) in this exchange's receive buffer (valid
        until the next fetch).  Blocks the host until the owner published it."""
        owner = self.owner(k)
        if owner == self.rank:
            raise ValueError(f"rank {self.rank} owns layer {k}: use its own result")
        self._wait([self._key("ready", k)])
        self._read_slot(owner, self._slot(k))
        floor = float(self.recv[-1:].item())  # synchronises the stream: the copy out is complete
        self._set(self._key("ack", k, self.rank))
        n = self.n
        return self.recv[:n], self.recv[n:n + n * n].view(n, n), floor

    def skip(self, k: int) -> None:
        """On a reader: layer k will not be fetched (its step was dropped); the owner may reuse its slot."""
        if self.owner(k) != self.rank:
            self._set(self._key("ack", k, self.rank))

    def close(self) -> None:
        if getattr(self, "_ptr", 0):
            self._close_transport()
