"""Per-layer set-up ahead of the solves.

Before a layer's rows can be solved, the adapters need layer-wide set-up: the randomized Hadamard rotations of W
and H, the unit-RMS scale and the floored fp64 eigendecomposition of the rotated Hessian
(mpq/adapters/quip_sharp.py:33-67, :468-520).  The reference runs it serially before each layer.  It depends only
on the layer's own W and H, so while the row blocks of layer k are solved, the set-up of a later layer runs here:
on one worker thread (the eigendecomposition blocks its calling thread on host synchronisations) and on one
lowest-priority stream, so the solve's kernels are scheduled first and the set-up takes the SMs they leave.

A set-up starts after the work its caller's stream had been given when it was submitted.  Results come back
through get(): the caller's stream waits for the set-up's completion event, and every tensor of the result is
recorded on the caller's stream, so the caching allocator does not hand its memory to the worker stream while the
solve still reads it.  drain() waits for every set-up still in flight (a timed region that submitted set-ups ends
after their work).
"""
from __future__ import annotations

from concurrent.futures import Future, ThreadPoolExecutor
from typing import Any, Callable, Dict, Hashable, Iterator

import torch


def _tensors(obj: Any) -> Iterator[torch.Tensor]:
    if torch.is_tensor(obj):
        yield obj
    elif isinstance(obj, dict):
        for v in obj.values():
            yield from _tensors(v)
    elif isinstance(obj, (list, tuple)):
        for v in obj:
            yield from _tensors(v)


class SetupPipeline:
    """A single worker thread with its own lowest-priority CUDA stream; set-ups run in submission order."""

    def __init__(self, device: torch.device):
        self.dev = torch.device(device)
        lo, _ = torch.cuda.Stream.priority_range()
        self.stream = torch.cuda.Stream(self.dev, priority=lo)
        self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="mpq-setup",
                                        initializer=torch.cuda.set_device, initargs=(self.dev,))
        self._pending: Dict[Hashable, Future] = {}

    def submit(self, key: Hashable, fn: Callable[..., Any], *args, **kwargs) -> None:
        """Queue fn(*args, **kwargs) on the worker; its CUDA work goes to the worker's stream, ordered after
        everything the caller's stream has been given so far (the inputs may still be in flight there)."""
        if key in self._pending:
            raise KeyError(f"set-up {key!r} is already queued")
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.dev))
        for t in _tensors((args, kwargs)):
            if t.is_cuda:
                t.record_stream(self.stream)

        def work():
            self.stream.wait_event(ready)
            with torch.inference_mode(), torch.cuda.stream(self.stream):
                out = fn(*args, **kwargs)
                ev = torch.cuda.Event()
                ev.record(self.stream)
            return out, ev

        self._pending[key] = self._pool.submit(work)

    def pending(self, key: Hashable) -> bool:
        return key in self._pending

    def keys(self):
        """Keys of the queued set-ups, in submission order."""
        return list(self._pending)

    def get(self, key: Hashable) -> Any:
        """The set-up's result, ordered before everything the caller's stream runs next (re-raises its error)."""
        out, ev = self._pending.pop(key).result()
        cur = torch.cuda.current_stream(self.dev)
        cur.wait_event(ev)
        for t in _tensors(out):
            if t.is_cuda:
                t.record_stream(cur)
        return out

    def wait(self, key: Hashable) -> None:
        """Block until the set-up has run and its device work has completed; its result stays queued for get()."""
        _, ev = self._pending[key].result()
        ev.synchronize()

    def drain(self) -> None:
        """Wait for every queued set-up; the caller's stream then waits for their device work.  Results are
        dropped."""
        for key in list(self._pending):
            self.get(key)

    def close(self) -> None:
        try:
            self.drain()
        finally:
            self._pool.shutdown(wait=True)

    def __enter__(self) -> "SetupPipeline":
        return self

    def __exit__(self, *exc) -> None:
        self.close()
