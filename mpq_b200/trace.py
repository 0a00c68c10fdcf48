"""Lightweight launch accounting: counts C-ABI kernel launches and, when asked, times the
dominant kernel family with CUDA events on the launching stream."""
from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager
from typing import Dict, List, Optional, Tuple

import torch

_launches = 0
_timed_names: Optional[set] = None
_events: Dict[str, List[Tuple[torch.cuda.Event, torch.cuda.Event, float]]] = defaultdict(list)


def count_launch(n: int = 1) -> None:
    global _launches
    _launches += n


def launches() -> int:
    return _launches


def begin_timing(name: str):
    """Return an event pair if `name` is being timed, else None."""
    if _timed_names is None or name not in _timed_names or torch.cuda.is_current_stream_capturing():
        return None
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    return s, e


def end_timing(name: str, tok, work: float) -> None:
    if tok is None:
        return
    s, e = tok
    e.record()
    _events[name].append((s, e, float(work)))


@contextmanager
def timing(names):
    """Record CUDA events around every launch of the named entry points inside the block."""
    global _timed_names
    prev = _timed_names
    _timed_names = set(names)
    _events.clear()
    try:
        yield
    finally:
        _timed_names = prev


def summary(name: str) -> Dict[str, float]:
    """Average duration (ms) and algorithmic work per launch of `name` (call after a synchronize)."""
    ev = _events.get(name, [])
    if not ev:
        return {"launches": 0, "ms_total": 0.0, "ms_avg": 0.0, "work_avg": 0.0}
    ms = [s.elapsed_time(e) for s, e, _ in ev]
    work = [w for _, _, w in ev]
    return {"launches": len(ev), "ms_total": float(sum(ms)), "ms_avg": float(sum(ms) / len(ms)),
            "work_avg": float(sum(work) / len(work)), "work_total": float(sum(work))}
