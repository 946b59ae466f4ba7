"""In-process world for threads with real semantics.

``local_world(n, timeout_s, faults)`` returns one communicator per rank; each
rank is driven by its own thread.  Point-to-point messages queue per (src, dst)
pair, ``recv`` blocks until a message arrives or the deadline passes
(``CommTimeout``), and the collectives combine every rank's contribution.  A
``FaultPlan`` injects host-side failures (drop a message, delay, kill a rank at
its k-th op); peers of a killed rank get ``CommError`` on their next op.
"""
from __future__ import annotations

import threading
from typing import Callable, List, Optional

from .._ext import host as _host
from .base import FaultPlan

_C = _host()
LocalCommunicator = _C.LocalCommunicator


def local_world(n: int, timeout_s: float = 30.0, faults: Optional[FaultPlan] = None) -> List[LocalCommunicator]:
    return _C.local_world(n, timeout_s, faults)


def run_threads(comms, fn: Callable, *args, timeout_s: float = 60.0):
    """Run ``fn(comm, *args)`` on one thread per rank; returns results (exceptions re-raised
    as a list entry)."""
    out: list = [None] * len(comms)

    def body(i):
        try:
            out[i] = fn(comms[i], *args)
        except BaseException as e:  # noqa: BLE001 - reported to the caller
            out[i] = e

    ts = [threading.Thread(target=body, args=(i,), daemon=True) for i in range(len(comms))]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout_s)
    return out


__all__ = ["LocalCommunicator", "local_world", "run_threads"]
