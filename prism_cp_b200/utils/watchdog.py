"""Stall watchdog: report where the host and the GPU stopped when a step makes no progress.

``StallWatchdog(stall_s)`` is fed ``beat(label)`` calls from the trainer and the
executor (microbatch and layer boundaries, forward and backward). Each beat
records a CUDA event on the current stream and re-arms ``faulthandler``'s
timer. When no beat arrives for ``stall_s`` seconds:

* ``faulthandler`` (a C thread that needs neither the GIL nor CUDA) dumps the
  Python stack of every thread to stderr: where the host is blocked;
* a Python thread queries the recorded events newest-first (``cudaEventQuery``
  does not block) and prints the last label the GPU completed and the first it
  has not: which layer and phase the device is stuck in.

Nothing is synchronised, so enabling it does not change the timing of the
work it watches. Enable with ``PRISM_WATCHDOG=<seconds>`` or by passing a
watchdog to the trainer. The reference's failure detection is host-side too
(process exit codes, peer kill on the first failure:
scripts/torchrun_launcher.py:44-118); this adds the in-process view.
"""

from __future__ import annotations

import collections
import faulthandler
import os
import sys
import threading
import time

import torch


class StallWatchdog:
    def __init__(self, stall_s: float, history: int = 1024, stream=None, fault_file=None):
        self.stall_s = float(stall_s)
        self.marks: collections.deque = collections.deque(maxlen=history)
        self.last_beat = time.monotonic()
        self.last_label = "start"
        self.reported = False
        self.stream = stream if stream is not None else sys.stderr
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self.cuda = torch.cuda.is_available()
        # faulthandler writes to a real file descriptor from its own C thread
        self.fault_file = fault_file if fault_file is not None else sys.__stderr__
        try:
            self.fault_file.fileno()
        except (AttributeError, OSError, ValueError):
            self.fault_file = None
        self._arm()
        self.thread = threading.Thread(target=self._run, daemon=True, name="prism-watchdog")
        self.thread.start()

    def beat(self, label: str) -> None:
        ev = None
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record()
        with self._lock:
            self.marks.append((label, ev))
            self.last_beat = time.monotonic()
            self.last_label = label
            self.reported = False
        self._arm()

    def _arm(self) -> None:
        if self.fault_file is not None:
            faulthandler.dump_traceback_later(self.stall_s, repeat=False, file=self.fault_file, exit=False)

    def gpu_position(self):
        """(last completed label, first pending label) among the recorded beats."""
        with self._lock:
            marks = list(self.marks)
        done, pending = None, None
        for label, ev in reversed(marks):
            if ev is None:
                continue
            if ev.query():
                done = label
                break
            pending = label
        return done, pending

    def report(self) -> str:
        done, pending = self.gpu_position() if self.cuda else (None, None)
        return (f"[watchdog] no progress for {time.monotonic() - self.last_beat:.0f} s after host beat "
                f"'{self.last_label}'; GPU completed up to '{done}', first pending '{pending}'")

    def _run(self) -> None:
        while not self._stop.wait(1.0):
            with self._lock:
                stalled = (time.monotonic() - self.last_beat) > self.stall_s and not self.reported
            if stalled:
                msg = self.report()
                print(msg, file=self.stream, flush=True)
                with self._lock:
                    self.reported = True

    def close(self) -> None:
        self._stop.set()
        if self.fault_file is not None:
            faulthandler.cancel_dump_traceback_later()


_ACTIVE: StallWatchdog | None = None


def from_env() -> StallWatchdog | None:
    """The process-wide watchdog if ``PRISM_WATCHDOG`` is set (created once)."""
    global _ACTIVE
    if _ACTIVE is None:
        s = os.environ.get("PRISM_WATCHDOG")
        if s:
            _ACTIVE = StallWatchdog(float(s))
    return _ACTIVE


def beat(label: str) -> None:
    """Beat the process-wide watchdog, if any."""
    if _ACTIVE is not None:
        _ACTIVE.beat(label)
