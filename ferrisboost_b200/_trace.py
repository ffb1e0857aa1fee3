"""FBGPU_TRACE=1: wall time of each phase of a training call on stderr."""
from __future__ import annotations

import os
import sys
import time


class PhaseTrace:
    def __init__(self, what: str):
        self.what, self.on, self.clock = what, bool(os.environ.get("FBGPU_TRACE")), time.perf_counter
        self.t = self.clock()

    def __call__(self, name: str) -> None:
        if not self.on:
            return
        now = self.clock()
        sys.stderr.write(f"[fbgpu] {self.what} {name:<30} {1000 * (now - self.t):9.3f} ms\n")
        self.t = now
