"""Step-phase timing (``THESEUS_PROFILE=1``).

The reference only hashes ``THESEUS_PROFILE`` into its run-agreement check (``train.py:67``). Here
the variable turns on device-timed phases of every training step: CUDA events around the teacher
forward, each layer's student micro-steps and each layer's reduction + update (which, with the
peer-memory exchange, only enqueues work on the exchange stream), plus NVTX ranges with the same
names for external timeline tools. ``summary()`` returns milliseconds per phase for the last step;
the trainer emits them as a ``profile`` event with the maximum over ranks. Without the variable every
call is a no-op.
"""
import os
import time
from contextlib import contextmanager

import torch


def enabled():
    return os.environ.get("THESEUS_PROFILE", "0") not in ("", "0")


class StepProfiler:
    def __init__(self, device, on=None):
        self.on = enabled() if on is None else on
        self.cuda = device.type == "cuda"
        self.marks = []  # (name, start, end)
        self.host = {}   # phase -> host seconds spent issuing it

    def reset(self):
        self.marks = []
        self.host = {}

    @contextmanager
    def phase(self, name):
        if not self.on:
            yield
            return
        if self.cuda:
            torch.cuda.nvtx.range_push(name)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            t0 = time.perf_counter()
            try:
                with torch.profiler.record_function("phase:" + name):  # kernel attribution under torch.profiler
                    yield
            finally:
                self.host[name] = self.host.get(name, 0.0) + time.perf_counter() - t0
                end.record()
                torch.cuda.nvtx.range_pop()
                self.marks.append((name, start, end))
        else:
            t0 = time.perf_counter()
            try:
                yield
            finally:
                self.marks.append((name, t0, time.perf_counter()))

    def host_summary(self):
        """{phase: ms} of host time spent issuing each phase in the last step (summed over repeats)."""
        return {name: 1000.0 * sec for name, sec in self.host.items()}

    def summary(self):
        """{phase: ms} summed over repeated phases of the step (synchronizes the device once)."""
        if not self.on or not self.marks:
            return {}
        if self.cuda:
            self.marks[-1][2].synchronize()
        out = {}
        for name, a, b in self.marks:
            ms = a.elapsed_time(b) if self.cuda else (b - a) * 1000.0
            out[name] = out.get(name, 0.0) + ms
        return out
