"""Per-section device timing with CUDA events (the reference's UlyssesRuntime.profile_start /
profile_end sections, src/inference/utils/ulysses_runtime.py:148-170, and the trainers'
phase timers). Off by default; when on, every section records an event pair on the current
stream and `report()` synchronises once and sums milliseconds per section name."""
from collections import defaultdict
from contextlib import contextmanager

import torch


class SectionTimer:
    def __init__(self, enabled=False):
        self.enabled = enabled
        self._pending = []
        self.totals = defaultdict(float)
        self.counts = defaultdict(int)

    @contextmanager
    def section(self, name):
        if not self.enabled:
            yield
            return
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        try:
            yield
        finally:
            end.record()
            self._pending.append((name, start, end))

    def flush(self):
        if not self._pending:
            return
        torch.cuda.synchronize()
        for name, s, e in self._pending:
            self.totals[name] += s.elapsed_time(e)
            self.counts[name] += 1
        self._pending.clear()

    def report(self, reset=True):
        self.flush()
        out = {k: round(v, 3) for k, v in sorted(self.totals.items(), key=lambda kv: -kv[1])}
        if reset:
            self.totals.clear()
            self.counts.clear()
        return out
