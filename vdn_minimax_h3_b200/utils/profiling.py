"""Per-section device timing with CUDA events (the reference's UlyssesRuntime.profile_start /
profile_end sections, src/inference/utils/ulysses_runtime.py:148-170, and the trainers'
phase timers). Off by default; when on, every section records an event pair on the current
stream (and an NVTX range, so a timeline profiler shows the same sections) and `report()`
synchronises once and sums milliseconds per section name.

`step_profiler(step)` is the training-side counterpart of the reference's H3_PROF_STEP
(src/training/train_stage_a2.py:83-120): with VDN_PROF_STEP=N (or H3_PROF_STEP=N) in the
environment, step N runs under torch.profiler and a kernel table is printed."""
import os
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
        torch.cuda.nvtx.range_push(name)
        start.record()
        try:
            yield
        finally:
            end.record()
            torch.cuda.nvtx.range_pop()
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


def profiled_step_index():
    """The 1-based training step to profile (VDN_PROF_STEP, or the reference's H3_PROF_STEP),
    or None."""
    v = os.environ.get("VDN_PROF_STEP") or os.environ.get("H3_PROF_STEP")
    return int(v) if v else None


@contextmanager
def step_profiler(step, row_limit=25, print_fn=print):
    """Profile this step when it is the one selected by the environment; prints the kernel
    table sorted by device (or CPU) time."""
    if profiled_step_index() != step:
        yield
        return
    from torch.profiler import ProfilerActivity, profile
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    with profile(activities=acts) as prof:
        yield
        if torch.cuda.is_available():
            torch.cuda.synchronize()
    key = "cuda_time_total" if torch.cuda.is_available() else "cpu_time_total"
    print_fn(f"profile of step {step}:\n" + prof.key_averages().table(sort_by=key, row_limit=row_limit))


def debug_memory_line(label, print_fn=print):
    """Print `label: alloc=.. peak=..GiB` (this process's CUDA allocator) when VDN_DEBUG_MEM
    or the reference's H3_DEBUG_MEM is set (reference train_stage_a1.py:92-94: one line per
    aligned block on rank 0). Returns the line, or None when the switch is off."""
    if not (os.environ.get("VDN_DEBUG_MEM") or os.environ.get("H3_DEBUG_MEM")):
        return None
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        alloc = torch.cuda.memory_allocated() / 2 ** 30
        peak = torch.cuda.max_memory_allocated() / 2 ** 30
    else:
        alloc = peak = 0.0
    line = f"    {label}: alloc={alloc:.1f} peak={peak:.1f}GiB"
    print_fn(line, flush=True)
    return line
