"""Per-kernel CUDA-event timing and launch counting for the libcbk wrappers.

Off by default.  When active, every wrapper call records a pair of CUDA events
on the stream it launches on, so durations are device time of that stream;
``summary()`` synchronises and returns {kernel: (launches, total_ms)}."""
from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager

import torch


class KernelTimes:
    def __init__(self):
        self.active = False
        self.spans = defaultdict(list)
        self.launches = defaultdict(int)

    def reset(self):
        self.spans.clear()
        self.launches.clear()

    @contextmanager
    def span(self, name: str, device, n_launches: int = 1):
        if not self.active:
            yield
            return
        stream = torch.cuda.current_stream(device)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        yield
        b.record(stream)
        self.spans[name].append((a, b))
        self.launches[name] += n_launches

    def summary(self):
        torch.cuda.synchronize()
        return {n: (len(ev), sum(a.elapsed_time(b) for a, b in ev)) for n, ev in self.spans.items()}


TIMES = KernelTimes()
