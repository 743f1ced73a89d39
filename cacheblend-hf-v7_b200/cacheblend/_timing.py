"""Per-kernel CUDA-event timing and launch counting for the libcbk wrappers.

Off by default.  When active, every wrapper call records a pair of CUDA events
on the stream it launches on, so durations are device time of that stream;
``summary()`` synchronises and returns {kernel: (launches, total_ms)}.

Inside a CUDA-graph capture the events are external event-record nodes of the
graph (``torch.cuda.Event(external=True)``): every replay records them again,
so ``read_graph_spans()`` after a replay gives each kernel's device time as it
ran inside the graph, with no host launch gaps in between.
"""
from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager

import torch


class KernelTimes:
    def __init__(self):
        self.active = False
        self.spans = defaultdict(list)
        self.launches = defaultdict(int)
        self.graph_spans = []          # (name, start event, end event, launches) recorded in a capture

    def reset(self):
        self.spans.clear()
        self.launches.clear()
        self.graph_spans = []

    @contextmanager
    def span(self, name: str, device, n_launches: int = 1):
        if not self.active:
            yield
            return
        stream = torch.cuda.current_stream(device)
        captured = torch.cuda.is_current_stream_capturing()
        a = torch.cuda.Event(enable_timing=True, external=captured)
        b = torch.cuda.Event(enable_timing=True, external=captured)
        a.record(stream)
        yield
        b.record(stream)
        if captured:
            self.graph_spans.append((name, a, b, n_launches))
        else:
            self.spans[name].append((a, b))
            self.launches[name] += n_launches

    def summary(self):
        torch.cuda.synchronize()
        return {n: (len(ev), sum(a.elapsed_time(b) for a, b in ev)) for n, ev in self.spans.items()}

    def read_graph_spans(self, spans, acc=None):
        """Add the last replay's durations of captured spans into acc
        ({name: [calls, total_ms, launches]}); the caller synchronises first."""
        acc = {} if acc is None else acc
        for name, a, b, n in spans:
            e = acc.setdefault(name, [0, 0.0, 0])
            e[0] += 1
            e[1] += a.elapsed_time(b)
            e[2] += n
        return acc


TIMES = KernelTimes()
