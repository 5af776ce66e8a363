"""Launch accounting for the C-ABI calls: a per-entry-point launch counter
(always on) and, inside a ``KernelTimer`` context, CUDA-event timing of each
launch on the current stream together with its algorithmic work (FLOPs or
bytes) as stated by the caller. Used by the benchmark to report achieved
TFLOP/s or GB/s of a kernel over exactly the timed region."""
from collections import defaultdict

import torch

launches = defaultdict(int)
_timer = None


class KernelTimer:
    def __init__(self, names=None):
        self.names = set(names) if names else None
        self.records = defaultdict(list)  # name -> [(start, end, work)]
        self._pool = []

    def reserve(self, n):
        """Create ``n`` events ahead of the timed region (each recorded once, which makes CUDA
        allocate it), so that timing a launch costs two event records and no event creation."""
        for _ in range(n):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._pool.append(ev)
        torch.cuda.synchronize()
        return self

    def event(self):
        return self._pool.pop() if self._pool else torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        global _timer
        _timer = self
        return self

    def __exit__(self, *exc):
        global _timer
        _timer = None
        return False

    def wants(self, name):
        return self.names is None or name in self.names

    def total(self, prefix):
        """Summed {launches, ms_total, work_total} over groups whose key starts with ``prefix``."""
        out = {"launches": 0, "ms_total": 0.0, "work_total": 0}
        for key, v in self.summary().items():
            if key.startswith(prefix):
                for f in out:
                    out[f] += v[f]
        return out

    def summary(self):
        """name -> {launches, ms_total, ms_per_launch, work_total} (synchronises)."""
        torch.cuda.synchronize()
        out = {}
        for name, recs in self.records.items():
            ms = sum(s.elapsed_time(e) for s, e, _ in recs)
            out[name] = {"launches": len(recs), "ms_total": ms, "ms_per_launch": ms / max(len(recs), 1),
                         "work_total": sum(w for _, _, w in recs)}
        return out


def active():
    return _timer


def total_launches():
    return sum(launches.values())
