"""Device time per named phase of a training step.

``with phase("allreduce"): ...`` records a CUDA event pair on the current stream around the
block when a :class:`PhaseTimer` is active (``PhaseTimer.activate()``), and does nothing
otherwise, so library code can be instrumented at no cost. Times are summed per name and read
after a synchronise (:meth:`PhaseTimer.collect`); nested phases each get their own time. Event
pairs are never recorded inside a CUDA-graph capture (the capture would own them).
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import Dict, List, Optional, Tuple

import torch

_active: Optional["PhaseTimer"] = None


class PhaseTimer:
    def __init__(self):
        self._pairs: Dict[str, List[Tuple[torch.cuda.Event, torch.cuda.Event]]] = {}

    @contextmanager
    def span(self, name: str):
        if torch.cuda.is_current_stream_capturing():
            yield
            return
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        try:
            yield
        finally:
            e.record()
            self._pairs.setdefault(name, []).append((s, e))

    def collect(self) -> Dict[str, float]:
        """Milliseconds per phase name, summed over every recorded span (synchronises)."""
        torch.cuda.synchronize()
        return {k: sum(s.elapsed_time(e) for s, e in v) for k, v in self._pairs.items()}

    def activate(self) -> "PhaseTimer":
        global _active
        _active = self
        return self

    def deactivate(self) -> None:
        global _active
        if _active is self:
            _active = None


@contextmanager
def phase(name: str):
    if _active is None:
        yield
    else:
        with _active.span(name):
            yield
