"""Host-side failure detection: store heartbeats, failure notes, diagnosed barriers.

The reference relies on the launcher noticing a dead worker process
(astrai/parallel/setup.py:198-205) and on PyTorch's default collective
timeouts. Here a rank that stops making progress is noticed by its peers on
the host, before they launch the next collective or peer-memory kernel (a
kernel that spins on a dead peer's flag would only give up at its own bounded
wait, and a collective would hang until the process-group timeout):

* :class:`Heartbeat` - every rank publishes a beat counter under
  ``{prefix}/beat/{rank}`` in the process group's key-value store from a
  daemon thread. :meth:`Heartbeat.check` raises :class:`PeerFailure` naming
  every peer whose counter has not moved for ``timeout`` seconds, or that
  recorded a failure with :meth:`Heartbeat.mark_failed` (a rank that catches an
  exception writes its reason before it exits, so peers fail fast with the
  cause instead of waiting out the timeout).
* :func:`diagnosed_barrier` - a barrier that names the ranks that did not
  arrive (``monitored_barrier`` on gloo; on NCCL a store-based arrival check
  with the same report).

Nothing here touches a GPU; the failure tests run as gloo ranks on CPU.
"""

from __future__ import annotations

import re
import threading
import time
from datetime import timedelta
from typing import Dict, List, Optional

import torch.distributed as dist


class PeerFailure(RuntimeError):
    """One or more peer ranks stopped or reported a failure."""

    def __init__(self, ranks: List[int], reasons: Dict[int, str]):
        self.ranks = sorted(ranks)
        self.reasons = reasons
        detail = ", ".join(f"rank {r}: {reasons.get(r, 'no heartbeat')}" for r in self.ranks)
        super().__init__(f"peer failure detected ({detail})")


def _default_store():
    if not (dist.is_available() and dist.is_initialized()):
        raise RuntimeError("Heartbeat needs an initialised process group or an explicit store")
    return dist.distributed_c10d._get_default_store()


class Heartbeat:
    def __init__(self, store=None, rank: Optional[int] = None, world_size: Optional[int] = None,
                 interval: float = 1.0, timeout: float = 10.0, prefix: str = "astrai/health"):
        self.store = store if store is not None else _default_store()
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world_size is None else world_size
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self._beat = 0
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        now = time.monotonic()
        # last value seen per peer and when it last changed (local clock: no cross-host clock sync needed)
        self._seen: Dict[int, tuple] = {r: (-1, now) for r in range(self.world) if r != self.rank}

    # ------------------------------------------------------------------ publishing
    def beat(self) -> None:
        self._beat += 1
        self.store.set(f"{self.prefix}/beat/{self.rank}", str(self._beat))

    def start(self) -> "Heartbeat":
        self.beat()
        if self._thread is None:
            self._stop.clear()
            self._thread = threading.Thread(target=self._loop, name=f"astrai-heartbeat-{self.rank}", daemon=True)
            self._thread.start()
        return self

    def _loop(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self.beat()
            except Exception:  # store gone (master exited): peers notice the missing beats
                return

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5.0)
        self._thread = None

    def mark_failed(self, reason: str) -> None:
        """Record this rank's failure so peers raise at their next :meth:`check`."""
        try:
            self.store.set(f"{self.prefix}/failed/{self.rank}", reason[:500])
        except Exception:
            pass

    # ------------------------------------------------------------------ checking
    def _get(self, key: str) -> Optional[str]:
        if not self.store.check([key]):
            return None
        return self.store.get(key).decode()

    def check(self) -> None:
        """Raise :class:`PeerFailure` if a peer reported a failure or its beat is older than ``timeout``."""
        now = time.monotonic()
        dead: List[int] = []
        reasons: Dict[int, str] = {}
        for r in list(self._seen):
            note = self._get(f"{self.prefix}/failed/{r}")
            if note is not None:
                dead.append(r)
                reasons[r] = f"reported failure: {note}"
                continue
            raw = self._get(f"{self.prefix}/beat/{r}")
            val = int(raw) if raw is not None else -1
            last, since = self._seen[r]
            if val != last:
                self._seen[r] = (val, now)
            elif now - since > self.timeout:
                dead.append(r)
                reasons[r] = f"no heartbeat for {now - since:.1f} s"
        if dead:
            raise PeerFailure(dead, reasons)

    def wait_all_alive(self, within: float) -> None:
        """Block until every peer has published at least one beat (or raise after ``within`` s)."""
        end = time.monotonic() + within
        missing = list(self._seen)
        while missing and time.monotonic() < end:
            missing = [r for r in missing if self._get(f"{self.prefix}/beat/{r}") is None]
            if missing:
                time.sleep(0.05)
        if missing:
            raise PeerFailure(missing, {r: "never started" for r in missing})


def diagnosed_barrier(timeout_s: float = 30.0, group=None, store=None, tag: str = "barrier") -> None:
    """Barrier that raises :class:`PeerFailure` naming the ranks that did not arrive within ``timeout_s``."""
    backend = dist.get_backend(group)
    if backend == "gloo":
        try:
            dist.monitored_barrier(group=group, timeout=timedelta(seconds=timeout_s), wait_all_ranks=True)
            return
        except RuntimeError as e:
            m = re.search(r"[Rr]anks?\s+([\d,\s]+?)\s+failed", str(e))
            ranks = [int(t) for t in re.findall(r"\d+", m.group(1))] if m else [-1]
            raise PeerFailure(ranks, {r: "did not reach the barrier" for r in ranks}) from e
    # NCCL: arrival keys in the store, then the device barrier once everyone is known to be there
    st = store if store is not None else _default_store()
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    gen = st.add(f"astrai/{tag}/gen/{rank}", 1)
    st.set(f"astrai/{tag}/{gen}/{rank}", "1")
    end = time.monotonic() + timeout_s
    missing = list(range(world))
    while time.monotonic() < end:
        missing = [r for r in missing if not st.check([f"astrai/{tag}/{gen}/{r}"])]
        if not missing:
            dist.barrier(group=group)
            return
        time.sleep(0.01)
    raise PeerFailure(missing, {r: "did not reach the barrier" for r in missing})
