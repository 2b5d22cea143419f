"""Host-side failure detection and fault injection.

The reference relies on a 24 h NCCL timeout and on skipping a step when the filter raises
(train.py:49, 261-269).  Here failures are detected on the host, between steps, before the next
collective is launched -- nothing waits on a dead peer inside a kernel:

* :class:`Heartbeat` -- every rank refreshes ``hb/<rank>`` (monotonic wall time) in the
  c10d store from a background thread; :meth:`Heartbeat.dead_peers` lists ranks whose beat is
  older than ``timeout``.
* :func:`report_failure` / :func:`failed_peers` -- a rank that hits an exception publishes
  ``fail/<rank>`` before it leaves, so the others learn of it immediately.
* :class:`Watchdog` -- combines both; ``check()`` raises :class:`PeerFailure` between steps.
* :class:`FaultInjector` -- host-only fault injection for tests and drills, configured by
  ``CFB_FAULT="rank=R,step=K,kind=raise|exit|stall"``: raise an exception, exit without notice,
  or stop heart-beating (a stalled host) at the start of step K on rank R.  No GPU fault, trap or
  hang is ever injected.
* Device-side waits (peer flags, mbarriers) are bounded in the kernels themselves and report
  through error words (see csrc/kernels/comm_sm100.cu and sm100_common.cuh).
"""
from __future__ import annotations

import os
import threading
import time
from typing import List, Optional


class PeerFailure(RuntimeError):
    def __init__(self, ranks: List[int], reason: str):
        super().__init__(f"peer rank(s) {ranks} failed: {reason}")
        self.ranks = ranks
        self.reason = reason


def _now() -> float:
    return time.time()


class Heartbeat:
    def __init__(self, store, rank: int, world: int, interval: float = 0.5,
                 timeout: float = 10.0, prefix: str = "cfb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self._stop = threading.Event()
        self._paused = threading.Event()
        self._th: Optional[threading.Thread] = None
        self.beat()

    def key(self, r: int) -> str:
        return f"{self.prefix}/hb/{r}"

    def beat(self) -> None:
        self.store.set(self.key(self.rank), repr(_now()))

    def _loop(self) -> None:
        while not self._stop.wait(self.interval):
            if not self._paused.is_set():
                try:
                    self.beat()
                except Exception:
                    return

    def start(self) -> "Heartbeat":
        self._th = threading.Thread(target=self._loop, daemon=True)
        self._th.start()
        return self

    def pause(self) -> None:
        """Stop beating (used by the fault injector to emulate a stalled host)."""
        self._paused.set()

    def stop(self) -> None:
        self._stop.set()
        if self._th:
            self._th.join(timeout=5)

    def dead_peers(self) -> List[int]:
        now = _now()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                t = float(self.store.get(self.key(r)).decode())
            except Exception:
                dead.append(r)
                continue
            if now - t > self.timeout:
                dead.append(r)
        return dead


def report_failure(store, rank: int, reason: str, prefix: str = "cfb") -> None:
    try:
        store.set(f"{prefix}/fail/{rank}", reason[:1000])
    except Exception:
        pass


def failed_peers(store, world: int, rank: int, prefix: str = "cfb"):
    out = []
    keys = [f"{prefix}/fail/{r}" for r in range(world) if r != rank]
    try:
        present = store.check(keys)
    except Exception:
        present = False
    if not present:
        # check() is all-or-nothing; probe individually
        for r in range(world):
            if r == rank:
                continue
            try:
                if store.check([f"{prefix}/fail/{r}"]):
                    out.append((r, store.get(f"{prefix}/fail/{r}").decode()))
            except Exception:
                pass
        return out
    return [(r, store.get(f"{prefix}/fail/{r}").decode()) for r in range(world) if r != rank]


class Watchdog:
    def __init__(self, store, rank: int, world: int, interval: float = 0.5, timeout: float = 10.0):
        self.store, self.rank, self.world = store, rank, world
        self.hb = Heartbeat(store, rank, world, interval, timeout).start()

    def check(self) -> None:
        """Raise :class:`PeerFailure` if a peer reported a failure or stopped beating."""
        failed = failed_peers(self.store, self.world, self.rank)
        if failed:
            raise PeerFailure([r for r, _ in failed], "; ".join(m for _, m in failed))
        dead = self.hb.dead_peers()
        if dead:
            raise PeerFailure(dead, f"no heartbeat for more than {self.hb.timeout:.1f}s")

    def report(self, exc: BaseException) -> None:
        report_failure(self.store, self.rank, f"{type(exc).__name__}: {exc}")

    def close(self) -> None:
        self.hb.stop()


class FaultInjector:
    """Host-only fault injection configured from ``CFB_FAULT`` (see module docstring)."""

    def __init__(self, spec: Optional[str] = None, rank: int = 0, heartbeat: Optional[Heartbeat] = None):
        spec = spec if spec is not None else os.environ.get("CFB_FAULT", "")
        self.rank, self.hb = rank, heartbeat
        self.cfg = {}
        for part in filter(None, spec.split(",")):
            k, v = part.split("=")
            self.cfg[k.strip()] = v.strip()

    def at_step(self, step: int) -> None:
        if not self.cfg:
            return
        if int(self.cfg.get("rank", -1)) != self.rank or int(self.cfg.get("step", -1)) != step:
            return
        kind = self.cfg.get("kind", "raise")
        if kind == "raise":
            raise RuntimeError(f"injected fault on rank {self.rank} at step {step}")
        if kind == "exit":
            os._exit(17)
        if kind == "stall":
            if self.hb is not None:
                self.hb.pause()
            time.sleep(float(self.cfg.get("seconds", "30")))
