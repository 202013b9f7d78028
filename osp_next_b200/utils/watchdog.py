"""Host-side failure detection (no GPU fault is ever used to test it).

* :class:`StepWatchdog` — a per-rank thread that fires ``on_timeout`` when the
  training / sampling loop stops calling :meth:`heartbeat` for ``timeout_s``
  (a hung collective or kernel); the default handler records the event and exits
  the process so the launcher / scheduler can restart from the newest checkpoint.
* :class:`RankHeartbeat` — ranks publish a heartbeat in the c10d store between
  steps; :meth:`dead_ranks` lists peers whose heartbeat is older than the
  timeout, so survivors learn of a lost rank *before* their next collective
  instead of blocking in it.
Device-side counterpart: every spin-wait in the sm_100a kernels is bounded and
reports a code through the error word (``ops.ext().get_error``).
"""
from __future__ import annotations

import json
import os
import threading
import time
from typing import Callable, List, Optional


class StepWatchdog:
    def __init__(self, timeout_s: float, on_timeout: Optional[Callable[[float], None]] = None,
                 report_path: Optional[str] = None, poll_s: float = 0.2):
        self.timeout_s = timeout_s
        self.on_timeout = on_timeout or self._default
        self.report_path = report_path
        self.poll_s = poll_s
        self._last = time.monotonic()
        self._stop = threading.Event()
        self.fired = False
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def heartbeat(self):
        self._last = time.monotonic()

    def stop(self):
        self._stop.set()
        self._t.join(timeout=2)

    def _run(self):
        while not self._stop.wait(self.poll_s):
            idle = time.monotonic() - self._last
            if idle > self.timeout_s and not self.fired:
                self.fired = True
                if self.report_path:
                    with open(self.report_path, "w") as f:
                        json.dump({"event": "step_timeout", "idle_s": idle, "pid": os.getpid(),
                                   "time": time.time()}, f)
                self.on_timeout(idle)

    @staticmethod
    def _default(idle):
        os._exit(3)


class RankHeartbeat:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "osp_hb"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix

    def beat(self, step: int):
        self.store.set(f"{self.prefix}/{self.rank}", json.dumps({"t": time.time(), "step": step}))

    def dead_ranks(self) -> List[int]:
        now, dead = time.time(), []
        for r in range(self.world):
            if r == self.rank:
                continue
            key = f"{self.prefix}/{r}"
            try:
                if not self.store.check([key]):
                    dead.append(r)
                    continue
                d = json.loads(self.store.get(key))
            except Exception:
                dead.append(r)
                continue
            if now - d["t"] > self.timeout_s:
                dead.append(r)
        return dead
