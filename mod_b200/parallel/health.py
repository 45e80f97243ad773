"""Rank liveness: host-side heartbeats and failure notices over the c10d store.

The reference has no failure detection beyond ``exit()`` on a CUDA error
(``src/inference_pio/plugins/cuda/c_src/tensor_ops_cuda.cu:10-18``) and
``try/except`` around generation (``src/inference_pio/models/qwen3_0_6b/plugin.py:150-152``).

Serving with collectives in every step needs more: when one rank dies, the
others must find out on the host *before* they launch the next step's fused
exchange kernels (whose device waits would otherwise run out one by one) or
the next NCCL collective.  Each rank runs a daemon thread that writes a beat
(wall-clock seconds) under ``hb/<rank>`` every ``interval`` seconds.
``check()`` -- called between steps -- raises ``RankFailure`` when a peer
posted a failure notice, announced that it left, or has not beaten for
``timeout`` seconds.  A rank leaves only between steps (none of its kernels or
collectives in flight); ``leave()`` and ``mark_failed()`` post the notice.

The store is the process group's own TCPStore by default, hosted by rank 0;
losing rank 0 therefore shows up as a store error, which ``check()`` also
reports as a ``RankFailure``.
"""
from __future__ import annotations

import threading
import time
from typing import Dict, List, Optional

_PREFIX = "mb_hb/"


class RankFailure(RuntimeError):
    def __init__(self, ranks: List[int], reasons: Dict[int, str]):
        self.ranks = sorted(ranks)
        self.reasons = reasons
        super().__init__("rank(s) %s unavailable: %s" % (self.ranks, "; ".join(
            f"{r}: {reasons[r]}" for r in self.ranks)))


def default_store():
    import torch.distributed as dist

    return dist.distributed_c10d._get_default_store()


class Heartbeat:
    def __init__(self, rank: int, world: int, store=None, interval: float = 0.2, timeout: float = 2.0,
                 namespace: str = ""):
        if timeout <= 2 * interval:
            raise ValueError("heartbeat timeout must exceed two beat intervals")
        self.rank, self.world = rank, world
        self.store = store if store is not None else default_store()
        self.interval, self.timeout = interval, timeout
        self.ns = _PREFIX + (namespace + "/" if namespace else "")
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._first_seen: Dict[int, float] = {}

    # ------------------------------------------------------------------ keys
    def _beat_key(self, r: int) -> str:
        return f"{self.ns}beat/{r}"

    def _note_key(self, r: int) -> str:
        return f"{self.ns}note/{r}"

    # ------------------------------------------------------------------ life cycle
    def start(self) -> "Heartbeat":
        self._beat()
        self._thread = threading.Thread(target=self._run, name=f"mb-heartbeat-{self.rank}", daemon=True)
        self._thread.start()
        return self

    def _beat(self) -> None:
        self.store.set(self._beat_key(self.rank), repr(time.time()))

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:  # store gone (rank 0 exited): the next check() reports it
                return

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.interval + 1.0)
            self._thread = None

    def leave(self) -> None:
        """Announce an orderly exit between steps, then stop beating."""
        self._post("left")
        self.stop()

    def mark_failed(self, reason: str) -> None:
        """Announce that this rank hit an error and will not take part in further steps."""
        self._post("failed: " + reason.replace("\n", " ")[:200])
        self.stop()

    def _post(self, note: str) -> None:
        try:
            self.store.set(self._note_key(self.rank), note)
        except Exception:
            pass

    # ------------------------------------------------------------------ detection
    def dead_peers(self) -> Dict[int, str]:
        now = time.time()
        bad: Dict[int, str] = {}
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                if self.store.check([self._note_key(r)]):
                    bad[r] = self.store.get(self._note_key(r)).decode()
                    continue
                if not self.store.check([self._beat_key(r)]):
                    # never beaten yet: allow it ``timeout`` from when we first looked
                    t0 = self._first_seen.setdefault(r, now)
                    if now - t0 > self.timeout:
                        bad[r] = "no heartbeat since start"
                    continue
                last = float(self.store.get(self._beat_key(r)).decode())
                if now - last > self.timeout:
                    bad[r] = f"last heartbeat {now - last:.2f} s ago"
            except Exception as e:  # store unreachable: its host (rank 0) is gone
                bad[0 if self.rank != 0 else r] = f"store unreachable ({type(e).__name__})"
                break
        return bad

    def check(self) -> None:
        bad = self.dead_peers()
        if bad:
            raise RankFailure(list(bad), bad)

    def __enter__(self) -> "Heartbeat":
        return self.start()

    def __exit__(self, *exc) -> None:
        self.stop()
