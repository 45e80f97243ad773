"""One request front-end over an engine that spans several processes (one per GPU).

Rank 0 owns the public interface (``submit_request`` / ``generate_stream`` /
``cancel`` / ``shutdown``, the :class:`mod_b200.api.managers.StreamingEngine`
shape, so :class:`~mod_b200.api.managers.AsyncEngine` and the HTTP server sit
on top unchanged).  Every rank runs the same loop; one iteration is

1. rank 0 broadcasts what arrived since the last iteration: new requests,
   cancellations, and whether to stop;
2. every rank applies it to its engine and runs one ``step``;
3. (expert or data parallelism) every rank sends the tokens its sequences
   produced to rank 0, which feeds the request streams.

Tensor parallelism (``mode="tp"``): every rank adds every request in the same
order, so the ranks' schedulers take the same decisions and each step's
collectives line up; rank 0's own engine produces the tokens.  Expert
parallelism with data-parallel attention (``mode="ep"``): rank 0 gives each
request to the rank with the fewest unfinished requests; the engines step in
lock-step (``LLMEngine._ep_step``).  ``mode="dp"``: independent replicas, one
per rank, placed and gathered the same way.  ``mode="single"``: one process.

The reference has no multi-process serving; its streaming engine is a thread
pool over one model (``pio/common/processing/streaming_computation.py:43-181``).
"""
from __future__ import annotations

import itertools
import queue
import threading
import time
from typing import Dict, List, Optional

import torch.distributed as dist

from ..engine.sequence import SamplingParams, SeqStatus


class DistributedFrontEnd:
    def __init__(self, engine, mode: str = "tp", group=None, idle_sleep: float = 0.001):
        if mode not in ("tp", "ep", "dp", "single"):
            raise ValueError(f"unknown mode {mode!r} (tp, ep, dp, single)")
        self.engine, self.mode, self.group = engine, mode, group
        multi = dist.is_available() and dist.is_initialized() and mode != "single"
        self.rank = dist.get_rank(group) if multi else 0
        self.world = dist.get_world_size(group) if multi else 1
        self.placed = mode in ("ep", "dp") and self.world > 1   # requests go to one rank each
        self.idle_sleep = idle_sleep
        self._lock = threading.Lock()
        self._count = itertools.count()
        self._new: List[tuple] = []          # (rid, token ids, params) not yet broadcast
        self._cancel: List[int] = []
        self._stop = False
        self._streams: Dict[int, "queue.Queue"] = {}
        self._owner: Dict[int, int] = {}     # rid -> rank serving it (rank 0's view, unfinished only)
        self._load = [0] * self.world        # unfinished requests per rank (rank 0's view)
        self._eng_id: Dict[int, int] = {}    # rid -> engine request id on this rank
        self._produced: List[tuple] = []     # (rid, token or None at the end, error) since the last delivery
        self.stats = {"submitted": 0, "completed": 0}
        self._thread: Optional[threading.Thread] = None
        if self.rank == 0:
            self._thread = threading.Thread(target=self.run, daemon=True)
            self._thread.start()

    # ------------------------------------------------------------------ rank 0 API
    def submit_request(self, token_ids: List[int], params: Optional[SamplingParams] = None, priority: int = 0,
                       images=None) -> int:
        if self.rank != 0:
            raise RuntimeError("requests enter through rank 0")
        if images is not None:
            raise ValueError("the multi-process front-end takes token requests")
        with self._lock:
            if self._stop:
                raise RuntimeError("front-end is shut down")
            rid = next(self._count)
            self._streams[rid] = queue.Queue()
            self._new.append((rid, [int(t) for t in token_ids], params))
            self.stats["submitted"] += 1
        return rid

    def cancel(self, rid: int) -> None:
        with self._lock:
            self._cancel.append(rid)

    def generate_stream(self, rid: int, timeout: float = 300.0):
        q = self._streams[rid]
        while True:
            item = q.get(timeout=timeout)
            if item is None:
                return
            if isinstance(item, Exception):
                raise item
            yield item

    def shutdown(self, timeout: float = 60.0) -> None:
        """Rank 0: every rank's loop ends after the next iteration (unfinished requests end
        with an error)."""
        with self._lock:
            self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=timeout)

    # ------------------------------------------------------------------ every rank
    def run(self) -> None:
        """The loop; rank 0 runs it in a thread, the other ranks call it and it returns
        when rank 0 shuts down."""
        while True:
            msg = self._exchange_commands()
            self._apply(msg)
            if msg["stop"]:
                self._finish_all("front-end shut down")
                return
            done = self.engine.step() if self._needs_step() else []
            for s in done:
                rid = getattr(s, "front_rid", None)
                if rid is not None:
                    err = s.error if s.status == SeqStatus.FAILED else None
                    self._produced.append((rid, None, err))
                    self._eng_id.pop(rid, None)
                    self.engine.seqs.pop(s.req_id, None)
            self._deliver()
            if not done and self._idle():
                time.sleep(self.idle_sleep)

    def _needs_step(self) -> bool:
        if getattr(self.engine, "_ep_lockstep", False):
            return True        # lock-step: the engine itself agrees with its peers on idle steps
        return self.engine.has_unfinished()

    def _idle(self) -> bool:
        if getattr(self.engine, "_ep_lockstep", False):
            return bool(getattr(self.engine, "_ep_all_done", False))
        return not self.engine.has_unfinished()

    def _exchange_commands(self) -> dict:
        msg = None
        if self.rank == 0:
            with self._lock:
                adds, self._new = self._new, []
                cancels, self._cancel = self._cancel, []
                stop = self._stop
            placed = []
            for rid, ids, params in adds:
                owner = 0
                if self.placed:
                    owner = min(range(self.world), key=lambda r: (self._load[r], r))
                    self._load[owner] += 1
                self._owner[rid] = owner
                placed.append((rid, ids, params, owner))
            msg = {"add": placed, "cancel": cancels, "stop": stop}
        if self.world > 1:
            box = [msg]
            dist.broadcast_object_list(box, src=0, group=self.group)
            msg = box[0]
        return msg

    def _apply(self, msg: dict) -> None:
        for rid, ids, params, owner in msg["add"]:
            if self.placed and owner != self.rank:
                continue

            def cb(seq, tok, rid=rid):
                self._produced.append((rid, int(tok), None))

            eid = self.engine.add_request(ids, params, callback=cb)
            self.engine.seqs[eid].front_rid = rid
            self._eng_id[rid] = eid
        for rid in msg["cancel"]:
            eid = self._eng_id.pop(rid, None)
            if eid is not None:     # the rank serving it ends the stream
                self.engine.abort(eid)
                self.engine.seqs.pop(eid, None)
                self._produced.append((rid, None, None))

    def _deliver(self) -> None:
        """Tokens to rank 0's streams (placed requests: gathered from every rank)."""
        produced, self._produced = self._produced, []
        if self.placed:
            lists = [None] * self.world if self.rank == 0 else None
            dist.gather_object(produced, lists, dst=0, group=self.group)
            if self.rank != 0:
                return
            produced = [item for part in lists for item in part]
        elif self.rank != 0:
            return
        for rid, tok, err in produced:
            q = self._streams.get(rid)
            if q is None or rid not in self._owner:
                continue        # unknown, or already ended
            if tok is not None:
                q.put(tok)
                continue
            q.put(RuntimeError(err) if err else None)
            owner = self._owner.pop(rid)
            if self.placed:
                self._load[owner] = max(0, self._load[owner] - 1)
            self.stats["completed"] += 1

    def _finish_all(self, why: str) -> None:
        for eid in list(self._eng_id.values()):
            self.engine.abort(eid)
            self.engine.seqs.pop(eid, None)
        self._eng_id.clear()
        if self.rank == 0:
            for rid in list(self._owner):
                self._streams[rid].put(RuntimeError(why))
            self._owner.clear()
