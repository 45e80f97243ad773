"""Request managers kept for API parity with the reference.

* :class:`BatchManager` - ``add_request`` / ``step`` / ``get_status`` as in
  ``pio/common/managers/batch_manager.py:9-84``, but each ``step`` advances the
  continuous batcher by one engine step instead of running one request to
  completion; a failed request is marked FAILED while the others continue.
* :class:`StreamingEngine` - asynchronous front-end: requests go to a
  priority queue; a worker thread drives the engine; ``generate_stream``
  yields tokens as they are produced
  (``pio/common/processing/streaming_computation.py:43-197``).
* :class:`AdaptiveAdmission` - admission control from free KV blocks and the
  measured step time (the role of ``AdaptiveBatchManager``,
  ``pio/common/processing/adaptive_batch_manager.py:42-251``).
"""
from __future__ import annotations

import heapq
import itertools
import queue
import threading
import time
from typing import Any, Dict, Iterator, List, Optional

from ..engine.sequence import SamplingParams, SeqStatus


class BatchManager:
    def __init__(self, plugin_or_engine):
        self.plugin = plugin_or_engine if hasattr(plugin_or_engine, "engine") else None
        self._engine = None if self.plugin else plugin_or_engine
        self.requests: Dict[Any, int] = {}

    @property
    def engine(self):
        return self.plugin.engine if self.plugin else self._engine

    def add_request(self, request_id, token_ids: List[int], params: Optional[SamplingParams] = None) -> None:
        self.requests[request_id] = self.engine.add_request([int(t) for t in token_ids], params)

    def step(self) -> List[Any]:
        """One engine step; returns the ids of requests that completed in it."""
        done = self.engine.step()
        inv = {v: k for k, v in self.requests.items()}
        return [inv[s.req_id] for s in done if s.req_id in inv]

    def get_status(self, request_id) -> str:
        seq = self.engine.seqs.get(self.requests.get(request_id))
        return "unknown" if seq is None else seq.status.value

    def get_output(self, request_id) -> List[int]:
        return list(self.engine.seqs[self.requests[request_id]].output)

    def run_all(self) -> Dict[Any, List[int]]:
        eng = self.engine
        if getattr(eng, "_ep_lockstep", False):
            eng._ep_all_done = False
        while eng.keep_stepping() if hasattr(eng, "keep_stepping") else eng.has_unfinished():
            self.step()
        return {rid: self.get_output(rid) for rid in self.requests}


class StreamingEngine:
    """Thread-safe streaming front-end over one engine."""

    def __init__(self, engine, max_queue: int = 1024):
        self.engine = engine
        self.max_queue = max_queue
        self._pq: List = []
        self._count = itertools.count()
        self._lock = threading.Lock()
        self._cv = threading.Condition(self._lock)
        self._streams: Dict[int, "queue.Queue"] = {}
        self._stop = False
        self._cancel: set = set()       # stream ids to abort before the next engine step
        self._eng_id: Dict[int, int] = {}
        self._thread = threading.Thread(target=self._loop, daemon=True)
        self._thread.start()
        self.stats = {"submitted": 0, "completed": 0, "rejected": 0}

    def submit_request(self, token_ids: List[int], params: Optional[SamplingParams] = None, priority: int = 0,
                       images=None) -> int:
        with self._lock:
            if len(self._pq) >= self.max_queue:
                self.stats["rejected"] += 1
                raise RuntimeError("queue full")
            rid = next(self._count)
            q: "queue.Queue" = queue.Queue()
            self._streams[rid] = q
            heapq.heappush(self._pq, (priority, rid, list(token_ids), params, images))
            self.stats["submitted"] += 1
            self._cv.notify()
        return rid

    def cancel(self, rid: int) -> None:
        """Abort a submitted request; its stream ends (None) once the engine thread applies it."""
        with self._lock:
            self._cancel.add(rid)
            self._cv.notify()

    def generate_stream(self, rid: int, timeout: float = 300.0) -> Iterator[int]:
        q = self._streams[rid]
        while True:
            item = q.get(timeout=timeout)
            if item is None:
                return
            if isinstance(item, Exception):
                raise item
            yield item

    def _loop(self):
        # expert parallelism: the engine steps in lock-step with the other ranks, so this loop keeps
        # stepping while idle (a short sleep when no rank has work) and stops when every rank has
        # asked to (``LLMEngine.request_stop``)
        lockstep = getattr(self.engine, "_ep_lockstep", False)
        while True:
            with self._lock:
                while (not lockstep and not self._stop and not self._pq and not self._cancel
                       and not self.engine.has_unfinished()):
                    self._cv.wait(timeout=0.1)
                if self._cancel:
                    for rid in self._cancel:
                        q = self._streams.get(rid)
                        queued = [e for e in self._pq if e[1] == rid]
                        if queued:       # not handed to the engine yet
                            self._pq = [e for e in self._pq if e[1] != rid]
                            heapq.heapify(self._pq)
                        elif rid in self._eng_id:
                            eid = self._eng_id.pop(rid)
                            self.engine.abort(eid)
                            self.engine.seqs.pop(eid, None)
                        if q is not None:
                            q.put(None)
                        self.stats["cancelled"] = self.stats.get("cancelled", 0) + 1
                    self._cancel.clear()
                # pending cancellations are applied even at shutdown, so their blocks are freed
                if self._stop:
                    if not lockstep:
                        return
                    self.engine.request_stop()
                while self._pq:
                    _, rid, ids, params, images = heapq.heappop(self._pq)
                    q = self._streams[rid]

                    def cb(seq, tok, q=q):
                        q.put(tok)

                    eng_id = self.engine.add_request(ids, params, images=images, callback=cb)
                    self.engine.seqs[eng_id].stream_id = rid
                    self._eng_id[rid] = eng_id
            done = self.engine.step()
            for s in done:
                self._eng_id.pop(getattr(s, "stream_id", -1), None)
                self.engine.seqs.pop(s.req_id, None)  # a long-running server keeps no finished sequences
                q = self._streams.get(getattr(s, "stream_id", -1))
                if q is not None:
                    q.put(RuntimeError(s.error) if s.status == SeqStatus.FAILED else None)
                    self.stats["completed"] += 1
            if lockstep:
                if self.engine.ep_stopped:
                    return
                if self.engine._ep_all_done:
                    time.sleep(0.001)

    def shutdown(self, timeout: float = 10.0):
        """Stops the engine thread.  Under expert parallelism the thread ends once every rank
        has shut down, so this waits up to ``timeout`` seconds for the peers."""
        with self._lock:
            self._stop = True
            self._cv.notify()
        self._thread.join(timeout=timeout)


class ReplicaRouter:
    """Data-parallel serving: requests spread over several engine replicas.

    Each replica (an engine on its own device, or a CPU engine) gets its own
    streaming thread, scheduler and KV cache; a new request goes to the
    replica with the fewest queued + running sequences.  The interface is the
    :class:`StreamingEngine` one, so :class:`AsyncEngine` and the HTTP server
    can sit on top of a router unchanged.
    """

    def __init__(self, engines, max_queue: int = 1024):
        if not engines:
            raise ValueError("ReplicaRouter needs at least one engine")
        self.replicas = [e if isinstance(e, StreamingEngine) else StreamingEngine(e, max_queue) for e in engines]
        self._count = itertools.count()
        self._lock = threading.Lock()
        self._route: Dict[int, tuple] = {}       # router id -> (replica index, replica id)
        self._streams = _RoutedStreams(self)

    def _load(self, r: "StreamingEngine") -> int:
        with r._lock:
            return len(r._pq) + len(r.engine.scheduler.running) + len(r.engine.scheduler.waiting)

    def submit_request(self, token_ids: List[int], params: Optional[SamplingParams] = None, priority: int = 0,
                       images=None) -> int:
        with self._lock:
            i = min(range(len(self.replicas)), key=lambda j: (self._load(self.replicas[j]), j))
            rid = next(self._count)
            self._route[rid] = (i, self.replicas[i].submit_request(token_ids, params, priority, images=images))
        return rid

    def replica_of(self, rid: int) -> int:
        return self._route[rid][0]

    def generate_stream(self, rid: int, timeout: float = 300.0) -> Iterator[int]:
        i, sub = self._route[rid]
        return self.replicas[i].generate_stream(sub, timeout)

    def cancel(self, rid: int) -> None:
        i, sub = self._route[rid]
        self.replicas[i].cancel(sub)

    @property
    def stats(self) -> Dict[str, int]:
        out: Dict[str, int] = {}
        for r in self.replicas:
            for k, v in r.stats.items():
                out[k] = out.get(k, 0) + v
        return out

    def shutdown(self) -> None:
        for r in self.replicas:
            r.shutdown()


class _RoutedStreams:
    """``router._streams[rid]`` / ``.pop(rid)``: the per-request token queue, as on a StreamingEngine."""

    def __init__(self, router: ReplicaRouter):
        self.router = router

    def __getitem__(self, rid: int):
        i, sub = self.router._route[rid]
        return self.router.replicas[i]._streams[sub]

    def pop(self, rid: int, default=None):
        route = self.router._route.pop(rid, None)
        if route is None:
            return default
        i, sub = route
        return self.router.replicas[i]._streams.pop(sub, default)


class AsyncEngine:
    """asyncio front-end over a :class:`StreamingEngine` (text or image + text requests).

    The reference's async multimodal manager only echoes its request
    (``src/inference_pio/models/qwen3_vl_2b/async_multimodal_processing.py:10-32``).
    Here ``await generate(...)`` returns the generated ids and ``stream(...)``
    yields them as the engine thread produces them; the engine keeps batching
    every pending request together.  ``process_request`` accepts the
    reference's request shape: a dict with ``input_ids`` and optional
    ``pixel_values`` / ``max_new_tokens``.
    """

    def __init__(self, engine, max_queue: int = 1024):
        # a streaming front-end (StreamingEngine, ReplicaRouter, DistributedFrontEnd) is used as is
        self.streaming = engine if hasattr(engine, "submit_request") else StreamingEngine(engine, max_queue)

    async def stream(self, token_ids: List[int], params: Optional[SamplingParams] = None, priority: int = 0,
                     images=None):
        import asyncio

        rid = self.streaming.submit_request(token_ids, params, priority, images=images)
        q = self.streaming._streams[rid]
        loop = asyncio.get_running_loop()
        finished = False
        try:
            while True:
                item = await loop.run_in_executor(None, q.get)
                if item is None:
                    finished = True
                    return
                if isinstance(item, Exception):
                    finished = True
                    raise item
                yield item
        finally:
            if not finished:  # the consumer stopped early (e.g. the HTTP client went away): free the request
                self.streaming.cancel(rid)
            self.streaming._streams.pop(rid, None)

    async def generate(self, token_ids: List[int], params: Optional[SamplingParams] = None, priority: int = 0,
                       images=None) -> List[int]:
        return [t async for t in self.stream(token_ids, params, priority, images)]

    async def process_request(self, request) -> List[int]:
        p = SamplingParams(max_new_tokens=int(request.get("max_new_tokens", 64)))
        return await self.generate(list(request["input_ids"]), p, images=request.get("pixel_values"))

    def shutdown(self) -> None:
        self.streaming.shutdown()


class AdaptiveAdmission:
    """Chooses how many new requests to admit per step: stays within free KV
    blocks (with headroom for decode growth) and backs off when the measured
    step time exceeds a latency target."""

    def __init__(self, target_step_s: float = 0.05, headroom_blocks: int = 64):
        self.target = target_step_s
        self.headroom = headroom_blocks
        self.ewma = None

    def observe(self, step_seconds: float) -> None:
        self.ewma = step_seconds if self.ewma is None else 0.8 * self.ewma + 0.2 * step_seconds

    def max_admit(self, free_blocks: int, blocks_per_request: int, running: int, max_batch: int) -> int:
        room = max(0, free_blocks - self.headroom) // max(1, blocks_per_request)
        n = min(room, max_batch - running)
        if self.ewma is not None and self.ewma > self.target:
            n = min(n, max(1, n // 2))
        return max(0, n)
