"""HTTP serving front-end (``python -m mod_b200 serve MODEL``).

The reference has no server; its CLI runs one prompt per process
(``src/inference_pio/__main__.py:266-343``).  This module exposes one engine
over HTTP with an OpenAI-style completions route, so concurrent clients share
the continuous batcher:

* ``POST /v1/completions`` -- ``{"prompt": str | [ids], "max_tokens": int,
  "temperature": float, "top_p": float, "top_k": int, "seed": int,
  "stream": bool}``; the reply carries the text (when a tokenizer is loaded),
  the token ids and usage counts; ``stream`` returns server-sent events, one
  per token;
* ``POST /v1/chat/completions`` -- ``{"messages": [{"role", "content"}...],
  "max_tokens", ..., "enable_thinking": bool}``: the messages go through the
  ChatML template (thinking mode on or off) and the reply is one assistant
  message with ``<think>`` blocks removed from ``content``;
* ``GET /health`` -- engine state (running / waiting sequences, free KV
  blocks);
* ``GET /v1/models`` -- the served model;
* ``GET /metrics`` -- Prometheus text format: request and token counters,
  request latency histogram, running / waiting sequences and free KV blocks.

Requests go through :class:`~mod_b200.api.managers.AsyncEngine`, whose engine
thread batches every pending request together.
"""
import contextlib
import json
import time
from typing import List, Optional, Union

from pydantic import BaseModel

from ..engine.sequence import SamplingParams
from .managers import AsyncEngine


class CompletionRequest(BaseModel):
    prompt: Union[str, List[int]]
    max_tokens: int = 64
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    seed: Optional[int] = None
    stop_token_ids: List[int] = []
    stream: bool = False
    n: int = 1                      # independent samples of one prompt (seed + i for sample i)
    stop: List[str] = []            # text stop strings (need a tokenizer); the reply ends before the first


class ChatRequest(BaseModel):
    messages: List[dict]
    max_tokens: int = 256
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    seed: Optional[int] = None
    stop_token_ids: List[int] = []
    enable_thinking: bool = False


def create_app(engine, tokenizer=None, model_name: str = "model"):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import StreamingResponse

    front = AsyncEngine(engine)

    @contextlib.asynccontextmanager
    async def lifespan(app):
        yield
        front.shutdown()

    app = FastAPI(title="mod_b200", version="0.1.0", lifespan=lifespan)
    app.state.front = front
    m = _Metrics(getattr(engine, "engine", engine))  # a front-end's engine

    def _ids(req: CompletionRequest) -> List[int]:
        if isinstance(req.prompt, list):
            return [int(t) for t in req.prompt]
        if tokenizer is None:
            raise HTTPException(400, "no tokenizer loaded: send the prompt as token ids")
        return tokenizer.encode(req.prompt)

    def _params(req: CompletionRequest) -> SamplingParams:
        if req.max_tokens < 1:
            raise HTTPException(400, "max_tokens must be >= 1")
        kw = dict(max_new_tokens=req.max_tokens, temperature=req.temperature, top_p=req.top_p, top_k=req.top_k)
        if req.seed is not None:
            kw["seed"] = req.seed
        if req.stop_token_ids:
            kw["stop_token_ids"] = tuple(int(t) for t in req.stop_token_ids)
        return SamplingParams(**kw)

    def _text(ids: List[int]) -> Optional[str]:
        return tokenizer.decode(ids) if tokenizer is not None else None

    async def _generate_stop(ids: List[int], params: SamplingParams, stop: List[str]):
        """Generate until a stop string appears in the decoded text; the request is cancelled
        there (the stream is closed at once, which frees its KV blocks), the text is cut before
        the stop string and the token ids are trimmed to the tokens whose text ends before it."""
        import contextlib

        out: List[int] = []
        async with contextlib.aclosing(front.stream(ids, params)) as gen:
            async for tok in gen:
                out.append(tok)
                text = tokenizer.decode(out)
                cut = min((text.find(x) for x in stop if x and x in text), default=-1)
                if cut >= 0:
                    keep = len(out)
                    while keep > 0 and len(tokenizer.decode(out[:keep])) > cut:
                        keep -= 1
                    return out[:keep], text[:cut], "stop"
        return out, tokenizer.decode(out), ("length" if len(out) >= params.max_new_tokens else "stop")

    @app.get("/health")
    def health():
        return {"status": "ok", "running": len(engine.scheduler.running), "waiting": len(engine.scheduler.waiting),
                "free_kv_blocks": engine.blocks.num_free}

    @app.get("/metrics")
    def metrics():
        from fastapi.responses import Response

        body, ctype = m.render()
        return Response(content=body, media_type=ctype)

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model"}]}

    @app.post("/v1/completions")
    async def completions(req: CompletionRequest):
        ids, params = _ids(req), _params(req)
        if req.n < 1 or (req.n > 1 and req.stream):
            raise HTTPException(400, "n must be >= 1 (and 1 when streaming)")
        if req.stop and (tokenizer is None or req.stream):
            raise HTTPException(400, "stop strings need a tokenizer and a non-streaming request")
        created = int(time.time())
        t0 = time.perf_counter()
        m.requests.inc()
        m.prompt_tokens.inc(len(ids))
        if req.stream:
            async def events():
                async for tok in front.stream(ids, params):
                    m.completion_tokens.inc()
                    yield "data: " + json.dumps({"object": "text_completion.chunk", "model": model_name,
                                                 "token": tok, "text": _text([tok])}) + "\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(events(), media_type="text/event-stream")
        import asyncio
        import dataclasses

        base_seed = params.seed if params.seed is not None else 0
        plist = [params] if req.n == 1 else [dataclasses.replace(params, seed=base_seed + i) for i in range(req.n)]
        try:
            if req.stop:
                res = await asyncio.gather(*(_generate_stop(ids, p, req.stop) for p in plist))
            else:
                outs = await asyncio.gather(*(front.generate(ids, p) for p in plist))
                res = [(o, _text(o), "length" if len(o) >= req.max_tokens else "stop") for o in outs]
        except RuntimeError as e:
            m.failures.inc()
            raise HTTPException(503, str(e))
        ntok = sum(len(o) for o, _, _ in res)
        m.completion_tokens.inc(ntok)
        m.latency.observe(time.perf_counter() - t0)
        return {"object": "text_completion", "created": created, "model": model_name,
                "choices": [{"index": i, "text": text, "token_ids": out, "finish_reason": why}
                            for i, (out, text, why) in enumerate(res)],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": ntok, "total_tokens": len(ids) + ntok}}

    @app.post("/v1/chat/completions")
    async def chat(req: ChatRequest):
        from ..io.prompts import apply_chat_template, strip_thinking

        if tokenizer is None:
            raise HTTPException(400, "no tokenizer loaded: chat needs one")
        if not req.messages:
            raise HTTPException(400, "messages must not be empty")
        text = apply_chat_template(tokenizer, req.messages, enable_thinking=req.enable_thinking)
        ids = tokenizer.encode(text)
        params = _params(CompletionRequest(prompt=ids, max_tokens=req.max_tokens, temperature=req.temperature,
                                           top_p=req.top_p, top_k=req.top_k, seed=req.seed,
                                           stop_token_ids=req.stop_token_ids))
        m.requests.inc()
        m.prompt_tokens.inc(len(ids))
        t0 = time.perf_counter()
        try:
            out = await front.generate(ids, params)
        except RuntimeError as e:
            m.failures.inc()
            raise HTTPException(503, str(e))
        m.completion_tokens.inc(len(out))
        m.latency.observe(time.perf_counter() - t0)
        reply = tokenizer.decode(out)
        return {"object": "chat.completion", "created": int(time.time()), "model": model_name,
                "choices": [{"index": 0, "message": {"role": "assistant", "content": strip_thinking(reply)},
                             "token_ids": out,
                             "finish_reason": "length" if len(out) >= req.max_tokens else "stop"}],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out),
                          "total_tokens": len(ids) + len(out)}}

    return app


class _Metrics:
    """Prometheus metrics of one served engine (own registry, so several apps can coexist)."""

    def __init__(self, engine):
        from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram

        self.engine = engine
        self.registry = r = CollectorRegistry()
        self.requests = Counter("mb_requests", "completion requests", registry=r)
        self.failures = Counter("mb_request_failures", "requests that failed", registry=r)
        self.prompt_tokens = Counter("mb_prompt_tokens", "prompt tokens received", registry=r)
        self.completion_tokens = Counter("mb_completion_tokens", "tokens generated", registry=r)
        self.latency = Histogram("mb_request_seconds", "non-streaming request latency", registry=r,
                                 buckets=(0.01, 0.05, 0.1, 0.25, 0.5, 1, 2, 5, 10, 30, 60))
        self.running = Gauge("mb_running_sequences", "sequences in the running batch", registry=r)
        self.waiting = Gauge("mb_waiting_sequences", "sequences waiting for admission", registry=r)
        self.free_blocks = Gauge("mb_free_kv_blocks", "free paged-KV blocks", registry=r)
        self.preempted = Gauge("mb_preemptions", "sequences preempted so far", registry=r)

    def render(self):
        from prometheus_client import CONTENT_TYPE_LATEST, generate_latest

        e = self.engine
        if not hasattr(e, "scheduler"):  # a router over several engines: no single scheduler to report
            return generate_latest(self.registry), CONTENT_TYPE_LATEST
        self.running.set(len(e.scheduler.running))
        self.waiting.set(len(e.scheduler.waiting))
        self.free_blocks.set(e.blocks.num_free)
        self.preempted.set(e.scheduler.num_preempted)
        return generate_latest(self.registry), CONTENT_TYPE_LATEST


def serve(engine, tokenizer=None, model_name: str = "model", host: str = "127.0.0.1", port: int = 8000) -> None:
    import uvicorn

    uvicorn.run(create_app(engine, tokenizer, model_name), host=host, port=port, log_level="info")
