"""Streaming and asyncio front-ends: concurrent requests are batched by one
engine thread and return the same tokens as a direct generate()."""
import asyncio

from mod_b200.engine.sequence import SamplingParams


def _engine():
    from mod_b200.config import get_preset
    from mod_b200.engine.llm_engine import LLMEngine

    return LLMEngine(get_preset("tiny-dense"), backend="torch", device="cpu", max_batch=4, max_model_len=64,
                     use_graphs=False)


PROMPTS = [[1, 2, 3, 4], [9, 8, 7], [5] * 10]


def test_streaming_engine_matches_generate():
    from mod_b200.api.managers import StreamingEngine

    ref = _engine().generate(PROMPTS, SamplingParams(max_new_tokens=5))
    se = StreamingEngine(_engine())
    try:
        rids = [se.submit_request(p, SamplingParams(max_new_tokens=5)) for p in PROMPTS]
        got = [list(se.generate_stream(r, timeout=60)) for r in rids]
    finally:
        se.shutdown()
    assert got == ref
    assert se.stats["completed"] == len(PROMPTS)


def test_async_engine_concurrent_requests():
    from mod_b200.api.managers import AsyncEngine

    ref = _engine().generate(PROMPTS, SamplingParams(max_new_tokens=5))
    ae = AsyncEngine(_engine())

    async def main():
        outs = await asyncio.gather(*(ae.generate(p, SamplingParams(max_new_tokens=5)) for p in PROMPTS))
        streamed = [t async for t in ae.stream(PROMPTS[0], SamplingParams(max_new_tokens=5))]
        via_request = await ae.process_request({"input_ids": PROMPTS[1], "max_new_tokens": 5})
        return outs, streamed, via_request

    try:
        outs, streamed, via_request = asyncio.run(asyncio.wait_for(main(), 120))
    finally:
        ae.shutdown()
    assert outs == ref and streamed == ref[0] and via_request == ref[1]


def test_engine_abort_frees_blocks():
    eng = _engine()
    free0 = eng.blocks.num_free
    a = eng.add_request(PROMPTS[2], SamplingParams(max_new_tokens=50))
    b = eng.add_request(PROMPTS[0], SamplingParams(max_new_tokens=3))
    eng.step()                                   # prefill both
    assert eng.abort(a) and not eng.abort(a)     # second abort: already finished
    while eng.has_unfinished():
        eng.step()
    assert eng.seqs[a].status.name == "ABORTED" and len(eng.seqs[b].output) == 3
    assert eng.blocks.num_free == free0
    w = eng.add_request(PROMPTS[1], SamplingParams(max_new_tokens=3))
    assert eng.abort(w) and not eng.has_unfinished()   # a waiting request leaves the queue


def test_async_stream_cancel_frees_the_request():
    from mod_b200.api.managers import AsyncEngine

    eng = _engine()
    free0 = eng.blocks.num_free
    ae = AsyncEngine(eng)

    async def main():
        got = []
        async for t in ae.stream(PROMPTS[2], SamplingParams(max_new_tokens=40)):
            got.append(t)
            if len(got) == 2:
                break                             # consumer goes away early
        return got

    try:
        got = asyncio.run(asyncio.wait_for(main(), 60))
        import time

        t0 = time.time()
        while (eng.has_unfinished() or eng.blocks.num_free != free0) and time.time() - t0 < 10:
            time.sleep(0.05)
    finally:
        ae.shutdown()
    assert len(got) == 2 and not eng.has_unfinished() and eng.blocks.num_free == free0
    assert ae.streaming.stats.get("cancelled", 0) == 1


def test_stop_token_ids_end_generation():
    ref = _engine().generate([PROMPTS[0]], SamplingParams(max_new_tokens=8))[0]
    stop = ref[3]
    got = _engine().generate([PROMPTS[0]], SamplingParams(max_new_tokens=8, stop_token_ids=(stop,)))[0]
    assert got == ref[:ref.index(stop) + 1]


def test_replica_router_spreads_requests_and_matches():
    from mod_b200.api.managers import AsyncEngine, ReplicaRouter

    ref = _engine().generate(PROMPTS, SamplingParams(max_new_tokens=5))
    router = ReplicaRouter([_engine(), _engine()])
    ae = AsyncEngine(router)

    async def main():
        return await asyncio.gather(*(ae.generate(p, SamplingParams(max_new_tokens=5)) for p in PROMPTS))

    try:
        rids = [router.submit_request(p, SamplingParams(max_new_tokens=5)) for p in PROMPTS]
        assert {router.replica_of(r) for r in rids} == {0, 1}      # both replicas got work
        direct = [list(router.generate_stream(r, timeout=60)) for r in rids]
        outs = asyncio.run(asyncio.wait_for(main(), 120))
    finally:
        ae.shutdown()
    assert direct == ref and outs == ref
    assert router.stats["completed"] == 2 * len(PROMPTS)
