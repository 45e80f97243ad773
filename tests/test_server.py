"""HTTP front-end: completions (ids and text), streaming, health, errors --
against a direct generate() on the same CPU engine configuration."""
import json

import pytest

pytest.importorskip("fastapi")
pytest.importorskip("httpx")

from fastapi.testclient import TestClient  # noqa: E402

from mod_b200.engine.sequence import SamplingParams  # noqa: E402
from mod_b200.io.tokenizer import load_tokenizer  # noqa: E402


def _engine():
    from mod_b200.config import get_preset
    from mod_b200.engine.llm_engine import LLMEngine

    return LLMEngine(get_preset("tiny-dense"), backend="torch", device="cpu", max_batch=4, max_model_len=96,
                     use_graphs=False)


def test_completions_stream_health_and_errors():
    from mod_b200.api.server import create_app

    prompt = [5, 6, 7, 8, 9]
    ref = _engine().generate([prompt], SamplingParams(max_new_tokens=6))[0]
    tok = load_tokenizer(None)
    app = create_app(_engine(), tok, "tiny-dense")
    with TestClient(app) as c:
        assert c.get("/health").json()["status"] == "ok"
        assert c.get("/v1/models").json()["data"][0]["id"] == "tiny-dense"
        r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 6})
        assert r.status_code == 200
        body = r.json()
        assert body["choices"][0]["token_ids"] == ref
        assert body["usage"] == {"prompt_tokens": 5, "completion_tokens": 6, "total_tokens": 11}
        with c.stream("POST", "/v1/completions", json={"prompt": prompt, "max_tokens": 6, "stream": True}) as s:
            toks = [json.loads(line[6:])["token"] for line in s.iter_lines()
                    if line.startswith("data: ") and line != "data: [DONE]"]
        assert toks == ref
        t = c.post("/v1/completions", json={"prompt": "hi", "max_tokens": 3})
        assert t.status_code == 200 and len(t.json()["choices"][0]["token_ids"]) == 3
        assert c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 0}).status_code == 400
        mt = c.get("/metrics").text
        assert "mb_requests_total 3.0" in mt and "mb_completion_tokens_total 15.0" in mt
        assert "mb_free_kv_blocks" in mt and "mb_request_seconds_count 2.0" in mt


def test_chat_completions_uses_the_chat_template():
    from mod_b200.api.server import create_app
    from mod_b200.io.prompts import apply_chat_template

    tok = load_tokenizer(None)
    msgs = [{"role": "user", "content": "Hi"}]
    ids = apply_chat_template(tok, msgs, enable_thinking=False, tokenize=True)
    ref = _engine().generate([ids], SamplingParams(max_new_tokens=4))[0]
    app = create_app(_engine(), tok, "tiny-dense")
    with TestClient(app) as c:
        r = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 4})
        assert r.status_code == 200
        body = r.json()
        assert body["choices"][0]["token_ids"] == ref and body["choices"][0]["message"]["role"] == "assistant"
        assert body["usage"]["prompt_tokens"] == len(ids)
        assert c.post("/v1/chat/completions", json={"messages": []}).status_code == 400


def test_n_samples_with_seeds():
    from mod_b200.api.server import create_app

    app = create_app(_engine(), None, "tiny-dense")
    with TestClient(app) as c:
        body = {"prompt": [5, 6, 7, 8], "max_tokens": 6, "temperature": 1.0, "seed": 11, "n": 3}
        r = c.post("/v1/completions", json=body).json()
        again = c.post("/v1/completions", json=body).json()
        outs = [ch["token_ids"] for ch in r["choices"]]
        assert len(outs) == 3 and r["usage"]["completion_tokens"] == 18
        assert outs == [ch["token_ids"] for ch in again["choices"]]        # seeded: reproducible
        assert len({tuple(o) for o in outs}) > 1                            # different seeds differ
        assert c.post("/v1/completions", json={**body, "stream": True}).status_code == 400


def test_stop_strings_cut_and_cancel():
    from mod_b200.api.server import create_app

    tok = load_tokenizer(None)
    eng = _engine()
    app = create_app(eng, tok, "tiny-dense")
    with TestClient(app) as c:
        full = c.post("/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 12}).json()["choices"][0]
        text = full["text"]
        stop = text[len(text) // 2:len(text) // 2 + 1] if len(text) > 2 else None
        if not stop:
            pytest.skip("the random model's text is too short to pick a stop string from")
        r = c.post("/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 12, "stop": [stop]}).json()
        ch = r["choices"][0]
        assert ch["finish_reason"] == "stop" and stop not in ch["text"] and text.startswith(ch["text"])
        assert len(ch["token_ids"]) <= len(full["token_ids"])
        assert c.post("/v1/completions", json={"prompt": [1], "stop": ["x"], "stream": True}).status_code == 400
    assert eng.blocks.num_free == eng.blocks.num_blocks          # the cancelled request released its blocks
