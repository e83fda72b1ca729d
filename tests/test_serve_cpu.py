"""The serving surface (lagunalab_b200/serve.py; lagunaLab scripts/serve_streaming.py:37-140)
without a GPU: the preset rules, the end-of-turn ids, the prompt cache, and the HTTP endpoints
over a fake engine on 127.0.0.1 (non-streaming and server-sent events, stop strings, errors)."""
import json
import threading
import urllib.error
import urllib.request

import pytest

from lagunalab_b200 import serve


def test_apply_preset_fills_missing_flags_and_explicit_flags_win():
    argv = ["--port", "9000", "--preset", "laptop16", "--max-tokens", "100"]
    cfg = {}
    p = serve.apply_preset(argv, cfg)
    assert "--preset" not in argv and "laptop16" not in argv
    assert cfg == {"pack": "models/Laguna-XS-2.1-pruned-50-packed", "slots": 64,
                   "cache_limit_gb": 1.0, "fused_decode": False}
    assert argv[argv.index("--max-tokens") + 1] == "100"  # explicit wins
    assert argv[argv.index("--prompt-cache-size") + 1] == "6"
    assert argv[argv.index("--prompt-cache-bytes") + 1] == "4294967296"
    assert p["server_args"] == {"--max-tokens": "100", "--prompt-cache-size": "6",
                                "--prompt-cache-bytes": "4294967296"}
    assert serve.apply_preset(["--port", "1"], {}) is None
    with pytest.raises(KeyError):
        serve.apply_preset(["--preset", "nope"], {})


def test_eos_ids_add_the_generation_config_ids(tmp_path):
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": [2, 24]}))

    class Tok:
        eos_token_id = 2
    assert serve.eos_ids(tmp_path, Tok()) == {2, 24}
    assert serve.eos_ids(tmp_path / "missing", Tok()) == {2}


def test_prompt_cache_longest_prefix_and_lru():
    pc = serve.PromptCache(size=2)
    pc.put([1, 2, 3], "a")
    pc.put([1, 2, 9, 9], "b")
    e, n = pc.take([1, 2, 9, 5])
    assert e[1] == "b" and n == 3 and len(pc.entries) == 1
    pc.put(e[0], e[1])
    pc.put([7], "c")  # evicts the oldest ("a")
    assert [x[1] for x in pc.entries] == ["b", "c"]
    assert pc.take([4]) == (None, 0)


class _Tok:
    """Character-level stand-in: id i <-> chr(ord('a') + i) for i < 26."""
    eos_token_id = None

    def encode(self, text):
        return [ord(c) - ord("a") for c in text]

    def decode(self, ids):
        return "".join(chr(ord("a") + i) for i in ids)

    def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=True):
        return self.encode("".join(m["content"] for m in messages))


class _FakeEngine:
    """generate() continues the alphabet after the prompt's last letter; id 25 ('z') stops."""

    def __init__(self):
        self.tokenizer = _Tok()
        self.lock = threading.Lock()
        self.calls = []

    def chat_ids(self, messages):
        return self.tokenizer.apply_chat_template(messages)

    def prompt_ids(self, prompt):
        return self.tokenizer.encode(prompt)

    def generate(self, ids, max_tokens, temperature=0.0):
        self.calls.append((list(ids), max_tokens, temperature))
        if not ids:
            raise ValueError("empty prompt")
        return self._gen(ids, max_tokens)

    def _gen(self, ids, max_tokens):
        t = ids[-1]
        for _ in range(max_tokens):
            t += 1
            if t >= 25:
                return "stop"
            yield t
        return "length"


@pytest.fixture()
def server():
    eng = _FakeEngine()
    httpd = serve.serve(eng, "127.0.0.1", 0, "fake", max_tokens=8)
    th = threading.Thread(target=httpd.serve_forever, daemon=True)
    th.start()
    yield eng, f"http://127.0.0.1:{httpd.server_address[1]}"
    httpd.shutdown()
    httpd.server_close()


def _post(url, body):
    req = urllib.request.Request(url, json.dumps(body).encode(),
                                 {"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=30) as r:
        return r.read().decode()


def test_completion_and_chat_completion(server):
    eng, base = server
    d = json.loads(_post(base + "/v1/completions", {"prompt": "abc", "max_tokens": 4}))
    assert d["object"] == "text_completion" and d["choices"][0]["text"] == "defg"
    assert d["choices"][0]["finish_reason"] == "length"
    assert d["usage"] == {"prompt_tokens": 3, "completion_tokens": 4, "total_tokens": 7}
    d = json.loads(_post(base + "/v1/chat/completions",
                         {"messages": [{"role": "user", "content": "uv"}], "max_tokens": 50}))
    assert d["object"] == "chat.completion"
    assert d["choices"][0]["message"] == {"role": "assistant", "content": "wxy"}
    assert d["choices"][0]["finish_reason"] == "stop"  # 'z' is the stop id
    d = json.loads(_post(base + "/v1/completions", {"prompt": "a"}))
    assert len(d["choices"][0]["text"]) == 8  # the server's default max_tokens
    m = json.loads(urllib.request.urlopen(base + "/v1/models", timeout=30).read())
    assert m["data"][0]["id"] == "fake"


def test_stop_strings_cut_the_text(server):
    eng, base = server
    d = json.loads(_post(base + "/v1/completions",
                         {"prompt": "a", "max_tokens": 20, "stop": ["ef"]}))
    assert d["choices"][0]["text"] == "bcd" and d["choices"][0]["finish_reason"] == "stop"


def test_streamed_events_have_no_comment_lines(server):
    eng, base = server
    raw = _post(base + "/v1/chat/completions",
                {"messages": [{"role": "user", "content": "pq"}], "max_tokens": 3,
                 "stream": True})
    events = [e for e in raw.split("\n\n") if e]
    assert all(e.startswith("data: ") for e in events), events
    assert events[-1] == "data: [DONE]"
    chunks = [json.loads(e[6:]) for e in events[:-1]]
    text = "".join(c["choices"][0]["delta"].get("content", "") for c in chunks)
    assert text == "rst"
    assert chunks[-1]["choices"][0]["finish_reason"] == "length"
    assert all(c["object"] == "chat.completion.chunk" for c in chunks)


def test_errors(server):
    eng, base = server
    with pytest.raises(urllib.error.HTTPError) as e:
        _post(base + "/v1/nothing", {})
    assert e.value.code == 404
    with pytest.raises(urllib.error.HTTPError) as e:
        _post(base + "/v1/completions", {"max_tokens": 3})  # no prompt
    assert e.value.code == 400
    for stream in (False, True):  # an empty prompt is refused before any response starts
        with pytest.raises(urllib.error.HTTPError) as e:
            _post(base + "/v1/completions", {"prompt": "", "stream": stream})
        assert e.value.code == 400


class _FakeKV:
    def __init__(self, n, trimmable=True):
        self.offset, self.trimmable = n, trimmable

    def is_trimmable(self):
        return self.trimmable

    def trim(self, n):
        self.offset -= n
        return n


def test_engine_reuses_the_longest_cached_prefix():
    eng = serve.Engine(model=None, tokenizer=_Tok(), make_cache=lambda: "fresh",
                       max_context=64, prompt_cache=serve.PromptCache(2))
    held = [_FakeKV(10), _FakeKV(10)]
    eng.prompt_cache.put(list(range(10)), held)
    cache, n = eng._cache_for(list(range(7)) + [30, 31])  # shares 7 tokens
    assert cache is held and n == 7 and all(c.offset == 7 for c in held)
    assert eng.prompt_cache.entries == []  # taken out while the request runs
    eng.prompt_cache.put(list(range(7)), held)
    cache, n = eng._cache_for(list(range(7)))  # the whole prompt cached: one token is re-fed
    assert cache is held and n == 6 and all(c.offset == 6 for c in held)
    ring = [_FakeKV(9, trimmable=False)]  # a wrapped sliding window cannot be cut back
    eng.prompt_cache.put(list(range(9)), ring)
    assert eng._cache_for(list(range(5)) + [40]) == ("fresh", 0)
