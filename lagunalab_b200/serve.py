"""OpenAI-compatible serving of the B200 engine: the ``scripts/serve_streaming.py`` surface of
lagunaLab (:37-140), which wraps mlx-lm's server around ``load_streaming``, rebuilt on the
Python standard library's HTTP server over this package's decoder.

    python -m lagunalab_b200.serve --pack DIR [--preset laptop16] [--fused-decode]
        [--slots N] [--host 127.0.0.1] [--port 8081] [--max-tokens 4096]
        [--prompt-cache-size 6] [--prompt-cache-bytes 4294967296]

Kept from the reference: the ``PRESETS`` table and ``apply_preset(argv)`` (a preset fills the
server flags that argv does not set; explicit flags win, ``--fused-decode`` and ``--slots``
too), the model load (``load_streaming(pack, slots, cache_limit_gb)``; with fused decode the
caches are ``make_quantized_cache(model, 8, fused_decode=True)``), the end-of-turn ids from the
pack's ``generation_config.json`` added to the tokenizer's EOS set (:86-94), and no SSE
keepalive comment lines on the wire (what ``_DropKeepalive`` strips, :50-74). Requests are
served one at a time, as the reference does with the fused cache, whose cache has no batch
merge (:27-30).

Endpoints: ``GET /v1/models``, ``POST /v1/completions``, ``POST /v1/chat/completions`` (the
prompt rendered with the tokenizer's chat template), non-streaming or ``"stream": true``
(server-sent events ending in ``data: [DONE]``). Decoding is greedy, one CUDA-graph replay per
token (``laguna.DecodeGraph``); ``temperature > 0`` samples on the device from the softmax of
the logits / temperature, one eager step per token. A prompt cache keeps the KV caches of the
last ``--prompt-cache-size`` conversations (bounded by ``--prompt-cache-bytes``) and reuses the
longest cached prefix of a new prompt (the reference relies on mlx-lm's prompt cache the same
way, :8-16).
"""
import argparse
import json
import sys
import threading
import time
import uuid
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path

PACK = "models/Laguna-XS-2.1-packed"

# the reference's preset table (scripts/serve_streaming.py:37-48)
PRESETS = {
    "laptop16": {"pack": "models/Laguna-XS-2.1-pruned-50-packed", "slots": 64,
                 "cache_limit_gb": 1.0, "fused_decode": False,
                 "server_args": {"--max-tokens": "4096", "--prompt-cache-size": "6",
                                 "--prompt-cache-bytes": "4294967296"}},
}


def apply_preset(argv, config):
    """Pop ``--preset NAME`` from argv, write the preset's pack, slots, cache limit and fused
    decode into ``config`` (a dict), and append its server flags that argv does not already set.
    Returns the resolved preset (its server flags as they end up in argv), or None without
    ``--preset``. An unknown name raises KeyError, as the reference's table lookup does."""
    if "--preset" not in argv:
        return None
    i = argv.index("--preset")
    p = PRESETS[argv[i + 1]]
    del argv[i:i + 2]
    config.update(pack=p["pack"], slots=p["slots"], cache_limit_gb=p["cache_limit_gb"],
                  fused_decode=p["fused_decode"])
    for flag, value in p["server_args"].items():
        if flag not in argv:
            argv += [flag, value]
    return {**p, "server_args": {f: argv[argv.index(f) + 1] for f in p["server_args"]}}


def eos_ids(pack_dir, tokenizer):
    """The tokenizer's EOS id(s) plus every id of the pack's generation_config.json
    ``eos_token_id`` (Laguna ends a turn with "</assistant>", id 24, besides EOS id 2)."""
    ids = set()
    tid = getattr(tokenizer, "eos_token_id", None)
    if tid is not None:
        ids.update(tid if isinstance(tid, (list, tuple)) else [tid])
    gc = Path(pack_dir) / "generation_config.json"
    if gc.exists():
        e = json.loads(gc.read_text()).get("eos_token_id", [])
        ids.update(e if isinstance(e, list) else [e])
    return {int(i) for i in ids}


class PromptCache:
    """The KV caches of the last ``size`` conversations (LRU), bounded by ``max_bytes``: each
    entry is (token ids the cache holds, the per-layer caches)."""

    def __init__(self, size=2, max_bytes=None):
        self.size, self.max_bytes = int(size), max_bytes
        self.entries = []  # most recent last

    def take(self, ids):
        """(entry, prefix length) of the entry sharing the longest prefix with ``ids``, removed
        from the cache (the caller puts it back after generating), or (None, 0)."""
        best, best_n = None, 0
        for e in self.entries:
            toks = e[0]
            n = 0
            for a, b in zip(toks, ids):
                if a != b:
                    break
                n += 1
            if n > best_n:
                best, best_n = e, n
        if best is not None:
            self.entries.remove(best)
        return best, best_n

    def put(self, toks, cache):
        self.entries.append((list(toks), cache))
        while len(self.entries) > max(1, self.size):
            self.entries.pop(0)
        if self.max_bytes:
            while len(self.entries) > 1 and self.nbytes() > self.max_bytes:
                self.entries.pop(0)

    def nbytes(self):
        return sum(sum(getattr(c, "nbytes", 0) for c in cache) for _, cache in self.entries)


class Engine:
    """One request at a time over ``model``: prefill the prompt (reusing the longest cached
    prefix), then decode greedily one CUDA-graph replay per token (``laguna.DecodeGraph``), or
    sample with a temperature one eager step per token. ``make_cache()`` builds a request's
    per-layer caches with room for ``max_context`` rows."""

    def __init__(self, model, tokenizer, stop_ids=(), make_cache=None, max_context=8192,
                 prompt_cache=None):
        self.model, self.tokenizer = model, tokenizer
        self.stop_ids = {int(i) for i in stop_ids}
        self.max_context = int(max_context)
        self.make_cache = make_cache or (lambda: model.make_cache(capacity=self.max_context))
        self.prompt_cache = prompt_cache if prompt_cache is not None else PromptCache(1)
        self.lock = threading.Lock()

    def chat_ids(self, messages):
        ids = self.tokenizer.apply_chat_template(messages, add_generation_prompt=True,
                                                 tokenize=True)
        return [int(i) for i in (ids["input_ids"] if isinstance(ids, dict) else ids)]

    def prompt_ids(self, prompt):
        if isinstance(prompt, list) and all(isinstance(i, int) for i in prompt):
            return list(prompt)
        if isinstance(prompt, list):
            prompt = "".join(prompt)
        return [int(i) for i in self.tokenizer.encode(prompt)]

    def _cache_for(self, ids):
        """(caches holding ids[:n], n) with n < len(ids): a cached conversation trimmed to its
        common prefix with ids, or fresh caches."""
        entry, n = self.prompt_cache.take(ids)
        n = min(n, len(ids) - 1)
        if entry is not None and n > 0:
            cache = entry[1]
            if all(c.is_trimmable() or c.offset == n for c in cache):
                for c in cache:
                    if c.offset > n:
                        c.trim(c.offset - n)
                if all(c.offset == n for c in cache):
                    return cache, n
        return self.make_cache(), 0

    def generate(self, ids, max_tokens, temperature=0.0):
        """A generator of the generated ids; a stop id ends the generation without being
        yielded, and the generator returns (through StopIteration) the finish reason, "stop" or
        "length". The prompt is checked here, before the generator runs (ValueError)."""
        if not ids:
            raise ValueError("empty prompt")
        if len(ids) >= self.max_context:
            raise ValueError(f"prompt of {len(ids)} tokens exceeds the context {self.max_context}")
        return self._generate(list(ids), int(max_tokens), float(temperature or 0.0))

    def _generate(self, ids, max_tokens, temperature):
        import torch

        from . import laguna, ops
        max_tokens = max(0, min(max_tokens, self.max_context - len(ids) - 1))
        cache, n = self._cache_for(ids)
        dev = self.model.lm_head.weight.device
        held = list(ids)
        reason = "length"
        try:
            new = torch.tensor(ids[n:], dtype=torch.int32, device=dev).view(1, -1)
            logits = self.model.last_logits(new, cache).reshape(1, -1)
            if max_tokens == 0:
                return reason
            if temperature and temperature > 0:
                for i in range(max_tokens):
                    p = torch.softmax(logits.float() / float(temperature), dim=-1)
                    t = int(torch.multinomial(p, 1))
                    if t in self.stop_ids:
                        return "stop"
                    yield t
                    if i + 1 == max_tokens:
                        break
                    held.append(t)
                    logits = self.model.last_logits(
                        torch.tensor([[t]], dtype=torch.int32, device=dev), cache).reshape(1, -1)
                return reason
            tok = ops.argmax(logits)
            t = int(tok)
            if t in self.stop_ids:
                return "stop"
            yield t
            if max_tokens == 1:
                return reason
            held.append(t)  # the graph's first (eager) step feeds it
            dg = laguna.DecodeGraph(self.model, cache, tok)
            try:
                for i in range(1, max_tokens):
                    if i > 1:
                        held.append(t)  # the previous token, fed by this step
                        dg.step()
                    t = int(dg.tok)
                    if t in self.stop_ids:
                        reason = "stop"
                        break
                    yield t
            finally:
                # the graph wrote rows up to its device position; the host offsets follow
                pos = dg.position()
                for c in cache:
                    (c.q if getattr(c, "q", None) is not None else c).offset = pos
                del dg
            return reason
        finally:
            if len(held) == cache[0].offset:
                self.prompt_cache.put(held, cache)


def _text_stream(tokenizer, gen):
    """(text piece, token count) per step of ``gen`` with incremental detokenisation: a piece
    is released once the decoded text no longer ends inside a multi-byte character. Returns
    (through StopIteration) gen's finish reason."""
    ids, sent = [], ""
    while True:
        try:
            t = next(gen)
        except StopIteration as e:
            text = tokenizer.decode(ids)
            if len(text) > len(sent):
                yield text[len(sent):], len(ids)
            return e.value
        ids.append(t)
        text = tokenizer.decode(ids)
        if not text.endswith("�") and len(text) > len(sent):
            yield text[len(sent):], len(ids)
            sent = text


def _now():
    return int(time.time())


def make_handler(engine, model_name, default_max_tokens=512):
    """The request handler class of the OpenAI-compatible endpoints over ``engine``."""

    class Handler(BaseHTTPRequestHandler):
        server_version = "lagunalab-b200"

        def log_message(self, fmt, *args):  # quiet: one line per request is the caller's choice
            pass

        def _send_json(self, code, obj):
            body = json.dumps(obj).encode()
            self.send_response(code)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def _event(self, obj):
            # one server-sent event; never a ":" comment line (keepalives), which some OpenAI
            # streaming clients reject
            self.wfile.write(b"data: " + (obj if isinstance(obj, bytes) else
                                          json.dumps(obj).encode()) + b"\n\n")
            self.wfile.flush()

        def do_GET(self):
            if self.path.rstrip("/") == "/v1/models":
                self._send_json(200, {"object": "list", "data": [
                    {"id": model_name, "object": "model", "created": _now(),
                     "owned_by": "lagunalab-b200"}]})
            elif self.path.rstrip("/") == "/health":
                self._send_json(200, {"status": "ok"})
            else:
                self._send_json(404, {"error": {"message": f"no route {self.path}"}})

        def do_POST(self):
            path = self.path.rstrip("/")
            chat = path == "/v1/chat/completions"
            if not chat and path != "/v1/completions":
                self._send_json(404, {"error": {"message": f"no route {self.path}"}})
                return
            try:
                req = json.loads(self.rfile.read(int(self.headers.get("Content-Length", 0))))
                ids = engine.chat_ids(req["messages"]) if chat else engine.prompt_ids(req["prompt"])
                max_tokens = int(req.get("max_tokens") or req.get("max_completion_tokens")
                                 or default_max_tokens)
                temperature = float(req.get("temperature") or 0.0)
                stop = req.get("stop") or []
                stop = [stop] if isinstance(stop, str) else list(stop)
            except (ValueError, KeyError, TypeError) as e:
                self._send_json(400, {"error": {"message": f"bad request: {e}"}})
                return
            rid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex[:24]
            with engine.lock:
                try:
                    gen = engine.generate(ids, max_tokens, temperature)
                except ValueError as e:
                    self._send_json(400, {"error": {"message": str(e)}})
                    return
                try:
                    if req.get("stream"):
                        self._stream(rid, chat, gen, stop)
                    else:
                        self._complete(rid, chat, gen, stop, len(ids))
                finally:
                    # a client that went away mid-stream leaves the generator suspended: close it
                    # here, under the lock, so its caches are synchronised and returned to the
                    # prompt cache before the next request
                    gen.close()

        def _pieces(self, gen, stop):
            """(piece, tokens so far) with the stop strings applied: text that could still be
            the start of a stop string is held back until it cannot; returns the reason."""
            stop = [s_ for s_ in stop if s_]
            text, sent, n = "", 0, 0
            stream = _text_stream(engine.tokenizer, gen)
            while True:
                try:
                    piece, n = next(stream)
                except StopIteration as e:
                    if len(text) > sent:
                        yield text[sent:], n
                    return e.value or "stop"
                text += piece
                hits = [j for j in (text.find(s_) for s_ in stop) if j >= 0]
                if hits:
                    cut = min(hits)
                    if cut > sent:
                        yield text[sent:cut], n
                    gen.close()
                    return "stop"
                hold = 0
                for s_ in stop:
                    for k in range(min(len(s_) - 1, len(text)), 0, -1):
                        if text.endswith(s_[:k]):
                            hold = max(hold, k)
                            break
                if len(text) - hold > sent:
                    yield text[sent:len(text) - hold], n
                    sent = len(text) - hold

        def _complete(self, rid, chat, gen, stop, n_prompt):
            out, n = [], 0
            it = self._pieces(gen, stop)
            while True:
                try:
                    piece, n = next(it)
                except StopIteration as e:
                    reason = e.value
                    break
                out.append(piece)
            text = "".join(out)
            choice = ({"index": 0, "message": {"role": "assistant", "content": text},
                       "finish_reason": reason} if chat else
                      {"index": 0, "text": text, "logprobs": None, "finish_reason": reason})
            self._send_json(200, {
                "id": rid, "object": "chat.completion" if chat else "text_completion",
                "created": _now(), "model": model_name, "choices": [choice],
                "usage": {"prompt_tokens": n_prompt, "completion_tokens": n,
                          "total_tokens": n_prompt + n}})

        def _stream(self, rid, chat, gen, stop):
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream")
            self.send_header("Cache-Control", "no-cache")
            self.end_headers()
            obj = "chat.completion.chunk" if chat else "text_completion"

            def chunk(piece, reason=None):
                c = ({"index": 0, "delta": {} if piece is None else
                      {"role": "assistant", "content": piece}, "finish_reason": reason} if chat
                     else {"index": 0, "text": piece or "", "logprobs": None,
                           "finish_reason": reason})
                return {"id": rid, "object": obj, "created": _now(), "model": model_name,
                        "choices": [c]}

            it = self._pieces(gen, stop)
            while True:
                try:
                    piece, _ = next(it)
                except StopIteration as e:
                    reason = e.value
                    break
                self._event(chunk(piece))
            self._event(chunk(None, reason))
            self._event(b"[DONE]")

    return Handler


def serve(engine, host="127.0.0.1", port=8081, model_name="laguna", max_tokens=512):
    """An HTTP server on (host, port) over ``engine`` (call ``serve_forever()`` on it)."""
    return ThreadingHTTPServer((host, port), make_handler(engine, model_name, max_tokens))


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    config = {"pack": PACK, "slots": 32, "cache_limit_gb": 1.0, "fused_decode": False}
    preset = apply_preset(argv, config)
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--pack", "--model", dest="pack", default=config["pack"])
    ap.add_argument("--slots", type=int, default=config["slots"])
    ap.add_argument("--fused-decode", action="store_true", default=config["fused_decode"])
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8081)
    ap.add_argument("--max-tokens", type=int, default=512)
    ap.add_argument("--max-context", type=int, default=16384)
    ap.add_argument("--prompt-cache-size", type=int, default=2)
    ap.add_argument("--prompt-cache-bytes", type=int, default=None)
    args = ap.parse_args(argv)

    from . import cache as qcache
    from .streaming import load_streaming
    model, tok = load_streaming(args.pack, args.slots, cache_limit_gb=config["cache_limit_gb"])
    if tok is None:
        raise SystemExit(f"{args.pack}: no tokenizer.json")
    if args.fused_decode:
        make = lambda: qcache.make_quantized_cache(model, 8, fused_decode=True,  # noqa: E731
                                                   capacity=args.max_context)
    else:
        make = lambda: model.make_cache(capacity=args.max_context)  # noqa: E731
    eng = Engine(model, tok, eos_ids(args.pack, tok), make, args.max_context,
                 PromptCache(args.prompt_cache_size, args.prompt_cache_bytes))
    print(f"serve: pack={args.pack} slots={args.slots} "
          f"kv={'q8-fused' if args.fused_decode else 'plain'}"
          + (f" preset={preset['server_args']}" if preset else "")
          + f" on http://{args.host}:{args.port}", flush=True)
    httpd = serve(eng, args.host, args.port, Path(args.pack).name, args.max_tokens)
    try:
        httpd.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        httpd.server_close()


if __name__ == "__main__":
    main()
