"""Serving on the B200 engine (lagunalab_b200/serve.py): a tiny random-init decoder behind the
OpenAI-compatible endpoints on 127.0.0.1. The greedy tokens that come back over HTTP equal
``laguna.generate``'s; a follow-up request that extends the first conversation reuses its
cached prefix and still gives the tokens of a fresh generation; the 8-bit fused cache serves
too."""
import json
import threading
import urllib.request

import pytest
import torch

pytestmark = pytest.mark.gpu


class _Tok:
    """Stand-in tokenizer over ids 0..511: id i <-> the 2-character hex string of i % 256
    prefixed by a bucket letter (no multi-byte characters)."""
    eos_token_id = None

    def encode(self, text):
        return [int(text[i + 1:i + 4], 16) for i in range(0, len(text), 4)]

    def decode(self, ids):
        return "".join(f"t{i:03x}" for i in ids)

    def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=True):
        return self.encode("".join(m["content"] for m in messages))


def _model():
    from lagunalab_b200 import synth
    args = synth.decoder_args(vocab=512, hidden=256, layers=3, heads=4, kv_heads=2, head_dim=128,
                              experts=8, top_k=2, moe_inter=128, shared_inter=128,
                              dense_inter=256, rope_theta=1e4)
    return synth.decoder(args, seed=5, std=0.05, norm_noise=0.1, router_bias_std=0.3)


def _post(url, body):
    req = urllib.request.Request(url, json.dumps(body).encode(),
                                 {"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=120) as r:
        return json.loads(r.read().decode())


def _ids(text):
    return [int(text[i + 1:i + 4], 16) for i in range(0, len(text), 4)]


@pytest.mark.parametrize("kv", ["bf16", "q8"])
def test_served_greedy_tokens_equal_generate(kv):
    from lagunalab_b200 import cache as qcache, laguna, serve
    model = _model()
    make = ((lambda: qcache.make_quantized_cache(model, 8, fused_decode=True, capacity=512))
            if kv == "q8" else (lambda: model.make_cache(capacity=512)))
    eng = serve.Engine(model, _Tok(), stop_ids=(), make_cache=make, max_context=512,
                       prompt_cache=serve.PromptCache(2))
    httpd = serve.serve(eng, "127.0.0.1", 0, "tiny")
    th = threading.Thread(target=httpd.serve_forever, daemon=True)
    th.start()
    base = f"http://127.0.0.1:{httpd.server_address[1]}"
    try:
        prompt = torch.randint(0, 512, (11,), generator=torch.Generator().manual_seed(6)).tolist()
        want = laguna.generate(model, torch.tensor(prompt).cuda(), 12, cache=make())
        d = _post(base + "/v1/completions", {"prompt": prompt, "max_tokens": 12})
        got = _ids(d["choices"][0]["text"])
        assert got == want and d["choices"][0]["finish_reason"] == "length"
        # the next turn extends the conversation: its cached prefix is reused
        follow = prompt + got[:7] + [3, 4, 5]
        want2 = laguna.generate(model, torch.tensor(follow).cuda(), 9, cache=make())
        d2 = _post(base + "/v1/completions", {"prompt": follow, "max_tokens": 9})
        assert _ids(d2["choices"][0]["text"]) == want2
        assert d2["usage"]["prompt_tokens"] == len(follow)
    finally:
        httpd.shutdown()
        httpd.server_close()
