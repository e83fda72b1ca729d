"""Replay harness host logic on CPU (lagunaLab replay/session.py, replay/replay.py): session
parsing and normalisation, tokenization with truncation, the assistant-position selection,
chunked prefill through one cache, the reference file round trip, the truncated-KL and
top-1 arithmetic against a hand computation, and the ``forward=`` contract. The model is a
small causal torch toy with a cache, so every path runs without a GPU."""
import json

import numpy as np
import pytest
import torch

from lagunalab_b200 import replay, session
from tests._replay_util import CharTokenizer, TokenizerWrapper, target_positions, write_capture

V, H = 512, 32


class _Cache:
    def __init__(self):
        self.offset = 0
        self.acc = torch.zeros(H)


class _Toy:
    """Causal toy LM: hidden(t) = tanh(emb[id_t] + pos[t] + 0.1 * sum of earlier embeddings),
    carried across calls by the cache."""

    def __init__(self, seed=0, noise=0.0):
        g = torch.Generator().manual_seed(seed)
        self.emb = torch.randn(V, H, generator=g)
        self.pos = torch.randn(4096, H, generator=g) * 0.3
        self.head = torch.randn(V, H, generator=g)
        if noise:
            self.head = self.head + noise * torch.randn(V, H, generator=torch.Generator()
                                                        .manual_seed(seed + 99))
        self.lm_head = lambda h: h @ self.head.T

    def _body(self, x, cache):
        e = self.emb[x[0].long()]
        L = e.shape[0]
        prev = cache.acc + torch.cumsum(e, 0) - e
        h = torch.tanh(e + self.pos[cache.offset:cache.offset + L] + 0.1 * prev)
        cache.acc = cache.acc + e.sum(0)
        cache.offset += L
        return h[None]

    def make_cache(self):
        return _Cache()

    def last_logits(self, x, cache):
        return self.lm_head(self.model(x, cache)[0][-1:])[None]


class _Dev:
    device = torch.device("cpu")


def _toy(**k):
    m = _Toy(**k)
    m.model = type("M", (), {"__call__": lambda s, x, cache=None: m._body(x, cache),
                             "embed_tokens": type("E", (), {"weight": _Dev()})()})()
    return m


def test_normalize_wire_format():
    m = session.normalize({"role": "user", "content": [{"type": "text", "text": "a"}, "x",
                                                        {"type": "text", "text": "b"}]})
    assert m["content"] == "ab"
    assert session.normalize({"role": "assistant", "content": None})["content"] == ""
    calls = [{"id": i, "function": {"name": "f", "arguments": a}}
             for i, a in enumerate(['{"p": 1}', '{bad', 'null', '[1, 2]', {"k": 2}])]
    got = [c["function"]["arguments"]
           for c in session.normalize({"role": "assistant", "content": "",
                                       "tool_calls": calls})["tool_calls"]]
    assert got == [{"p": 1}, {"_raw": "{bad"}, {"_raw": "null"}, {"_raw": "[1, 2]"}, {"k": 2}]


def test_load_session_takes_last_chat_request(tmp_path):
    msgs, tools = session.load_session(write_capture(tmp_path / "s.jsonl"))
    assert len(msgs) == 5 and tools == []
    assert msgs[1]["content"] == "List the files."
    assert msgs[2]["tool_calls"][0]["function"]["arguments"] == {"path": "."}
    bad = tmp_path / "none.jsonl"
    bad.write_text(json.dumps({"path": "/v1/models", "request": None}) + "\n")
    with pytest.raises(ValueError, match="no chat requests"):
        session.load_session(bad)


def test_tokenize_truncates_and_unwraps(tmp_path):
    msgs, tools = session.load_session(write_capture(tmp_path / "s.jsonl"))
    tok = CharTokenizer()
    ids, mask, tr = session.tokenize(TokenizerWrapper(tok), msgs, tools)
    assert ids.dtype == np.int32 and mask.dtype == bool and not tr and mask.any()
    ids2, mask2, tr2 = session.tokenize(tok, msgs, tools, max_tokens=30)
    assert tr2 and len(ids2) == 30 and (ids2 == ids[:30]).all() and (mask2 == mask[:30]).all()


def test_assistant_positions_and_chunking(tmp_path):
    msgs, tools = session.load_session(write_capture(tmp_path / "s.jsonl"))
    ids, mask, _ = session.tokenize(CharTokenizer(), msgs, tools)
    m = _toy()
    whole = list(replay.assistant_logprobs(m, ids, mask))
    pos = np.concatenate([p for p, _ in whole])
    assert (pos == target_positions(mask)).all()
    lp = torch.cat([l for _, l in whole])
    assert torch.allclose(lp.exp().sum(-1), torch.ones(len(pos)), atol=1e-5)
    pieces = list(replay.assistant_logprobs(m, ids, mask, chunk=7))
    assert (np.concatenate([p for p, _ in pieces]) == pos).all()
    assert torch.allclose(torch.cat([l for _, l in pieces]), lp, atol=1e-5)


def test_ref_round_trip_and_kl_arithmetic(tmp_path):
    cap = write_capture(tmp_path / "s.jsonl")
    tok = CharTokenizer()
    ref_model, other = _toy(seed=0), _toy(seed=0, noise=0.3)
    out = tmp_path / "s.npz"
    replay.build_ref(ref_model, tok, cap, out, n_actions=2, max_new=6, model_id="toy")
    ref = np.load(out)
    assert ref["top_ids"].shape[1] == replay.TOPK and str(ref["model"]) == "toy"
    assert (np.diff(ref["top_lp"], axis=1) <= 0).all()  # descending
    same = replay.score(ref_model, out, chunk=5)
    assert same["kl_top64_mean"] < 1e-5 and same["top1_agree"] == 1.0
    assert same["ref_model"] == "toy" and same["assistant_tokens"] == len(ref["pos"])
    # the other model's truncated KL by hand, over its full log-softmax
    got = replay.score(other, out)
    full = torch.cat([l for _, l in replay.assistant_logprobs(other, ref["ids"], ref["mask"])])
    rlp = torch.from_numpy(ref["top_lp"])
    mlp = torch.gather(full, 1, torch.from_numpy(ref["top_ids"]).long())
    kl = (rlp.exp() * (rlp - mlp)).sum(1).numpy()
    agree = (full.argmax(1).numpy() == ref["top_ids"][:, 0]).mean()
    assert got["kl_top64_mean"] == pytest.approx(float(kl.mean()), rel=1e-5)
    assert got["kl_top64_p99"] == pytest.approx(float(np.percentile(kl, 99)), rel=1e-5)
    assert got["top1_agree"] == pytest.approx(float(agree))
    assert got["kl_top64_mean"] > 1e-3
    assert replay.score_actions(ref_model, tok, out) == 1.0


def test_forward_contract_and_position_check(tmp_path):
    cap = write_capture(tmp_path / "s.jsonl")
    m = _toy()
    out = tmp_path / "s.npz"
    replay.build_ref(m, CharTokenizer(), cap, out, n_actions=0)
    fwd = lambda x, c: m.lm_head(m._body(x, c)[0])[None]
    got = replay.score(None, out, make_cache=_Cache, forward=fwd)
    assert got["kl_top64_mean"] < 1e-5 and got["top1_agree"] == 1.0
    ref = dict(np.load(out))
    ref["pos"] = ref["pos"] + 1
    np.savez(tmp_path / "bad.npz", **ref)
    with pytest.raises(AssertionError, match="position mismatch"):
        replay.score(m, tmp_path / "bad.npz")


def test_load_needs_weight_shards(tmp_path):
    from lagunalab_b200 import laguna, pack, synth
    args = synth.decoder_args(vocab=512, hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128,
                              experts=8, top_k=2, moe_inter=128, shared_inter=128,
                              dense_inter=256)
    (tmp_path / "config.json").write_text(json.dumps(pack.model_config(args)))
    with pytest.raises(FileNotFoundError, match="safetensors"):
        laguna.load(tmp_path)
