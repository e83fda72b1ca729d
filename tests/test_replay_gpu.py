"""Replay scoring through the B200 decoder (lagunaLab replay/replay.py:23-124): a reference
built by the sm_100a engine scores against itself (whole and chunked prefill through one
cache), the CPU oracle decoder scored through the ``forward=`` contract against that
reference agrees within bf16 noise, and the stored greedy actions reproduce."""
import numpy as np
import pytest
import torch

from oracle import model_ref
from tests._replay_util import CharTokenizer, write_capture

pytestmark = pytest.mark.gpu


def _tiny():
    from lagunalab_b200 import synth
    args = synth.decoder_args(vocab=512, hidden=256, layers=3, heads=4, kv_heads=2, head_dim=128,
                              experts=8, top_k=2, moe_inter=128, shared_inter=128, dense_inter=256,
                              rope_theta=1e4)
    model = synth.decoder(args, seed=4, std=0.05, norm_noise=0.1, router_bias_std=0.3)
    return args, model, synth.oracle_weights(model), synth.oracle_args(args)


def _agrees_off_ties(ref, pieces, margin=0.05, min_frac=1.0):
    """Top-1 agrees with the reference wherever the reference's top-2 log-probs are more
    than ``margin`` apart, on at least ``min_frac`` of those positions (this random tiny
    model's logits are nearly flat, so bf16 rounding-order differences may flip near-ties;
    between two different engines a router near-tie can also flip an expert, which moves
    every later position of the sequence)."""
    lp = torch.cat([l.cpu() for _, l in pieces])
    clear = (ref["top_lp"][:, 0] - ref["top_lp"][:, 1]) > margin
    got = lp.argmax(-1).numpy()
    assert clear.sum() >= len(clear) // 2
    frac = float((got[clear] == ref["top_ids"][clear, 0]).mean())
    assert frac >= min_frac, f"top-1 agreement {frac:.3f} off near-ties"


def test_replay_scores_on_b200(tmp_path):
    from lagunalab_b200 import replay
    args, model, W, oargs = _tiny()
    tok = CharTokenizer(vocab=512)
    out = tmp_path / "s.npz"
    replay.build_ref(model, tok, write_capture(tmp_path / "s.jsonl"), out, n_actions=2,
                     max_new=4, model_id="tiny")
    ref = np.load(out)
    assert ref["top_ids"].shape == (len(ref["pos"]), replay.TOPK)

    same = replay.score(model, out)
    assert same["kl_top64_mean"] < 1e-4 and same["peak_mem_gb"] > 0
    _agrees_off_ties(ref, replay.assistant_logprobs(model, ref["ids"], ref["mask"]))
    chunked = replay.score(model, out, chunk=16)
    assert chunked["kl_top64_mean"] < 1e-3
    _agrees_off_ties(ref, replay.assistant_logprobs(model, ref["ids"], ref["mask"], chunk=16))

    n_layers = len(W["layers"])
    fwd = lambda x, c: model_ref.forward(W, oargs, x[0].long(), c)[None]
    mk = lambda: model_ref.Cache(n_layers)
    oracle = replay.score(None, out, make_cache=mk, forward=fwd)
    assert oracle["kl_top64_mean"] < 1e-2, oracle
    _agrees_off_ties(ref, replay.assistant_logprobs(None, ref["ids"], ref["mask"],
                                                    make_cache=mk, forward=fwd), min_frac=0.8)

    # the greedy actions replay on the same engine, which is deterministic (the prefill
    # combine sums each token's picks in a fixed order), so both match
    assert replay.score_actions(model, tok, out) == 1.0


def test_checkpoint_round_trip_scores_like_the_original(tmp_path):
    """``pack.save_checkpoint`` -> ``laguna.load`` (MLX checkpoint directory) gives a model
    that scores against the original's replay reference within bf16 noise."""
    from lagunalab_b200 import laguna, pack, replay
    args, model, W, oargs = _tiny()
    out = tmp_path / "s.npz"
    replay.build_ref(model, CharTokenizer(vocab=512), write_capture(tmp_path / "s.jsonl"), out,
                     n_actions=0)
    pack.save_checkpoint(model, tmp_path / "ckpt")
    loaded, tok = laguna.load(tmp_path / "ckpt")
    assert tok is None
    got = replay.score(loaded, out)
    assert got["kl_top64_mean"] < 1e-4, got
    ref = np.load(out)
    _agrees_off_ties(ref, replay.assistant_logprobs(loaded, ref["ids"], ref["mask"]))
