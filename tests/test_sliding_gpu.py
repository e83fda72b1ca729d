"""Sliding-window layers and YaRN / partial-rotary RoPE on the GPU (laguna_mlx/laguna.py:62-72,
:183-186, :209-214; the real XS 2.1 layer mix) against the oracle, whose forms
tests/test_model_oracle_cpu.py pins to the vendored PyTorch model.

A 4-layer model (full, sliding, sliding, full; window 16): full layers use YaRN with half of
the 128 head dims rotated, sliding layers the default rope; every sequence runs past the
window. Checks: prefill logits, a prefill split in two (the window's previous rows carried
over), greedy decoding teacher-forced against the oracle (every step compared; a differing
token only where the oracle's top-2 margin is a near-tie), graph-replayed decoding (ring rows
written at position mod window on the device) equal to eager decoding, and the 8-bit cache
whose sliding layers keep their bf16 window.
"""
import pytest
import torch

from oracle import model_ref
from tests._util import COS_TOL, cos, rel_err

pytestmark = pytest.mark.gpu

YARN = {"rope_theta": 500000.0, "rope_type": "yarn", "factor": 32.0,
        "original_max_position_embeddings": 8192, "beta_slow": 1.0, "beta_fast": 64.0,
        "attention_factor": 1.3465735902799727, "partial_rotary_factor": 0.5}
ROPE = {"full_attention": YARN,
        "sliding_attention": {"rope_type": "default", "rope_theta": 10000.0,
                              "partial_rotary_factor": 1.0}}
W = 16
NEAR_TIE = 0.05  # logit margin below which a routing-flip may change the token


def _model(seed=0, window=W):
    from lagunalab_b200 import synth
    args = synth.decoder_args(vocab=512, hidden=256, layers=4, heads=4, kv_heads=2,
                              head_dim=128, experts=8, top_k=2, moe_inter=128, shared_inter=128,
                              dense_inter=256, rope_parameters=ROPE, sliding_window=window,
                              layer_types=["full_attention", "sliding_attention",
                                           "sliding_attention", "full_attention"],
                              heads_per_layer=[4, 4, 8, 4])
    model = synth.decoder(args, seed=seed, std=0.05, norm_noise=0.1, router_bias_std=0.3)
    return args, model, synth.oracle_weights(model), synth.oracle_args(args)


def _ids(n, seed):
    return torch.randint(0, 512, (n,), generator=torch.Generator().manual_seed(seed))


def test_prefill_logits_past_the_window():
    """Logits of every position within 3e-2 of the largest oracle logit (four layers of bf16
    rounding: measured 0.011-0.024), but for at most 2 of 40 positions: a router whose 2nd
    and 3rd scores nearly tie may pick another expert for one token (measured: one position
    at 0.27)."""
    args, model, Wt, oa = _model(0)
    ids = _ids(40, 1)
    got = model(ids.cuda().to(torch.int32), model.make_cache())[0].float().cpu()
    want = model_ref.forward(Wt, oa, ids, model_ref.Cache(4))
    per_pos = (got - want).abs().max(-1).values / want.abs().max()
    keep = per_pos <= 3e-2
    assert int((~keep).sum()) <= 2, per_pos
    # the flipped positions are excluded from the cosine too: one of them alone pulls the
    # whole tensor's cosine to 0.9988
    assert cos(got[keep], want[keep]) >= COS_TOL


def test_prefill_in_two_parts_equals_one():
    args, model, _, _ = _model(1)
    ids = _ids(41, 2).cuda().to(torch.int32)
    one = model.last_logits(ids.view(1, -1), model.make_cache())
    c = model.make_cache()
    model.last_logits(ids[:23].view(1, -1), c)
    two = model.last_logits(ids[23:].view(1, -1), c)
    assert all(x.offset == 41 for x in c)
    # the two parts (23 and 18 tokens) take the decode-size linears, the whole prompt the
    # dequantized GEMM: the same fp32-accumulated values up to summation order
    assert rel_err(two, one) <= 2e-2 and cos(two, one) >= 0.9999


def _teacher_forced(model, cache, prompt, toks, gaps):
    from lagunalab_b200 import ops
    logits = model.last_logits(prompt.cuda().to(torch.int32).view(1, -1), cache)
    flips = 0
    for i, t in enumerate(toks):
        got = int(ops.argmax(logits.view(1, -1)))
        if got != t:
            assert gaps[i] < NEAR_TIE, f"step {i}: {got} != {t} (oracle margin {gaps[i]:.4f})"
            flips += 1
        logits = model.last_logits(torch.tensor([[t]], dtype=torch.int32, device="cuda"), cache)
    return flips


def test_greedy_decode_teacher_forced_matches_oracle():
    args, model, Wt, oa = _model(2)
    prompt = _ids(21, 3)
    toks, gaps = model_ref.greedy(Wt, oa, prompt, 24)
    flips = _teacher_forced(model, model.make_cache(), prompt, toks, gaps)
    assert flips <= 2


def test_graph_replayed_decode_equals_eager_on_sliding_layers():
    from lagunalab_b200 import laguna, ops
    args, model, _, _ = _model(3)
    prompt = _ids(19, 4).cuda()
    eager = laguna.generate(model, prompt, 22)
    cache = model.make_cache(capacity=256)
    tok = ops.argmax(model.last_logits(prompt.to(torch.int32).view(1, -1), cache).view(1, -1))
    dg = laguna.DecodeGraph(model, cache, tok)
    toks = [int(tok), int(dg.tok)]
    for _ in range(20):
        dg.step()
        toks.append(int(dg.tok))
    assert toks == eager
    assert ops.decode_status() == (0, 0, 0, 0)


def test_graph_replayed_decode_with_a_multi_tile_window():
    """A 48-row window spans three 16-key attention tiles: once the ring has wrapped, the
    newest row sits in any of them, and the graph-replayed step (programmatic dependent launch:
    the attention streams tiles before the prologue that appends the newest row finishes) must
    not read that row early. Tokens equal eager decoding over 70 steps past the window."""
    from lagunalab_b200 import laguna, ops
    args, model, _, _ = _model(5, window=48)
    prompt = _ids(30, 6).cuda()
    eager = laguna.generate(model, prompt, 72)
    cache = model.make_cache(capacity=256)
    tok = ops.argmax(model.last_logits(prompt.to(torch.int32).view(1, -1), cache).view(1, -1))
    dg = laguna.DecodeGraph(model, cache, tok)
    toks = [int(tok), int(dg.tok)]
    for _ in range(70):
        dg.step()
        toks.append(int(dg.tok))
    assert toks == eager


def test_quantized_cache_keeps_bf16_windows():
    from lagunalab_b200 import cache as qcache, laguna
    args, model, Wt, oa = _model(4)
    c = qcache.make_quantized_cache(model, fused_decode=True, capacity=256)
    assert [type(x).__name__ for x in c] == ["DequantKVCache", "RotatingKVCache",
                                             "RotatingKVCache", "DequantKVCache"]
    prompt = _ids(20, 5)
    toks, gaps = model_ref.greedy(Wt, oa, prompt, 20, kv_bits=[8, None, None, 8])
    flips = _teacher_forced(model, c, prompt, toks, gaps)
    assert flips <= 2
