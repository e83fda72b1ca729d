"""Full Laguna decoder on the GPU vs the CPU oracle (oracle/model_ref.py, pinned to
Poolside's PyTorch model by tests/test_model_oracle_cpu.py).

Kernel level: RMSNorm (+ residual), the 4-bit decode GEMV, the quantized embedding, the
attention prologue (q/k norm, RoPE, cache append, gate), the bf16 split-KV decode attention
(host- and device-side lengths, GQA groups 2/8/16, the fused head gate) and argmax. Model
level: prefill logits, and greedy decoding token by token against the oracle's greedy
decoding (BASELINE: greedy decode tokens identical; a step whose oracle top-2 logits are
within a bf16 rounding of each other is reported as a near-tie and not counted).
"""
import ctypes

import pytest
import torch

from oracle import model_ref, moe_ref
from tests._util import COS_TOL, REL_TOL, cos, rel_err

pytestmark = pytest.mark.gpu


def _bf16_close(got, want, ulps=1):
    """Elementwise within `ulps` bf16 ulps of the oracle (rounding-order differences)."""
    got, want = got.float().cpu(), want.float().cpu()
    tol = ulps * torch.clamp(want.abs(), min=1e-30) * 2.0 ** -7 + 1e-30
    return bool(((got - want).abs() <= tol).all())


def test_rmsnorm_with_and_without_residual():
    from lagunalab_b200 import ops
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5, 2048, generator=g).to(torch.bfloat16)
    r = torch.randn(5, 2048, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16)
    got = ops.rmsnorm(x.cuda(), w.cuda(), 1e-6)
    assert _bf16_close(got, model_ref.rmsnorm(x.float(), w.float(), 1e-6))
    h, got = ops.rmsnorm(x.cuda(), w.cuda(), 1e-6, residual=r.cuda())
    hw = (x.float() + r.float()).to(torch.bfloat16).float()
    assert torch.equal(h.float().cpu(), hw)
    assert _bf16_close(got, model_ref.rmsnorm(hw, w.float(), 1e-6))


@pytest.mark.parametrize("T,K,N", [(1, 2048, 5152), (3, 4096, 2048), (16, 2048, 100), (9, 8192, 2048),
                                   (17, 2048, 1000), (40, 4096, 2048), (64, 2048, 5152)])
def test_qlinear_decode_gemv(T, K, N):
    from lagunalab_b200 import ops
    from tests._util import quant_np
    g = torch.Generator().manual_seed(T + K + N)
    w = torch.randn(N, K, generator=g) * 0.02
    mat = quant_np(w, 4)
    x = torch.randn(T, K, generator=g).to(torch.bfloat16)
    res = torch.randn(T, N, generator=g).to(torch.bfloat16)
    want = moe_ref.qlinear(x, mat)
    got = ops.qlinear(x.cuda(), tuple(t.cuda() for t in mat))
    assert rel_err(got, want) <= 1e-2 and cos(got, want) >= 0.9999
    got = ops.qlinear(x.cuda(), tuple(t.cuda() for t in mat), residual=res.cuda())
    want = (want + res.float()).to(torch.bfloat16).float()
    assert rel_err(got, want) <= 1e-2


def test_embedding_rows():
    from lagunalab_b200 import ops
    from tests._util import quant_np
    g = torch.Generator().manual_seed(1)
    table = quant_np(torch.randn(1000, 256, generator=g) * 0.5, 4)
    ids = torch.tensor([0, 999, 17, 17, 512], dtype=torch.int32)
    got = ops.embed(ids.cuda(), tuple(t.cuda() for t in table))
    want = moe_ref.dequantize(*table, 64, 4)[ids.long()]
    assert _bf16_close(got, want)
    bad = ops.embed(torch.tensor([1000, -1], dtype=torch.int32, device="cuda"),
                    tuple(t.cuda() for t in table))
    assert torch.isnan(bad.float()).all()


@pytest.mark.parametrize("T,pos", [(1, 0), (1, 300), (7, 0), (5, 11)])
def test_attention_prologue(T, pos):
    from lagunalab_b200 import ops
    Hq, Hkv, D, cap = 8, 2, 128, 512
    g = torch.Generator().manual_seed(T * 100 + pos)
    qkvg = (torch.randn(T, (Hq + 2 * Hkv) * D + Hq, generator=g)).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    kc = torch.zeros(Hkv, cap, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    q, gate = ops.attn_prep(qkvg.cuda(), Hq, Hkv, D, qn.cuda(), kn.cuda(), 1e-6, 1e6, kc, vc, pos=pos)
    x = qkvg.float()
    qw = x[:, :Hq * D].view(T, Hq, D).transpose(0, 1)
    kw = x[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D).transpose(0, 1)
    vw = x[:, (Hq + Hkv) * D:(Hq + 2 * Hkv) * D].view(T, Hkv, D).transpose(0, 1)
    qr = model_ref.rope(model_ref.rmsnorm(qw, qn.float(), 1e-6), pos, 1e6)
    kr = model_ref.rope(model_ref.rmsnorm(kw, kn.float(), 1e-6), pos, 1e6)
    assert _bf16_close(q, qr, ulps=2)
    assert _bf16_close(kc[:, pos:pos + T], kr, ulps=2)
    assert torch.equal(vc[:, pos:pos + T].float().cpu(), vw)
    assert kc[:, :pos].abs().sum() == 0 and kc[:, pos + T:].abs().sum() == 0
    gw = model_ref.softplus(x[:, (Hq + 2 * Hkv) * D:])
    assert _bf16_close(gate, gw.to(torch.bfloat16).float())


def _kv(B, Hkv, cap, seed):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, Hkv, cap, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, cap, 128, generator=g).to(torch.bfloat16)
    return k, v


@pytest.mark.parametrize("n,G,B", [(1, 8, 1), (15, 8, 1), (17, 2, 1), (1000, 8, 1),
                                   (8448, 8, 1), (3000, 16, 1), (700, 8, 3)])
def test_bf16_decode_attention(n, G, B):
    from lagunalab_b200 import ops
    Hkv = 4 if B == 1 else 2
    Hq = G * Hkv
    cap = (n + 255) // 256 * 256 + 256
    k, v = _kv(B, Hkv, cap, seed=n + G)
    g = torch.Generator().manual_seed(n)
    q = torch.randn(B, Hq, 128, generator=g).to(torch.bfloat16)
    gate = torch.nn.functional.softplus(torch.randn(B, Hq, generator=g)).to(torch.bfloat16)
    scale = 128 ** -0.5
    got = ops.bf16_decode_attention(q.cuda(), k.cuda(), v.cuda(), n, scale, gate=gate.cuda())
    for b in range(B):
        o = model_ref.sdpa(q[b].float()[:, None], k[b, :, :n].float(), v[b, :, :n].float(), scale, n - 1)
        want = (o[:, 0] * gate[b].float()[:, None]).to(torch.bfloat16).float()
        assert rel_err(got[b], want) <= REL_TOL and cos(got[b], want) >= COS_TOL, b
        assert (got[b].float().cpu() - want).abs().max() < 2e-2


def test_bf16_decode_attention_device_length_and_repeat():
    from lagunalab_b200 import ops
    Hkv, G, cap = 4, 8, 4096
    k, v = _kv(1, Hkv, cap, seed=3)
    q = torch.randn(1, Hkv * G, 128, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    pos = torch.tensor([2999], dtype=torch.int32, device="cuda")  # n = pos + 1
    for _ in range(3):
        got = ops.bf16_decode_attention(q.cuda(), k.cuda(), v.cuda(), 0, 0.1, n_dev=pos, n_add=1)
        o = model_ref.sdpa(q[0].float()[:, None], k[0, :, :3000].float(), v[0, :, :3000].float(), 0.1, 2999)
        assert rel_err(got[0], o[:, 0]) <= REL_TOL


def test_argmax_first_max_and_position():
    from lagunalab_b200 import ops
    x = torch.randn(3, 100352, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
    x[1, 5] = x[1, 70000] = 100.0  # a tie: first index wins
    pos = torch.tensor([41], dtype=torch.int32, device="cuda")
    ids = ops.argmax(x.cuda(), pos=pos, inc=1)
    assert ids.tolist() == [int(torch.argmax(x[0].float())), 5, int(torch.argmax(x[2].float()))]
    assert int(pos) == 42


def _tiny(seed=0):
    from lagunalab_b200 import synth
    args = synth.decoder_args(vocab=512, hidden=256, layers=3, heads=4, kv_heads=2, head_dim=128,
                              experts=8, top_k=2, moe_inter=128, shared_inter=128, dense_inter=256,
                              rope_theta=1e4)
    model = synth.decoder(args, seed=seed, std=0.05, norm_noise=0.1, router_bias_std=0.3)
    return args, model, synth.oracle_weights(model), synth.oracle_args(args)


def test_model_prefill_logits():
    args, model, W, oargs = _tiny(0)
    ids = torch.randint(0, 512, (12,), generator=torch.Generator().manual_seed(1))
    got = model(ids.cuda().to(torch.int32), model.make_cache())[0]
    want = model_ref.forward(W, oargs, ids)
    assert rel_err(got, want) <= REL_TOL and cos(got, want) >= COS_TOL


def _teacher_forced(model, cache, prompt, toks, gaps, near_tie=0.02):
    """Feed the oracle's greedy tokens one at a time and compare the engine's argmax at every
    step: a step may differ only where the oracle's top-2 logit margin is a near-tie. Returns
    the number of differing steps."""
    from lagunalab_b200 import ops
    logits = model.last_logits(prompt.cuda().to(torch.int32).view(1, -1), cache)
    flips = 0
    for i, t in enumerate(toks):
        got = int(ops.argmax(logits.view(1, -1)))
        if got != t:
            assert gaps[i] < near_tie, f"step {i}: {got} != {t} (oracle margin {gaps[i]:.4f})"
            flips += 1
        logits = model.last_logits(torch.tensor([[t]], dtype=torch.int32, device="cuda"), cache)
    return flips


def test_model_greedy_decode_matches_oracle():
    """Teacher-forced against the oracle's greedy decode: every one of 16 steps is compared
    (the engine is fed the oracle's previous token, so a near-tie flip does not end the
    comparison); at most 2 steps may differ, each on a near-tie."""
    args, model, W, oargs = _tiny(2)
    prompt = torch.randint(0, 512, (9,), generator=torch.Generator().manual_seed(3))
    toks, gaps = model_ref.greedy(W, oargs, prompt, 16)
    assert _teacher_forced(model, model.make_cache(), prompt, toks, gaps) <= 2


def test_graph_replayed_decode_equals_eager_decode():
    """DecodeGraph (token id and position on the device, one replay per token) produces the
    same greedy tokens as eager decoding."""
    from lagunalab_b200 import laguna, ops
    args, model, _, _ = _tiny(4)
    prompt = torch.randint(0, 512, (9,), generator=torch.Generator().manual_seed(5)).cuda()
    eager = laguna.generate(model, prompt, 8)
    cache = model.make_cache(capacity=256)
    logits = model.last_logits(prompt.to(torch.int32).view(1, -1), cache)
    tok = ops.argmax(logits.view(1, -1))
    dg = laguna.DecodeGraph(model, cache, tok)
    toks = [int(tok), int(dg.tok)]
    for _ in range(6):
        dg.step()
        toks.append(int(dg.tok))
    assert toks == eager
    assert dg.position() == 9 + 7


def test_decode_with_dependent_launch_equals_plain_launch():
    """The same decode steps eagerly with programmatic dependent launch on and off, and a
    graph captured without it: identical tokens."""
    from lagunalab_b200 import _lib, laguna, ops
    args, model, _, _ = _tiny(6)
    prompt = torch.randint(0, 512, (7,), generator=torch.Generator().manual_seed(8)).cuda()
    plain = laguna.generate(model, prompt, 6)
    prev = _lib.lib().lg_set_pdl(1)
    try:
        with_pdl = laguna.generate(model, prompt, 6)
    finally:
        _lib.lib().lg_set_pdl(prev)
    assert with_pdl == plain
    cache = model.make_cache(capacity=256)
    tok = ops.argmax(model.last_logits(prompt.to(torch.int32).view(1, -1), cache).view(1, -1))
    dg = laguna.DecodeGraph(model, cache, tok, pdl=False)
    toks = [int(tok), int(dg.tok)]
    for _ in range(4):
        dg.step()
        toks.append(int(dg.tok))
    assert toks == plain
