"""The decoder over an 8-bit quantized KV cache (DequantKVCache with fused_decode,
laguna_mlx/cache.py:66-106) on the GPU.

Kernel level, bit for bit against the library's own separate steps: the attention prologue
that quantizes the new k/v rows straight into the packed cache equals the bf16 prologue
followed by the quantizer (host and device positions); the device-length q8 attention with the
fused head gate equals the host-length kernel times the gate when both plan for the same
length (and agrees within 1e-2 relative when the plan is longer than the valid length: the same
keys split differently, only the fp32 merge order changes). Model level: greedy decoding
against the oracle with the same 8-bit cache semantics (oracle/model_ref.py Cache(kv_bits=8)),
and graph-replayed decoding against eager decoding.
"""
import pytest
import torch

from oracle import model_ref
from tests._util import cos, rel_err

pytestmark = pytest.mark.gpu


def _tiny(seed=0):
    from lagunalab_b200 import synth
    args = synth.decoder_args(vocab=512, hidden=256, layers=3, heads=4, kv_heads=2, head_dim=128,
                              experts=8, top_k=2, moe_inter=128, shared_inter=128, dense_inter=256,
                              rope_theta=1e4)
    model = synth.decoder(args, seed=seed, std=0.05, norm_noise=0.1, router_bias_std=0.3)
    return args, model, synth.oracle_weights(model), synth.oracle_args(args)


def _packed(Hkv, cap, D, dev="cuda"):
    return (torch.zeros(1, Hkv, cap, D // 4, dtype=torch.int32, device=dev),
            torch.zeros(1, Hkv, cap, D // 64, dtype=torch.bfloat16, device=dev),
            torch.zeros(1, Hkv, cap, D // 64, dtype=torch.bfloat16, device=dev))


@pytest.mark.parametrize("T,pos,dev_pos", [(1, 37, False), (1, 255, True), (9, 0, False),
                                           (5, 100, False)])
def test_prologue_quantizes_rows_like_the_quantizer(T, pos, dev_pos):
    from lagunalab_b200 import ops
    Hq, Hkv, D, cap = 8, 2, 128, 256
    g = torch.Generator().manual_seed(T + pos)
    qkvg = (2 * torch.randn(T, (Hq + 2 * Hkv) * D + Hq, generator=g)).to(torch.bfloat16).cuda()
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).cuda()
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).cuda()
    pd = torch.tensor([pos], dtype=torch.int32).cuda() if dev_pos else None
    kc = torch.zeros(Hkv, cap, D, dtype=torch.bfloat16).cuda()
    vc = torch.zeros_like(kc)
    q1, g1 = ops.attn_prep(qkvg, Hq, Hkv, D, qn, kn, 1e-6, 1e4, kc, vc, pos=pos, pos_dev=pd)
    keys, values = _packed(Hkv, cap, D), _packed(Hkv, cap, D)
    q2, g2 = ops.attn_prep_q8(qkvg, Hq, Hkv, D, qn, kn, 1e-6, 1e4, keys, values, pos=pos,
                              pos_dev=pd)
    assert torch.equal(q1, q2) and torch.equal(g1, g2)
    rk, rv = _packed(Hkv, cap, D), _packed(Hkv, cap, D)
    ops.quantize_into(kc[None, :, pos:pos + T], rk, pos, 64, 8)
    ops.quantize_into(vc[None, :, pos:pos + T], rv, pos, 64, 8)
    for a, b in zip(keys + values, rk + rv):
        assert torch.equal(a, b)


@pytest.mark.parametrize("n,n_plan,G", [(300, 4096, 8), (4096, 4096, 8), (77, 9000, 4),
                                        (5000, 82944, 8)])
def test_device_length_attention_with_gate_equals_host_form(n, n_plan, G):
    from lagunalab_b200 import ops
    Hkv, D = 4, 128
    Hq = G * Hkv
    cap = n_plan
    g = torch.Generator(device="cuda")
    g.manual_seed(n)
    x = torch.randn(1, Hkv, cap, D, generator=g, device="cuda").to(torch.bfloat16)
    keys, values = _packed(Hkv, cap, D), _packed(Hkv, cap, D)
    ops.quantize_into(x, keys, 0, 64, 8)
    ops.quantize_into(x.flip(-1), values, 0, 64, 8)
    q = torch.randn(1, Hq, D, generator=g, device="cuda").to(torch.bfloat16)
    gate = torch.rand(1, Hq, generator=g, device="cuda").to(torch.bfloat16)
    want = ops.q8_decode_attention(q.view(1, Hq, 1, D), keys, values, n, D ** -0.5)
    want = (want.view(1, Hq, D) * gate.view(1, Hq, 1))
    nd = torch.tensor([n - 1], dtype=torch.int32, device="cuda")
    got = ops.q8_decode_attention_dev(q, keys, values, n_plan, nd, 1, D ** -0.5, gate=gate)
    plain = ops.q8_decode_attention_dev(q, keys, values, n_plan, nd, 1, D ** -0.5)
    host = ops.q8_decode_attention(q.view(1, Hq, 1, D), keys, values, n, D ** -0.5).view(1, Hq, D)
    if n == n_plan:  # the same work split: the same bits
        assert torch.equal(got, want)
        assert torch.equal(plain, host)
    else:  # a plan for more keys splits the same keys differently: fp32 merge order only
        assert rel_err(got, want) <= 1e-2 and cos(got, want) >= 0.9999
        assert rel_err(plain, host) <= 1e-2 and cos(plain, host) >= 0.9999
    # the gate is applied to the bf16 attention output (the kernel's own, same plan)
    assert torch.equal(got, (plain * gate.view(1, Hq, 1)))


def test_greedy_decode_with_quantized_cache_matches_oracle():
    from lagunalab_b200 import cache as qcache, laguna
    args, model, W, oargs = _tiny(7)
    prompt = torch.randint(0, 512, (11,), generator=torch.Generator().manual_seed(9))
    steps = 10
    c = qcache.make_quantized_cache(model, fused_decode=True, capacity=256)
    want, gaps = model_ref.greedy(W, oargs, prompt, steps, kv_bits=8)
    # teacher-forced: every step compared, a differing step only on an oracle near-tie
    from tests.test_decoder_gpu import _teacher_forced
    assert _teacher_forced(model, c, prompt, want, gaps) <= 2
    assert all(x.fused_step for x in c)  # the last step ran the fused q8 kernel


def test_graph_replayed_decode_with_quantized_cache_equals_eager():
    from lagunalab_b200 import cache as qcache, laguna, ops
    args, model, _, _ = _tiny(3)
    prompt = torch.randint(0, 512, (9,), generator=torch.Generator().manual_seed(4)).cuda()
    eager = laguna.generate(model, prompt, 8, qcache.make_quantized_cache(
        model, fused_decode=True, capacity=256))
    c = qcache.make_quantized_cache(model, fused_decode=True, capacity=256)
    tok = ops.argmax(model.last_logits(prompt.to(torch.int32).view(1, -1), c).view(1, -1))
    dg = laguna.DecodeGraph(model, c, tok)
    toks = [int(tok), int(dg.tok)]
    for _ in range(6):
        dg.step()
        toks.append(int(dg.tok))
    assert toks == eager
    assert dg.position() == 9 + 7
