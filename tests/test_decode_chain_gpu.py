"""One-token decode kernels (lg_decode_gemv, lg_router_decode, lg_moe_decode) on the GPU.

Against the oracle (oracle/moe_ref.py) on the same packed weights: the dense GEMV with and
without the fused input RMSNorm / residual / SwiGLU pair, at sizes that take one tile per CTA,
a ring of staged tiles per CTA, and a partial last tile. Against the standalone kernels,
bit for bit: the fused norm gives the same bits as lg_rmsnorm followed by the GEMV, and the
fused router the same normalised input, logits, picks and weights as lg_rmsnorm followed by
lg_router_topk. The fused experts against the oracle's
SwitchGLU + combine + shared expert + residual, with and without a shared expert, with an
empty pick, and at the bs1 decode shapes of the 64- and 128-expert models.
"""
import pytest
import torch

from oracle import moe_ref
from tests._util import COS_TOL, REL_TOL, cos, gen, quant_np, rel_err

pytestmark = pytest.mark.gpu


def _mat(N, K, seed, std=0.02, bits=4):
    g = gen(seed)
    return quant_np(torch.randn(N, K, generator=g) * std, bits)


def _cuda(m):
    return tuple(t.cuda() for t in m)


@pytest.mark.parametrize("K,N", [(2048, 5152), (4096, 2048), (256, 37), (8192, 2048),
                                 (2048, 24013), (1024, 100)])
def test_decode_gemv_plain_and_residual(K, N):
    from lagunalab_b200 import ops
    mat = _mat(N, K, K + N)
    g = gen(N)
    x = torch.randn(1, K, generator=g).to(torch.bfloat16)
    res = torch.randn(1, N, generator=g).to(torch.bfloat16)
    want = moe_ref.qlinear(x, mat)
    got = ops.decode_gemv(x.cuda(), _cuda(mat))
    assert rel_err(got, want) <= 1e-2 and cos(got, want) >= 0.9999
    got = ops.decode_gemv(x.cuda(), _cuda(mat), residual=res.cuda())
    want = (want + res.float()).to(torch.bfloat16).float()
    assert rel_err(got, want) <= 1e-2
    assert ops.decode_status() == (0, 0, 0, 0)


@pytest.mark.parametrize("K,N", [(2048, 5152), (256, 40), (2048, 100352)])
def test_decode_gemv_fused_norm_is_bitwise_the_two_kernel_form(K, N):
    from lagunalab_b200 import ops
    mat = _cuda(_mat(N, K, 7 + N))
    g = gen(K)
    x = (3 * torch.randn(1, K, generator=g)).to(torch.bfloat16).cuda()
    w = (1 + 0.2 * torch.randn(K, generator=g)).to(torch.bfloat16).cuda()
    two = ops.decode_gemv(ops.rmsnorm(x, w, 1e-6), mat)
    one = ops.decode_gemv(x, mat, norm=(w, 1e-6))
    assert torch.equal(one, two)


@pytest.mark.parametrize("K,N", [(2048, 8192), (256, 48), (512, 200)])
def test_decode_gemv_swiglu_pair(K, N):
    from lagunalab_b200 import ops
    gm, um = _mat(N, K, 1), _mat(N, K, 2)
    g = gen(3)
    x = torch.randn(1, K, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    xn = ops.rmsnorm(x.cuda(), w.cuda(), 1e-6)
    got = ops.decode_gemv(x.cuda(), _cuda(gm), norm=(w.cuda(), 1e-6), up=_cuda(um))
    gv = moe_ref.qlinear(xn.cpu(), gm)
    uv = moe_ref.qlinear(xn.cpu(), um)
    want = moe_ref._bf(moe_ref.silu_bf16(gv) * uv)
    assert rel_err(got, want) <= 1e-2 and cos(got, want) >= 0.9999


@pytest.mark.parametrize("E,k,H,score", [(64, 8, 2048, "sigmoid"), (8, 2, 256, "sigmoid"),
                                         (64, 8, 2048, "softmax"), (128, 8, 1024, "sigmoid")])
def test_router_decode_is_bitwise_norm_plus_router(E, k, H, score):
    from lagunalab_b200 import ops
    g = gen(E + H)
    h = (2 * torch.randn(1, H, generator=g)).to(torch.bfloat16).cuda()
    nw = (1 + 0.2 * torch.randn(H, generator=g)).to(torch.bfloat16).cuda()
    gate = _cuda(_mat(E, H, E, std=0.05, bits=8))
    bias = 0.3 * torch.randn(E, generator=g)
    bias[::7] = float("-inf")  # pruned experts
    bias = bias.cuda()
    xn, inds, w, lg = ops.router_decode(h, nw, 1e-6, gate, bias, k, True, score, logits=True)
    xn2 = ops.rmsnorm(h, nw, 1e-6)
    inds2, w2, lg2 = ops.router_topk(xn2, gate, bias, k, True, score)
    assert torch.equal(xn, xn2)
    assert torch.equal(lg, lg2)
    assert torch.equal(inds, inds2) and torch.equal(w, w2)
    assert ops.decode_status() == (0, 0, 0, 0)


def _stack(mats):
    return tuple(torch.stack([m[i] for m in mats]) for i in range(3))


def _gpu_mats(gc, *shape):
    from lagunalab_b200 import ops
    return ops.quantize(torch.randn(*shape, device="cuda", generator=gc) * 0.02, 64, 4)


@pytest.mark.parametrize("E,k,H,I,Ish,scale", [(64, 8, 2048, 1024, 1024, 1.0),
                                               (128, 8, 2048, 1024, 1024, 2.5),
                                               (8, 2, 256, 128, 128, 2.5),
                                               (16, 4, 512, 256, 0, 1.0),
                                               (16, 4, 256, 128, 192, 1.0)])
def test_moe_decode_matches_oracle(E, k, H, I, Ish, scale):
    from lagunalab_b200 import ops
    gc = torch.Generator(device="cuda")
    gc.manual_seed(E * 3 + H)
    experts = tuple(_gpu_mats(gc, E, *shp) for shp in ((I, H), (I, H), (H, I)))
    shared = tuple(_gpu_mats(gc, *shp) for shp in ((Ish, H), (Ish, H), (H, Ish))) if Ish else None
    g = gen(E + H)
    xn = torch.randn(1, H, generator=g).to(torch.bfloat16)
    res = torch.randn(1, H, generator=g).to(torch.bfloat16)
    inds = torch.randperm(E, generator=g)[:k].to(torch.int32).view(1, k)
    w = torch.rand(1, k, generator=g).to(torch.bfloat16)
    got = ops.moe_decode(xn.cuda(), inds.cuda(), w.cuda(), scale, experts, shared,
                         residual=res.cuda())
    # oracle on the picked experts only (re-indexed 0..k-1)
    sub = [tuple(t[inds[0].long().cuda()].cpu() for t in m) for m in experts]
    y = moe_ref.switch_glu(xn, torch.arange(k).view(1, k), *sub)
    sh = moe_ref.mlp(xn, *(tuple(t.cpu() for t in m) for m in shared)) if shared \
        else torch.zeros(1, H)
    moe = moe_ref.combine(y, w, scale, sh)
    want = (moe + res.float()).to(torch.bfloat16).float()
    assert rel_err(got, want) <= REL_TOL and cos(got, want) >= COS_TOL
    got0 = ops.moe_decode(xn.cuda(), inds.cuda(), w.cuda(), scale, experts, shared)
    assert rel_err(got0, moe) <= REL_TOL and cos(got0, moe) >= COS_TOL
    assert ops.decode_status() == (0, 0, 0, 0)


def test_moe_decode_skips_an_empty_pick():
    """A pick outside [0, E) contributes nothing (the general expert path's rule)."""
    from lagunalab_b200 import ops
    E, k, H, I = 8, 3, 256, 128
    g = gen(11)
    qm = lambda *s: quant_np(torch.randn(*s, generator=g) * 0.02)
    gate = _stack([qm(I, H) for _ in range(E)])
    up = _stack([qm(I, H) for _ in range(E)])
    down = _stack([qm(H, I) for _ in range(E)])
    xn = torch.randn(1, H, generator=g).to(torch.bfloat16)
    w = torch.rand(1, k, generator=g).to(torch.bfloat16)
    inds = torch.tensor([[3, -1, 5]], dtype=torch.int32)
    mats = tuple(map(_cuda, (gate, up, down)))
    got = ops.moe_decode(xn.cuda(), inds.cuda(), w.cuda(), 1.0, mats)
    inds2 = torch.tensor([[3, 5]], dtype=torch.int32)
    w2 = w[:, [0, 2]].contiguous()
    want = ops.moe_decode(xn.cuda(), inds2.cuda(), w2.cuda(), 1.0, mats)
    assert torch.equal(got, want)


def test_one_token_model_step_equals_general_path():
    """A decoder layer's one-token MLP sub-block (fused norm, router, experts, combine,
    residual) against the module path the prefill uses on the same input (rmsnorm, route,
    moe_experts / qmlp, bf16 residual add)."""
    from lagunalab_b200 import synth
    args = synth.decoder_args(vocab=512, hidden=2048, layers=2, heads=32, kv_heads=4,
                              head_dim=128, experts=64, top_k=8, moe_inter=1024,
                              shared_inter=1024, dense_inter=2048, rope_theta=1e6)
    model = synth.decoder(args, seed=3, std=0.02, norm_noise=0.1, router_bias_std=0.3)
    g = gen(5)
    h = (torch.randn(1, 1, 2048, generator=g)).to(torch.bfloat16).cuda()
    for layer in model.layers:  # layer 0 dense, layer 1 MoE
        got = layer.mlp.token(h, layer.post_attention_layernorm)
        assert got is not None
        want = h + layer.mlp(layer.post_attention_layernorm(h))
        assert rel_err(got, want) <= REL_TOL and cos(got, want) >= COS_TOL


def test_routing_hooks_still_see_decode_steps():
    """With the routing recorder installed, one-token steps go through ``route`` (counts grow
    by k per MoE layer and token)."""
    from lagunalab_b200 import hooks, laguna, synth
    args = synth.decoder_args(vocab=512, hidden=256, layers=3, heads=4, kv_heads=2, head_dim=128,
                              experts=8, top_k=2, moe_inter=128, shared_inter=128,
                              dense_inter=256, rope_theta=1e4)
    model = synth.decoder(args, seed=0, std=0.05)
    prompt = torch.arange(5, dtype=torch.int32).cuda()
    with hooks.RoutingRecorder(model) as rec:
        laguna.generate(model, prompt, 3)
    for c in rec.counts.values():
        assert c.sum() == (5 + 3) * 2  # prefill tokens + three one-token steps, k = 2


def test_moe_decode_workspace_shared_by_growing_sizes():
    """Calls of growing hidden size share one workspace: each finds its completion counters
    zeroed (a small call's outputs never land where a larger call keeps counters)."""
    from lagunalab_b200 import ops
    outs = []
    for H in (256, 512, 2048):
        gc = torch.Generator(device="cuda")
        gc.manual_seed(H)
        experts = tuple(_gpu_mats(gc, 8, *shp) for shp in ((128, H), (128, H), (H, 128)))
        xn = torch.randn(1, H, generator=gen(H)).to(torch.bfloat16).cuda()
        inds = torch.tensor([[1, 6]], dtype=torch.int32).cuda()
        w = torch.tensor([[0.7, 0.3]]).to(torch.bfloat16).cuda()
        got = ops.moe_decode(xn, inds, w, 1.0, experts)
        y = moe_ref.switch_glu(xn.cpu(), torch.arange(2).view(1, 2),
                               *[tuple(t[inds[0].long()].cpu() for t in m) for m in experts])
        want = moe_ref.combine(y, w.cpu(), 1.0, torch.zeros(1, H))
        assert rel_err(got, want) <= REL_TOL and cos(got, want) >= COS_TOL, H
