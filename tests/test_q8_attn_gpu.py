"""Fused 8-bit KV decode attention vs the oracle (laguna_mlx/q8_attn.py:102-130).

Mirrors lagunaLab tests/test_q8_attn.py:19-31: lengths 1, 7, BLOCK, BLOCK+1, 3*BLOCK+100 on
48 query / 8 KV heads with buffers longer than n, max abs error < 2e-2; plus BASELINE
config 4's 32/4 heads (G = 8, which the reference Metal kernel refuses) at 82,671 keys."""
import ctypes

import pytest
import torch

from oracle import attn_ref
from tests._util import COS_TOL, REL_TOL, cos, rel_err

pytestmark = pytest.mark.gpu


def _cache(B, hkv, n, cap, seed):
    from lagunalab_b200 import ops
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, hkv, cap, 128, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, hkv, cap, 128, generator=g).to(torch.bfloat16).cuda()
    mk = lambda: (torch.zeros(B, hkv, cap, 32, dtype=torch.int32, device="cuda"),
                  torch.zeros(B, hkv, cap, 2, dtype=torch.bfloat16, device="cuda"),
                  torch.zeros(B, hkv, cap, 2, dtype=torch.bfloat16, device="cuda"))
    kt, vt = mk(), mk()
    ops.quantize_into(k[:, :, :n], kt, 0, 64, 8)
    ops.quantize_into(v[:, :, :n], vt, 0, 64, 8)
    return kt, vt


@pytest.mark.parametrize("n", [1, 7, 512, 513, 3 * 512 + 100])
def test_matches_dequantize_then_attention(n):
    from lagunalab_b200.q8_attn import q8_decode_attention
    cap = (n + 255) // 256 * 256 + 256   # buffers longer than n: the kernel must stop at n
    kt, vt = _cache(1, 8, n, cap, seed=n)
    q = torch.randn(1, 48, 1, 128, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    scale = 128 ** -0.5
    got = q8_decode_attention(q.cuda(), kt, vt, n, scale)
    want = attn_ref.q8_decode_attention_ref(q.float(), tuple(t.cpu() for t in kt),
                                            tuple(t.cpu() for t in vt), n, scale)
    assert got.shape == q.shape and got.dtype == q.dtype
    assert (got.cpu().float() - want.float()).abs().max() < 2e-2


@pytest.mark.parametrize("n,B", [(82671, 1), (5000, 2), (300, 3)])
def test_gqa8_config4_shape(n, B):
    from lagunalab_b200.q8_attn import q8_decode_attention
    cap = (n + 255) // 256 * 256
    kt, vt = _cache(B, 4, n, cap, seed=n + B)
    q = torch.randn(B, 32, 1, 128, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    got = q8_decode_attention(q.cuda(), kt, vt, n, 128 ** -0.5)
    want = attn_ref.q8_decode_attention_ref(q.float(), tuple(t.cpu() for t in kt),
                                            tuple(t.cpu() for t in vt), n, 128 ** -0.5)
    assert (got.cpu().float() - want.float()).abs().max() < 2e-2
    assert rel_err(got, want) <= REL_TOL and cos(got, want) >= COS_TOL


@pytest.mark.parametrize("G", [1, 2, 6, 16])
def test_other_group_sizes(G):
    from lagunalab_b200.q8_attn import q8_decode_attention
    n = 1000
    kt, vt = _cache(1, 2, n, 1024, seed=G)
    q = torch.randn(1, 2 * G, 1, 128, generator=torch.Generator().manual_seed(G)).to(torch.bfloat16)
    got = q8_decode_attention(q.cuda(), kt, vt, n, 0.1)
    want = attn_ref.q8_decode_attention_ref(q.float(), tuple(t.cpu() for t in kt),
                                            tuple(t.cpu() for t in vt), n, 0.1)
    assert (got.cpu().float() - want.float()).abs().max() < 2e-2


def test_peaked_scores_and_repeat_calls():
    """A near one-hot softmax and repeated calls on the same workspace (counters reset)."""
    from lagunalab_b200.q8_attn import q8_decode_attention
    n = 4097
    kt, vt = _cache(1, 4, n, 4352, seed=3)
    q = (torch.randn(1, 32, 1, 128, generator=torch.Generator().manual_seed(9)) * 8).to(torch.bfloat16)
    want = attn_ref.q8_decode_attention_ref(q.float(), tuple(t.cpu() for t in kt),
                                            tuple(t.cpu() for t in vt), n, 128 ** -0.5)
    for _ in range(3):
        got = q8_decode_attention(q.cuda(), kt, vt, n, 128 ** -0.5)
        assert (got.cpu().float() - want.float()).abs().max() < 2e-2


def test_fused_cache_decode_matches_dequant_path():
    """DequantKVCache: fused single-token attend() vs the dequantize path on the same cache."""
    from lagunalab_b200.cache import DequantKVCache
    g = torch.Generator().manual_seed(0)
    kv = lambda L: torch.randn(1, 4, L, 128, generator=g).to(torch.bfloat16).cuda()
    fused, plain = DequantKVCache(fused_decode=True), DequantKVCache()
    k0, v0 = kv(300), kv(300)
    for c in (fused, plain):
        c.update_and_fetch(k0, v0)
    for step in range(3):
        k1, v1 = kv(1), kv(1)
        fused.update_and_fetch(k1, v1)
        kd, vd = plain.update_and_fetch(k1, v1)
        assert fused.fused_step and not plain.fused_step
        q = torch.randn(1, 32, 1, 128, generator=g).to(torch.bfloat16).cuda()
        got = fused.attend(q, 128 ** -0.5)
        want = attn_ref.sdpa_decode_ref(q.cpu(), kd.cpu(), vd.cpu(), kd.shape[2], 128 ** -0.5)
        assert (got.cpu().float() - want.float()).abs().max() < 2e-2
    assert fused.offset == 303 and fused.q.keys[0].shape[2] == 512


def test_one_workspace_serves_mixed_shapes():
    """One zeroed workspace, calls of different (batch, kv head) counts in turn: each call
    must find its completion counters at zero wherever the previous call put its partials."""
    from lagunalab_b200 import _lib
    shapes = [(1, 4, 32, 20000), (4, 8, 64, 3000), (1, 2, 16, 9000), (4, 8, 64, 3000),
              (1, 4, 32, 20000)]
    need = max(_lib.lib().lg_q8_decode_workspace_bytes(B, Hq, hkv, n) for B, hkv, Hq, n in shapes)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    for i, (B, hkv, Hq, n) in enumerate(shapes):
        cap = (n + 255) // 256 * 256
        kt, vt = _cache(B, hkv, n, cap, seed=100 + i)
        q = torch.randn(B, Hq, 1, 128, generator=torch.Generator().manual_seed(i)).to(torch.bfloat16).cuda()
        out = torch.empty_like(q)
        _lib.call("lg_q8_decode_attention", q.data_ptr(), B, Hq, hkv, 128,
                  *(t.data_ptr() for t in kt), *(t.data_ptr() for t in vt), cap, n,
                  ctypes.c_float(128 ** -0.5), out.data_ptr(), ws.data_ptr(), ws.numel(),
                  torch.cuda.current_stream().cuda_stream)
        want = attn_ref.q8_decode_attention_ref(q.float().cpu(), tuple(t.cpu() for t in kt),
                                                tuple(t.cpu() for t in vt), n, 128 ** -0.5)
        assert (out.cpu().float() - want.float()).abs().max() < 2e-2, (B, hkv, Hq, n)
    assert int(ws[:16384].count_nonzero()) == 0  # counters left at zero
