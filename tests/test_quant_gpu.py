"""The CUDA quantizer is bit-exact against the oracle's restatement; dequantize matches the
MLX formula; the KV-cache append follows mlx-lm's capacity rules."""
import numpy as np
import pytest
import torch

from oracle import attn_ref, mlx_quant

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits,group", [(4, 64), (8, 64), (8, 32), (4, 128)])
def test_quantize_bit_exact(bits, group):
    from lagunalab_b200 import ops
    g = torch.Generator().manual_seed(bits * group)
    x = torch.randn(257, 512, generator=g) * 0.5
    x[3, :64] = 1.25          # constant group: scale 0
    x[4, 7] = 40.0            # outlier
    for dt in (torch.float32, torch.bfloat16):
        xs = x.to(dt)
        q, s, b = ops.quantize(xs.cuda(), group, bits)
        rq, rs, rb = attn_ref.quantize_rows(xs.float().numpy(), group, bits)
        assert np.array_equal(q.cpu().numpy().view(np.uint32), rq)
        assert np.array_equal(s.cpu().view(torch.int16).numpy().view(np.uint16), rs)
        assert np.array_equal(b.cpu().view(torch.int16).numpy().view(np.uint16), rb)


def test_dequantize_matches_formula():
    from lagunalab_b200 import ops
    x = torch.randn(64, 256, generator=torch.Generator().manual_seed(0))
    q, s, b = ops.quantize(x.cuda(), 64, 4)
    d = ops.dequantize(q, s, b, 64, 4).cpu().float()
    ref = mlx_quant.dequantize(q.cpu().numpy().view(np.uint32),
                               s.cpu().view(torch.int16).numpy().view(np.uint16),
                               b.cpu().view(torch.int16).numpy().view(np.uint16), 64, 4)
    ref = torch.from_numpy(ref).to(torch.bfloat16).float()
    assert torch.equal(d, ref)


def test_kv_append_capacity_and_offsets():
    from lagunalab_b200.cache import QuantizedKVCache
    c = QuantizedKVCache()
    ref = attn_ref.QuantizedKVCacheRef()
    g = torch.Generator().manual_seed(0)
    chunks = [200, 60, 1, 1, 250, 1]
    allk = []
    for L in chunks:
        k = torch.randn(1, 2, L, 128, generator=g).to(torch.bfloat16)
        allk.append(k)
        c.update_and_fetch(k.cuda(), k.cuda())
        prev, cap = ref.append(L)
        assert c.offset == prev + L and c.keys[0].shape[2] == cap
    ks, _ = c.state
    full = torch.cat(allk, dim=2).float().numpy()
    rq, rs, rb = attn_ref.quantize_rows(full, 64, 8)
    assert np.array_equal(ks[0].cpu().numpy().view(np.uint32), rq)
