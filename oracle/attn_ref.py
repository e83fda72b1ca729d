"""PyTorch-CPU restatement of the fused 8-bit KV decode attention and of the
quantized KV cache append (test infrastructure only).

* ``q8_decode_attention_ref`` follows laguna_mlx/q8_attn.py:102-130 and the Metal
  source at :17-92: dequantize ``scale * code + bias`` per 64-group (:50, :55), scale
  the query in fp32 (:117), an fp32 softmax over the first ``n`` rows, output cast
  to the query dtype (:130).
* ``q8_decode_attention_blocks`` is the same computation in the reference's
  block-split form: 512-key blocks with per-block (max, sum, acc) partials and
  the log-sum-exp merge of q8_attn.py:126-130.
* ``quantize_rows`` restates the build's own affine quantizer (min/max per group,
  bf16 scale and bias, codes rounded half-to-even and clamped), which the CUDA
  append kernel must reproduce bit for bit. MLX's own ``mx.quantize`` rounding
  rule cannot be run here, so KV parity tests feed the same packed buffers to
  both sides.
"""
import numpy as np
import torch

from . import mlx_quant

BLOCK = 512  # laguna_mlx/q8_attn.py:14


def _deq_rows(packed, scales, biases, n):
    """Dequantize rows [..., :n, :] of an 8-bit g64 packed buffer to fp32."""
    from .moe_ref import dequantize
    return dequantize(packed[..., :n, :], scales[..., :n, :], biases[..., :n, :],
                      group_size=64, bits=8)


def q8_decode_attention_ref(q, keys, values, n, scale):
    """q [B, Hq, 1, D] -> [B, Hq, 1, D] in q's dtype (q8_attn.py:102-130)."""
    B, Hq, L, D = q.shape
    assert L == 1 and D == 128
    k = _deq_rows(*keys, n)      # [B, hkv, n, D]
    v = _deq_rows(*values, n)
    hkv = k.shape[1]
    G = Hq // hkv
    qs = q.to(torch.float32).reshape(B, hkv, G, D) * scale
    s = torch.einsum("bhgd,bhnd->bhgn", qs, k)
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("bhgn,bhnd->bhgd", p, v)
    return o.reshape(B, Hq, 1, D).to(q.dtype)


def q8_decode_attention_blocks(q, keys, values, n, scale, block=BLOCK):
    """Block-split form with the reference's partials and merge (q8_attn.py:116-130)."""
    B, Hq, _, D = q.shape
    k = _deq_rows(*keys, n)
    v = _deq_rows(*values, n)
    hkv = k.shape[1]
    G = Hq // hkv
    qs = q.to(torch.float32).reshape(B, hkv, G, D) * scale
    nblk = max(1, -(-n // block))
    pm, pl, pa = [], [], []
    for b0 in range(0, nblk * block, block):
        kb, vb = k[:, :, b0:b0 + block], v[:, :, b0:b0 + block]
        s = torch.einsum("bhgd,bhnd->bhgn", qs, kb)
        m = s.max(dim=-1).values
        e = torch.exp(s - m[..., None])
        pm.append(m)
        pl.append(e.sum(-1))
        pa.append(torch.einsum("bhgn,bhnd->bhgd", e, vb))
    pm, pl, pa = torch.stack(pm, -1), torch.stack(pl, -1), torch.stack(pa, -2)
    M = pm.max(dim=-1, keepdim=True).values
    w = torch.exp(pm - M)
    out = (w[..., None] * pa).sum(-2) / (w * pl).sum(-1)[..., None]
    return out.reshape(B, Hq, 1, D).to(q.dtype)


def sdpa_decode_ref(q, k, v, n, scale):
    """Plain decode attention over bf16 K/V rows [:n] (laguna.py:107 SDPA), fp32 math."""
    B, Hq, _, D = q.shape
    hkv = k.shape[1]
    G = Hq // hkv
    qs = q.to(torch.float32).reshape(B, hkv, G, D) * scale
    kk = k[:, :, :n].to(torch.float32)
    vv = v[:, :, :n].to(torch.float32)
    p = torch.softmax(torch.einsum("bhgd,bhnd->bhgn", qs, kk), dim=-1)
    o = torch.einsum("bhgn,bhnd->bhgd", p, vv)
    return o.reshape(B, Hq, 1, D).to(q.dtype)


def quantize_rows(x, group_size=64, bits=8):
    """The build's affine quantizer on float rows [..., D] -> (uint32 packed, bf16 scales,
    bf16 biases) as numpy arrays (scales/biases as uint16 bf16 bit patterns).

    Per group: lo = min, hi = max, scale = bf16((hi - lo) / (2^bits - 1)),
    bias = bf16(lo); code = clamp(rint((x - bias) / scale), 0, 2^bits - 1), with
    code 0 everywhere when scale rounds to 0."""
    x = np.asarray(x, dtype=np.float32)
    D = x.shape[-1]
    g = x.reshape(*x.shape[:-1], D // group_size, group_size)
    lo = g.min(-1)
    hi = g.max(-1)
    nb = np.float32((1 << bits) - 1)
    s_bits = mlx_quant.f32_to_bf16_bits((hi - lo) / nb)
    b_bits = mlx_quant.f32_to_bf16_bits(lo)
    s = mlx_quant.bf16_bits_to_f32(s_bits)
    b = mlx_quant.bf16_bits_to_f32(b_bits)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.rint((g - b[..., None]) / s[..., None])
    q = np.where(s[..., None] == 0, 0, q)
    q = np.clip(q, 0, (1 << bits) - 1).astype(np.int64)
    packed = mlx_quant.pack_codes(q.reshape(*x.shape[:-1], D), bits)
    return packed, s_bits, b_bits


class QuantizedKVCacheRef:
    """Capacity and offset rules of mlx-lm's QuantizedKVCache as used by
    laguna_mlx/cache.py:83-90: buffers grow by whole 256-row steps; a buffer whose
    offset is not on a step boundary is first cut back to the offset."""

    step = 256

    def __init__(self):
        self.cap = 0
        self.offset = 0

    def append(self, L):
        prev = self.offset
        if self.cap == 0 or prev + L > self.cap:
            new = (self.step + L - 1) // self.step * self.step
            if self.cap and prev % self.step != 0:
                self.cap = prev
            self.cap += new
        self.offset += L
        return prev, self.cap
