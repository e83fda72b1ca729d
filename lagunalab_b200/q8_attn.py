"""Fused single-token attention over an 8-bit quantized KV cache (laguna_mlx/q8_attn.py).

``q8_decode_attention(q, keys, values, n, scale)`` keeps the reference signature: q
[B, Hq, 1, 128]; keys/values are the cache's full-capacity (packed, scales, biases) tuples,
of which the first ``n`` rows are valid; returns [B, Hq, 1, 128] in q's dtype (bf16).
The B200 kernel is a split-KV flash-decode on the tensor cores over the raw 8-bit codes,
with the per-split merge done inside the same launch.
"""
from . import ops

BLOCK = 512  # the reference kernel's keys per threadgroup; kept for callers that import it


def q8_decode_attention(q, keys, values, n, scale):
    B, Hq, L, D = q.shape
    if L != 1 or D != 128:
        raise ValueError("decode only, head_dim 128")
    if keys[0].shape[-1] != D // 4:
        raise ValueError("8-bit, group_size 64 only")
    return ops.q8_decode_attention(q, keys, values, n, scale).to(q.dtype)
