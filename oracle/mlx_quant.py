"""MLX affine quantization layout, restated in numpy (test infrastructure only).

Layout (laguna_mlx/q8_attn.py:8-10 for 8 bits; the same convention at 4 bits,
as read by scripts/pack_experts.py:19-30 and stacked per expert by
laguna_mlx/laguna.py:216-228):

* ``weight``  uint32 [..., in * bits / 32]; word ``j`` holds the ``32 / bits``
  consecutive codes ``j * (32 / bits) + i`` at bit offset ``i * bits``
  (low bits first, little endian).
* ``scales``, ``biases``  [..., in / group_size] (bf16 on the real checkpoint,
  streaming.py:30-31).
* value = scale * code + bias (laguna_mlx/q8_attn.py:50, :55).
"""
import numpy as np


def bf16_bits_to_f32(u16):
    """bf16 bit patterns (uint16) -> float32 values, exactly."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    """float32 -> bf16 bit patterns with round-to-nearest-even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = np.where(nan, np.uint16(0x7FC0), rounded)
    return rounded


def round_bf16(x):
    """Round float32 values to the nearest bf16 and return them as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def unpack_codes(packed, bits):
    """uint32 [..., W] -> uint8/int codes [..., W * 32 / bits] (low bits first)."""
    packed = np.asarray(packed, dtype=np.uint32)
    per = 32 // bits
    mask = np.uint32((1 << bits) - 1)
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    codes = (packed[..., None] >> shifts) & mask
    return codes.reshape(*packed.shape[:-1], packed.shape[-1] * per).astype(np.int64)


def pack_codes(codes, bits):
    """Inverse of ``unpack_codes``: integer codes [..., n] -> uint32 [..., n * bits / 32]."""
    codes = np.asarray(codes, dtype=np.uint64)
    per = 32 // bits
    c = codes.reshape(*codes.shape[:-1], codes.shape[-1] // per, per)
    shifts = (np.arange(per, dtype=np.uint64) * bits)
    return np.bitwise_or.reduce(c << shifts, axis=-1).astype(np.uint32)


def dequantize(packed, scales, biases, group_size, bits):
    """MLX affine dequantize to float32 (laguna_mlx/q8_attn.py:50: ``ks * q + kb``).

    ``scales``/``biases`` may be float arrays or bf16 bit patterns (uint16).
    The product ``scale * code`` and the add are done in float32, as the Metal
    kernel does in registers.
    """
    codes = unpack_codes(packed, bits).astype(np.float32)
    s = _as_f32(scales)
    b = _as_f32(biases)
    n = codes.shape[-1]
    g = codes.reshape(*codes.shape[:-1], n // group_size, group_size)
    out = g * s[..., None] + b[..., None]
    return out.reshape(codes.shape).astype(np.float32)


def _as_f32(a):
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return bf16_bits_to_f32(a)
    return a.astype(np.float32)
