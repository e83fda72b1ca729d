"""Quantized KV cache objects with the surface of laguna_mlx/cache.py:66-157.

``QuantizedKVCache`` restates the capacity rules of mlx-lm's QuantizedKVCache that
``DequantKVCache`` wraps (cache.py:83): packed uint32 words plus bf16 scales/biases per
row, full-capacity buffers grown by whole 256-row steps (a buffer whose offset is not on a
step boundary is first cut back to the offset). Appends are quantized on the GPU by the
library's affine quantizer. ``DequantKVCache`` keeps the reference's switches and its
attribute contract: no ``bits`` attribute except on ``quantized_decode`` single-token steps
(cache.py:108-112), ``fused_step`` set on single-token steps with ``fused_decode``.
"""
import torch

from . import ops


class QuantizedKVCache:
    step = 256

    def __init__(self, group_size=64, bits=8, capacity=0):
        self.group_size, self.bits = group_size, bits
        self.keys = self.values = None
        self.offset = 0
        self.capacity_hint = capacity

    def reserve(self, B, H, D, L, device):
        """Room for L more rows without moving the valid ones: a first buffer holds at least
        ``capacity`` rows; growth keeps the 256-row steps."""
        need = self.offset + L
        if self.keys is not None and self.keys[0].shape[2] >= need:
            return
        rows = max(self.capacity_hint, (need + self.step - 1) // self.step * self.step)
        k, v = self._alloc(B, H, rows, D, device), self._alloc(B, H, rows, D, device)
        if self.keys is not None and self.offset:
            for dst, src in zip(k + v, self.keys + self.values):
                dst[:, :, :self.offset] = src[:, :, :self.offset]
        self.keys, self.values = k, v

    def _alloc(self, B, H, rows, D, device):
        wpr = D * self.bits // 32
        gpr = D // self.group_size
        return (torch.zeros(B, H, rows, wpr, dtype=torch.int32, device=device),
                torch.zeros(B, H, rows, gpr, dtype=torch.bfloat16, device=device),
                torch.zeros(B, H, rows, gpr, dtype=torch.bfloat16, device=device))

    def update_and_fetch(self, keys, values):
        B, H, L, Dk = keys.shape
        Dv = values.shape[-1]
        prev = self.offset
        if self.keys is None or prev + L > self.keys[0].shape[2]:
            new = (self.step + L - 1) // self.step * self.step
            if self.keys is not None:
                if prev % self.step != 0:
                    self.keys = tuple(t[:, :, :prev] for t in self.keys)
                    self.values = tuple(t[:, :, :prev] for t in self.values)
                ek = self._alloc(B, H, new, Dk, keys.device)
                ev = self._alloc(B, H, new, Dv, keys.device)
                self.keys = tuple(torch.cat([a, b], dim=2) for a, b in zip(self.keys, ek))
                self.values = tuple(torch.cat([a, b], dim=2) for a, b in zip(self.values, ev))
            else:
                self.keys = self._alloc(B, H, new, Dk, keys.device)
                self.values = self._alloc(B, H, new, Dv, keys.device)
        ops.quantize_into(keys, self.keys, prev, self.group_size, self.bits)
        ops.quantize_into(values, self.values, prev, self.group_size, self.bits)
        self.offset += L
        return self.state

    @property
    def state(self):
        if self.keys is None:
            return None, None
        n = self.offset
        return (tuple(t[:, :, :n] for t in self.keys), tuple(t[:, :, :n] for t in self.values))

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n

    def is_trimmable(self):
        return True

    def empty(self):
        return self.keys is None

    def make_mask(self, N, return_array=False, window_size=None):
        """mlx-lm convention: None for a single query, "causal" otherwise."""
        return None if N == 1 else "causal"

    @property
    def nbytes(self):
        if self.keys is None:
            return 0
        return sum(t.numel() * t.element_size() for t in (*self.keys, *self.values))


class DequantKVCache:
    """laguna_mlx/cache.py:66-145 on B200. Single-token steps with ``fused_decode`` run the
    fused q8 decode kernel through ``attend``; other steps hand attention bf16 K/V."""

    def __init__(self, group_size=64, bits=8, quantized_decode=False, fused_decode=False,
                 capacity=0):
        if fused_decode and (bits, group_size) != (8, 64):
            raise ValueError("fused_decode needs 8-bit, group_size 64")
        self.q = QuantizedKVCache(group_size=group_size, bits=bits, capacity=capacity)
        self.quantized_decode = quantized_decode
        self.fused_decode = fused_decode
        self._quantized_step = False
        self.fused_step = False

    def update_and_fetch(self, keys, values):
        qk, qv = self.q.update_and_fetch(keys, values)
        self.fused_step = self.fused_decode and keys.shape[2] == 1
        if self.fused_step:
            return qk, qv
        self._quantized_step = self.quantized_decode and keys.shape[2] == 1
        if self._quantized_step:
            return qk, qv
        g, b, n = self.q.group_size, self.q.bits, self.q.offset
        return (ops.dequantize_rows(self.q.keys, n, g, b),
                ops.dequantize_rows(self.q.values, n, g, b))

    def attend(self, queries, scale):
        """Single-token attention straight off the packed cache (the fused q8 kernel)."""
        from .q8_attn import q8_decode_attention

        return q8_decode_attention(queries, self.q.keys, self.q.values, self.q.offset, scale)

    @property
    def bits(self):
        if not self._quantized_step:
            raise AttributeError("bits")
        return self.q.bits

    @property
    def offset(self):
        return self.q.offset

    @property
    def kv_bits(self):
        return self.q.bits

    @property
    def group_size(self):
        return self.q.group_size

    def make_mask(self, *args, **kwargs):
        return self.q.make_mask(*args, **kwargs)

    @property
    def state(self):
        return self.q.state

    def is_trimmable(self):
        return True

    def trim(self, n):
        return self.q.trim(n)

    def empty(self):
        return self.q.empty()

    @property
    def nbytes(self):
        return self.q.nbytes


def make_quantized_cache(model, bits=8, group_size=64, quantized_decode=False, fused_decode=False,
                         capacity=0):
    """laguna_mlx/cache.py:147-157: quantized K/V on full-attention layers (``capacity``
    preallocates rows, as one-token steps replayed from a CUDA graph need); sliding-window
    layers keep a bf16 ring of their window."""
    a = model.args
    if a.head_dim % group_size:
        raise ValueError(f"head_dim {a.head_dim} is not a multiple of group_size {group_size}")
    from .laguna import RotatingKVCache
    caches = []
    for lt in a.layer_types:
        if lt == "sliding_attention":  # sliding layers keep their bf16 window (cache.py:153)
            caches.append(RotatingKVCache(a.sliding_window))
            continue
        caches.append(DequantKVCache(group_size=group_size, bits=bits,
                                     quantized_decode=quantized_decode, fused_decode=fused_decode,
                                     capacity=capacity))
    return caches
