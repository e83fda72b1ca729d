"""The fixed-scratch q8 decode entry point, called through the C ABI.

Some callers cannot allocate device memory when they call (a plugin host that only passes
input and output pointers, code running where CUDA forbids allocation calls, or a path that
cannot take cudaMalloc's implicit synchronisation). lg_q8_decode_attention_noalloc serves
them from a fixed array inside the library. Two calls in a row (different shapes, so the
shared scratch is reused) must match the workspace entry point within the decode-attention
tolerance, and an oversized request must be refused. This file is collected last.
"""
import ctypes

import pytest
import torch

from lagunalab_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _case(B, Hq, Hkv, n, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    cap = (n + 255) // 256 * 256
    mk = lambda: (torch.zeros(B, Hkv, cap, 32, dtype=torch.int32, device="cuda"),
                  torch.zeros(B, Hkv, cap, 2, dtype=torch.bfloat16, device="cuda"),
                  torch.zeros(B, Hkv, cap, 2, dtype=torch.bfloat16, device="cuda"))
    kt, vt = mk(), mk()
    for t in (kt, vt):
        x = torch.randn(B, Hkv, n, 128, generator=g, device="cuda").to(torch.bfloat16)
        ops.quantize_into(x, t, 0, 64, 8)
    q = torch.randn(B, Hq, 1, 128, generator=g, device="cuda").to(torch.bfloat16)
    return q, kt, vt, cap


def _noalloc(q, kt, vt, cap, n, scale):
    B, Hq, _, D = q.shape
    Hkv = kt[0].shape[1]
    out = torch.empty_like(q)
    _lib.call("lg_q8_decode_attention_noalloc", q.data_ptr(), B, Hq, Hkv, D,
              *(t.data_ptr() for t in kt), *(t.data_ptr() for t in vt), cap, n,
              ctypes.c_float(scale), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return out


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    scale = 128 ** -0.5
    for (B, Hq, Hkv, n, seed) in [(1, 32, 4, 20000, 1), (2, 48, 8, 1537, 2)]:
        q, kt, vt, cap = _case(B, Hq, Hkv, n, seed)
        got = _noalloc(q, kt, vt, cap, n, scale)
        want = ops.q8_decode_attention(q, kt, vt, n, scale)
        torch.cuda.synchronize()
        assert (got.float() - want.float()).abs().max().item() < 2e-2


def test_noalloc_rejects_requests_beyond_the_fixed_scratch():
    limit = _lib.lib().lg_q8_decode_fixed_scratch_bytes()
    # a group of 16 query heads split over the whole GPU needs more partials than the array
    B, Hq, Hkv, n = 1, 64, 4, 82671
    assert _lib.lib().lg_q8_decode_workspace_bytes(B, Hq, Hkv, n) > limit
    q, kt, vt, cap = _case(1, 16, 1, 64, 3)
    fake = ctypes.c_void_p(kt[0].data_ptr())
    with pytest.raises(ValueError, match="fixed"):
        _lib.call("lg_q8_decode_attention_noalloc", q.data_ptr(), B, Hq, Hkv, 128,
                  fake, fake, fake, fake, fake, fake, n, n, ctypes.c_float(0.1), q.data_ptr(),
                  None)
