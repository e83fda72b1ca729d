"""The one-token q/k/v/g projection with the attention prologue fused behind it
(lg_decode_qkv_prep) on the GPU.

Bit for bit against the library's own two-launch form, lg_decode_gemv with the fused input
RMSNorm followed by lg_attn_prep / lg_attn_prep_q8 (laguna.py:94-106): the projection row, the
rotated q, the gates and every cache tensor, for the bf16 and the 8-bit cache, host and device
positions, per-head and per-element gates. Repeated calls on one workspace check that the
per-head tile counters are back at zero after each call; a device position at the capacity
writes no cache row, like the two-launch form.
"""
import pytest
import torch

from tests._util import gen, quant_np

pytestmark = pytest.mark.gpu


def _case(K, Hq, Hkv, D, per_head, seed):
    g = gen(seed)
    N = (Hq + 2 * Hkv) * D + (Hq if per_head else Hq * D)
    mat = tuple(t.cuda() for t in quant_np(torch.randn(N, K, generator=g) * 0.05, 4))
    x = (3 * torch.randn(1, K, generator=g)).to(torch.bfloat16).cuda()
    w = (1 + 0.2 * torch.randn(K, generator=g)).to(torch.bfloat16).cuda()
    qn = (1 + 0.2 * torch.randn(D, generator=g)).to(torch.bfloat16).cuda()
    kn = (1 + 0.2 * torch.randn(D, generator=g)).to(torch.bfloat16).cuda()
    return mat, x, w, qn, kn


def _caches(q8, Hkv, cap, D):
    if q8:
        def one():
            return (torch.zeros(1, Hkv, cap, D // 4, dtype=torch.int32, device="cuda"),
                    torch.zeros(1, Hkv, cap, D // 64, dtype=torch.bfloat16, device="cuda"),
                    torch.zeros(1, Hkv, cap, D // 64, dtype=torch.bfloat16, device="cuda"))
        return one(), one()
    return (torch.zeros(Hkv, cap, D, dtype=torch.bfloat16, device="cuda"),
            torch.zeros(Hkv, cap, D, dtype=torch.bfloat16, device="cuda"))


def _flat(c):
    return list(c) if isinstance(c, tuple) else [c]


@pytest.mark.parametrize("q8", [False, True])
@pytest.mark.parametrize("dev_pos", [False, True])
@pytest.mark.parametrize("K,Hq,Hkv,D,per_head", [(2048, 32, 4, 128, True),
                                                 (256, 4, 2, 128, False),
                                                 (1024, 8, 2, 256, True),
                                                 (512, 6, 3, 64, True)])
def test_fused_prologue_is_bitwise_the_two_launch_form(q8, dev_pos, K, Hq, Hkv, D, per_head):
    from lagunalab_b200 import ops
    cap = 300
    mat, x, w, qn, kn = _case(K, Hq, Hkv, D, per_head, K + Hq + D)
    ka, va = _caches(q8, Hkv, cap, D)
    kb, vb = _caches(q8, Hkv, cap, D)
    prep2 = ops.attn_prep_q8 if q8 else ops.attn_prep
    for step, pos in enumerate([0, 1, 77, cap - 1]):
        xs = (x * (1 + step)).to(torch.bfloat16)
        pd = torch.tensor([pos], dtype=torch.int32, device="cuda") if dev_pos else None
        qkvg1, q1, g1 = ops.decode_qkv_prep(xs, mat, (w, 1e-6), Hq, Hkv, D, qn, kn, 1e-6, 5e5,
                                            ka, va, pos=pos, pos_dev=pd,
                                            gate_per_head=per_head)
        qkvg2 = ops.decode_gemv(xs, mat, norm=(w, 1e-6))
        q2, g2 = prep2(qkvg2, Hq, Hkv, D, qn, kn, 1e-6, 5e5, kb, vb, pos=pos, pos_dev=pd,
                       gate_per_head=per_head)
        assert torch.equal(qkvg1, qkvg2)
        assert torch.equal(q1, q2) and torch.equal(g1, g2)
        for a, b in zip(_flat(ka) + _flat(va), _flat(kb) + _flat(vb)):
            assert torch.equal(a, b)
        ws = ops.workspace(x.device, "qkv_prep", 0)
        assert not ws.any(), "per-head counters left non-zero"
    assert ops.decode_status() == (0, 0, 0, 0)


def test_device_position_at_capacity_writes_no_row():
    from lagunalab_b200 import ops
    K, Hq, Hkv, D, cap = 512, 4, 2, 128, 16
    mat, x, w, qn, kn = _case(K, Hq, Hkv, D, True, 3)
    for q8 in (False, True):
        kc, vc = _caches(q8, Hkv, cap, D)
        pd = torch.tensor([cap], dtype=torch.int32, device="cuda")
        _, q, _ = ops.decode_qkv_prep(x, mat, (w, 1e-6), Hq, Hkv, D, qn, kn, 1e-6, 1e4, kc, vc,
                                      pos_dev=pd)
        assert all(not t.any() for t in _flat(kc) + _flat(vc))
        assert q.float().abs().sum() > 0


def test_projection_rows_must_match_the_heads():
    from lagunalab_b200 import ops
    K, Hq, Hkv, D = 256, 4, 2, 128
    mat, x, w, qn, kn = _case(K, Hq, Hkv, D, True, 5)
    kc, vc = _caches(False, Hkv, 8, D)
    with pytest.raises(ValueError):
        ops.decode_qkv_prep(x, mat, (w, 1e-6), Hq, Hkv + 1, D, qn, kn, 1e-6, 1e4, kc, vc)
