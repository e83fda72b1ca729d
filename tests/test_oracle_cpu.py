"""The CPU oracle, pinned against the reference's own PyTorch model (golden fixtures made
by tests/golden/make_golden.py) and against known-answer layouts; no GPU."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attn_ref, mlx_quant, moe_ref

GOLD = Path(__file__).resolve().parent / "golden"


def _load(name):
    d = np.load(GOLD / f"{name}.npz")
    return {k: torch.from_numpy(np.asarray(v)) for k, v in d.items()}, d


@pytest.mark.parametrize("name", ["moe_tiny", "moe_mid"])
def test_fp32_block_matches_reference_model(name):
    t, d = _load(name)
    out, inds, w, logits = moe_ref.moe_block_fp32(
        t["x"], t["gate_w"], t["bias"], t["gate_up"], t["down"], t["sh_gate"], t["sh_up"],
        t["sh_down"], int(d["k"]), float(d["scale"]))
    assert torch.equal(logits, t["ref_logits"])
    assert torch.equal(inds, t["ref_inds"])  # same order: both sorted by biased score
    torch.testing.assert_close(w, t["ref_w"], atol=0, rtol=0)
    torch.testing.assert_close(out, t["ref_out"], atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("name", ["moe_tiny", "moe_mid"])
def test_router_matches_reference_router(name):
    t, d = _load(name)
    k = int(d["k"])
    inds, w, logits, scores, sel = moe_ref.route(t["x"].to(torch.bfloat16).float(), t["gate_w"],
                                                 t["bias"], k)
    # the reference router on the same (bf16-rounded) input
    x = t["x"].to(torch.bfloat16).float()
    ref_scores = torch.sigmoid(x @ t["gate_w"].T)
    ref_inds = torch.topk(ref_scores + t["bias"], k, dim=-1).indices
    assert torch.equal(torch.sort(inds, -1).values, torch.sort(ref_inds, -1).values)
    assert not moe_ref.tie_rows(sel, k).any()


def test_tie_rule_lower_index_first_and_masked_experts():
    sel = torch.tensor([[0.5, 0.9, 0.5, 0.9, 0.1, 0.5]])
    assert moe_ref.topk_indices(sel, 3).tolist() == [[1, 3, 0]]
    assert moe_ref.tie_rows(sel, 3).tolist() == [True]   # 3rd and 4th are both 0.5
    assert moe_ref.tie_rows(sel, 2).tolist() == [False]
    # pruned experts carry bias -inf (lagunaLab pruning masks the router that way)
    logits = torch.tensor([[3.0, 2.0, 1.0, 0.0]])
    bias = torch.tensor([float("-inf"), 0.0, float("-inf"), 0.0])
    inds, w, *_ = moe_ref.route(logits.to(torch.bfloat16), torch.eye(4), bias, 2)
    assert inds.tolist() == [[1, 3]]
    # with more picks than live experts the masked ones come last, lower index first
    inds, *_ = moe_ref.route(logits.to(torch.bfloat16), torch.eye(4), bias, 3)
    assert inds.tolist() == [[1, 3, 0]]


def test_pack_layout_known_answer_8bit():
    # laguna_mlx/q8_attn.py:8-10: a key row is 32 uint32, each holding 4 consecutive values,
    # low byte first
    codes = np.arange(128, dtype=np.int64).reshape(1, 128)
    words = mlx_quant.pack_codes(codes, 8)
    assert words.shape == (1, 32)
    assert words[0, 0] == 0x03020100 and words[0, 31] == 0x7F7E7D7C
    assert np.array_equal(mlx_quant.unpack_codes(words, 8), codes)


def test_pack_layout_known_answer_4bit():
    codes = np.array([[1, 2, 3, 4, 5, 6, 7, 8, 15, 0, 0, 0, 0, 0, 0, 9]], dtype=np.int64)
    words = mlx_quant.pack_codes(codes, 4)
    assert words.tolist() == [[0x87654321, 0x9000000F]]
    assert np.array_equal(mlx_quant.unpack_codes(words, 4), codes)
    # the torch restatement decodes the same bits
    t = torch.from_numpy(words.view(np.int32))
    assert moe_ref.unpack_codes(t, 4).tolist() == codes.tolist()


def test_dequantize_formula():
    codes = np.array([[0, 255] + [7] * 62], dtype=np.int64)
    words = mlx_quant.pack_codes(codes, 8)
    s = mlx_quant.f32_to_bf16_bits(np.array([[0.5]], np.float32))
    b = mlx_quant.f32_to_bf16_bits(np.array([[-2.0]], np.float32))
    v = mlx_quant.dequantize(words, s, b, 64, 8)
    assert v[0, 0] == -2.0 and v[0, 1] == 125.5 and v[0, 2] == 1.5


def test_bf16_bit_helpers_round_trip():
    x = np.array([0.0, -0.0, 1.0, -1.0, 3.38e38, 1.18e-38, np.inf, -np.inf, 1.00390625],
                 np.float32)
    bits = mlx_quant.f32_to_bf16_bits(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, ref)


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_rows_error_bound(bits):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 128)).astype(np.float32)
    q, s, b = attn_ref.quantize_rows(x, 64, bits)
    back = mlx_quant.dequantize(q, s, b, 64, bits)
    step = mlx_quant.bf16_bits_to_f32(s)
    # half a step from rounding plus the bf16 rounding of scale and bias
    err = np.abs(back - x).reshape(64, 2, 64).max(-1)
    assert (err <= 0.5 * step * 1.02 + 2 ** -7 * np.abs(x).reshape(64, 2, 64).max(-1)).all()


@pytest.mark.parametrize("n", [1, 7, 512, 513, 3 * 512 + 100])
def test_q8_block_merge_equals_direct_softmax(n):
    # the reference's block split + LSE merge (q8_attn.py:116-130) is the same function
    g = torch.Generator().manual_seed(n)
    cap = (n + 255) // 256 * 256
    k = torch.randn(1, 8, cap, 128, generator=g)
    v = torch.randn(1, 8, cap, 128, generator=g)
    kt = tuple(torch.from_numpy(a.astype(np.int32) if a.dtype == np.uint32 else a.view(np.int16))
               for a in attn_ref.quantize_rows(k.numpy(), 64, 8))
    vt = tuple(torch.from_numpy(a.astype(np.int32) if a.dtype == np.uint32 else a.view(np.int16))
               for a in attn_ref.quantize_rows(v.numpy(), 64, 8))
    kt = (kt[0], kt[1].view(torch.bfloat16), kt[2].view(torch.bfloat16))
    vt = (vt[0], vt[1].view(torch.bfloat16), vt[2].view(torch.bfloat16))
    q = torch.randn(1, 48, 1, 128, generator=g).to(torch.bfloat16)
    a = attn_ref.q8_decode_attention_ref(q, kt, vt, n, 128 ** -0.5)
    b = attn_ref.q8_decode_attention_blocks(q, kt, vt, n, 128 ** -0.5)
    assert (a.float() - b.float()).abs().max() < 1e-2


def test_kv_cache_capacity_rules():
    c = attn_ref.QuantizedKVCacheRef()
    assert c.append(300) == (0, 512)
    c = attn_ref.QuantizedKVCacheRef()
    c.append(200)
    assert c.append(60) == (200, 456)   # cut back to 200, then one 256-row step
    c = attn_ref.QuantizedKVCacheRef()
    c.append(256)
    assert c.append(1) == (256, 512)


def test_quantized_oracle_matches_fp32_structure_on_dequantized_weights():
    # The quantized restatement (bf16 materialisation points) against the reference-pinned
    # fp32 block evaluated on the same dequantized weights.
    from tests._util import moe_weights, quant_np, rel_err, cos
    E, H, I, Ish, k, T = 8, 128, 64, 64, 2, 12
    w = moe_weights(E, H, I, Ish, seed=3, std=0.05)
    qg, qu, qd = (quant_np(w[n]) for n in ("gate", "up", "down"))
    sg, su, sd = (quant_np(w[n]) for n in ("sh_gate", "sh_up", "sh_down"))
    deq = lambda t: moe_ref.dequantize(*t, group_size=64, bits=4)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    bias = torch.randn(E, generator=g) * 0.01
    out_q, inds_q, _ = moe_ref.moe_block(x, w["router"], bias, (qg, qu, qd), (sg, su, sd), k,
                                         routed_scaling_factor=2.5)
    out_f, inds_f, _, _ = moe_ref.moe_block_fp32(
        x.float(), w["router"], bias, torch.cat([deq(qg), deq(qu)], 1), deq(qd), deq(sg),
        deq(su), deq(sd), k, routed_scaling_factor=2.5)
    assert torch.equal(inds_q, inds_f)
    assert rel_err(out_q, out_f) < 2e-2 and cos(out_q, out_f) > 0.999
