"""Expert pack format and streaming loader, host side (laguna_mlx/streaming.py,
scripts/pack_experts.py): every expert round-trips bit for bit through its layer file, the
stride is whole 16 KiB pages, the resident file holds everything but the routed experts, and a
model rebuilt from the pack's weights carries the same tensors (mirrors the reference's
test_streaming.py pack tests)."""
import json

import numpy as np
import torch

from tests._util import gen, quant_np


def _cpu_model():
    from lagunalab_b200 import laguna, synth
    args = synth.decoder_args(vocab=96, hidden=128, layers=3, heads=2, kv_heads=1, head_dim=128,
                              experts=4, top_k=2, moe_inter=64, shared_inter=64, dense_inter=128,
                              rope_theta=1e4)
    g = gen(3)
    ql = lambda *s, bits=4: laguna.QuantizedLinear(*quant_np(torch.randn(*s, generator=g) * 0.05,
                                                             bits), 64, bits)
    sl = lambda *s: laguna.SwitchLinear(*quant_np(torch.randn(*s, generator=g) * 0.05), 64, 4)
    norm = lambda n: laguna.RMSNorm(n, 1e-6, (1 + 0.1 * torch.randn(n, generator=g)).to(
        torch.bfloat16))
    H, D = args.hidden_size, args.head_dim
    layers = []
    for i in range(args.num_hidden_layers):
        Hq, Hkv = args.num_attention_heads, args.num_key_value_heads
        at = laguna.Attention(args, i, ql(Hq * D, H), ql(Hkv * D, H), ql(Hkv * D, H),
                              ql(H, Hq * D), ql(Hq, H), norm(D), norm(D))
        if i in args.mlp_only_layers:
            mlp = laguna.MLP(H, 128, ql(128, H), ql(128, H), ql(H, 128))
        else:
            E, I = args.num_experts, args.moe_intermediate_size
            sw = laguna.SwitchGLU(H, I, E, sl(E, I, H), sl(E, I, H), sl(E, H, I))
            sh = laguna.MLP(H, 64, ql(64, H), ql(64, H), ql(H, 64))
            mlp = laguna.SparseMoeBlock(args, ql(E, H, bits=8), 0.1 * torch.randn(E, generator=g),
                                        sw, sh)
        layers.append(laguna.DecoderLayer(args, i, at, mlp, norm(H), norm(H)))
    emb = ql(args.vocab_size, H)
    model = laguna.LagunaModel(args, laguna.QuantizedEmbedding(*emb.mat), layers, norm(H))
    return laguna.Model(args, model, ql(args.vocab_size, H))


def test_pack_round_trips_every_expert_bit_exact(tmp_path):
    from lagunalab_b200 import pack
    m = _cpu_model()
    layout = pack.pack_model(m, tmp_path)
    assert layout["layers"] == [1, 2] and layout["stride"] % 16384 == 0
    assert json.loads((tmp_path / "layout.json").read_text()) == layout
    for l in layout["layers"]:
        sw = m.layers[l].mlp.switch_mlp
        stacked = pack.read_layer(tmp_path, layout, l)
        for e in range(layout["num_experts"]):
            got = pack.read_expert(tmp_path, layout, l, e)
            for proj in ("gate_proj", "up_proj", "down_proj"):
                for i, part in enumerate(("weight", "scales", "biases")):
                    want = getattr(sw, proj).mat[i][e]
                    have = got[f"{proj}.{part}"]
                    assert have.dtype == want.dtype
                    assert torch.equal(have.view(torch.int16) if have.dtype == torch.bfloat16
                                       else have, want.view(torch.int16)
                                       if want.dtype == torch.bfloat16 else want)
                    assert torch.equal(stacked[f"{proj}.{part}"][e], have)
    from safetensors.torch import load_file
    resident = load_file(str(tmp_path / "resident.safetensors"))
    assert not any("switch_mlp" in k for k in resident)
    assert "model.layers.1.mlp.gate.weight" in resident
    assert resident["model.layers.1.mlp.gate.weight"].dtype == torch.uint32


def test_bfloat16_edge_values_round_trip():
    from lagunalab_b200 import pack
    edge = torch.tensor([0.0, -0.0, 1.0, -1.0, 3.38e38, 1.18e-38, float("inf"), float("-inf")])
    a = torch.cat([edge, torch.randn(24, generator=gen(0))]).to(torch.bfloat16)
    raw = pack._to_bytes(a)
    layout = {"arrays": {"x": {"offset": 0, "shape": list(a.shape), "dtype": "bfloat16"}}}
    got = pack.expert_from_bytes(raw, layout)["x"]
    assert got.dtype == torch.bfloat16
    assert pack._to_bytes(got) == raw  # including the sign of -0.0


def test_model_from_pack_weights_has_the_same_tensors(tmp_path):
    from lagunalab_b200 import laguna, pack
    from safetensors.torch import load_file
    m = _cpu_model()
    pack.pack_model(m, tmp_path)
    cfg = json.loads((tmp_path / "config.json").read_text())
    args = laguna.ModelArgs.from_dict(cfg)
    w = load_file(str(tmp_path / "resident.safetensors"))
    layout = json.loads((tmp_path / "layout.json").read_text())
    for l in layout["layers"]:  # the routed experts from the layer files
        for name, t in pack.read_layer(tmp_path, layout, l).items():
            w[f"model.layers.{l}.mlp.switch_mlp.{name}"] = t
    m2 = laguna.model_from_weights(args, w, cfg["quantization"], device="cpu")
    a, b = pack.model_weights(m), pack.model_weights(m2)
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k].view(torch.int16) if a[k].dtype == torch.bfloat16 else a[k],
                           b[k].view(torch.int16) if b[k].dtype == torch.bfloat16 else b[k]), k
    assert m2.layers[1].mlp.gate.bits == 8 and m2.layers[1].self_attn.q_proj.bits == 4
