"""The streaming surface on the GPU (laguna_mlx/streaming.py; reference tests
test_streaming.py:55-97): a model loaded from an expert pack gives exactly the resident
model's logits (prefill, and decode with a cache), through the module call surface and the
fused decode path; every expert is resident (no misses, no bytes read after loading) and the
statistics count the picks served."""
import pytest
import torch

from tests.test_streaming_cpu import _cpu_model

pytestmark = pytest.mark.gpu


def _resident_on_gpu(tmp_path):
    import json
    from lagunalab_b200 import laguna, pack
    from safetensors.torch import load_file
    m = _cpu_model()
    pack.pack_model(m, tmp_path)
    cfg = json.loads((tmp_path / "config.json").read_text())
    layout = json.loads((tmp_path / "layout.json").read_text())
    w = load_file(str(tmp_path / "resident.safetensors"))
    for l in layout["layers"]:
        for name, t in pack.read_layer(tmp_path, layout, l).items():
            w[f"model.layers.{l}.mlp.switch_mlp.{name}"] = t
    return laguna.model_from_weights(laguna.ModelArgs.from_dict(cfg), w, cfg["quantization"])


def _ids(n, seed):
    return torch.randint(0, 96, (n,), generator=torch.Generator().manual_seed(seed)).to(
        torch.int32).cuda()


def test_streamed_model_equals_resident_model(tmp_path):
    from lagunalab_b200 import streaming
    resident = _resident_on_gpu(tmp_path)
    streamed, tok = streaming.load_streaming(tmp_path, slots=3)
    assert tok is None
    ids = _ids(20, 6)
    assert torch.equal(streamed(ids[None]), resident(ids[None]))
    s = streaming.stream_stats(streamed)
    assert s["hits"] > 0 and s["misses"] == 0 and s["bytes_read"] == 0 and s["hit_rate"] == 1.0


def test_streamed_decode_with_cache_equals_resident(tmp_path):
    from lagunalab_b200 import laguna, streaming
    resident = _resident_on_gpu(tmp_path)
    streamed, _ = streaming.load_streaming(tmp_path, slots=4)
    ids = _ids(12, 7)
    want = laguna.generate(resident, ids, 6)
    before = streaming.stream_stats(streamed)["hits"]
    got = laguna.generate(streamed, ids, 6)
    assert got == want
    s = streaming.stream_stats(streamed)
    # prefill (12 tokens) + 6 one-token steps, k = 2 picks each, per MoE layer (2 layers)
    assert s["hits"] - before == 2 * 2 * (12 + 6) and s["misses"] == 0


def test_streaming_switchglu_call_surface(tmp_path):
    from lagunalab_b200 import streaming
    streamed, _ = streaming.load_streaming(tmp_path if (tmp_path / "layout.json").exists()
                                           else _pack(tmp_path), slots=2)
    sw = streamed.layers[1].mlp.switch_mlp
    assert isinstance(sw, streaming.StreamingSwitchGLU)
    x = torch.randn(5, 128, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    idx = torch.tensor([[0, 3], [1, 2], [3, 3], [2, 0], [1, 1]], dtype=torch.int32).cuda()
    y = sw(x, idx)
    assert y.shape == (5, 2, 128)
    assert torch.equal(y, sw.resident_glu()(x, idx))
    assert sw.store.load([3, 1]) == {3: 3, 1: 1}


def _pack(tmp_path):
    from lagunalab_b200 import pack
    pack.pack_model(_cpu_model(), tmp_path)
    return tmp_path
