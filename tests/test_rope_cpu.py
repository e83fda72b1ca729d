"""The product's RoPE set-up (laguna.rope_setup: partial rotary and YaRN frequencies, the
attention factor) against the oracle's restatement (oracle/model_ref.rope_params), which
tests/test_model_oracle_cpu.py pins to the vendored PyTorch model; and the ring cache's
window rows."""
import torch

from lagunalab_b200 import laguna
from oracle import model_ref

YARN = {"rope_theta": 500000.0, "rope_type": "yarn", "factor": 32.0,
        "original_max_position_embeddings": 8192, "beta_slow": 1.0, "beta_fast": 64.0,
        "attention_factor": 1.3465735902799727, "partial_rotary_factor": 0.5}


def test_yarn_and_partial_rotary_tables_match_the_oracle():
    for p, D in ((YARN, 128), (dict(YARN, attention_factor=None), 256),
                 ({"rope_type": "default", "rope_theta": 1e4, "partial_rotary_factor": 0.5}, 128),
                 (dict(YARN, partial_rotary_factor=1.0, factor=8.0), 128)):
        got = laguna.rope_setup(p, D, "cpu")
        R, inv, ms = model_ref.rope_params(p, D)
        assert got[1] == R and abs(got[2] - ms) < 1e-12
        assert torch.allclose(got[0], inv, rtol=2e-7, atol=0), (p, (got[0] - inv).abs().max())


def test_default_full_rope_uses_the_kernel_frequencies():
    assert laguna.rope_setup({"rope_type": "default", "rope_theta": 1e6}, 128, "cpu") is None


def test_ring_cache_window_rows():
    c = laguna.RotatingKVCache(5)
    c.reserve(1, 2, 128, "cpu")
    c.offset = 3
    assert c.window_rows().tolist() == [0, 1, 2]
    c.offset = 12
    assert c.window_rows().tolist() == [2, 3, 4, 0, 1]  # positions 7..11
    assert not c.is_trimmable() and c.trim(3) == 0
