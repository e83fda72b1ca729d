"""Generate golden MoE-block vectors from the reference's vendored PyTorch model.

Run in a container where the lagunaLab sources are available:

    python tests/golden/make_golden.py /path/to/lagunaLab

It imports ``tests/reference/modeling_laguna.py`` and ``configuration_laguna.py``
from that tree (Poolside's HF model, the ground truth the MLX port is tested
against in lagunaLab's tests/test_laguna.py:12-19), builds ``LagunaSparseMoeBlock``
with random fp32 weights (a random ``e_score_correction_bias`` too, as
lagunaLab's tests/tiny.py:33-45 does, so selection-only bias is exercised), and
stores inputs and outputs as ``.npz``. The fixtures are committed; the tests read
only the ``.npz`` files.

Cases:
* ``moe_tiny``    lagunaLab's TINY MoE shape (hidden 64, 8 experts, top-2,
                  intermediate 32, shared 32, routed scale 2.5), 10 tokens.
* ``moe_mid``     Laguna-proportioned: hidden 128, 32 experts, top-8,
                  intermediate 32, shared 32, routed scale 1.0, 16 tokens.
* ``model_tiny``  the whole ``LagunaForCausalLM`` (3 layers: layer 0 dense, 1-2 MoE; hidden
                  64, 4 query / 2 kv heads of 32, per-head gate, RoPE theta 1e4, 8 experts
                  top-2, vocab 96), fp32, 12 tokens; stores the state dict under its own
                  parameter names and the logits of every position.
* ``model_swa``   the same family with the real checkpoint's layer mix: sliding-window layers
                  (window 5) with default RoPE, full layers with YaRN and partial rotary
                  (half of the head dims), per-layer head counts; 16 tokens at positions
                  3000..3015.
"""
import copy
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent

CASES = {
    "moe_tiny": dict(hidden_size=64, num_experts=8, num_experts_per_tok=2,
                     moe_intermediate_size=32, shared_expert_intermediate_size=32,
                     moe_routed_scaling_factor=2.5, T=10, seed=0),
    "moe_mid": dict(hidden_size=128, num_experts=32, num_experts_per_tok=8,
                    moe_intermediate_size=32, shared_expert_intermediate_size=32,
                    moe_routed_scaling_factor=1.0, T=16, seed=1),
}


def main(ref_root):
    sys.path.insert(0, str(ref_root))
    from tests.reference.configuration_laguna import LagunaConfig
    from tests.reference.modeling_laguna import LagunaSparseMoeBlock

    for name, c in CASES.items():
        c = copy.deepcopy(c)
        T, seed = c.pop("T"), c.pop("seed")
        torch.manual_seed(seed)
        cfg = LagunaConfig(norm_topk_prob=True, **c)
        blk = LagunaSparseMoeBlock(cfg).float().eval()
        with torch.no_grad():
            for _, p in blk.named_parameters():
                p.copy_(0.05 * torch.randn_like(p))
            x = torch.randn(1, T, c["hidden_size"])
            logits, w, inds = blk.gate(x.reshape(T, -1))
            out = blk(x).reshape(T, -1)
        np.savez_compressed(
            OUT / f"{name}.npz",
            x=x.reshape(T, -1).numpy(),
            gate_w=blk.gate.weight.detach().numpy(),
            bias=blk.gate.e_score_correction_bias.detach().numpy(),
            gate_up=blk.experts.gate_up_proj.detach().numpy(),
            down=blk.experts.down_proj.detach().numpy(),
            sh_gate=blk.shared_expert.gate_proj.weight.detach().numpy(),
            sh_up=blk.shared_expert.up_proj.weight.detach().numpy(),
            sh_down=blk.shared_expert.down_proj.weight.detach().numpy(),
            k=np.int64(c["num_experts_per_tok"]),
            scale=np.float32(c["moe_routed_scaling_factor"]),
            ref_logits=logits.numpy(),
            ref_w=w.numpy(),
            ref_inds=inds.numpy(),
            ref_out=out.numpy(),
        )
        print(name, "written", out.shape)


def model_tiny(ref_root):
    sys.path.insert(0, str(ref_root))
    from tests.reference.configuration_laguna import LagunaConfig
    from tests.reference.modeling_laguna import LagunaForCausalLM

    torch.manual_seed(2)
    cfg = LagunaConfig(vocab_size=96, hidden_size=64, intermediate_size=128, num_hidden_layers=3,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                       gating="per-head", num_experts=8, num_experts_per_tok=2,
                       moe_intermediate_size=32, shared_expert_intermediate_size=32,
                       mlp_only_layers=[0], moe_routed_scaling_factor=2.5, norm_topk_prob=True,
                       rope_parameters={"rope_type": "default", "rope_theta": 10000.0},
                       rms_norm_eps=1e-6, tie_word_embeddings=False, max_position_embeddings=128)
    cfg._attn_implementation = "eager"
    model = LagunaForCausalLM(cfg).float().eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight"):
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
            else:
                p.copy_(0.08 * torch.randn_like(p))
        for name, b in model.named_buffers():
            if name.endswith("e_score_correction_bias"):
                b.copy_(0.3 * torch.randn_like(b))
        ids = torch.randint(0, 96, (1, 12))
        logits = model(input_ids=ids, use_cache=False).logits[0]
    state = {k: v.detach().float().numpy() for k, v in model.state_dict().items()}
    np.savez_compressed(OUT / "model_tiny.npz", ids=ids[0].numpy(), ref_logits=logits.numpy(),
                        **{"w." + k: v for k, v in state.items()})
    print("model_tiny written", logits.shape)


# the real checkpoint's layer mix (lagunaLab tests/tiny.py:11-18): YaRN with half the head dims
# rotated on full-attention layers, default RoPE on sliding-window layers
SWA_ROPE = {
    "full_attention": {
        "rope_theta": 500000.0, "rope_type": "yarn", "factor": 32.0,
        "original_max_position_embeddings": 8192, "beta_slow": 1.0, "beta_fast": 64.0,
        "attention_factor": 1.3465735902799727, "partial_rotary_factor": 0.5,
    },
    "sliding_attention": {"rope_type": "default", "rope_theta": 10000.0,
                          "partial_rotary_factor": 1.0},
}


def model_swa(ref_root):
    """``model_swa``: 4 layers (full, sliding, sliding, full; window 5) with the YaRN /
    partial-rotary full layers of the real checkpoint, 16 tokens (past the window)."""
    sys.path.insert(0, str(ref_root))
    from tests.reference.configuration_laguna import LagunaConfig
    from tests.reference.modeling_laguna import LagunaForCausalLM

    torch.manual_seed(3)
    cfg = LagunaConfig(vocab_size=96, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
                       num_attention_heads=4, num_attention_heads_per_layer=[4, 4, 8, 4],
                       num_key_value_heads=2, head_dim=32, gating="per-head", num_experts=8,
                       num_experts_per_tok=2, moe_intermediate_size=32,
                       shared_expert_intermediate_size=32, mlp_only_layers=[0],
                       moe_routed_scaling_factor=2.5, norm_topk_prob=True,
                       rope_parameters=copy.deepcopy(SWA_ROPE), sliding_window=5,
                       layer_types=["full_attention", "sliding_attention", "sliding_attention",
                                    "full_attention"],
                       rms_norm_eps=1e-6, tie_word_embeddings=False,
                       max_position_embeddings=262144)
    cfg._attn_implementation = "eager"
    model = LagunaForCausalLM(cfg).float().eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight"):
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
            else:
                p.copy_(0.08 * torch.randn_like(p))
        for name, b in model.named_buffers():
            if name.endswith("e_score_correction_bias"):
                b.copy_(0.3 * torch.randn_like(b))
        ids = torch.randint(0, 96, (1, 16))
        pos = torch.arange(16)[None] + 3000  # far past the window, and into YaRN's ramp
        logits = model(input_ids=ids, position_ids=pos, use_cache=False).logits[0]
    state = {k: v.detach().float().numpy() for k, v in model.state_dict().items()}
    np.savez_compressed(OUT / "model_swa.npz", ids=ids[0].numpy(), pos0=np.int64(3000),
                        ref_logits=logits.numpy(), **{"w." + k: v for k, v in state.items()})
    print("model_swa written", logits.shape)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <lagunaLab source root>")
    main(sys.argv[1])
    model_tiny(sys.argv[1])
    model_swa(sys.argv[1])
