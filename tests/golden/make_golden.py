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


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <lagunaLab source root>")
    main(sys.argv[1])
