"""Shared helpers for the parity tests: seeded weights, MLX-layout quantization and the
tolerance metrics (max relative error = max|a - b| / max|b|, cosine similarity)."""
import numpy as np
import torch

# BASELINE bar for layer outputs: max relative error <= 2e-2 and cosine >= 0.999.
REL_TOL = 2e-2
COS_TOL = 0.999


def rel_err(a, b):
    a = a.detach().float().cpu()
    b = b.detach().float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def cos(a, b):
    a = a.detach().float().cpu().reshape(-1)
    b = b.detach().float().cpu().reshape(-1)
    return float(torch.nn.functional.cosine_similarity(a, b, dim=0))


def gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def normal(shape, std, g):
    return torch.randn(*shape, generator=g) * std


def moe_weights(E, H, I, I_sh, seed, std=0.02):
    """fp32 CPU weights: experts gate/up [E, I, H], down [E, H, I]; shared [I_sh, H] x2,
    [H, I_sh]; router fp32 [E, H]."""
    g = gen(seed)
    w = dict(
        gate=normal((E, I, H), std, g), up=normal((E, I, H), std, g),
        down=normal((E, H, I), std, g), router=normal((E, H), std, g),
    )
    if I_sh:
        w.update(sh_gate=normal((I_sh, H), std, g), sh_up=normal((I_sh, H), std, g),
                 sh_down=normal((H, I_sh), std, g))
    return w


def to_cpu(t):
    return tuple(x.cpu() for x in t)


def quant_np(w, bits=4, group=64):
    """The oracle's restated quantizer on a CPU fp32 tensor -> (int32 words, bf16 scales,
    bf16 biases) torch tensors."""
    from oracle import attn_ref

    q, s, b = attn_ref.quantize_rows(w.numpy(), group, bits)
    return (torch.from_numpy(q.view(np.int32)),
            torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
            torch.from_numpy(b.view(np.int16)).view(torch.bfloat16))
