"""Seeded synthetic inputs with the BASELINE shapes (no datasets or checkpoints are used).

Weights are drawn N(0, std) on the GPU from a seeded generator and quantized to the MLX
4-bit affine group-64 layout (bf16 scales/biases) by this library's quantizer; the same
packed tensors feed the kernels and, in tests, the CPU oracle.

Skewed routing (Zipf(1.1) expert popularity): the router's selection-only
bias ``e_score_correction_bias`` (laguna_mlx/laguna.py:133, :140) is set to
``beta * log p_{pi(e)}`` with p proportional to r^-1.1 over ranks r = 1..E and pi a seeded
permutation. beta = 0.045 puts the busiest of 128 experts at ~1,200 of 4,096 x 8 picks.
"""
import torch

from . import laguna, ops

ZIPF_S = 1.1
ZIPF_BETA = 0.045


def zipf_bias(E, seed, beta=ZIPF_BETA, s=ZIPF_S, device="cuda"):
    g = torch.Generator().manual_seed(seed + 7919)
    perm = torch.randperm(E, generator=g)
    r = torch.arange(1, E + 1, dtype=torch.float64)
    logp = -s * torch.log(r)
    bias = beta * (logp - logp.max())
    out = torch.empty(E, dtype=torch.float64)
    out[perm] = bias
    return out.to(torch.float32).to(device)


def _randn(shape, std, gen, device):
    return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std


def moe_block(T, E=128, k=8, H=2048, I=1024, I_sh=1024, seed=0, std=0.02, zipf=False,
              routed_scaling_factor=1.0, device="cuda"):
    """A Laguna-shaped SparseMoeBlock with random 4-bit weights and bf16 N(0,1) input x."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    router = _randn((E, H), std, gen, dev)
    q = lambda shape: laguna.SwitchLinear(*ops.quantize(_randn(shape, std, gen, dev), 64, 4))
    sw = laguna.SwitchGLU(H, I, E, q((E, I, H)), q((E, I, H)), q((E, H, I)))
    sh = None
    if I_sh:
        ql = lambda shape: laguna.QuantizedLinear(*ops.quantize(_randn(shape, std, gen, dev), 64, 4))
        sh = laguna.MLP(H, I_sh, ql((I_sh, H)), ql((I_sh, H)), ql((H, I_sh)))
    bias = zipf_bias(E, seed, device=dev) if zipf else torch.zeros(E, device=dev)
    args = laguna.ModelArgs(
        model_type="laguna", vocab_size=100352, hidden_size=H, intermediate_size=8192,
        num_hidden_layers=1, num_attention_heads=32, num_key_value_heads=4, head_dim=128,
        rms_norm_eps=1e-6, num_experts=E, num_experts_per_tok=k, moe_intermediate_size=I,
        shared_expert_intermediate_size=I_sh, rope_parameters={"rope_theta": 1e6},
        moe_routed_scaling_factor=routed_scaling_factor, mlp_only_layers=[])
    blk = laguna.SparseMoeBlock(args, router, bias, sw, sh)
    x = torch.randn(T, H, generator=gen, device=dev).to(torch.bfloat16)
    return blk, x


def q8_layers(L, n, B=1, Hq=32, Hkv=4, seed=0, device="cuda"):
    """L independent 8-bit group-64 caches of n keys (K, V ~ N(0,1) bf16) plus a query each."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    cap = (n + 255) // 256 * 256
    layers = []
    for _ in range(L):
        kv = []
        for _ in range(2):
            x = torch.randn(B, Hkv, n, 128, generator=gen, device=dev).to(torch.bfloat16)
            t = (torch.zeros(B, Hkv, cap, 32, dtype=torch.int32, device=dev),
                 torch.zeros(B, Hkv, cap, 2, dtype=torch.bfloat16, device=dev),
                 torch.zeros(B, Hkv, cap, 2, dtype=torch.bfloat16, device=dev))
            ops.quantize_into(x, t, 0, 64, 8)
            del x
            kv.append(t)
        q = torch.randn(B, Hq, 1, 128, generator=gen, device=dev).to(torch.bfloat16)
        layers.append((q, kv[0], kv[1]))
    return layers


def q8_bytes_per_layer(n, B=1, Hkv=4, D=128):
    """Algorithmic bytes of one layer's decode attention: K and V codes plus their bf16
    scales and biases for n keys (query and output are negligible)."""
    per_key = 2 * (D + 2 * (D // 64) * 2)
    return B * Hkv * n * per_key


def moe_flops(T, k, H, I, I_sh):
    """Algorithmic FLOPs of one MoE block forward: 3 products of 2*H*I per routed pick and
    2*H*I_sh per shared row (the router and elementwise work are not counted)."""
    return 2.0 * 3 * H * (T * k * I + T * I_sh)


def gateup_flops(T, k, H, I, I_sh):
    return 2.0 * 2 * H * (T * k * I + T * I_sh)

