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



# ----------------------------------------------------------------------------------------
# Full decoder (BASELINE config 3 and small test shapes)
# ----------------------------------------------------------------------------------------

def decoder_args(vocab=100352, hidden=2048, layers=40, heads=32, kv_heads=4, head_dim=128,
                 experts=64, top_k=8, moe_inter=1024, shared_inter=1024, dense_inter=8192,
                 rope_theta=1e6, routed_scale=2.5, gating="per-head"):
    """ModelArgs of a Laguna decoder; the defaults are BASELINE config 3 (the 50%-pruned
    model: 64 experts per layer, top-8, 40 layers, hidden 2048, GQA 32/4, head_dim 128,
    layer 0 dense with intermediate 8192, vocabulary 100,352, RoPE theta 1e6)."""
    return laguna.ModelArgs(
        model_type="laguna", vocab_size=vocab, hidden_size=hidden,
        intermediate_size=dense_inter, num_hidden_layers=layers, num_attention_heads=heads,
        num_key_value_heads=kv_heads, head_dim=head_dim, rms_norm_eps=1e-6, num_experts=experts,
        num_experts_per_tok=top_k, moe_intermediate_size=moe_inter,
        shared_expert_intermediate_size=shared_inter,
        rope_parameters={"rope_type": "default", "rope_theta": rope_theta},
        mlp_only_layers=[0], moe_routed_scaling_factor=routed_scale, gating=gating)


def decoder(args, seed=0, std=0.02, norm_noise=0.0, router_bias_std=0.0, device="cuda"):
    """A random-init Laguna ``Model``: every linear and the embedding 4-bit g64, the router
    8-bit g64 (laguna.py:236-238), bf16 norms (ones, plus ``norm_noise`` N(0,1) noise)."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    H, D = args.hidden_size, args.head_dim
    ql = lambda shape, bits=4: laguna.QuantizedLinear(
        *ops.quantize(_randn(shape, std, gen, dev), 64, bits), 64, bits)
    qs = lambda shape: laguna.SwitchLinear(*ops.quantize(_randn(shape, std, gen, dev), 64, 4))

    def norm(n):
        w = torch.ones(n, device=dev)
        if norm_noise:
            w = w + norm_noise * torch.randn(n, generator=gen, device=dev)
        return laguna.RMSNorm(n, args.rms_norm_eps, w.to(torch.bfloat16))

    emb = ql((args.vocab_size, H))
    embed = laguna.QuantizedEmbedding(emb.weight, emb.scales, emb.biases)
    layers = []
    for i in range(args.num_hidden_layers):
        Hq, Hkv = args.num_attention_heads_per_layer[i], args.num_key_value_heads
        G = Hq if args.gating == "per-head" else Hq * D
        attn = laguna.Attention(args, i, ql((Hq * D, H)), ql((Hkv * D, H)), ql((Hkv * D, H)),
                                ql((H, Hq * D)), ql((G, H)), norm(D), norm(D))
        if i in args.mlp_only_layers:
            I = args.intermediate_size
            mlp = laguna.MLP(H, I, ql((I, H)), ql((I, H)), ql((H, I)))
        else:
            E, I, Ish = args.num_experts, args.moe_intermediate_size, args.shared_expert_intermediate_size
            sw = laguna.SwitchGLU(H, I, E, qs((E, I, H)), qs((E, I, H)), qs((E, H, I)))
            sh = laguna.MLP(H, Ish, ql((Ish, H)), ql((Ish, H)), ql((H, Ish))) if Ish else None
            bias = (router_bias_std * torch.randn(E, generator=gen, device=dev)
                    if router_bias_std else torch.zeros(E, device=dev))
            mlp = laguna.SparseMoeBlock(args, ql((E, H), bits=8), bias, sw, sh)
        layers.append(laguna.DecoderLayer(args, i, attn, mlp, norm(H), norm(H)))
    model = laguna.LagunaModel(args, embed, layers, norm(H))
    return laguna.Model(args, model, ql((args.vocab_size, H)))


def oracle_weights(model):
    """The model's weights as the CPU oracle's dict (oracle/model_ref.py)."""
    cpu = lambda m: tuple(t.cpu() for t in m.mat)
    W = {"embed": cpu(model.model.embed_tokens), "norm": model.model.norm.weight.float().cpu(),
         "lm_head": cpu(model.lm_head), "layers": []}
    for L in model.layers:
        a = L.self_attn
        d = {"in_norm": L.input_layernorm.weight.float().cpu(),
             "post_norm": L.post_attention_layernorm.weight.float().cpu(),
             "q_norm": a.q_norm.weight.float().cpu(), "k_norm": a.k_norm.weight.float().cpu(),
             "q": cpu(a.q_proj), "k": cpu(a.k_proj), "v": cpu(a.v_proj), "o": cpu(a.o_proj),
             "g": cpu(a.g_proj)}
        m = L.mlp
        if isinstance(m, laguna.MLP):
            d["mlp"] = ("dense", tuple(cpu(p) for p in (m.gate_proj, m.up_proj, m.down_proj)))
        else:
            sw = m.switch_mlp
            d["mlp"] = ("moe", {
                "gate": cpu(m.gate) if isinstance(m.gate, laguna.QuantizedLinear) else m.gate.cpu(),
                "bias": m.e_score_correction_bias.float().cpu(),
                "experts": tuple(cpu(p) for p in (sw.gate_proj, sw.up_proj, sw.down_proj)),
                "shared": tuple(cpu(p) for p in (m.shared_expert.gate_proj, m.shared_expert.up_proj,
                                                 m.shared_expert.down_proj))})
        W["layers"].append(d)
    return W


def oracle_args(args):
    return dict(head_dim=args.head_dim, heads=list(args.num_attention_heads_per_layer),
                kv_heads=args.num_key_value_heads, eps=args.rms_norm_eps,
                rope_theta=float(args.rope_for("full_attention")["rope_theta"]),
                gating="per-head" if args.gating == "per-head" else "element",
                k=args.num_experts_per_tok, routed_scale=args.moe_routed_scaling_factor,
                norm_topk_prob=args.norm_topk_prob)
