"""Seeded synthetic inputs with the BASELINE shapes (no datasets or checkpoints are used).

MoE-block weights are drawn N(0, std) on the GPU from a seeded generator and quantized to
the MLX 4-bit affine group-64 layout (bf16 scales/biases) by this library's quantizer; the
same packed tensors feed the kernels and, in tests, the CPU oracle. Full decoders (BASELINE
config 3) draw their weights from ``hash_normal``, a counter-based generator that gives the
same bits on the CPU and the GPU, so a CPU checker can rebuild the exact model a GPU run
used without copying 1.8 GB of packed weights.

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
                 rope_theta=1e6, routed_scale=2.5, gating="per-head", layer_types=None,
                 sliding_window=None, rope_parameters=None, heads_per_layer=None):
    """ModelArgs of a Laguna decoder; the defaults are BASELINE config 3 (the 50%-pruned
    model: 64 experts per layer, top-8, 40 layers, hidden 2048, GQA 32/4, head_dim 128,
    layer 0 dense with intermediate 8192, vocabulary 100,352, RoPE theta 1e6)."""
    return laguna.ModelArgs(
        model_type="laguna", vocab_size=vocab, hidden_size=hidden,
        intermediate_size=dense_inter, num_hidden_layers=layers, num_attention_heads=heads,
        num_key_value_heads=kv_heads, head_dim=head_dim, rms_norm_eps=1e-6, num_experts=experts,
        num_experts_per_tok=top_k, moe_intermediate_size=moe_inter,
        shared_expert_intermediate_size=shared_inter,
        rope_parameters=rope_parameters or {"rope_type": "default", "rope_theta": rope_theta},
        mlp_only_layers=[0], moe_routed_scaling_factor=routed_scale, gating=gating,
        layer_types=layer_types, sliding_window=sliding_window,
        num_attention_heads_per_layer=heads_per_layer)


_M32 = 0xFFFFFFFF
# Irwin-Hall(4) over bytes: the sum of four uniform bytes has mean 510 and standard deviation
# sqrt(4 * (256^2 - 1) / 12)
_IH_MEAN = 510.0
_IH_SD = (4 * (256 ** 2 - 1) / 12) ** 0.5


def _mix32(x):
    """A 32-bit integer hash (xor-shift / multiply rounds) on an int64 tensor holding values in
    [0, 2^32). The multipliers are odd and below 2^31, so every product stays below 2^63 and
    CPU and CUDA compute the same bits."""
    x = x ^ (x >> 16)
    x = (x * 0x7FEB352D) & _M32
    x = x ^ (x >> 15)
    x = (x * 0x2C1B3C6D) & _M32
    return x ^ (x >> 16)


def _mix32_int(v):
    return int(_mix32(torch.tensor([v & _M32], dtype=torch.int64))[0])


def hash_normal(shape, seed, stream, std=1.0, device="cuda", chunk=1 << 24):
    """Seeded approximately-normal fp32 values (mean 0, standard deviation ``std``, |x| <=
    3.45 std) that are bit-identical on the CPU and on the GPU: element i of (seed, stream) is
    the Irwin-Hall sum of the four bytes of a two-round integer hash of i, centred and scaled
    by one fp32 multiply. Used wherever a CPU checker must rebuild the exact weights or
    inputs a GPU run used (torch's CPU and CUDA generators draw different numbers)."""
    shape = tuple(int(d) for d in (shape if isinstance(shape, (tuple, list)) else (shape,)))
    n = 1
    for d in shape:
        n *= d
    if n >= 1 << 32:
        raise ValueError("hash_normal: at most 2^32 values per stream")
    k1 = _mix32_int(seed * 0x9E3779B1 + 0x632BE5AB)
    k2 = _mix32_int(stream * 0x85EBCA77 + k1)
    c = torch.tensor(std / _IH_SD, dtype=torch.float32, device=device)
    out = torch.empty(n, dtype=torch.float32, device=device)
    for a in range(0, n, chunk):
        b = min(n, a + chunk)
        x = torch.arange(a, b, dtype=torch.int64, device=device)
        x = _mix32(_mix32(x ^ k1) ^ k2)
        s = (x & 255) + ((x >> 8) & 255) + ((x >> 16) & 255) + (x >> 24)
        out[a:b] = (s.to(torch.float32) - _IH_MEAN) * c
    return out.view(shape)


def decoder_tensors(args, seed=0, std=0.02, norm_noise=0.0, router_bias_std=0.0, device="cuda",
                    want=None):
    """Every parameter of a random-init Laguna decoder, lazily, in one fixed order:
    (MLX parameter name, kind, fp32 tensor) with kind "q4" (a linear, the embedding or a
    stacked expert tensor, to be quantized 4-bit g64), "q8" (the router, 8-bit g64,
    laguna.py:236-238), "norm" (an RMSNorm weight: ones, plus ``norm_noise`` noise) or "bias"
    (the router's fp32 ``e_score_correction_bias``). Values come from ``hash_normal`` with one
    stream per tensor, so a CPU checker rebuilds the GPU model bit for bit. ``want(name)``
    (optional) selects the tensors to produce; the others are skipped without being drawn
    (their streams are still consumed, so the selected ones keep their values)."""
    for name, kind, make in _decoder_thunks(args, seed, std, norm_noise, router_bias_std,
                                            device):
        if want is None or want(name):
            yield name, kind, make()


def _decoder_thunks(args, seed, std, norm_noise, router_bias_std, device):
    """(name, kind, thunk) per decoder parameter; each thunk owns its stream id."""
    H, D, V = args.hidden_size, args.head_dim, args.vocab_size
    stream = iter(range(1 << 30))

    def normal(shape, s=std):
        sid = next(stream)
        return lambda: hash_normal(shape, seed, sid, s, device)

    def norm(n):
        sid = next(stream)

        def make():
            w = torch.ones(n, dtype=torch.float32, device=device)
            if norm_noise:
                w = w + hash_normal(n, seed, sid, norm_noise, device)
            return w
        return make

    yield "model.embed_tokens", "q4", normal((V, H))
    for i in range(args.num_hidden_layers):
        p = f"model.layers.{i}"
        Hq, Hkv = args.num_attention_heads_per_layer[i], args.num_key_value_heads
        G = Hq if args.gating == "per-head" else Hq * D
        for n, shape in (("q_proj", (Hq * D, H)), ("k_proj", (Hkv * D, H)),
                         ("v_proj", (Hkv * D, H)), ("o_proj", (H, Hq * D)), ("g_proj", (G, H))):
            yield f"{p}.self_attn.{n}", "q4", normal(shape)
        yield f"{p}.self_attn.q_norm", "norm", norm(D)
        yield f"{p}.self_attn.k_norm", "norm", norm(D)
        if i in args.mlp_only_layers:
            I = args.intermediate_size
            yield f"{p}.mlp.gate_proj", "q4", normal((I, H))
            yield f"{p}.mlp.up_proj", "q4", normal((I, H))
            yield f"{p}.mlp.down_proj", "q4", normal((H, I))
        else:
            E, I = args.num_experts, args.moe_intermediate_size
            Ish = args.shared_expert_intermediate_size
            yield f"{p}.mlp.switch_mlp.gate_proj", "q4", normal((E, I, H))
            yield f"{p}.mlp.switch_mlp.up_proj", "q4", normal((E, I, H))
            yield f"{p}.mlp.switch_mlp.down_proj", "q4", normal((E, H, I))
            if Ish:
                yield f"{p}.mlp.shared_expert.gate_proj", "q4", normal((Ish, H))
                yield f"{p}.mlp.shared_expert.up_proj", "q4", normal((Ish, H))
                yield f"{p}.mlp.shared_expert.down_proj", "q4", normal((H, Ish))
            sid = next(stream)
            bias = ((lambda sid=sid: hash_normal(E, seed, sid, router_bias_std, device))
                    if router_bias_std
                    else (lambda: torch.zeros(E, dtype=torch.float32, device=device)))
            yield f"{p}.mlp.e_score_correction_bias", "bias", bias
            yield f"{p}.mlp.gate", "q8", normal((E, H))
        yield f"{p}.input_layernorm", "norm", norm(H)
        yield f"{p}.post_attention_layernorm", "norm", norm(H)
    yield "model.norm", "norm", norm(H)
    yield "lm_head", "q4", normal((V, H))


def decoder_quantization(args):
    """The "quantization" config entry of these models: 4-bit g64, the routers 8-bit g64."""
    q = {"group_size": 64, "bits": 4}
    for i in range(args.num_hidden_layers):
        if i not in args.mlp_only_layers:
            q[f"model.layers.{i}.mlp.gate"] = {"group_size": 64, "bits": 8}
    return q


def decoder(args, seed=0, std=0.02, norm_noise=0.0, router_bias_std=0.0, device="cuda"):
    """A random-init Laguna ``Model``: every linear and the embedding 4-bit g64, the router
    8-bit g64 (laguna.py:236-238), bf16 norms; the tensors of ``decoder_tensors`` quantized on
    the GPU by the library's quantizer (bit-exact with the CPU checker's) and loaded through
    the MLX-name loader ``laguna.model_from_weights``."""
    weights = {}
    for name, kind, t in decoder_tensors(args, seed, std, norm_noise, router_bias_std, device):
        if kind in ("q4", "q8"):
            q, s, b = ops.quantize(t, 64, 4 if kind == "q4" else 8)
            weights[name + ".weight"], weights[name + ".scales"], weights[name + ".biases"] = q, s, b
        elif kind == "norm":
            weights[name + ".weight"] = t.to(torch.bfloat16)
        else:
            weights[name] = t
        del t
    return laguna.model_from_weights(args, weights, decoder_quantization(args), device)


KV_SEED_OFFSET = 7777


def kv_rows(layer, n, Hkv=4, D=128, seed=0, device="cuda"):
    """Synthetic K and V rows of one layer's cache, bf16 [Hkv, n, D] each: hash_normal N(0, 1)
    values (streams 2 * layer and 2 * layer + 1 of ``seed + KV_SEED_OFFSET``), the same bits on
    the CPU and the GPU. A decode that starts from such a cache state exercises attention at
    a long context without a prefill of that length (the CPU checker cannot run one)."""
    s = seed + KV_SEED_OFFSET
    k = hash_normal((Hkv, n, D), s, 2 * layer, 1.0, device).to(torch.bfloat16)
    v = hash_normal((Hkv, n, D), s, 2 * layer + 1, 1.0, device).to(torch.bfloat16)
    return k, v


def fill_q8_cache(cache, n, seed=0):
    """Fill rows [0, n) of every layer of a ``make_quantized_cache`` list with ``kv_rows``
    quantized 8-bit g64 by the library's quantizer, and set each layer's offset to n."""
    for i, c in enumerate(cache):
        qc = c.q
        k, v = kv_rows(i, n, seed=seed)
        Hkv, _, D = k.shape
        qc.reserve(1, Hkv, D, n, k.device)
        ops.quantize_into(k[None], qc.keys, 0, qc.group_size, qc.bits)
        ops.quantize_into(v[None], qc.values, 0, qc.group_size, qc.bits)
        qc.offset = n
        del k, v


def zipf_router(model, seed=0):
    """Zipf(1.1)-skewed routing for every MoE layer of a decoder: each
    layer's selection-only bias becomes ``zipf_bias`` with its own seeded permutation."""
    for i, L in enumerate(model.layers):
        m = L.mlp
        if isinstance(m, laguna.SparseMoeBlock):
            dev = m.e_score_correction_bias.device
            m.e_score_correction_bias = zipf_bias(m.num_experts, seed + 1000 * i, device=dev)


STREAM_KV_BASE = 1 << 20  # hash_normal stream ids of the batched-decode caches


def fill_stream_cache(cache, n, first_stream=0, seed=0):
    """Synthetic context for batched decode: rows [0, n) of every stream of every layer of a
    ``Model.make_stream_cache`` list get hash_normal N(0, 1) K and V rows (one generator stream
    per (layer, global stream index), so the rows of a stream do not depend on how the streams
    are split over ranks); a sliding layer's ring gets the last window's rows at position mod
    window. A decode step over such a cache reads the same bytes as one after a prefill."""
    s = seed + KV_SEED_OFFSET
    for i, c in enumerate(cache):
        B, Hkv, cap, D = c.keys.shape
        ring = isinstance(c, laguna.RotatingKVCache)
        for b in range(B):
            sid = STREAM_KV_BASE + 2 * (i * 4096 + first_stream + b)
            k = hash_normal((Hkv, n, D), s, sid, 1.0, c.keys.device).to(torch.bfloat16)
            v = hash_normal((Hkv, n, D), s, sid + 1, 1.0, c.keys.device).to(torch.bfloat16)
            if ring:
                p = torch.arange(max(0, n - cap), n, device=c.keys.device)
                c.keys[b][:, p % cap] = k[:, p]
                c.values[b][:, p % cap] = v[:, p]
            else:
                c.keys[b, :, :n] = k
                c.values[b, :, :n] = v
            del k, v


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
    """The CPU oracle's model arguments: per layer the RoPE parameters (None where the default
    rope rotates every head dim), their theta and the sliding window (None on full layers)."""
    rps = [args.rope_for(lt) for lt in args.layer_types]
    plain = lambda p: (p.get("rope_type", "default") == "default"
                       and p.get("partial_rotary_factor", 1.0) == 1.0)
    return dict(head_dim=args.head_dim, heads=list(args.num_attention_heads_per_layer),
                kv_heads=args.num_key_value_heads, eps=args.rms_norm_eps,
                rope_theta=float(args.rope_for("full_attention")["rope_theta"]),
                rope_thetas=[float(p["rope_theta"]) for p in rps],
                rope=[None if plain(p) else dict(p) for p in rps],
                window=[args.sliding_window if lt == "sliding_attention" else None
                        for lt in args.layer_types],
                gating="per-head" if args.gating == "per-head" else "element",
                k=args.num_experts_per_tok, routed_scale=args.moe_routed_scaling_factor,
                norm_topk_prob=args.norm_topk_prob)
