"""TEST INFRASTRUCTURE — CPU restatement of the full Laguna decoder (laguna_mlx/laguna.py:75-206).

Used only by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline, as the checker
of the B200 decoder; never by the library.

Two forms:
* ``forward`` follows the MLX graph of the reference: MLX-layout quantized weights
  (4-bit g64 linears and embedding, 8-bit router) dequantized to fp32, fp32 arithmetic,
  and every op output materialised in bf16 where MLX materialises it (RMSNorm, each
  quantized matmul, q/k norm, RoPE, SDPA output, gate, residual adds, MoE block).
* ``forward_fp32`` is the same architecture on unquantized fp32 weights with no rounding;
  it is pinned against Poolside's PyTorch model (tests/reference/modeling_laguna.py,
  LagunaForCausalLM) by the golden fixture ``tests/golden/model_tiny.npz``.

Weights are a dict:
  {"embed": mat, "norm": w, "lm_head": mat, "layers": [layer...]}
  layer = {"in_norm": w, "post_norm": w, "q": mat, "k": mat, "v": mat, "o": mat, "g": mat,
           "q_norm": w, "k_norm": w, "mlp": ("dense", (gate, up, down)) or
           ("moe", {"gate": router weight, "bias": fp32 [E], "experts": (gate, up, down),
                    "shared": (gate, up, down)})}
  mat = (uint32 packed, bf16 scales, bf16 biases) in ``forward``; an fp32 [out, in] matrix
  in ``forward_fp32``.
"""
import math

import torch

from . import moe_ref


def _bf(t):
    return t.to(torch.bfloat16).to(torch.float32)


def _deq(mat, bits=4):
    q, s, b = mat
    return moe_ref.dequantize(q, s, b, 64, bits)


def rmsnorm(x, w, eps):
    """mx.fast.rms_norm: bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w), fp32 statistics."""
    xf = x.to(torch.float32)
    r = 1.0 / torch.sqrt((xf * xf).mean(-1, keepdim=True) + eps)
    return _bf(_bf(xf * r) * w.to(torch.float32))


def rope_params(p, head_dim):
    """(rotated dims R, inv_freq fp32 [R/2], mscale) of one layer type's RoPE parameters.

    default (laguna.py:69-72 -> mx.fast.rope): inv_freq_i = theta^(-2i/R).
    yarn (YaRN, Peng et al. 2023, as transformers 5.5's ``_compute_yarn_parameters`` computes
    it for the vendored PyTorch model): per frequency, a linear ramp between the
    ``factor``-interpolated and the original frequency over the dims whose wavelength falls
    between ``beta_fast`` and ``beta_slow`` rotations of ``original_max_position_embeddings``;
    mscale = ``attention_factor`` (default 0.1 ln(factor) + 1).
    ``partial_rotary_factor`` f rotates the first R = int(head_dim * f) dims only."""
    R = int(head_dim * p.get("partial_rotary_factor", 1.0))
    base = float(p["rope_theta"])
    idx = torch.arange(0, R, 2, dtype=torch.float64)
    if p.get("rope_type", "default") == "default":
        return R, (base ** (-idx / R)).to(torch.float32), 1.0
    if p["rope_type"] != "yarn":
        raise NotImplementedError(p["rope_type"])
    factor = float(p["factor"])
    orig = float(p.get("original_max_position_embeddings", 4096))
    fast, slow = float(p.get("beta_fast", 32.0)), float(p.get("beta_slow", 1.0))
    mscale = p.get("attention_factor")
    if mscale is None:
        mscale = 0.1 * math.log(factor) + 1.0 if factor > 1 else 1.0

    def corr_dim(rot):
        return R * math.log(orig / (rot * 2 * math.pi)) / (2 * math.log(base))

    lo = max(math.floor(corr_dim(fast)), 0)
    hi = min(math.ceil(corr_dim(slow)), R - 1)
    if lo == hi:
        hi += 0.001
    ramp = ((torch.arange(R // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0, 1)
    extra = 1 - ramp  # weight of the original (extrapolated) frequency
    pos_freq = base ** (idx / R)
    inv = (1 / (factor * pos_freq)) * (1 - extra) + (1 / pos_freq) * extra
    return R, inv.to(torch.float32), float(mscale)


def rope(x, pos0, theta, R=None, inv=None, mscale=1.0):
    """RoPE of the mlx-lm layer (laguna.py:62-72, 99-100; mx.fast.rope, traditional=False):
    pairs (i, i + R/2) of the first R dims, positions pos0 + t along dim -2, fp32 angles and
    one bf16 rounding; dims past R pass through. Default: R = D, inv_freq_i = theta^(-2i/D).
    mscale != 1 (YaRN) scales the rotated dims first, rounded to the input's bf16 as
    mlx-lm's YaRN layer does before its fast rope."""
    D = x.shape[-1]
    R = D if R is None else R
    half = R // 2
    if inv is None:
        i = torch.arange(half, dtype=torch.float32, device=x.device)
        inv = torch.exp2(-(2.0 * i) / R * math.log2(theta))
    inv = inv.to(device=x.device, dtype=torch.float32)
    pos = torch.arange(x.shape[-2], dtype=torch.float32, device=x.device) + float(pos0)
    ang = pos[:, None] * inv[None, :]
    c, s = torch.cos(ang), torch.sin(ang)
    xr = x[..., :R].to(torch.float32)
    if mscale != 1.0:
        xr = _bf(xr * mscale)
    x1, x2 = xr[..., :half], xr[..., half:]
    out = torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)
    if R < D:
        out = torch.cat([out, x[..., R:].to(torch.float32)], dim=-1)
    return _bf(out)


def softplus(x):
    """nn.softplus = logaddexp(x, 0), in fp32."""
    return torch.clamp(x, min=0) + torch.log1p(torch.exp(-x.abs()))


def sdpa(q, k, v, scale, q_pos0, q_chunk=512, window=None):
    """Causal attention for queries at positions q_pos0 + t over keys 0..S-1 (fp32, GQA),
    output rounded to bf16. q [Hq, T, D], k/v [Hkv, S, D]. ``window`` W (sliding-window
    layers, laguna.py:183-186): a query at p sees keys p - W < j <= p only. Rows of queries
    are independent, so long prompts are processed ``q_chunk`` queries at a time (same
    values, bounded memory)."""
    Hq, T, D = q.shape
    Hkv, S, _ = k.shape
    G = Hq // Hkv
    kk = k.to(torch.float32)
    vv = v.to(torch.float32)
    out = torch.empty(Hq, T, D, dtype=torch.float32, device=q.device)
    kpos = torch.arange(S, device=q.device)[None, :]
    for a in range(0, T, q_chunk):
        b = min(T, a + q_chunk)
        qc = q[:, a:b].to(torch.float32).reshape(Hkv, G * (b - a), D)
        s = (qc @ kk.transpose(1, 2)).view(Hkv, G, b - a, S) * scale
        qpos = torch.arange(a, b, device=q.device)[:, None] + q_pos0
        hide = kpos > qpos
        if window:
            hide = hide | (kpos <= qpos - window)
        s = s.masked_fill(hide, float("-inf"))
        pr = torch.softmax(s, dim=-1).view(Hkv, G * (b - a), S)
        out[:, a:b] = (pr @ vv).view(Hq, b - a, D)
    return _bf(out)


class Cache:
    """K/V per layer ([Hkv, S, D] fp32 tensors): bf16-valued, or with ``kv_bits=8`` the rows
    as an 8-bit group-64 DequantKVCache holds them (laguna_mlx/cache.py:66-106): quantized by
    the build's quantizer on append, dequantized as fp32 scale * code + bias (the fused
    single-token kernel's view, q8_attn.py:50) — multi-token steps see them rounded to bf16
    (mx.dequantize's output, cache.py:99-100).

    Rows live in per-layer buffers of ``capacity`` rows that grow by doubling, so an append
    copies only the new rows. ``preload`` installs rows a test made elsewhere (for a decode
    that starts from a given cache state)."""

    def __init__(self, n_layers, kv_bits=None, capacity=256):
        self.kb = [None] * n_layers
        self.vb = [None] * n_layers
        self.n = [0] * n_layers
        self.offset = 0
        self.kv_bits = kv_bits
        self.capacity = capacity

    def _bits(self, i):
        """KV bits of layer i: ``kv_bits`` may be a per-layer list (None: bf16 rows, as the
        sliding-window layers of a quantized cache keep, laguna_mlx/cache.py:147-157)."""
        return self.kv_bits[i] if isinstance(self.kv_bits, (list, tuple)) else self.kv_bits

    def _qdq(self, x, bits):
        from . import attn_ref, mlx_quant
        packed, s_bits, b_bits = attn_ref.quantize_rows(x.cpu().numpy(), 64, bits)
        return torch.from_numpy(mlx_quant.dequantize(packed, s_bits, b_bits, 64,
                                                     bits)).to(x.device)

    def _room(self, i, Hkv, D, need, device="cpu"):
        buf = self.kb[i]
        if buf is not None and buf.shape[1] >= need:
            return
        cap = max(self.capacity, need, 2 * (buf.shape[1] if buf is not None else 0))
        k = torch.zeros(Hkv, cap, D, device=device)
        v = torch.zeros(Hkv, cap, D, device=device)
        if buf is not None:
            k[:, :self.n[i]] = self.kb[i][:, :self.n[i]]
            v[:, :self.n[i]] = self.vb[i][:, :self.n[i]]
        self.kb[i], self.vb[i] = k, v

    def preload(self, i, k, v):
        """Layer i holds exactly the fp32 rows k, v [Hkv, S, D] (already in the cache's
        representation: bf16 values, or dequantized 8-bit rows)."""
        Hkv, S, D = k.shape
        self.kb[i] = self.vb[i] = None
        self.n[i] = 0
        self._room(i, Hkv, D, S, k.device)
        self.kb[i][:, :S] = k
        self.vb[i][:, :S] = v
        self.n[i] = S

    @property
    def k(self):
        return [None if b is None else b[:, :n] for b, n in zip(self.kb, self.n)]

    @property
    def v(self):
        return [None if b is None else b[:, :n] for b, n in zip(self.vb, self.n)]

    def update(self, i, k, v):
        bits = self._bits(i)
        if bits:
            k, v = self._qdq(k, bits), self._qdq(v, bits)
        Hkv, T, D = k.shape
        n0 = self.n[i]
        self._room(i, Hkv, D, n0 + T, k.device)
        self.kb[i][:, n0:n0 + T] = k
        self.vb[i][:, n0:n0 + T] = v
        self.n[i] = n0 + T
        ck, cv = self.kb[i][:, :n0 + T], self.vb[i][:, :n0 + T]
        if bits and T > 1:
            return _bf(ck), _bf(cv)
        return ck, cv


def _attention(L, x, cache, i, args, pos0, lin):
    T = x.shape[0]
    D = args["head_dim"]
    Hq, Hkv = args["heads"][i], args["kv_heads"]
    eps = args["eps"]
    q = lin(x, L["q"]).view(T, Hq, D).transpose(0, 1)
    k = lin(x, L["k"]).view(T, Hkv, D).transpose(0, 1)
    v = lin(x, L["v"]).view(T, Hkv, D).transpose(0, 1)
    q = rmsnorm(q, L["q_norm"], eps)
    k = rmsnorm(k, L["k_norm"], eps)
    rp = args.get("rope", [None] * (i + 1))[i]
    if isinstance(rp, dict):
        rp = rope_params(rp, D)
    if rp is None:
        theta = args.get("rope_thetas", [args["rope_theta"]] * (i + 1))[i]
        q = rope(q, pos0, theta)
        k = rope(k, pos0, theta)
    else:
        q = rope(q, pos0, None, *rp)
        k = rope(k, pos0, None, *rp)
    if cache is not None:
        k, v = cache.update(i, k, v)
    window = args.get("window", [None] * (i + 1))[i]
    o = sdpa(q, k, v, D ** -0.5, pos0, window=window).transpose(0, 1)  # [T, Hq, D]
    g = _bf(softplus(lin(x, L["g"]).to(torch.float32)))
    g = g[..., None] if args["gating"] == "per-head" else g.view(T, Hq, D)
    return lin(_bf(o * g).reshape(T, Hq * D), L["o"])


def _qlin(x, mat):
    return moe_ref.qlinear(x, mat)


def forward(W, args, ids, cache=None, last_only=False):
    """Logits (bf16-valued fp32 [T, V]) of token ids [T] at positions cache.offset + t;
    ``last_only`` returns the last position's logits only ([1, V])."""
    ids = torch.as_tensor(ids, dtype=torch.int64)
    pos0 = cache.offset if cache is not None else 0
    eps = args["eps"]
    x = _bf(_deq_rows(W["embed"], ids))
    for i, L in enumerate(W["layers"]):
        a = _attention(L, rmsnorm(x, L["in_norm"], eps), cache, i, args, pos0, _qlin)
        h = _bf(x + a)
        hn = rmsnorm(h, L["post_norm"], eps)
        kind, m = L["mlp"]
        if kind == "dense":
            y = moe_ref.mlp(hn, *m)
        else:
            y, _, _ = moe_ref.moe_block(hn, m["gate"], m["bias"], m["experts"], m["shared"],
                                        args["k"], args["routed_scale"], args["norm_topk_prob"])
        x = _bf(h + y)
    if cache is not None:
        cache.offset += ids.shape[0]
    if last_only:
        x = x[-1:]
    return moe_ref.qlinear(rmsnorm(x, W["norm"], eps), W["lm_head"])


def _deq_rows(mat, ids):
    """Rows ``ids`` of a 4-bit embedding table, dequantized (only the rows looked up)."""
    q, s, b = mat
    return moe_ref.dequantize(q[ids], s[ids], b[ids], 64, 4)


def greedy(W, args, prompt, steps, kv_bits=None, top=0, forced=None):
    """Greedy decode (prefill, then one token at a time). Returns (tokens, gaps): gaps[i] is
    the logit margin between the chosen token and the runner-up at step i (a margin within
    a bf16 rounding of the logits marks a near-tie that other rounding orders may flip).
    ``kv_bits=8``: an 8-bit quantized KV cache (see ``Cache``). ``top=n`` also returns the n
    largest logits and their ids per step. ``forced`` (a token list): step i + 1 is fed
    forced[i] instead of the chosen token (teacher forcing), so every step's logits are
    defined by the given sequence."""
    cache = Cache(len(W["layers"]), kv_bits, capacity=len(prompt) + steps + 1)
    logits = forward(W, args, prompt, cache, last_only=True)
    toks, gaps, tops = [], [], []
    for i in range(steps):
        last = logits[-1]
        top2 = torch.topk(last, max(2, top))
        t = int(torch.argmax(last))
        toks.append(t)
        gaps.append(float(top2.values[0] - top2.values[1]))
        if top:
            tops.append((top2.values[:top].tolist(), top2.indices[:top].tolist()))
        if i + 1 < steps:
            nxt = forced[i] if forced is not None else t
            logits = forward(W, args, [nxt], cache)
    return (toks, gaps, tops) if top else (toks, gaps)


def weights_from_named(items, n_layers, quantize):
    """The oracle's weight dict from (MLX parameter name, kind, fp32 tensor) items — kind "q4"
    / "q8" (quantized by ``quantize(tensor, bits) -> (int32 words, bf16 scales, bf16
    biases)``), "norm" (rounded to bf16) or "bias" (fp32) — named as laguna.py:169-241 names
    them after ``sanitize``."""
    W = {"layers": [dict() for _ in range(n_layers)]}
    moe = [dict() for _ in range(n_layers)]
    dense = [dict() for _ in range(n_layers)]
    for name, kind, t in items:
        if kind in ("q4", "q8"):
            v = quantize(t, 4 if kind == "q4" else 8)
        elif kind == "norm":
            v = _bf(t)
        else:
            v = t.to(torch.float32)
        if name == "model.embed_tokens":
            W["embed"] = v
        elif name == "model.norm":
            W["norm"] = v
        elif name == "lm_head":
            W["lm_head"] = v
        else:
            parts = name.split(".")
            i = int(parts[2])
            L = W["layers"][i]
            rest = ".".join(parts[3:])
            simple = {"self_attn.q_proj": "q", "self_attn.k_proj": "k", "self_attn.v_proj": "v",
                      "self_attn.o_proj": "o", "self_attn.g_proj": "g",
                      "self_attn.q_norm": "q_norm", "self_attn.k_norm": "k_norm",
                      "input_layernorm": "in_norm", "post_attention_layernorm": "post_norm"}
            if rest in simple:
                L[simple[rest]] = v
            elif rest.startswith("mlp.switch_mlp."):
                moe[i][rest.split(".")[2]] = v
            elif rest.startswith("mlp.shared_expert."):
                moe[i]["sh_" + rest.split(".")[2]] = v
            elif rest == "mlp.gate":
                moe[i]["router"] = v
            elif rest == "mlp.e_score_correction_bias":
                moe[i]["bias"] = v
            elif rest in ("mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
                dense[i][rest.split(".")[1]] = v
            else:
                raise KeyError(name)
    for i, L in enumerate(W["layers"]):
        if dense[i]:
            d = dense[i]
            L["mlp"] = ("dense", (d["gate_proj"], d["up_proj"], d["down_proj"]))
        else:
            m = moe[i]
            L["mlp"] = ("moe", {
                "gate": m["router"], "bias": m["bias"],
                "experts": (m["gate_proj"], m["up_proj"], m["down_proj"]),
                "shared": (m["sh_gate_proj"], m["sh_up_proj"], m["sh_down_proj"])})
    return W


# ---------------------------------------------------------------------------------------
# Unquantized, unrounded form (pinned against the vendored PyTorch model).
# ---------------------------------------------------------------------------------------

def _rms32(x, w, eps):
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * w


def _rope32(x, pos0, theta, R=None, inv=None, mscale=1.0):
    """The vendored PyTorch model's RoPE (modeling_laguna.py:68-128, :277-312): cos and sin of
    position x inv_freq times the attention scaling, rotate_half over the first R dims."""
    D = x.shape[-1]
    R = D if R is None else R
    half = R // 2
    if inv is None:
        inv = 1.0 / (theta ** (torch.arange(0, R, 2, dtype=torch.float32) / R))
    pos = torch.arange(x.shape[-2], dtype=torch.float32) + float(pos0)
    ang = pos[:, None] * inv[None, :]
    c, s = torch.cos(ang) * mscale, torch.sin(ang) * mscale
    x1, x2 = x[..., :half], x[..., half:R]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c, x[..., R:]], dim=-1)


def forward_fp32(W, args, ids, pos0=0):
    """fp32 logits [T, V] of a whole sequence at positions pos0 + t (no cache)."""
    ids = torch.as_tensor(ids, dtype=torch.int64)
    T = ids.shape[0]
    eps, D = args["eps"], args["head_dim"]
    x = W["embed"][ids].to(torch.float32)
    for i, L in enumerate(W["layers"]):
        Hq, Hkv = args["heads"][i], args["kv_heads"]
        xn = _rms32(x, L["in_norm"], eps)
        q = (xn @ L["q"].T).view(T, Hq, D).transpose(0, 1)
        k = (xn @ L["k"].T).view(T, Hkv, D).transpose(0, 1)
        v = (xn @ L["v"].T).view(T, Hkv, D).transpose(0, 1)
        rp = args.get("rope", [None] * (i + 1))[i] or (None, None, 1.0)
        q = _rope32(_rms32(q, L["q_norm"], eps), pos0, args["rope_theta"], *rp)
        k = _rope32(_rms32(k, L["k_norm"], eps), pos0, args["rope_theta"], *rp)
        G = Hq // Hkv
        s = (q @ k.repeat_interleave(G, 0).transpose(1, 2)) * D ** -0.5
        hide = torch.ones(T, T, dtype=torch.bool).triu(1)
        window = args.get("window", [None] * (i + 1))[i]
        if window:
            hide = hide | torch.ones(T, T, dtype=torch.bool).tril(-window)
        s = s.masked_fill(hide, float("-inf"))
        o = (torch.softmax(s, -1) @ v.repeat_interleave(G, 0)).transpose(0, 1)
        g = softplus(xn @ L["g"].T)
        g = g[..., None] if args["gating"] == "per-head" else g.view(T, Hq, D)
        h = x + (o * g).reshape(T, Hq * D) @ L["o"].T
        hn = _rms32(h, L["post_norm"], eps)
        kind, m = L["mlp"]
        if kind == "dense":
            gw, uw, dw = m
            y = (torch.nn.functional.silu(hn @ gw.T) * (hn @ uw.T)) @ dw.T
        else:
            gu = torch.cat([m["experts"][0], m["experts"][1]], dim=1)
            y = moe_ref.moe_block_fp32(hn, m["gate"], m["bias"], gu, m["experts"][2],
                                       *m["shared"], args["k"], args["routed_scale"],
                                       args["norm_topk_prob"])[0]
        x = h + y
    return _rms32(x, W["norm"], eps) @ W["lm_head"].T
