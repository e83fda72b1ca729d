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


def rope(x, pos0, theta):
    """Default RoPE (laguna.py:69-72; mx.fast.rope, traditional=False): pairs (i, i + D/2),
    inv_freq_i = theta^(-2i/D), positions pos0 + t along dim -2. fp32, one bf16 rounding."""
    D = x.shape[-1]
    half = D // 2
    i = torch.arange(half, dtype=torch.float32)
    inv = torch.exp2(-(2.0 * i) / D * math.log2(theta))
    pos = torch.arange(x.shape[-2], dtype=torch.float32) + float(pos0)
    ang = pos[:, None] * inv[None, :]
    c, s = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :half].to(torch.float32), x[..., half:].to(torch.float32)
    return _bf(torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1))


def softplus(x):
    """nn.softplus = logaddexp(x, 0), in fp32."""
    return torch.clamp(x, min=0) + torch.log1p(torch.exp(-x.abs()))


def sdpa(q, k, v, scale, q_pos0):
    """Causal attention for queries at positions q_pos0 + t over keys 0..S-1 (fp32, GQA),
    output rounded to bf16. q [Hq, T, D], k/v [Hkv, S, D]."""
    Hq, T, D = q.shape
    Hkv, S, _ = k.shape
    G = Hq // Hkv
    kk = k.repeat_interleave(G, dim=0).to(torch.float32)
    vv = v.repeat_interleave(G, dim=0).to(torch.float32)
    s = (q.to(torch.float32) @ kk.transpose(1, 2)) * scale
    qpos = torch.arange(T)[:, None] + q_pos0
    kpos = torch.arange(S)[None, :]
    s = s.masked_fill(kpos > qpos, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return _bf(p @ vv)


class Cache:
    """K/V per layer ([Hkv, S, D] fp32 tensors): bf16-valued, or with ``kv_bits=8`` the rows
    as an 8-bit group-64 DequantKVCache holds them (laguna_mlx/cache.py:66-106): quantized by
    the build's quantizer on append, dequantized as fp32 scale * code + bias (the fused
    single-token kernel's view, q8_attn.py:50) — multi-token steps see them rounded to bf16
    (mx.dequantize's output, cache.py:99-100)."""

    def __init__(self, n_layers, kv_bits=None):
        self.k = [None] * n_layers
        self.v = [None] * n_layers
        self.offset = 0
        self.kv_bits = kv_bits

    def _qdq(self, x):
        from . import attn_ref, mlx_quant
        packed, s_bits, b_bits = attn_ref.quantize_rows(x.numpy(), 64, self.kv_bits)
        return torch.from_numpy(mlx_quant.dequantize(packed, s_bits, b_bits, 64, self.kv_bits))

    def update(self, i, k, v):
        if self.kv_bits:
            k, v = self._qdq(k), self._qdq(v)
        self.k[i] = k if self.k[i] is None else torch.cat([self.k[i], k], dim=1)
        self.v[i] = v if self.v[i] is None else torch.cat([self.v[i], v], dim=1)
        if self.kv_bits and k.shape[1] > 1:
            return _bf(self.k[i]), _bf(self.v[i])
        return self.k[i], self.v[i]


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
    q = rope(q, pos0, args["rope_theta"])
    k = rope(k, pos0, args["rope_theta"])
    if cache is not None:
        k, v = cache.update(i, k, v)
    o = sdpa(q, k, v, D ** -0.5, pos0).transpose(0, 1)  # [T, Hq, D]
    g = _bf(softplus(lin(x, L["g"]).to(torch.float32)))
    g = g[..., None] if args["gating"] == "per-head" else g.view(T, Hq, D)
    return lin(_bf(o * g).reshape(T, Hq * D), L["o"])


def _qlin(x, mat):
    return moe_ref.qlinear(x, mat)


def forward(W, args, ids, cache=None):
    """Logits (bf16-valued fp32 [T, V]) of token ids [T] at positions cache.offset + t."""
    ids = torch.as_tensor(ids, dtype=torch.int64)
    pos0 = cache.offset if cache is not None else 0
    eps = args["eps"]
    x = _bf(_deq(W["embed"])[ids])
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
    return moe_ref.qlinear(rmsnorm(x, W["norm"], eps), W["lm_head"])


def greedy(W, args, prompt, steps, kv_bits=None):
    """Greedy decode (prefill, then one token at a time). Returns (tokens, gaps): gaps[i] is
    the logit margin between the chosen token and the runner-up at step i (a margin within
    a bf16 rounding of the logits marks a near-tie that other rounding orders may flip).
    ``kv_bits=8``: an 8-bit quantized KV cache (see ``Cache``)."""
    cache = Cache(len(W["layers"]), kv_bits)
    logits = forward(W, args, prompt, cache)
    toks, gaps = [], []
    for _ in range(steps):
        last = logits[-1]
        top2 = torch.topk(last, 2)
        t = int(torch.argmax(last))
        toks.append(t)
        gaps.append(float(top2.values[0] - top2.values[1]))
        logits = forward(W, args, [t], cache)
    return toks, gaps


# ---------------------------------------------------------------------------------------
# Unquantized, unrounded form (pinned against the vendored PyTorch model).
# ---------------------------------------------------------------------------------------

def _rms32(x, w, eps):
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * w


def _rope32(x, pos0, theta):
    D = x.shape[-1]
    half = D // 2
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    pos = torch.arange(x.shape[-2], dtype=torch.float32) + float(pos0)
    ang = pos[:, None] * inv[None, :]
    c, s = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


def forward_fp32(W, args, ids):
    """fp32 logits [T, V] of a whole sequence from position 0 (no cache)."""
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
        q = _rope32(_rms32(q, L["q_norm"], eps), 0, args["rope_theta"])
        k = _rope32(_rms32(k, L["k_norm"], eps), 0, args["rope_theta"])
        G = Hq // Hkv
        s = (q @ k.repeat_interleave(G, 0).transpose(1, 2)) * D ** -0.5
        s = s.masked_fill(torch.ones(T, T, dtype=torch.bool).triu(1), float("-inf"))
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
