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
    i = torch.arange(half, dtype=torch.float32, device=x.device)
    inv = torch.exp2(-(2.0 * i) / D * math.log2(theta))
    pos = torch.arange(x.shape[-2], dtype=torch.float32, device=x.device) + float(pos0)
    ang = pos[:, None] * inv[None, :]
    c, s = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :half].to(torch.float32), x[..., half:].to(torch.float32)
    return _bf(torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1))


def softplus(x):
    """nn.softplus = logaddexp(x, 0), in fp32."""
    return torch.clamp(x, min=0) + torch.log1p(torch.exp(-x.abs()))


def sdpa(q, k, v, scale, q_pos0, q_chunk=512):
    """Causal attention for queries at positions q_pos0 + t over keys 0..S-1 (fp32, GQA),
    output rounded to bf16. q [Hq, T, D], k/v [Hkv, S, D]. Rows of queries are independent,
    so long prompts are processed ``q_chunk`` queries at a time (same values, bounded
    memory)."""
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
        s = s.masked_fill(kpos > qpos, float("-inf"))
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

    def _qdq(self, x):
        from . import attn_ref, mlx_quant
        packed, s_bits, b_bits = attn_ref.quantize_rows(x.cpu().numpy(), 64, self.kv_bits)
        return torch.from_numpy(mlx_quant.dequantize(packed, s_bits, b_bits, 64,
                                                     self.kv_bits)).to(x.device)

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
        if self.kv_bits:
            k, v = self._qdq(k), self._qdq(v)
        Hkv, T, D = k.shape
        n0 = self.n[i]
        self._room(i, Hkv, D, n0 + T, k.device)
        self.kb[i][:, n0:n0 + T] = k
        self.vb[i][:, n0:n0 + T] = v
        self.n[i] = n0 + T
        ck, cv = self.kb[i][:, :n0 + T], self.vb[i][:, :n0 + T]
        if self.kv_bits and T > 1:
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
