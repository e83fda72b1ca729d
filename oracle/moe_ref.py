"""PyTorch-CPU restatement of the Laguna MoE block (test infrastructure only).

Follows laguna_mlx/laguna.py:114-150 and the SwitchGLU semantics of mlx-lm
0.31.3 (called at laguna.py:149): per (token, pick) the gate and up products,
SwiGLU, the down product, then the weighted sum over picks, the routed scale and
the shared expert.

Rounding: every tensor that the MLX graph materialises in bf16 is rounded to
bf16 here (``_bf``): the quantized matmul outputs, silu's sigmoid and product,
the SwiGLU product, the per-pick weighted outputs, the pick sum, the scaled sum
and the final add. Matmuls accumulate in float32 on float32-dequantized weights.

Weights are MLX-layout tuples ``(packed, scales, biases)``: ``packed`` holds the
uint32 words as torch.int32 (same bits), ``scales``/``biases`` are bf16 or f32.
A stacked expert tensor has a leading expert axis ``[E, out, ...]``.
"""
import torch

_MASK32 = 0xFFFFFFFF


def _bf(t):
    """Round to bf16 and back to float32 (an MLX bf16 materialisation point)."""
    return t.to(torch.bfloat16).to(torch.float32)


def unpack_codes(packed, bits):
    """int32/uint32 words [..., W] -> int64 codes [..., W * 32 / bits], low bits first."""
    p = packed.to(torch.int64) & _MASK32
    per = 32 // bits
    shifts = torch.arange(per, dtype=torch.int64, device=packed.device) * bits
    codes = (p.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)
    return codes.reshape(*packed.shape[:-1], packed.shape[-1] * per)


def dequantize(packed, scales, biases, group_size=64, bits=4):
    """MLX affine dequantize (value = scale * code + bias, laguna_mlx/q8_attn.py:50) in fp32."""
    codes = unpack_codes(packed, bits).to(torch.float32)
    n = codes.shape[-1]
    g = codes.reshape(*codes.shape[:-1], n // group_size, group_size)
    out = g * scales.to(torch.float32).unsqueeze(-1) + biases.to(torch.float32).unsqueeze(-1)
    return out.reshape(codes.shape)


def qlinear(x, wq, group_size=64, bits=4):
    """QuantizedLinear forward: bf16(x @ W^T), fp32 accumulation on dequantized W."""
    w = dequantize(*wq, group_size=group_size, bits=bits)
    return _bf(x.to(torch.float32) @ w.T)


def silu_bf16(g):
    """nn.silu on a bf16 array: g * sigmoid(g), each op materialised in bf16."""
    return _bf(g * _bf(torch.sigmoid(g)))


def mlp(x, gate, up, down, group_size=64, bits=4):
    """laguna.py:114-122 ``down(silu(gate(x)) * up(x))`` on 4-bit quantized linears."""
    deq = lambda q: dequantize(*q, group_size=group_size, bits=bits)
    return mlp_deq(x, deq(gate), deq(up), deq(down))


def mlp_deq(x, wg, wu, wd):
    """The same MLP on already-dequantized fp32 weights (bf16 materialisation points kept)."""
    xf = x.to(torch.float32)
    g = _bf(xf @ wg.T)
    u = _bf(xf @ wu.T)
    h = _bf(silu_bf16(g) * u)
    return _bf(h @ wd.T)


def router_logits(x, gate):
    """``gate(x).astype(f32)`` (laguna.py:138). ``gate`` is an fp32 [E, H] weight, or an
    8-bit g64 tuple (laguna.py:236-238); the quantized form's bf16 output is what MLX
    casts to fp32."""
    xf = x.to(torch.float32)
    if isinstance(gate, tuple):
        return qlinear(x, gate, group_size=64, bits=8)
    return xf @ gate.to(torch.float32).T


def topk_indices(sel, k):
    """Top-k of ``sel`` per row, larger first, ties broken by the lower expert index.

    MLX's ``argpartition`` (laguna.py:141) returns an unordered top-k and leaves the
    order of equal keys unspecified; this fixed rule is the build's tie rule."""
    order = torch.sort(-sel, dim=-1, stable=True).indices
    return order[..., :k]


def tie_rows(sel, k):
    """Rows whose k-th and (k+1)-th selection scores are equal or 1 ulp apart.

    On those rows the chosen set depends on the tie rule and on last-ulp rounding of
    the sigmoid, so parity checks them as a set up to the tie."""
    s = torch.sort(sel, dim=-1, descending=True).values
    if s.shape[-1] <= k:
        return torch.zeros(s.shape[:-1], dtype=torch.bool)
    a, b = s[..., k - 1], s[..., k]
    gap = (a - b).abs()
    ulp = torch.maximum(a.abs(), b.abs()) * 2.0 ** -23
    return (a == b) | (gap <= 2 * ulp)


def route(x, gate, bias, k, norm_topk_prob=True, score_fn="sigmoid"):
    """laguna.py:137-145 ``SparseMoeBlock.route``.

    Returns ``inds`` int64 [T, k] (sorted by biased score, larger first), ``w`` bf16
    [T, k], and the fp32 ``logits``/``scores``/``sel`` for parity reports.
    ``score_fn="softmax"`` is an extra mode (BASELINE wording), not the reference's."""
    logits = router_logits(x, gate)
    if score_fn == "sigmoid":
        scores = torch.sigmoid(logits)
    elif score_fn == "softmax":
        scores = torch.softmax(logits, dim=-1)
    else:
        raise ValueError(score_fn)
    sel = scores + bias.to(torch.float32)
    inds = topk_indices(sel, k)
    w = torch.gather(scores, -1, inds)
    if norm_topk_prob:
        w = w / w.sum(dim=-1, keepdim=True)
    return inds, w.to(torch.bfloat16), logits, scores, sel


def weights_from_logits(logits, bias, inds, norm_topk_prob=True):
    """Routing weights for given indices from given fp32 logits (laguna.py:138-145)."""
    scores = torch.sigmoid(logits.to(torch.float32))
    w = torch.gather(scores, -1, inds.to(torch.int64))
    if norm_topk_prob:
        w = w / w.sum(dim=-1, keepdim=True)
    return w


def switch_glu(x, inds, gate, up, down, group_size=64, bits=4):
    """SwitchGLU(x, inds) -> bf16-valued [T, k, H]: per pick
    ``down(silu(gate x) * up x)`` on the picked expert's 4-bit weights."""
    sel = lambda q, e: dequantize(*(t[e] for t in q), group_size=group_size, bits=bits)
    return _switch(x, inds, down[0].shape[1],
                   lambda e: (sel(gate, e), sel(up, e), sel(down, e)))


def switch_glu_deq(x, inds, wg, wu, wd):
    """SwitchGLU on already-dequantized stacked fp32 weights [E, out, in]."""
    return _switch(x, inds, wd.shape[1], lambda e: (wg[e], wu[e], wd[e]))


def _switch(x, inds, H_out, weights_of):
    T = x.shape[0]
    k = inds.shape[-1]
    out = torch.zeros(T, k, H_out, dtype=torch.float32, device=x.device)
    flat = inds.reshape(-1)
    for e in torch.unique(flat).tolist():
        if e < 0:
            continue
        picks = (flat == e).nonzero().squeeze(-1)
        ye = mlp_deq(x[picks // k], *weights_of(e))
        out.view(T * k, -1)[picks] = ye
    return out


def combine(y, w, routed_scaling_factor, shared):
    """laguna.py:149-150: ``(y * w[..., None]).sum(-2) * scale + shared`` with bf16 ops."""
    yw = _bf(y * w.to(torch.float32).unsqueeze(-1))
    s = _bf(yw.sum(dim=-2))
    s = _bf(s * float(routed_scaling_factor))
    return _bf(s + shared)


def moe_block(x, gate, bias, experts, shared, k, routed_scaling_factor=1.0,
              norm_topk_prob=True, group_size=64, bits=4):
    """laguna.py:147-150 ``SparseMoeBlock.__call__``. ``experts``/``shared`` are
    ``(gate, up, down)`` tuples of MLX-layout weights. Returns (out bf16-valued fp32
    [T, H], inds, w)."""
    inds, w, *_ = route(x, gate, bias, k, norm_topk_prob)
    y = switch_glu(x, inds, *experts, group_size=group_size, bits=bits)
    sh = mlp(x, *shared, group_size=group_size, bits=bits)
    return combine(y, w, routed_scaling_factor, sh), inds, w


# ---------------------------------------------------------------------------
# Unquantized fp32 form, used only to pin this restatement against the vendored
# PyTorch model (tests/reference/modeling_laguna.py:146-266), which has no
# quantization and no bf16 rounding.
# ---------------------------------------------------------------------------

def moe_block_fp32(x, gate_w, bias, gate_up, down, sh_gate, sh_up, sh_down, k,
                   routed_scaling_factor=1.0, norm_topk_prob=True):
    """fp32 MoE block: router (modeling_laguna.py:174-190), experts loop (:206-230),
    routed scale + shared (:254-266). ``gate_up`` is [E, 2I, H] (gate rows first)."""
    x = x.to(torch.float32)
    logits = x @ gate_w.T
    scores = torch.sigmoid(logits)
    sel = scores + bias
    inds = topk_indices(sel, k)
    w = torch.gather(scores, -1, inds)
    if norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    I = down.shape[-1]
    out = torch.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(k):
            e = int(inds[t, j])
            gu = gate_up[e] @ x[t]
            h = torch.nn.functional.silu(gu[:I]) * gu[I:]
            out[t] += w[t, j] * (down[e] @ h)
    sh = sh_down @ (torch.nn.functional.silu(x @ sh_gate.T) * (x @ sh_up.T)).T
    return out * routed_scaling_factor + sh.T, inds, w, logits
