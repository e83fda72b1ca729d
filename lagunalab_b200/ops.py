"""Torch-facing wrappers of the C-ABI kernels (device tensors in, device tensors out).

Every op runs on the CUDA stream that is current for the input's device and raises if the
library is missing or an input is not a contiguous CUDA tensor; nothing runs on the CPU.
Packed MLX words are carried as ``torch.int32`` tensors holding the uint32 bit patterns
(``torch.uint32`` has too few kernels to be practical); ``torch.uint32`` inputs are viewed
as int32.
"""
import torch

from . import _lib

_WS = {}


def _dev(t):
    if not (isinstance(t, torch.Tensor) and t.is_cuda):
        raise ValueError("lagunalab_b200 ops take CUDA tensors (there is no CPU path)")
    return t.device


def _c(t, dtype=None):
    """Contiguous CUDA tensor (optionally checked dtype); uint32 is viewed as int32."""
    if t is None:
        return None
    _dev(t)
    if t.dtype == torch.uint32:
        t = t.view(torch.int32)
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"expected {dtype}, got {t.dtype}")
    return t if t.is_contiguous() else t.contiguous()


def _p(t):
    return None if t is None else t.data_ptr()


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def workspace(device, kind, nbytes, zero=False):
    """A cached device workspace per (device, kind), grown on demand (256-byte aligned).

    ``zero=True`` workspaces are zero-filled when (re)allocated; the kernels that use them
    leave their counters at zero. Calls on one device that share a kind must not overlap in
    time on different streams."""
    key = (device.index, kind)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        n = max(int(nbytes), 256)
        buf = torch.zeros(n, dtype=torch.uint8, device=device) if zero else \
            torch.empty(n, dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def _qm(mat):
    """(weight, scales, biases) -> contiguous tuple."""
    q, s, b = mat
    return _c(q, torch.int32), _c(s, torch.bfloat16), _c(b, torch.bfloat16)


# ---------------------------------------------------------------------------------------
# Router (laguna_mlx/laguna.py:137-145)
# ---------------------------------------------------------------------------------------

def router_topk(x, gate, e_bias, k, norm_topk_prob=True, score_fn="sigmoid", counts=False):
    """Fused router. ``gate`` is an fp32 [E, H] weight or an MLX 8-bit tuple
    (weight, scales, biases). Returns (inds int32 [T, k], w bf16 [T, k], logits fp32 [T, E]
    [, counts int32 [E]])."""
    x = _c(x, torch.bfloat16)
    dev = x.device
    T, H = x.shape
    if isinstance(gate, tuple):
        gw, gs, gb = _qm(gate)
        bits = 8
    else:
        gw, gs, gb = _c(gate, torch.float32), None, None
        bits = 0
    E = gw.shape[0]
    eb = _c(e_bias.to(torch.float32)) if e_bias is not None else None
    inds = torch.empty(T, k, dtype=torch.int32, device=dev)
    w = torch.empty(T, k, dtype=torch.bfloat16, device=dev)
    logits = torch.empty(T, E, dtype=torch.float32, device=dev)
    cnt = torch.empty(E, dtype=torch.int32, device=dev) if counts else None
    sf = _lib.LG_SCORE_SOFTMAX if score_fn == "softmax" else _lib.LG_SCORE_SIGMOID
    _lib.call("lg_router_topk", _p(x), T, H, _p(gw), _p(gs), _p(gb), bits, _p(eb), E, k,
              int(bool(norm_topk_prob)), sf, _p(inds), _p(w), _p(logits), _p(cnt), _stream(dev))
    return (inds, w, logits, cnt) if counts else (inds, w, logits)


def moe_plan(inds, E, with_shared=True):
    """Expert histogram and expert-contiguous permutation of the picks (deterministic)."""
    inds = _c(inds, torch.int32)
    dev = inds.device
    T, k = inds.shape
    counts = torch.empty(E + 1, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 2, dtype=torch.int32, device=dev)
    perm = torch.empty(T * k + T, dtype=torch.int32, device=dev)
    _lib.call("lg_moe_plan", _p(inds), T, k, E, int(with_shared), _p(counts), _p(offsets),
              _p(perm), _stream(dev))
    return counts, offsets, perm


# ---------------------------------------------------------------------------------------
# Experts (SwitchGLU + combine, laguna_mlx/laguna.py:147-150; MLP, laguna.py:114-122)
# ---------------------------------------------------------------------------------------

_PATHS = {"auto": _lib.LG_PATH_AUTO, "gemv": _lib.LG_PATH_GEMV, "tensor": _lib.LG_PATH_TENSOR}


def moe_experts(x, inds, w, routed_scaling_factor, experts, shared=None, path="auto",
                group_size=64, bits=4, out=None):
    """(SwitchGLU(x, inds) * w).sum(-2) * routed_scaling_factor + shared(x) -> bf16 [T, H]."""
    x = _c(x, torch.bfloat16)
    dev = x.device
    T, H = x.shape
    inds = _c(inds, torch.int32)
    w = _c(w, torch.bfloat16)
    k = inds.shape[-1]
    g, u, d = (_qm(m) for m in experts)
    E, I = g[0].shape[0], g[0].shape[1]
    if shared is not None:
        sg, su, sd = (_qm(m) for m in shared)
        Ish = sg[0].shape[0]
    else:
        sg = su = sd = (None, None, None)
        Ish = 0
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    if T == 0:
        return out
    nb = _lib.lib().lg_moe_workspace_bytes(T, H, I, E, k, Ish)
    ws = workspace(dev, "moe", nb)
    _lib.call("lg_moe_experts", _p(x), T, H, I, E, k, _p(inds), _p(w),
              float(routed_scaling_factor),
              *map(_p, g), *map(_p, u), *map(_p, d),
              Ish, *map(_p, sg), *map(_p, su), *map(_p, sd),
              group_size, bits, _PATHS[path], _p(out), _p(ws), ws.numel(), _stream(dev))
    return out


def moe_status(device, T, H, I, E, k, I_sh):
    """Status word of the last tensor-core expert launch on ``device`` with these sizes
    (0 = ok; nonzero = a bounded pipeline wait expired). Synchronises."""
    import ctypes
    ws = _WS.get((torch.device(device).index, "moe"))
    if ws is None:
        return 0
    st = ctypes.c_int(0)
    _lib.call("lg_moe_status", _p(ws), T, H, I, E, k, I_sh, ctypes.byref(st))
    return st.value


def switch_glu(x, inds, experts, path="auto", group_size=64, bits=4):
    """SwitchGLU(x, indices): per-pick outputs bf16 [T, k, H] (unweighted)."""
    x = _c(x, torch.bfloat16)
    dev = x.device
    T, H = x.shape
    inds = _c(inds, torch.int32)
    k = inds.shape[-1]
    g, u, d = (_qm(m) for m in experts)
    E, I = g[0].shape[0], g[0].shape[1]
    y = torch.empty(T, k, H, dtype=torch.bfloat16, device=dev)
    nb = _lib.lib().lg_moe_workspace_bytes(T, H, I, E, k, 0)
    ws = workspace(dev, "moe", nb)
    _lib.call("lg_switch_glu", _p(x), T, H, I, E, k, _p(inds),
              *map(_p, g), *map(_p, u), *map(_p, d),
              group_size, bits, _PATHS[path], _p(y), _p(ws), ws.numel(), _stream(dev))
    return y


def qmlp(x, mats, path="auto", group_size=64, bits=4, out=None, ws=None):
    """Dense quantized SwiGLU MLP: down(silu(gate x) * up x) -> bf16 [T, H] (into ``out``, a
    contiguous [T, H] bf16 tensor, when given). ``ws``: the caller's own workspace (a uint8
    CUDA tensor of at least ``lg_moe_workspace_bytes(T, H, 0, 0, 0, I)`` bytes) instead of the
    shared one, for calls that overlap other MoE calls on another stream."""
    x = _c(x, torch.bfloat16)
    dev = x.device
    T, H = x.shape
    g, u, d = (_qm(m) for m in mats)
    I = g[0].shape[0]
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    elif not (out.is_contiguous() and out.dtype == torch.bfloat16 and tuple(out.shape) == (T, H)):
        raise ValueError("qmlp: out must be a contiguous bf16 [T, H] tensor")
    nb = _lib.lib().lg_moe_workspace_bytes(T, H, 0, 0, 0, I)
    if ws is None:
        ws = workspace(dev, "moe", nb)
    elif ws.numel() < nb:
        raise ValueError(f"qmlp: workspace of {ws.numel()} bytes, need {nb}")
    _lib.call("lg_qmlp", _p(x), T, H, I, *map(_p, g), *map(_p, u), *map(_p, d),
              group_size, bits, _PATHS[path], _p(out), _p(ws), ws.numel(), _stream(dev))
    return out


# ---------------------------------------------------------------------------------------
# Quantization (MLX affine layout) and the q8 decode attention
# ---------------------------------------------------------------------------------------

def quantize(w, group_size=64, bits=4):
    """MLX-layout affine quantization of the last axis: (int32 words, bf16 scales, bf16 biases)."""
    w = _c(w)
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.to(torch.float32)
    dev = w.device
    D = w.shape[-1]
    rows = w.numel() // D
    q = torch.empty(*w.shape[:-1], D * bits // 32, dtype=torch.int32, device=dev)
    s = torch.empty(*w.shape[:-1], D // group_size, dtype=torch.bfloat16, device=dev)
    b = torch.empty_like(s)
    _lib.call("lg_quantize_rows", _p(w), int(w.dtype == torch.float32), 1, 1, rows, D,
              0, 0, D, bits, group_size, _p(q), _p(s), _p(b), rows, 0, _stream(dev))
    return q, s, b


def quantize_into(x, dst, offset, group_size=64, bits=8):
    """Quantize x [B, H, L, D] (bf16, any strides with unit last stride) into rows
    [offset, offset + L) of packed buffers dst = (q [B,H,cap,*], s, b)."""
    _dev(x)
    if x.stride(-1) != 1:
        x = x.contiguous()
    B, H, L, D = x.shape
    q, s, b = dst
    cap = q.shape[2]
    if x.dtype not in (torch.bfloat16, torch.float32):
        x = x.to(torch.bfloat16)
    _lib.call("lg_quantize_rows", _p(x), int(x.dtype == torch.float32), B, H, L, D,
              x.stride(0), x.stride(1), x.stride(2), bits, group_size,
              _p(q), _p(s), _p(b), cap, offset, _stream(x.device))


def dequantize_rows(dst, n, group_size=64, bits=8):
    """Rows [0, n) of packed [B, H, cap, *] buffers -> bf16 [B, H, n, D]."""
    q, s, b = dst
    _dev(q)
    B, H, cap, W = q.shape
    D = W * 32 // bits
    out = torch.empty(B, H, n, D, dtype=torch.bfloat16, device=q.device)
    _lib.call("lg_dequantize_rows", _p(q), _p(s), _p(b), B, H, cap, n, D, bits, group_size,
              _p(out), _stream(q.device))
    return out


def dequantize(q, s, b, group_size=64, bits=4):
    """MLX-layout words -> bf16 matrix (for checks and model conversion)."""
    q = _c(q, torch.int32)
    rows = q.numel() // q.shape[-1]
    D = q.shape[-1] * 32 // bits
    out = dequantize_rows((q.reshape(1, 1, rows, -1), _c(s).reshape(1, 1, rows, -1),
                           _c(b).reshape(1, 1, rows, -1)), rows, group_size, bits)
    return out.reshape(*q.shape[:-1], D)


def q8_decode_attention(q, keys, values, n, scale, out=None):
    """Single-token attention over 8-bit group-64 packed K/V (first n rows valid).
    q [B, Hq, 1, D] bf16; keys/values = (uint32 words [B, Hkv, cap, D/4], bf16 scales,
    bf16 biases [B, Hkv, cap, D/64]). Returns [B, Hq, 1, D] bf16."""
    B, Hq, L, D = q.shape
    if L != 1:
        raise ValueError("decode only: q must have one token")
    q = _c(q, torch.bfloat16)
    kq, ks, kb = (_c(t) for t in keys)
    vq, vs, vb = (_c(t) for t in values)
    Hkv, cap = kq.shape[1], kq.shape[2]
    if kq.shape[-1] != D // 4:
        raise ValueError("8-bit, group_size 64 only")
    dev = q.device
    if out is None:
        out = torch.empty(B, Hq, 1, D, dtype=torch.bfloat16, device=dev)
    nb = _lib.lib().lg_q8_decode_workspace_bytes(B, Hq, Hkv, int(n))
    ws = workspace(dev, "q8", nb, zero=True)
    _lib.call("lg_q8_decode_attention", _p(q), B, Hq, Hkv, D, _p(kq), _p(ks), _p(kb),
              _p(vq), _p(vs), _p(vb), cap, int(n), float(scale), _p(out), _p(ws), ws.numel(),
              _stream(dev))
    return out


# ----------------------------------------------------------------------------------------
# Full-decoder ops (laguna.py:75-206)
# ----------------------------------------------------------------------------------------

def rmsnorm(x, w, eps, residual=None, sum_out=None):
    """RMSNorm over the last dim (bf16). With ``residual``, normalises h = x + residual and
    returns (h, norm(h)); else returns norm(x)."""
    H = x.shape[-1]
    x2 = _c(x, torch.bfloat16).reshape(-1, H)
    w = _c(w, torch.bfloat16)
    out = torch.empty_like(x2)
    h = None
    if residual is not None:
        residual = _c(residual, torch.bfloat16).reshape(-1, H)
        h = sum_out if sum_out is not None else torch.empty_like(x2)
    _lib.call("lg_rmsnorm", _p(x2), _p(residual), _p(w), x2.shape[0], H, float(eps), _p(h),
              _p(out), _stream(x2.device))
    if residual is not None:
        return h.reshape(x.shape), out.reshape(x.shape)
    return out.reshape(x.shape)


def qlinear(x, mat, residual=None, group_size=64, bits=4, out=None):
    """x [..., K] bf16 @ W^T for an MLX 4-bit [N, K] matrix -> [..., N] bf16 (+ residual).
    Decode sizes (<= 64 rows: a bs1 step, or one token of each of up to 64 streams) run the
    tensor-core GEMV; larger inputs dequantize W to bf16 and use a dense GEMM (fp32
    accumulate, one bf16 rounding)."""
    q, s, b = _qm(mat)
    K = x.shape[-1]
    N = q.shape[0]
    x2 = _c(x, torch.bfloat16).reshape(-1, K)
    T = x2.shape[0]
    if T > 64:
        w = dequantize(q, s, b, group_size, bits)
        y = x2 @ w.t()
        if residual is not None:
            y = y + _c(residual, torch.bfloat16).reshape(-1, N)
        if out is not None:
            out.reshape(-1, N).copy_(y)
            return out
        return y.reshape(*x.shape[:-1], N)
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    res = None if residual is None else _c(residual, torch.bfloat16)
    if T == 1 and _stageable(x2, q, s, b, group_size, bits):
        _lib.call("lg_decode_gemv", _p(x2), K, N, _p(q), _p(s), _p(b), None, None, None, None,
                  0.0, _p(res), _p(out), _stream(x2.device))
        return out
    _lib.call("lg_qlinear", _p(x2), T, K, N, _p(q), _p(s), _p(b), group_size, bits, _p(res),
              _p(out), _stream(x2.device))
    return out


def _stageable(x, q, s, b, group_size, bits):
    """Operands the shared-memory-staged one-token kernels take (16-byte aligned)."""
    return (bits == 4 and group_size == 64 and x.shape[-1] % 64 == 0
            and all(t.data_ptr() % 16 == 0 for t in (x, q, s, b)))


def decode_gemv(x, mat, norm=None, residual=None, up=None, out=None, group_size=64, bits=4):
    """One token through an MLX 4-bit [N, K] linear: ``W @ x`` (+ ``residual``), where x is
    first RMS-normalised when ``norm=(weight, eps)`` is given. With ``up`` (the up projection of
    the same shape), returns the SwiGLU ``silu(W_gate x) * (W_up x)`` instead. x [K] or [1, K]
    bf16 -> [..., N] bf16."""
    if (group_size, bits) != (64, 4):
        raise ValueError("decode_gemv: 4-bit group-64 weights only")
    q, s, b = _qm(mat)
    K = x.shape[-1]
    N = q.shape[0]
    x2 = _c(x, torch.bfloat16).reshape(-1, K)
    if x2.shape[0] != 1:
        raise ValueError("decode_gemv: one token")
    uq = us = ub = None
    if up is not None:
        uq, us, ub = _qm(up)
    nw, eps = (None, 0.0) if norm is None else (_c(norm[0], torch.bfloat16), float(norm[1]))
    res = None if residual is None else _c(residual, torch.bfloat16)
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    _lib.call("lg_decode_gemv", _p(x2), K, N, _p(q), _p(s), _p(b), _p(uq), _p(us), _p(ub),
              _p(nw), eps, _p(res), _p(out), _stream(x2.device))
    return out


def decode_qkv_prep(x, mat, norm, Hq, Hkv, D, qn_w, kn_w, qk_eps, theta, cache_k, cache_v,
                    pos=0, pos_dev=None, gate_per_head=True, rope=None, ring=0, row0=0):
    """One token's q/k/v/g projection (input RMSNorm ``norm=(weight, eps)`` fused in) and its
    attention prologue in one launch; returns (qkvg [1, N], q [Hq, 1, D], gate). ``cache_k`` /
    ``cache_v``: the bf16 cache [Hkv, cap, D] tensors, or the 8-bit cache's (words, scales,
    biases) tuples; the new rows go to row ``pos`` (or ``pos_dev[0]``). The same bits as
    ``decode_gemv`` followed by ``attn_prep`` / ``attn_prep_q8``."""
    q_, s_, b_ = _qm(mat)
    K = x.shape[-1]
    N = q_.shape[0]
    if N != (Hq + 2 * Hkv) * D + (Hq if gate_per_head else Hq * D):
        raise ValueError(f"decode_qkv_prep: {N} projection rows for heads {Hq}/{Hkv} x {D}")
    x2 = _c(x, torch.bfloat16).reshape(1, K)
    dev = x2.device
    qkvg = torch.empty(1, N, dtype=torch.bfloat16, device=dev)
    q = torch.empty(Hq, 1, D, dtype=torch.bfloat16, device=dev)
    gate = torch.empty(1, Hq if gate_per_head else Hq * D, dtype=torch.bfloat16, device=dev)
    if isinstance(cache_k, tuple):
        kq, ks, kb = cache_k
        vq, vs, vb = cache_v
        cap = kq.shape[-2]
        kc = vc = None
    else:
        kq = ks = kb = vq = vs = vb = None
        kc, vc = cache_k, cache_v
        cap = kc.shape[-2]
    nws = _lib.lib().lg_decode_qkv_prep_workspace_bytes(Hq, Hkv)
    ws = workspace(dev, "qkv_prep", nws, zero=True)
    _lib.call("lg_decode_qkv_prep", _p(x2), K, _p(q_), _p(s_), _p(b_),
              _p(_c(norm[0], torch.bfloat16)), float(norm[1]), Hq, Hkv, D, _p(_c(qn_w)),
              _p(_c(kn_w)), float(qk_eps), float(theta), _p(pos_dev), int(pos),
              int(bool(gate_per_head)), _p(qkvg), _p(q), _p(gate), _p(kc), _p(vc), _p(kq),
              _p(ks), _p(kb), _p(vq), _p(vs), _p(vb), cap, *_rope_args(rope, ring, row0),
              _p(ws), ws.numel(), _stream(dev))
    return qkvg, q, gate


def router_decode(h, norm_w, eps, gate, e_bias, k, norm_topk_prob=True, score_fn="sigmoid",
                  logits=False):
    """One token's post-attention RMSNorm and router in one launch: from the residual stream
    h [1, H] returns (xn [1, H] normalised, inds int32 [1, k], w bf16 [1, k][, logits fp32
    [1, E]]). ``gate`` is the 8-bit group-64 router (weight, scales, biases)."""
    H = h.shape[-1]
    h2 = _c(h, torch.bfloat16).reshape(1, H)
    gw, gs, gb = _qm(gate)
    E = gw.shape[0]
    dev = h2.device
    eb = _c(e_bias.to(torch.float32)) if e_bias is not None else None
    xn = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
    inds = torch.empty(1, k, dtype=torch.int32, device=dev)
    w = torch.empty(1, k, dtype=torch.bfloat16, device=dev)
    lg = torch.empty(1, E, dtype=torch.float32, device=dev) if logits else None
    sf = _lib.LG_SCORE_SOFTMAX if score_fn == "softmax" else _lib.LG_SCORE_SIGMOID
    ws = workspace(dev, "router_decode", _lib.lib().lg_router_decode_workspace_bytes(E), zero=True)
    _lib.call("lg_router_decode", _p(h2), _p(_c(norm_w, torch.bfloat16)), float(eps), H,
              _p(gw), _p(gs), _p(gb), _p(eb), E, k, int(bool(norm_topk_prob)), sf, _p(xn),
              _p(inds), _p(w), _p(lg), _p(ws), ws.numel(), _stream(dev))
    return (xn, inds, w, lg) if logits else (xn, inds, w)


def moe_decode(xn, inds, w, routed_scaling_factor, experts, shared=None, residual=None,
               out=None):
    """One token through the MoE experts: ``sum_j w_j * SwitchGLU_j(xn) * scale + shared(xn)``
    (+ ``residual``), bf16 [1, H]. inds int32 [1, k], w bf16 [1, k]."""
    xn = _c(xn, torch.bfloat16)
    dev = xn.device
    H = xn.shape[-1]
    inds = _c(inds, torch.int32)
    w = _c(w, torch.bfloat16)
    k = inds.shape[-1]
    g, u, d = (_qm(m) for m in experts)
    E, I = g[0].shape[0], g[0].shape[1]
    if shared is not None:
        sg, su, sd = (_qm(m) for m in shared)
        Ish = sg[0].shape[0]
    else:
        sg = su = sd = (None, None, None)
        Ish = 0
    res = None if residual is None else _c(residual, torch.bfloat16)
    if out is None:
        out = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
    nb = _lib.lib().lg_moe_decode_workspace_bytes(H, I, Ish, k)
    ws = workspace(dev, "moe_decode", nb, zero=True)
    _lib.call("lg_moe_decode", _p(xn), _p(inds), _p(w), H, I, E, k,
              float(routed_scaling_factor), *map(_p, g), *map(_p, u), *map(_p, d), Ish,
              *map(_p, sg), *map(_p, su), *map(_p, sd), _p(res), _p(out), _p(ws), ws.numel(),
              _stream(dev))
    return out


def router_decode_supported(H, E):
    """Whether the one-token router kernel takes an E x H router (one CTA's shared memory)."""
    return bool(_lib.lib().lg_router_decode_supported(H, E))


def moe_decode_supported(H, I, Ish, k):
    """Whether the one-token expert kernels take these sizes (shared memory bound)."""
    return bool(_lib.lib().lg_moe_decode_supported(H, I, Ish, k))



def decode_status(reset=True):
    """Check word of the one-token kernels' staging copies: (failed, smem offset, source
    address, block/thread) of the first copy that failed its alignment or bounds check, all
    zero when none did. Synchronises."""
    import ctypes
    buf = (ctypes.c_ulonglong * 4)()
    _lib.call("lg_decode_status", ctypes.addressof(buf), int(bool(reset)))
    return tuple(int(v) for v in buf)


def embed(ids, mat, group_size=64, bits=4):
    """Quantized embedding rows for device int32 ids [...] -> [..., H] bf16."""
    q, s, b = _qm(mat)
    ids = _c(ids.to(torch.int32) if ids.dtype != torch.int32 else ids)
    V, H = q.shape[0], q.shape[1] * 32 // bits
    out = torch.empty(*ids.shape, H, dtype=torch.bfloat16, device=ids.device)
    _lib.call("lg_embed", _p(ids), ids.numel(), _p(q), _p(s), _p(b), V, H, group_size, bits,
              _p(out), _stream(ids.device))
    return out


def _rope_args(rope, ring, row0):
    """(inv_freq pointer, rotated dims, mscale, ring, row0) for the prologue entry points.
    ``rope``: None (default RoPE over all dims) or (inv_freq fp32 CUDA tensor [R/2], R,
    mscale)."""
    if rope is None:
        return None, 0, 1.0, int(ring), int(row0)
    inv, R, ms = rope
    return _p(_c(inv, torch.float32)), int(R), float(ms), int(ring), int(row0)


def attn_prep(qkvg, Hq, Hkv, D, qn_w, kn_w, eps, theta, k_cache, v_cache, pos=0, pos_dev=None,
              gate_per_head=True, rope=None, ring=0, row0=0):
    """From fused q|k|v|g projections [T, .] write k, v rows into the caches [Hkv, cap, D] at
    positions pos + t and return (q [Hq, T, D] normed + roped, gate [T, Hq or Hq*D]).
    ``rope``: (inv_freq, rotated dims, mscale) for partial rotary / YaRN (laguna.py:62-72);
    ``ring`` > 0: the caches are a sliding window's ring (row = position mod ring); else row =
    position - ``row0``."""
    qkvg = _c(qkvg, torch.bfloat16)
    T = qkvg.shape[0]
    cap = k_cache.shape[-2]
    q = torch.empty(Hq, T, D, dtype=torch.bfloat16, device=qkvg.device)
    gate = torch.empty(T, Hq if gate_per_head else Hq * D, dtype=torch.bfloat16, device=qkvg.device)
    _lib.call("lg_attn_prep", _p(qkvg), T, Hq, Hkv, D, _p(_c(qn_w)), _p(_c(kn_w)), float(eps),
              float(theta), _p(pos_dev), int(pos), int(bool(gate_per_head)), _p(q), _p(k_cache),
              _p(v_cache), cap, _p(gate), *_rope_args(rope, ring, row0), _stream(qkvg.device))
    return q, gate


def attn_prep_streams(qkvg, Hq, Hkv, D, qn_w, kn_w, eps, theta, k_cache, v_cache, pos_dev,
                      gate_per_head=True, rope=None, ring=0):
    """One decode step of B independent streams: row t of the fused projections qkvg [B, .] is
    stream t's newest token, at position pos_dev[t] (device int32 [B]); its k, v rows go into
    stream t's caches [B, Hkv, cap, D] (row = position, or position mod ``ring``). Returns
    (q [B, Hq, D] normed + roped, gate [B, Hq or Hq*D])."""
    qkvg = _c(qkvg, torch.bfloat16)
    B = qkvg.shape[0]
    cap = k_cache.shape[-2]
    q = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=qkvg.device)
    gate = torch.empty(B, Hq if gate_per_head else Hq * D, dtype=torch.bfloat16, device=qkvg.device)
    inv, rot, ms, ring, _ = _rope_args(rope, ring, 0)
    _lib.call("lg_attn_prep_streams", _p(qkvg), B, Hq, Hkv, D, _p(_c(qn_w)), _p(_c(kn_w)),
              float(eps), float(theta), _p(_c(pos_dev, torch.int32)), int(bool(gate_per_head)),
              _p(q), _p(k_cache), _p(v_cache), cap, _p(gate), inv, rot, ms, ring,
              _stream(qkvg.device))
    return q, gate


def attn_prep_q8(qkvg, Hq, Hkv, D, qn_w, kn_w, eps, theta, keys, values, pos=0, pos_dev=None,
                 gate_per_head=True, rope=None, ring=0, row0=0):
    """attn_prep with an 8-bit group-64 cache: the new k, v rows are quantized into rows
    pos + t of the packed caches keys/values = (words [B=1, Hkv, cap, D/4], scales, biases)."""
    qkvg = _c(qkvg, torch.bfloat16)
    T = qkvg.shape[0]
    kq, ks, kb = keys
    vq, vs, vb = values
    cap = kq.shape[-2]
    q = torch.empty(Hq, T, D, dtype=torch.bfloat16, device=qkvg.device)
    gate = torch.empty(T, Hq if gate_per_head else Hq * D, dtype=torch.bfloat16, device=qkvg.device)
    _lib.call("lg_attn_prep_q8", _p(qkvg), T, Hq, Hkv, D, _p(_c(qn_w)), _p(_c(kn_w)), float(eps),
              float(theta), _p(pos_dev), int(pos), int(bool(gate_per_head)), _p(q),
              _p(kq), _p(ks), _p(kb), _p(vq), _p(vs), _p(vb), cap, _p(gate),
              *_rope_args(rope, ring, row0), _stream(qkvg.device))
    return q, gate


def q8_decode_attention_dev(q, keys, values, n_plan, n_dev, n_add, scale, gate=None, out=None):
    """Single-token attention over the packed 8-bit cache with the valid length on the device
    (n_dev[0] + n_add), planned for n_plan keys; optional per-head gate [B, Hq]. q [B, Hq, D]
    -> [B, Hq, D] bf16."""
    q = _c(q, torch.bfloat16)
    B, Hq, D = q.shape[0], q.shape[1], q.shape[-1]
    kq, ks, kb = (_c(t) for t in keys)
    vq, vs, vb = (_c(t) for t in values)
    Hkv, cap = kq.shape[1], kq.shape[2]
    nb = _lib.lib().lg_q8_decode_workspace_bytes(B, Hq, Hkv, int(n_plan))
    ws = workspace(q.device, "q8", nb, zero=True)
    if out is None:
        out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=q.device)
    _lib.call("lg_q8_decode_attention_dev", _p(q), B, Hq, Hkv, D, _p(kq), _p(ks), _p(kb), _p(vq),
              _p(vs), _p(vb), cap, int(n_plan), _p(n_dev), int(n_add), float(scale),
              _p(_c(gate)), _p(out), _p(ws), ws.numel(), _stream(q.device))
    return out


def bf16_decode_attention(q, k_cache, v_cache, n, scale, gate=None, n_dev=None, n_add=0,
                          n_plan=None, out=None):
    """Single-token attention over a bf16 cache. q [B, Hq, D]; caches [B, Hkv, cap, D];
    n valid keys (or n_dev[0] + n_add on the device); gate [B, Hq] per-head or None.
    Returns out [B, Hq, D] bf16 (gated)."""
    q = _c(q, torch.bfloat16)
    B, Hq, D = q.shape
    Hkv, cap = k_cache.shape[1], k_cache.shape[2]
    n_plan = cap if n_plan is None else int(n_plan)
    nb = _lib.lib().lg_bf16_decode_workspace_bytes(B, Hq, Hkv, n_plan)
    ws = workspace(q.device, "bf16_attn", nb, zero=True)
    if out is None:
        out = torch.empty_like(q)
    _lib.call("lg_bf16_decode_attention", _p(q), B, Hq, Hkv, D, _p(k_cache), _p(v_cache), cap,
              int(n), _p(n_dev), int(n_add), n_plan, float(scale), _p(_c(gate)), _p(out),
              _p(ws), ws.numel(), _stream(q.device))
    return out


def bf16_decode_attention_streams(q, k_cache, v_cache, n_dev, n_add, scale, gate=None,
                                  n_plan=None, out=None):
    """Single-token attention of B independent streams over their bf16 caches [B, Hkv, cap, D]:
    stream b attends over n_dev[b] + n_add keys (device int32 [B]; clamped to cap, so a
    sliding window's ring gives min(position + 1, window)). q [B, Hq, D]; gate [B, Hq]
    per-head or None. Returns [B, Hq, D] bf16 (gated)."""
    q = _c(q, torch.bfloat16)
    B, Hq, D = q.shape
    Hkv, cap = k_cache.shape[1], k_cache.shape[2]
    n_plan = cap if n_plan is None else int(n_plan)
    nb = _lib.lib().lg_bf16_decode_workspace_bytes(B, Hq, Hkv, n_plan)
    ws = workspace(q.device, "bf16_attn", nb, zero=True)
    if out is None:
        out = torch.empty_like(q)
    _lib.call("lg_bf16_decode_attention_streams", _p(q), B, Hq, Hkv, D, _p(k_cache),
              _p(v_cache), cap, _p(_c(n_dev, torch.int32)), int(n_add), n_plan, float(scale),
              _p(_c(gate)), _p(out), _p(ws), ws.numel(), _stream(q.device))
    return out


def argmax(logits, ids=None, pos=None, inc=1):
    """Greedy token per row of bf16 logits [T, V] into int32 ids [T]; optionally advances the
    device position counter ``pos`` by ``inc``."""
    logits = _c(logits, torch.bfloat16)
    V = logits.shape[-1]
    l2 = logits.reshape(-1, V)
    if ids is None:
        ids = torch.empty(l2.shape[0], dtype=torch.int32, device=logits.device)
    _lib.call("lg_argmax", _p(l2), l2.shape[0], V, _p(ids), _p(pos), int(inc),
              _stream(logits.device))
    return ids
