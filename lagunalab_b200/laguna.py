"""Laguna decoder on B200, with the module surface of laguna_mlx/laguna.py.

Same names and call semantics as the reference (laguna.py:18-241): ``ModelArgs`` with its
validation, ``MLP(dim, hidden)``, ``SwitchGLU(input_dims, hidden_dims, num_experts)`` called
as ``switch_mlp(x, indices) -> [..., k, hidden]``, ``SparseMoeBlock`` with a separate,
patchable ``route(x) -> (inds, w)`` (hooks and pruning wrap it), ``Attention``,
``DecoderLayer``, ``LagunaModel`` and ``Model`` (``layers``, ``make_cache``, ``sanitize``,
``quant_predicate``). Tensors are torch CUDA tensors; weights use the MLX packed layout
(uint32 words as int32, bf16 scales/biases). All arithmetic runs in the sm_100a kernels of
``liblaguna_b200.so`` (prefill-sized dense linears dequantize to bf16 for a dense GEMM, and
prefill attention uses torch's fused SDPA).
"""
import inspect
import math
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import torch

from . import _lib, ops


@dataclass
class ModelArgs:
    """laguna_mlx/laguna.py:18-66 (fields, defaults and the unsupported-config checks)."""
    model_type: str
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float
    num_experts: int
    num_experts_per_tok: int
    moe_intermediate_size: int
    shared_expert_intermediate_size: int
    rope_parameters: Dict[str, Any]
    layer_types: Optional[List[str]] = None
    sliding_window: Optional[int] = None
    swa_rope_parameters: Optional[Dict[str, Any]] = None
    num_attention_heads_per_layer: Optional[List[int]] = None
    mlp_only_layers: List[int] = field(default_factory=lambda: [0])
    norm_topk_prob: bool = True
    moe_routed_scaling_factor: float = 1.0
    max_position_embeddings: int = 262144
    tie_word_embeddings: bool = False
    gating: Any = True
    moe_router_logit_softcapping: float = 0.0
    swa_attention_sink_enabled: bool = False
    moe_apply_router_weight_on_input: bool = False

    def __post_init__(self):
        if self.moe_router_logit_softcapping:
            raise ValueError("Laguna: moe_router_logit_softcapping is not supported")
        if self.swa_attention_sink_enabled:
            raise ValueError("Laguna: swa_attention_sink_enabled is not supported")
        if self.moe_apply_router_weight_on_input:
            raise ValueError("Laguna: moe_apply_router_weight_on_input is not supported")
        if self.gating not in ("per-head", True):
            raise ValueError(f"Laguna: gating={self.gating!r} is not supported")
        if self.layer_types is None:
            self.layer_types = ["full_attention"] * self.num_hidden_layers
        if self.num_attention_heads_per_layer is None:
            self.num_attention_heads_per_layer = [self.num_attention_heads] * self.num_hidden_layers

    @classmethod
    def from_dict(cls, params):
        """Keep the keys that are fields (mlx-lm BaseModelArgs.from_dict behaviour)."""
        names = inspect.signature(cls).parameters
        return cls(**{k: v for k, v in params.items() if k in names})

    def rope_for(self, layer_type):
        rp = self.rope_parameters
        if layer_type == "sliding_attention":
            return self.swa_rope_parameters or rp.get("sliding_attention", rp)
        return rp.get("full_attention", rp)


class QuantizedLinear:
    """MLX QuantizedLinear storage: ``weight`` uint32 words (int32 tensor) [out, in*bits/32],
    ``scales``/``biases`` bf16 [out, in/group_size]."""

    def __init__(self, weight, scales, biases, group_size=64, bits=4):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits = group_size, bits

    @classmethod
    def from_float(cls, w, group_size=64, bits=4):
        return cls(*ops.quantize(w, group_size, bits), group_size, bits)

    @property
    def mat(self):
        return self.weight, self.scales, self.biases

    def dequantize(self):
        return ops.dequantize(self.weight, self.scales, self.biases, self.group_size, self.bits)

    def __call__(self, x, residual=None):
        """nn.QuantizedLinear: x @ W^T (bf16 out), optionally + residual (bf16)."""
        if self.bits != 4:
            raise ValueError("only 4-bit linears are callable (the 8-bit router has its own kernel)")
        return ops.qlinear(x, self.mat, residual, self.group_size, self.bits)


class MLP:
    """laguna_mlx/laguna.py:114-122: ``down(silu(gate(x)) * up(x))`` (shared expert, dense
    layer 0), 4-bit quantized projections."""

    def __init__(self, dim, hidden, gate_proj=None, up_proj=None, down_proj=None):
        self.dim, self.hidden = dim, hidden
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj

    @classmethod
    def from_float(cls, gate, up, down, group_size=64, bits=4):
        q = lambda w: QuantizedLinear.from_float(w, group_size, bits)
        return cls(gate.shape[1], gate.shape[0], q(gate), q(up), q(down))

    @property
    def mats(self):
        return (self.gate_proj.mat, self.up_proj.mat, self.down_proj.mat)

    def __call__(self, x):
        shape = x.shape
        out = ops.qmlp(x.reshape(-1, shape[-1]), self.mats, group_size=self.gate_proj.group_size,
                       bits=self.gate_proj.bits)
        return out.reshape(shape)

    def token(self, h, norm):
        """One token's dense MLP sub-block from the residual stream h [1, H]:
        ``h + self(norm(h))`` as two launches (norm + gate/up + SwiGLU, down + residual)."""
        if (self.gate_proj.bits, self.gate_proj.group_size) != (4, 64):
            return None
        H = h.shape[-1]
        a = ops.decode_gemv(h.reshape(1, H), self.gate_proj.mat, norm=(norm.weight, norm.eps),
                            up=self.up_proj.mat)
        return ops.decode_gemv(a, self.down_proj.mat, residual=h.reshape(1, H))


class SwitchLinear(QuantizedLinear):
    """mlx-lm QuantizedSwitchLinear storage: stacked [E, out, in*bits/32] words and
    [E, out, in/group] bf16 scales/biases; ``weight[slot] = ...`` replaces one expert
    (what lagunaLab's ExpertStore does per slot, streaming.py:70-74)."""


class SwitchGLU:
    """mlx-lm switch_layers.SwitchGLU surface (laguna.py:134, :149): ``__call__(x, indices)``
    returns the per-pick outputs [..., k, hidden] of ``down(silu(gate x) * up x)``."""

    def __init__(self, input_dims, hidden_dims, num_experts, gate_proj=None, up_proj=None,
                 down_proj=None):
        self.input_dims, self.hidden_dims, self.num_experts = input_dims, hidden_dims, num_experts
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj

    @classmethod
    def from_float(cls, gate, up, down, group_size=64, bits=4):
        q = lambda w: SwitchLinear.from_float(w, group_size, bits)
        return cls(gate.shape[2], gate.shape[1], gate.shape[0], q(gate), q(up), q(down))

    @property
    def mats(self):
        return (self.gate_proj.mat, self.up_proj.mat, self.down_proj.mat)

    def __call__(self, x, indices):
        H = x.shape[-1]
        k = indices.shape[-1]
        y = ops.switch_glu(x.reshape(-1, H), indices.reshape(-1, k).to(torch.int32), self.mats,
                           group_size=self.gate_proj.group_size, bits=self.gate_proj.bits)
        return y.reshape(*indices.shape, H)


class SparseMoeBlock:
    """laguna_mlx/laguna.py:125-150.

    ``gate`` is the router weight: fp32 [E, H] (``nn.Linear`` kept in fp32) or a
    ``QuantizedLinear`` with 8 bits / group 64 (laguna.py:236-238). ``route`` stays a separate
    method so instrumentation can wrap it; ``__call__`` uses the fused expert kernels when
    ``switch_mlp`` is this package's SwitchGLU (or a resident StreamingSwitchGLU) and the
    generic ``(switch_mlp(x, inds) * w).sum(-2)`` form otherwise."""

    def __init__(self, args, gate=None, e_score_correction_bias=None, switch_mlp=None,
                 shared_expert=None, score_fn="sigmoid"):
        self.top_k = args.num_experts_per_tok
        self.norm_topk_prob = args.norm_topk_prob
        self.routed_scaling_factor = args.moe_routed_scaling_factor
        self.num_experts = args.num_experts
        self.gate = gate
        self.e_score_correction_bias = e_score_correction_bias
        self.switch_mlp = switch_mlp
        self.shared_expert = shared_expert
        self.score_fn = score_fn

    def _gate_arg(self):
        g = self.gate
        if isinstance(g, QuantizedLinear):
            if (g.bits, g.group_size) != (8, 64):
                raise ValueError("router gate must be fp32 or 8-bit group-64")
            return g.mat
        return g

    def route(self, x):
        """laguna.py:137-145: (inds [..., k] int32, w [..., k] in x's dtype)."""
        H = x.shape[-1]
        inds, w, _ = ops.router_topk(x.reshape(-1, H).to(torch.bfloat16), self._gate_arg(),
                                     self.e_score_correction_bias, self.top_k,
                                     self.norm_topk_prob, self.score_fn)
        lead = x.shape[:-1]
        return inds.reshape(*lead, self.top_k), w.reshape(*lead, self.top_k).to(x.dtype)

    def __call__(self, x):
        inds, w = self.route(x)
        H = x.shape[-1]
        sw = self.switch_mlp
        fused = _fused_experts(sw)
        if fused is not None:
            _note_picks(sw, inds.numel())
            sh = self.shared_expert.mats if self.shared_expert is not None else None
            out = ops.moe_experts(x.reshape(-1, H), inds.reshape(-1, self.top_k),
                                  w.reshape(-1, self.top_k), self.routed_scaling_factor,
                                  fused.mats, sh, group_size=fused.gate_proj.group_size,
                                  bits=fused.gate_proj.bits)
            return out.reshape(x.shape)
        y = (sw(x, inds) * w[..., None]).sum(dim=-2)
        y = y * self.routed_scaling_factor
        if self.shared_expert is not None:
            y = y + self.shared_expert(x)
        return y


    def token_experts(self, H):
        """The SwitchGLU the one-token router + expert kernels can use, or None: ``route`` not
        wrapped or overridden (instrumentation sees every routing), an 8-bit router, 4-bit
        experts and sizes the kernels take."""
        if "route" in self.__dict__ or type(self).route is not SparseMoeBlock.route:
            return None
        g = self.gate
        if not isinstance(g, QuantizedLinear) or (g.bits, g.group_size) != (8, 64):
            return None
        fused = _fused_experts(self.switch_mlp)
        if fused is None or (fused.gate_proj.bits, fused.gate_proj.group_size) != (4, 64):
            return None
        Ish = 0
        if self.shared_expert is not None:
            sh = self.shared_expert
            if not isinstance(sh, MLP) or (sh.gate_proj.bits, sh.gate_proj.group_size) != (4, 64):
                return None
            Ish = sh.hidden
        if not ops.moe_decode_supported(H, fused.hidden_dims, Ish, self.top_k):
            return None
        if not ops.router_decode_supported(H, self.num_experts):
            return None
        return fused

    def token(self, h, norm):
        """One token's MoE sub-block from the residual stream h [1, H]:
        ``h + self(norm(h))`` (laguna.py:163-164) as a router launch and two expert launches;
        None when ``token_experts`` declines."""
        H = h.shape[-1]
        fused = self.token_experts(H)
        if fused is None:
            return None
        xn, inds, w = ops.router_decode(h.reshape(1, H), norm.weight, norm.eps, self.gate.mat,
                                        self.e_score_correction_bias, self.top_k,
                                        self.norm_topk_prob, self.score_fn)
        sh = self.shared_expert.mats if self.shared_expert is not None else None
        _note_picks(self.switch_mlp, self.top_k)
        return ops.moe_decode(xn, inds, w, self.routed_scaling_factor, fused.mats, sh,
                              residual=h.reshape(1, H))


def _note_picks(sw, n):
    """Expert picks served by the fused kernels, for a resident expert store's statistics."""
    note = getattr(sw, "note_picks", None)
    if note is not None:
        note(n)


def _fused_experts(sw):
    """The SwitchGLU whose weights the fused kernel can read directly, or None."""
    if isinstance(sw, SwitchGLU):
        return sw
    resident = getattr(sw, "resident_glu", None)
    return resident() if callable(resident) else None


# ----------------------------------------------------------------------------------------
# The rest of the decoder (laguna.py:75-113, :153-241)
# ----------------------------------------------------------------------------------------

class RMSNorm:
    """nn.RMSNorm (laguna.py:92-93, :160-161, :178): bf16 weight [dims]."""

    def __init__(self, dims, eps=1e-5, weight=None, device="cuda"):
        self.eps = eps
        self.weight = weight if weight is not None else torch.ones(dims, dtype=torch.bfloat16,
                                                                    device=device)

    def __call__(self, x):
        return ops.rmsnorm(x, self.weight, self.eps)


class QuantizedEmbedding(QuantizedLinear):
    """nn.QuantizedEmbedding (laguna.py:174 after nn.quantize): 4-bit table [V, H]."""

    def __call__(self, ids):
        return ops.embed(ids, self.mat, self.group_size, self.bits)

    def as_linear(self, x):
        return ops.qlinear(x, self.mat, None, self.group_size, self.bits)


class KVCache:
    """mlx-lm KVCache surface with bf16 keys/values [B, Hkv, cap, D]: ``offset`` rows are
    valid; capacity grows in 256-row steps (``capacity`` preallocates)."""
    step = 256

    def __init__(self, capacity=0):
        self.keys = self.values = None
        self.offset = 0
        self.capacity_hint = capacity

    def reserve(self, B, Hkv, D, T, device):
        need = self.offset + T
        if self.keys is None or self.keys.shape[2] < need:
            cap = max(self.capacity_hint, (need + self.step - 1) // self.step * self.step)
            k = torch.zeros(B, Hkv, cap, D, dtype=torch.bfloat16, device=device)
            v = torch.zeros_like(k)
            if self.keys is not None and self.offset:
                k[:, :, :self.offset] = self.keys[:, :, :self.offset]
                v[:, :, :self.offset] = self.values[:, :, :self.offset]
            self.keys, self.values = k, v

    def update_and_fetch(self, keys, values):
        B, Hkv, T, D = keys.shape
        self.reserve(B, Hkv, D, T, keys.device)
        self.keys[:, :, self.offset:self.offset + T] = keys
        self.values[:, :, self.offset:self.offset + T] = values
        self.offset += T
        return self.keys[:, :, :self.offset], self.values[:, :, :self.offset]

    @property
    def state(self):
        if self.keys is None:
            return None, None
        return self.keys[:, :, :self.offset], self.values[:, :, :self.offset]

    def is_trimmable(self):
        return True

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n

    def empty(self):
        return self.keys is None

    @property
    def nbytes(self):
        return 0 if self.keys is None else 2 * self.keys.numel() * self.keys.element_size()


def rope_setup(p, head_dim, device):
    """A layer type's RoPE for the prologue kernels (laguna.py:62-72): None for the default
    rope over every head dim (the kernel computes theta^(-2i/D) itself), else (inv_freq fp32
    [R/2] on ``device``, R, mscale) for partial rotary (R = head_dim * partial_rotary_factor)
    and/or YaRN scaling. YaRN (Peng et al., "YaRN: Efficient Context Window Extension of Large
    Language Models", 2023): frequencies whose wavelength exceeds the original context
    (below ``beta_slow`` rotations over it) are divided by ``factor``, those above
    ``beta_fast`` rotations are kept, a linear ramp in between; the rotated dims are scaled by
    ``attention_factor`` (default 0.1 ln(factor) + 1)."""
    R = int(head_dim * p.get("partial_rotary_factor", 1.0))
    kind = p.get("rope_type", "default")
    if kind == "default" and R == head_dim:
        return None
    if R % 64 or R <= 0:
        raise NotImplementedError(f"rotary dims {R}: the prologue kernels rotate multiples of 64")
    theta = float(p["rope_theta"])
    exps = [2.0 * i / R for i in range(R // 2)]
    base_freq = [theta ** -e for e in exps]
    mscale = 1.0
    if kind == "yarn":
        factor = float(p["factor"])
        ctx = float(p.get("original_max_position_embeddings", 4096))
        fast, slow = float(p.get("beta_fast", 32.0)), float(p.get("beta_slow", 1.0))

        def dim_of(rotations):  # the dim whose wavelength fits `rotations` times into ctx
            return R * math.log(ctx / (2 * math.pi * rotations)) / (2 * math.log(theta))

        lo, hi = max(math.floor(dim_of(fast)), 0), min(math.ceil(dim_of(slow)), R - 1)
        width = (hi - lo) if hi != lo else 0.001
        freqs = []
        for i, f in enumerate(base_freq):
            keep = 1.0 - min(max((i - lo) / width, 0.0), 1.0)  # 1: original, 0: interpolated
            freqs.append(f * keep + (f / factor) * (1.0 - keep))
        base_freq = freqs
        ms = p.get("attention_factor")
        mscale = float(ms) if ms is not None else (0.1 * math.log(factor) + 1.0 if factor > 1
                                                   else 1.0)
    elif kind != "default":
        raise NotImplementedError(f"rope_type {kind!r}")
    inv = torch.tensor(base_freq, dtype=torch.float64).to(torch.float32).to(device)
    return inv, R, mscale


class RotatingKVCache:
    """mlx-lm RotatingKVCache surface for sliding-window layers (laguna.py:209-214): the last
    ``max_size`` keys/values in a bf16 ring buffer [B, Hkv, max_size, D] (row = position mod
    max_size); ``offset`` counts every token seen. Attention over the ring is order-free
    (each key carries its own rotary position), so decode attends the filled rows as they
    lie."""

    def __init__(self, max_size, keep=0):
        if keep:
            raise NotImplementedError("keep > 0 (attention sinks) is not supported")
        self.max_size = int(max_size)
        self.keys = self.values = None
        self.offset = 0

    def reserve(self, B, Hkv, D, device):
        if self.keys is None:
            self.keys = torch.zeros(B, Hkv, self.max_size, D, dtype=torch.bfloat16, device=device)
            self.values = torch.zeros_like(self.keys)

    def window_rows(self):
        """Ring rows of the last min(offset, max_size) positions, oldest first."""
        n = min(self.offset, self.max_size)
        pos = torch.arange(self.offset - n, self.offset, device=self.keys.device)
        return pos % self.max_size

    @property
    def state(self):
        if self.keys is None:
            return None, None
        r = self.window_rows()
        return self.keys[:, :, r], self.values[:, :, r]

    def is_trimmable(self):
        return self.offset < self.max_size

    def trim(self, n):
        n = min(self.offset, n) if self.offset < self.max_size else 0
        self.offset -= n
        return n

    def empty(self):
        return self.keys is None

    @property
    def nbytes(self):
        return 0 if self.keys is None else 2 * self.keys.numel() * self.keys.element_size()


def _concat_rows(mats):
    """Row-concatenate MLX-layout matrices (words, scales, biases) with the same K."""
    return tuple(torch.cat([m[i] for m in mats], dim=0).contiguous() for i in range(3))


class Attention:
    """laguna.py:75-107: q/k/v/o/g projections (4-bit), per-head q/k RMSNorm, default RoPE,
    softplus output gate (per head or per element), GQA. The four input projections are
    stored as one row-concatenated matrix (one GEMV per token); ``q_proj``..``g_proj`` are
    row views of it."""

    def __init__(self, args, layer_idx, q_proj, k_proj, v_proj, o_proj, g_proj, q_norm=None,
                 k_norm=None):
        self.n_heads = args.num_attention_heads_per_layer[layer_idx]
        self.n_kv_heads = args.num_key_value_heads
        self.head_dim = hd = args.head_dim
        self.scale = hd ** -0.5
        self.per_head_gate = args.gating == "per-head"
        lt = args.layer_types[layer_idx]
        self.window = args.sliding_window if lt == "sliding_attention" else None
        if lt == "sliding_attention" and not self.window:
            raise ValueError("a sliding-window layer needs args.sliding_window")
        rp = args.rope_for(lt)
        self.rope_theta = float(rp["rope_theta"])
        self.eps = args.rms_norm_eps
        dev = q_proj.weight.device
        self.rope = rope_setup(rp, hd, dev)  # None: the default rope over every head dim
        self.q_norm = q_norm or RMSNorm(hd, args.rms_norm_eps, device=dev)
        self.k_norm = k_norm or RMSNorm(hd, args.rms_norm_eps, device=dev)
        mats = [q_proj.mat, k_proj.mat, v_proj.mat, g_proj.mat]
        fused = QuantizedLinear(*_concat_rows(mats), q_proj.group_size, q_proj.bits)
        self._qkvg = fused
        rows, r0 = [m[0].shape[0] for m in mats], 0
        views = []
        for n in rows:
            views.append(QuantizedLinear(fused.weight[r0:r0 + n], fused.scales[r0:r0 + n],
                                         fused.biases[r0:r0 + n], q_proj.group_size, q_proj.bits))
            r0 += n
        self.q_proj, self.k_proj, self.v_proj, self.g_proj = views
        self.o_proj = o_proj

    def __call__(self, x, mask=None, cache=None, residual=None, pos_dev=None, in_norm=None):
        """``pos_dev`` (device int32 [1]): the cache position lives on the device (one-token
        steps replayed from a CUDA graph); the cache must already hold the capacity and its
        host ``offset`` is left alone. ``in_norm`` (an RMSNorm): x is the un-normalised
        residual stream and the norm runs fused into the q/k/v/g projection."""
        B, L, H = x.shape
        if B != 1:
            raise NotImplementedError("batch size 1 only on this path")
        Hq, Hkv, D = self.n_heads, self.n_kv_heads, self.head_dim
        if in_norm is not None and L == 1 and pos_dev is not None and cache is not None:
            out = self._fused_token(x.reshape(1, H), cache, residual, pos_dev, in_norm)
            if out is not None:
                return out.reshape(B, L, H)
        if in_norm is None:
            qkvg = self._qkvg(x.reshape(L, H))
        elif L == 1:
            qkvg = ops.decode_gemv(x.reshape(1, H), self._qkvg.mat,
                                   norm=(in_norm.weight, in_norm.eps))
        else:
            qkvg = self._qkvg(in_norm(x).reshape(L, H))
        if cache is None:
            cache = RotatingKVCache(self.window) if self.window else KVCache()
        if isinstance(cache, RotatingKVCache):
            o = self._window_attention(qkvg, L, cache, pos_dev, x.device)
            out = self.o_proj(o, residual=None if residual is None else residual.reshape(L, H))
            return out.reshape(B, L, H)
        if getattr(cache, "q", None) is not None:  # 8-bit quantized cache (DequantKVCache)
            o = self._q8_attention(qkvg, L, cache, pos_dev, x.device)
            out = self.o_proj(o, residual=None if residual is None else residual.reshape(L, H))
            return out.reshape(B, L, H)
        if pos_dev is not None:
            if L != 1 or cache.keys is None:
                raise ValueError("device-position steps are single-token steps on a sized cache")
            q, gate = ops.attn_prep(qkvg, Hq, Hkv, D, self.q_norm.weight, self.k_norm.weight,
                                    self.eps, self.rope_theta, cache.keys[0], cache.values[0],
                                    pos_dev=pos_dev, gate_per_head=self.per_head_gate,
                                    rope=self.rope)
            o = ops.bf16_decode_attention(q.view(1, Hq, D), cache.keys, cache.values, 0,
                                          self.scale, gate=gate if self.per_head_gate else None,
                                          n_dev=pos_dev, n_add=1)
            o = o.view(1, Hq * D)
            if not self.per_head_gate:
                o = o * gate.view(1, Hq * D)
            out = self.o_proj(o, residual=None if residual is None else residual.reshape(1, H))
            return out.reshape(B, L, H)
        cache.reserve(1, Hkv, D, L, x.device)
        pos = cache.offset
        q, gate = ops.attn_prep(qkvg, Hq, Hkv, D, self.q_norm.weight, self.k_norm.weight,
                                self.eps, self.rope_theta, cache.keys[0], cache.values[0],
                                pos=pos, gate_per_head=self.per_head_gate, rope=self.rope)
        cache.offset += L
        if L == 1:
            o = ops.bf16_decode_attention(q.view(1, Hq, D), cache.keys, cache.values, pos + 1,
                                          self.scale,
                                          gate=gate if self.per_head_gate else None)
            o = o.view(1, Hq * D)
            if not self.per_head_gate:
                o = o * gate.view(1, Hq * D)
        else:
            k = cache.keys[:, :, :pos + L]
            v = cache.values[:, :, :pos + L]
            mask_ = None
            if pos:
                qp = torch.arange(L, device=x.device)[:, None] + pos
                mask_ = torch.arange(pos + L, device=x.device)[None, :] <= qp
            o = torch.nn.functional.scaled_dot_product_attention(
                q.unsqueeze(0), k, v, attn_mask=mask_, is_causal=mask_ is None, scale=self.scale,
                enable_gqa=True)[0].transpose(0, 1)  # [L, Hq, D]
            g = gate[..., None] if self.per_head_gate else gate.view(L, Hq, D)
            o = (o * g).reshape(L, Hq * D)
        out = self.o_proj(o, residual=None if residual is None else residual.reshape(L, H))
        return out.reshape(B, L, H)

    def step_streams(self, xn, cache, pos_dev, residual=None):
        """One decode step of B independent streams (batched decode, BASELINE config 5; the
        reference decodes one sequence per cache, laguna_mlx/cache.py has no batch merge):
        ``xn`` [B, H] the normalised inputs, one token per stream; ``cache`` a KVCache (or a
        sliding layer's RotatingKVCache) reserved for the B streams [B, Hkv, cap, D];
        ``pos_dev`` device int32 [B], the new tokens' positions. Returns o_proj(attention)
        [+ residual] as [B, H]."""
        B, H = xn.shape
        Hq, Hkv, D = self.n_heads, self.n_kv_heads, self.head_dim
        if getattr(cache, "q", None) is not None:
            raise NotImplementedError("batched decode runs over bf16 caches")
        ring = cache.max_size if isinstance(cache, RotatingKVCache) else 0
        if cache.keys is None or cache.keys.shape[0] != B:
            raise ValueError(f"the cache must be reserved for the {B} streams")
        qkvg = self._qkvg(xn)
        per_head = self.per_head_gate
        q, gate = ops.attn_prep_streams(qkvg, Hq, Hkv, D, self.q_norm.weight, self.k_norm.weight,
                                        self.eps, self.rope_theta, cache.keys, cache.values,
                                        pos_dev, gate_per_head=per_head, rope=self.rope,
                                        ring=ring)
        o = ops.bf16_decode_attention_streams(q, cache.keys, cache.values, pos_dev, 1, self.scale,
                                              gate=gate if per_head else None)
        o = o.view(B, Hq * D)
        if not per_head:
            o = o * gate.view(B, Hq * D)
        return self.o_proj(o, residual=residual)

    def _fused_token(self, x, cache, residual, pos_dev, in_norm):
        """A device-position single-token step with the q/k/v/g projection and the attention
        prologue in one launch (``ops.decode_qkv_prep``); None when the shape needs the
        two-launch form."""
        Hq, Hkv, D = self.n_heads, self.n_kv_heads, self.head_dim
        per_head = self.per_head_gate
        q8 = getattr(cache, "q", None) is not None
        if q8:
            if not cache.fused_decode:
                return None
            qc = cache.q
            qc.reserve(1, Hkv, D, 1, x.device)
            ck, cv = qc.keys, qc.values
        else:
            if isinstance(cache, RotatingKVCache):
                cache.reserve(1, Hkv, D, x.device)
            if cache.keys is None:
                return None
            ck, cv = cache.keys[0], cache.values[0]
        ring = cache.max_size if isinstance(cache, RotatingKVCache) else 0
        try:
            _, q, gate = ops.decode_qkv_prep(x, self._qkvg.mat, (in_norm.weight, in_norm.eps),
                                             Hq, Hkv, D, self.q_norm.weight, self.k_norm.weight,
                                             self.eps, self.rope_theta, ck, cv, pos_dev=pos_dev,
                                             gate_per_head=per_head, rope=self.rope, ring=ring)
        except _lib.LagunaError as e:
            if e.code != _lib.LG_ERR_UNSUPPORTED:
                raise
            return None
        if q8:
            cap = ck[0].shape[2]
            o = ops.q8_decode_attention_dev(q.view(1, Hq, D), ck, cv, cap, pos_dev, 1,
                                            self.scale, gate=gate if per_head else None)
        else:
            o = ops.bf16_decode_attention(q.view(1, Hq, D), cache.keys, cache.values, 0,
                                          self.scale, gate=gate if per_head else None,
                                          n_dev=pos_dev, n_add=1)
        o = o.view(1, Hq * D)
        if not per_head:
            o = o * gate.view(1, Hq * D)
        return self.o_proj(o, residual=None if residual is None else residual.reshape(1, -1))

    def _window_attention(self, qkvg, L, cache, pos_dev, device):
        """Sliding-window attention over a RotatingKVCache (laguna.py:183-186, :209-214): a
        query at position p sees the keys of positions p - W < j <= p. Single-token steps write
        the new row into the ring (row = p mod W) and attend its filled rows; multi-token steps
        attend over the window's previous rows and the new ones with a window mask, then keep
        the last W rows in the ring."""
        Hq, Hkv, D, W = self.n_heads, self.n_kv_heads, self.head_dim, cache.max_size
        per_head = self.per_head_gate
        cache.reserve(1, Hkv, D, device)
        kr, vr = cache.keys[0], cache.values[0]
        if L == 1:
            pos = cache.offset
            q, gate = ops.attn_prep(qkvg, Hq, Hkv, D, self.q_norm.weight, self.k_norm.weight,
                                    self.eps, self.rope_theta, kr, vr, pos=pos, pos_dev=pos_dev,
                                    gate_per_head=per_head, rope=self.rope, ring=W)
            g = gate if per_head else None
            if pos_dev is not None:  # the valid rows min(p + 1, W): the kernel clamps to cap
                o = ops.bf16_decode_attention(q.view(1, Hq, D), cache.keys, cache.values, 0,
                                              self.scale, gate=g, n_dev=pos_dev, n_add=1)
            else:
                cache.offset += 1
                o = ops.bf16_decode_attention(q.view(1, Hq, D), cache.keys, cache.values,
                                              min(pos + 1, W), self.scale, gate=g)
            o = o.view(1, Hq * D)
            return o if per_head else o * gate.view(1, Hq * D)
        if pos_dev is not None:
            raise ValueError("device-position steps are single-token steps")
        pos = cache.offset
        n_prev = min(pos, W)
        kt = torch.empty(Hkv, n_prev + L, D, dtype=torch.bfloat16, device=device)
        vt = torch.empty_like(kt)
        if n_prev:
            rows = cache.window_rows()
            kt[:, :n_prev] = kr[:, rows]
            vt[:, :n_prev] = vr[:, rows]
        q, gate = ops.attn_prep(qkvg, Hq, Hkv, D, self.q_norm.weight, self.k_norm.weight,
                                self.eps, self.rope_theta, kt, vt, pos=pos,
                                gate_per_head=per_head, rope=self.rope, row0=pos - n_prev)
        qi = torch.arange(L, device=device)[:, None] + n_prev
        kj = torch.arange(n_prev + L, device=device)[None, :]
        mask = (kj <= qi) & (kj > qi - W)
        o = torch.nn.functional.scaled_dot_product_attention(
            q.unsqueeze(0), kt.unsqueeze(0), vt.unsqueeze(0), attn_mask=mask, scale=self.scale,
            enable_gqa=True)[0].transpose(0, 1)  # [L, Hq, D]
        keep = min(W, n_prev + L)
        newpos = torch.arange(pos + L - keep, pos + L, device=device)
        kr[:, newpos % W] = kt[:, n_prev + L - keep:]
        vr[:, newpos % W] = vt[:, n_prev + L - keep:]
        cache.offset = pos + L
        g = gate[..., None] if per_head else gate.view(L, Hq, D)
        return (o * g).reshape(L, Hq * D)

    def _q8_attention(self, qkvg, L, cache, pos_dev, device):
        """Attention over an 8-bit group-64 DequantKVCache (laguna_mlx/cache.py:89-106): the new
        k, v rows are quantized into the packed cache; single-token steps with ``fused_decode``
        attend straight off the packed rows (q8 kernel), other steps over dequantized rows."""
        Hq, Hkv, D = self.n_heads, self.n_kv_heads, self.head_dim
        qc = cache.q
        qc.reserve(1, Hkv, D, L, device)
        cap = qc.keys[0].shape[2]
        per_head = self.per_head_gate
        if pos_dev is not None:
            if L != 1 or not cache.fused_decode:
                raise ValueError("device-position steps are fused single-token steps")
            q, gate = ops.attn_prep_q8(qkvg, Hq, Hkv, D, self.q_norm.weight, self.k_norm.weight,
                                       self.eps, self.rope_theta, qc.keys, qc.values,
                                       pos_dev=pos_dev, gate_per_head=per_head, rope=self.rope)
            o = ops.q8_decode_attention_dev(q.view(1, Hq, D), qc.keys, qc.values, cap, pos_dev,
                                            1, self.scale, gate=gate if per_head else None)
            o = o.view(1, Hq * D)
            return o if per_head else o * gate.view(1, Hq * D)
        pos = qc.offset
        q, gate = ops.attn_prep_q8(qkvg, Hq, Hkv, D, self.q_norm.weight, self.k_norm.weight,
                                   self.eps, self.rope_theta, qc.keys, qc.values, pos=pos,
                                   gate_per_head=per_head, rope=self.rope)
        qc.offset += L
        n = pos + L
        cache.fused_step = cache.fused_decode and L == 1
        if cache.fused_step:
            o = ops.q8_decode_attention(q.view(1, Hq, 1, D), qc.keys, qc.values, n, self.scale)
            g = gate.view(1, Hq, 1) if per_head else gate.view(1, Hq, D)
            return (o.view(1, Hq, D) * g).reshape(1, Hq * D)
        k = ops.dequantize_rows(qc.keys, n, qc.group_size, qc.bits)
        v = ops.dequantize_rows(qc.values, n, qc.group_size, qc.bits)
        mask_ = None
        if pos:
            qp = torch.arange(L, device=device)[:, None] + pos
            mask_ = torch.arange(n, device=device)[None, :] <= qp
        o = torch.nn.functional.scaled_dot_product_attention(
            q.unsqueeze(0), k, v, attn_mask=mask_, is_causal=mask_ is None and L > 1,
            scale=self.scale, enable_gqa=True)[0].transpose(0, 1)  # [L, Hq, D]
        g = gate[..., None] if per_head else gate.view(L, Hq, D)
        return (o * g).reshape(L, Hq * D)


class DecoderLayer:
    """laguna.py:153-166: pre-norm attention and MLP (dense in ``mlp_only_layers``, MoE
    otherwise) with residual adds."""

    def __init__(self, args, layer_idx, self_attn, mlp, input_layernorm=None,
                 post_attention_layernorm=None):
        self.self_attn = self_attn
        self.mlp = mlp
        dev = self_attn.o_proj.weight.device
        self.input_layernorm = input_layernorm or RMSNorm(args.hidden_size, args.rms_norm_eps,
                                                          device=dev)
        self.post_attention_layernorm = post_attention_layernorm or RMSNorm(
            args.hidden_size, args.rms_norm_eps, device=dev)

    def __call__(self, x, mask=None, cache=None):
        h = self.self_attn(self.input_layernorm(x), mask, cache, residual=x)
        return h + self.mlp(self.post_attention_layernorm(h))  # bf16 add, one rounding


class LagunaModel:
    """laguna.py:169-193. The layer loop fuses each residual add into the next RMSNorm (and
    the attention residual into the o_proj GEMV epilogue)."""

    def __init__(self, args, embed_tokens, layers, norm=None):
        self.args = args
        self.embed_tokens = embed_tokens
        self.layers = layers
        self.norm = norm or RMSNorm(args.hidden_size, args.rms_norm_eps,
                                    device=embed_tokens.weight.device)
        self.layer_types = args.layer_types

    def __call__(self, inputs, cache=None, pos_dev=None, normed=True):
        """Final hidden states (normalised; ``normed=False`` returns the residual stream of a
        one-token step un-normalised, for a consumer that fuses the final norm)."""
        if inputs.dim() == 1:
            inputs = inputs[None]
        x = self.embed_tokens(inputs)
        if cache is None:
            cache = [None] * len(self.layers)
        if x.shape[0] == 1 and x.shape[1] == 1:
            x = self._token(x, cache, pos_dev)
            return ops.rmsnorm(x, self.norm.weight, self.norm.eps) if normed else x
        if not normed:
            raise ValueError("normed=False is for one-token steps")
        xn = self.layers[0].input_layernorm(x)
        for i, (layer, c) in enumerate(zip(self.layers, cache)):
            h = layer.self_attn(xn, None, c, residual=x, pos_dev=pos_dev)
            m = layer.mlp(layer.post_attention_layernorm(h))
            nxt = self.layers[i + 1].input_layernorm if i + 1 < len(self.layers) else self.norm
            x, xn = ops.rmsnorm(m, nxt.weight, nxt.eps, residual=h)
        return xn

    def step_streams(self, ids, cache, pos_dev, moe=None):
        """Final normalised hidden states [B, H] of one decode step of B independent streams:
        ``ids`` device int32 [B] (each stream's newest token), ``cache`` from
        ``Model.make_stream_cache``, ``pos_dev`` device int32 [B] (the tokens' positions).
        ``moe``: per layer a callable that replaces the MLP sub-block's forward on the
        normalised [B, H] rows (the expert-parallel block), or None for the layer's own."""
        x = self.embed_tokens(ids.reshape(1, -1)).reshape(ids.shape[0], -1)
        xn = self.layers[0].input_layernorm(x)
        for i, (layer, c) in enumerate(zip(self.layers, cache)):
            h = layer.self_attn.step_streams(xn, c, pos_dev, residual=x)
            fwd = moe[i] if moe is not None and moe[i] is not None else layer.mlp
            m = fwd(layer.post_attention_layernorm(h))
            nxt = self.layers[i + 1].input_layernorm if i + 1 < len(self.layers) else self.norm
            x, xn = ops.rmsnorm(m, nxt.weight, nxt.eps, residual=h)
        return xn

    def _token(self, x, cache, pos_dev):
        """One token through every layer: per layer the input norm runs inside the q/k/v/g
        GEMV, the attention residual inside o_proj, and the MLP sub-block (norm, router,
        experts, combine, residual) in the one-token kernels."""
        for layer, c in zip(self.layers, cache):
            h = layer.self_attn(x, None, c, residual=x, pos_dev=pos_dev,
                                in_norm=layer.input_layernorm)
            mlp, pn = layer.mlp, layer.post_attention_layernorm
            tok = getattr(mlp, "token", None)
            y = tok(h, pn) if tok is not None else None
            x = y.reshape(h.shape) if y is not None else h + mlp(pn(h))  # bf16 add
        return x


class Model:
    """laguna.py:196-241: ``model`` (LagunaModel) + untied ``lm_head``."""

    def __init__(self, args, model, lm_head):
        self.args = args
        self.model_type = args.model_type
        self.model = model
        self.lm_head = lm_head

    def __call__(self, inputs, cache=None):
        return self.lm_head(self.model(inputs, cache))

    def last_logits(self, inputs, cache=None, pos_dev=None):
        """Logits of the last position only (what generation needs after a prefill). A
        one-token step runs the final norm inside the head's GEMV."""
        ids = inputs if inputs.dim() > 1 else inputs[None]
        if ids.shape[0] == 1 and ids.shape[1] == 1:
            x = self.model(ids, cache, pos_dev=pos_dev, normed=False)
            n = self.model.norm
            H = x.shape[-1]
            return ops.decode_gemv(x.reshape(1, H), self.lm_head.mat,
                                   norm=(n.weight, n.eps)).reshape(1, 1, -1)
        h = self.model(ids, cache, pos_dev=pos_dev)
        return self.lm_head(h[:, -1:])

    def step_streams(self, ids, cache, pos_dev, moe=None):
        """Logits [B, V] of one decode step of B independent streams (see
        ``LagunaModel.step_streams``); the caller advances ``pos_dev``."""
        return self.lm_head(self.model.step_streams(ids, cache, pos_dev, moe))

    def make_stream_cache(self, B, capacity, device="cuda"):
        """Per layer a bf16 cache holding B streams of ``capacity`` rows each ([B, Hkv,
        capacity, D]; a sliding layer's ring holds its window), for ``step_streams``."""
        a = self.args
        out = []
        for L in self.layers:
            at = L.self_attn
            c = RotatingKVCache(at.window) if at.window else KVCache(capacity)
            if at.window:
                c.reserve(B, a.num_key_value_heads, a.head_dim, device)
            else:
                c.reserve(B, a.num_key_value_heads, a.head_dim, capacity, device)
            out.append(c)
        return out

    @property
    def layers(self):
        return self.model.layers

    def make_cache(self, capacity=0):
        """laguna.py:209-214: a ring of the window for sliding-window layers, a growing cache
        (``capacity`` rows preallocated) for full-attention layers."""
        return [RotatingKVCache(self.args.sliding_window) if lt == "sliding_attention"
                else KVCache(capacity) for lt in self.args.layer_types]

    def sanitize(self, weights):
        """laguna.py:216-228 on a dict of tensors: per-expert weights stacked into
        ``switch_mlp``, the router bias moved to ``mlp.e_score_correction_bias``."""
        E = self.args.num_experts
        for l in range(self.args.num_hidden_layers):
            p = f"model.layers.{l}.mlp"
            if f"{p}.experts.0.gate_proj.weight" in weights:
                for n in ("gate_proj", "up_proj", "down_proj"):
                    weights[f"{p}.switch_mlp.{n}.weight"] = torch.stack(
                        [weights.pop(f"{p}.experts.{e}.{n}.weight") for e in range(E)])
            bias = weights.pop(f"{p}.experts.e_score_correction_bias", None)
            if bias is not None:
                weights[f"{p}.e_score_correction_bias"] = bias
        return weights

    def cast_predicate(self, key):
        return "e_score_correction_bias" not in key

    @property
    def quant_predicate(self):
        def predicate(path, _):
            if path.endswith("mlp.gate"):
                return {"group_size": 64, "bits": 8}
            return True

        return predicate


def model_from_weights(args, weights, quantization=None, device="cuda", switch_mlps=None):
    """A ``Model`` from MLX parameter names (laguna.py:169-241 after ``sanitize`` and
    ``nn.quantize``): quantized linears as ``<path>.weight`` (uint32 words), ``.scales``,
    ``.biases``; norms as ``<path>.weight``; the router's ``e_score_correction_bias`` in fp32.
    ``quantization``: {"group_size", "bits", "<path>": {...} per-module overrides} (the
    config's "quantization" entry). ``switch_mlps``: {layer: SwitchGLU-like} for MoE layers
    whose routed experts come from elsewhere (an expert pack)."""
    q = dict(quantization or {"group_size": 64, "bits": 4})
    dev = torch.device(device)

    def t(name, dtype=None):
        v = weights[name]
        if v.dtype == torch.uint32:
            v = v.view(torch.int32)
        v = v.to(dev)
        return v.to(dtype) if dtype is not None else v

    def qcfg(path):
        o = q.get(path, {})
        return o.get("group_size", q["group_size"]), o.get("bits", q["bits"])

    def lin(path, cls=QuantizedLinear):
        if f"{path}.scales" not in weights:  # unquantized (fp32 router)
            return t(f"{path}.weight", torch.float32)
        g, b = qcfg(path)
        return cls(t(f"{path}.weight"), t(f"{path}.scales", torch.bfloat16),
                   t(f"{path}.biases", torch.bfloat16), g, b)

    def norm(path, n):
        return RMSNorm(n, args.rms_norm_eps, t(f"{path}.weight", torch.bfloat16))

    H, D = args.hidden_size, args.head_dim
    layers = []
    for i in range(args.num_hidden_layers):
        p = f"model.layers.{i}"
        at = Attention(args, i, *(lin(f"{p}.self_attn.{n}") for n in
                                  ("q_proj", "k_proj", "v_proj", "o_proj", "g_proj")),
                       norm(f"{p}.self_attn.q_norm", D), norm(f"{p}.self_attn.k_norm", D))
        if i in args.mlp_only_layers:
            I = args.intermediate_size
            mlp = MLP(H, I, *(lin(f"{p}.mlp.{n}") for n in ("gate_proj", "up_proj", "down_proj")))
        else:
            if switch_mlps is not None and i in switch_mlps:
                sw = switch_mlps[i]
            else:
                sw = SwitchGLU(H, args.moe_intermediate_size, args.num_experts,
                               *(lin(f"{p}.mlp.switch_mlp.{n}", SwitchLinear)
                                 for n in ("gate_proj", "up_proj", "down_proj")))
            sh = None
            if f"{p}.mlp.shared_expert.gate_proj.weight" in weights:
                sh = MLP(H, args.shared_expert_intermediate_size,
                         *(lin(f"{p}.mlp.shared_expert.{n}")
                           for n in ("gate_proj", "up_proj", "down_proj")))
            bias_key = f"{p}.mlp.e_score_correction_bias"
            bias = t(bias_key, torch.float32) if bias_key in weights else \
                torch.zeros(args.num_experts, device=dev)
            mlp = SparseMoeBlock(args, lin(f"{p}.mlp.gate"), bias, sw, sh)
        layers.append(DecoderLayer(args, i, at, mlp, norm(f"{p}.input_layernorm", H),
                                   norm(f"{p}.post_attention_layernorm", H)))
    emb = lin("model.embed_tokens")
    embed = QuantizedEmbedding(emb.weight, emb.scales, emb.biases, emb.group_size, emb.bits)
    model = LagunaModel(args, embed, layers, norm("model.norm", H))
    return Model(args, model, lin("lm_head"))


def load(path, device="cuda"):
    """(model, tokenizer) from an MLX-format checkpoint directory (what mlx-lm's ``load``
    reads for this architecture, laguna.py:196-241): ``config.json`` with its
    "quantization" entry and the ``*.safetensors`` shards. Per-expert (unstacked) weights
    and the experts' router bias are rearranged by ``Model.sanitize``. The tokenizer is the
    directory's Hugging Face tokenizer when it has one, else None."""
    import json
    from pathlib import Path

    from safetensors.torch import load_file

    path = Path(path)
    config = json.loads((path / "config.json").read_text())
    args = ModelArgs.from_dict(config)
    shards = sorted(path.glob("*.safetensors"))
    if not shards:
        raise FileNotFoundError(f"{path}: no *.safetensors weights")
    weights = {}
    for f in shards:
        weights.update(load_file(str(f)))
    weights = Model.sanitize(Model(args, None, None), weights)
    model = model_from_weights(args, weights, config.get("quantization"), device)
    tok = None
    if (path / "tokenizer.json").exists() or (path / "tokenizer_config.json").exists():
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(str(path))
    return model, tok


class DecodeGraph:
    """Greedy bs1 decoding one CUDA-graph replay per token. The token id and the cache
    position live on the device: each step embeds ``tok``, runs every layer at position
    ``pos`` (all kernels read it there), and the argmax kernel writes the next id into
    ``tok`` and advances ``pos`` — so consecutive steps need no host work but the replay.

    ``cache`` is a prefilled ``make_cache(capacity)`` list with room for the tokens to come;
    ``tok`` (device int32 [1]) is the next input token. The first step runs eagerly (it also
    sizes every workspace) before the graph is captured."""

    def __init__(self, model, cache, tok, pdl=True):
        self.model, self.cache = model, cache
        self.tok = tok.reshape(1).to(torch.int32).clone()
        self.pos = torch.tensor([cache[0].offset], dtype=torch.int32, device=self.tok.device)
        full = [c for c in cache if not isinstance(c, RotatingKVCache)]
        if full:
            c0 = full[0]
            self.cap = (c0.q.keys[0].shape[2] if getattr(c0, "q", None) is not None
                        else c0.keys.shape[2])
        else:  # only sliding windows: rings never fill up
            self.cap = 1 << 30
        self.steps = 0
        self._body()  # one real step, eagerly
        self.first_logits = self.logits.clone()  # that step's logits (the capture reuses names)
        self.steps = 1
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        # the step's kernels are captured with programmatic dependent launch: each starts
        # while its predecessor runs and streams its weights before waiting for it
        from . import _lib
        prev = _lib.lib().lg_set_pdl(1 if pdl else 0)
        try:
            with torch.cuda.graph(self.graph):
                self._body()
        finally:
            _lib.lib().lg_set_pdl(prev)

    def _body(self):
        logits = self.model.last_logits(self.tok.view(1, 1), self.cache, pos_dev=self.pos)
        ops.argmax(logits.view(1, -1), ids=self.tok, pos=self.pos, inc=1)
        # the captured step's logits buffer (graph memory): valid after each replay
        self.logits = logits.view(-1)

    def step(self):
        """One token (asynchronous); ``tok`` holds it afterwards."""
        if self.cache[0].offset + self.steps + 1 > self.cap:
            raise ValueError(f"the cache holds {self.cap} rows")
        self.graph.replay()
        self.steps += 1

    def position(self):
        """Tokens in the cache now (host copy of the device counter)."""
        return int(self.pos.item())


class StreamDecodeGraph:
    """Greedy decoding of B independent streams, one CUDA-graph replay per step (BASELINE
    config 5's batched decode). The streams' newest tokens ``tok`` and positions ``pos``
    (device int32 [B]) stay on the device: each replay embeds the B tokens, runs every layer
    over the B streams' own caches, writes each stream's argmax into ``tok`` and advances every
    position. ``moe`` (optional, per layer): expert-parallel MoE forwards with device-held
    epochs, whose exchanges replay with the graph. The first step runs eagerly (it also sizes
    every workspace) before the graph is captured."""

    def __init__(self, model, cache, tok, pos, moe=None, pdl=False):
        self.model, self.cache, self.moe = model, cache, moe
        self.tok = tok.reshape(-1).to(torch.int32).clone()
        self.pos = pos.reshape(-1).to(torch.int32).clone()
        full = [c for c in cache if not isinstance(c, RotatingKVCache)]
        self.cap = full[0].keys.shape[2] if full else 1 << 30
        self.pos0 = int(self.pos.max()) if self.pos.numel() else 0  # the furthest stream's row
        if self.pos0 >= self.cap:
            raise ValueError(f"a stream is at position {self.pos0}; the caches hold {self.cap}")
        self._body()
        self.first_logits = self.logits.clone()
        self.steps = 1
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        # ``pdl``: capture with programmatic dependent launch, as DecodeGraph's step does. Off
        # by default: at 64 streams the early-started CTAs of the next kernel hold SM resources
        # the running one needs (measured 27.95 against 21.91 ms per step at 64 x 8k, 40 layers)
        from . import _lib
        prev = _lib.lib().lg_set_pdl(1 if pdl else 0)
        try:
            with torch.cuda.graph(self.graph):
                self._body()
        finally:
            _lib.lib().lg_set_pdl(prev)

    def _body(self):
        logits = self.model.step_streams(self.tok, self.cache, self.pos, self.moe)
        ops.argmax(logits, ids=self.tok)
        self.pos.add_(1)
        self.logits = logits  # the captured step's logits buffer: valid after each replay

    def step(self):
        """One token per stream (asynchronous); ``tok`` holds them afterwards."""
        if self.pos0 + self.steps >= self.cap:  # the row this replay would write
            raise ValueError(f"the caches hold {self.cap} rows")
        self.graph.replay()
        self.steps += 1


def generate(model, prompt, max_tokens, cache=None):
    """Greedy decoding: prefill ``prompt`` (device int tensor [L]), then ``max_tokens`` steps;
    returns the generated ids (list of int)."""
    if cache is None:
        cache = model.make_cache()
    ids = prompt.to(torch.int32).reshape(1, -1)
    logits = model.last_logits(ids, cache)
    out = []
    tok = ops.argmax(logits.reshape(1, -1))
    for _ in range(max_tokens):
        out.append(tok)
        logits = model.last_logits(tok.view(1, 1), cache)
        tok = ops.argmax(logits.reshape(1, -1))
    return [int(t) for t in torch.cat(out).tolist()]
