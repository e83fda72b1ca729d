"""Laguna MoE block on B200, with the module surface of laguna_mlx/laguna.py.

Same names and call semantics as the reference (laguna.py:18-150): ``ModelArgs`` with its
validation, ``MLP(dim, hidden)``, ``SwitchGLU(input_dims, hidden_dims, num_experts)`` called
as ``switch_mlp(x, indices) -> [..., k, hidden]``, and ``SparseMoeBlock`` with a separate,
patchable ``route(x) -> (inds, w)`` (hooks and pruning wrap it). Tensors are torch CUDA
tensors; weights use the MLX packed layout (uint32 words as int32, bf16 scales/biases).
All arithmetic runs in the sm_100a kernels of ``liblaguna_b200.so``.
"""
import inspect
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import torch

from . import ops


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


def _fused_experts(sw):
    """The SwitchGLU whose weights the fused kernel can read directly, or None."""
    if isinstance(sw, SwitchGLU):
        return sw
    resident = getattr(sw, "resident_glu", None)
    return resident() if callable(resident) else None
