"""The expert pack format of lagunaLab (scripts/pack_experts.py:33-88): a model split into
``resident.safetensors`` (every weight but the routed experts), one file per MoE layer
``experts/layer_NN.bin`` holding expert e's arrays at byte ``e * stride`` (stride rounded up
to 16 KiB pages), and ``layout.json`` = {num_experts, stride, layers, arrays: {"proj.part":
{offset, shape, dtype}}}; ``config.json`` carries the model arguments and the quantization.

Reading (``expert_from_bytes``, ``read_expert``) gives torch tensors with the same bits;
``pack_model`` writes the format from an in-memory ``laguna.Model`` (the reference packs an
MLX checkpoint directory; this writer serves tests and conversions done on this side).
"""
import json
from pathlib import Path

import numpy as np
import torch

PAGE = 16384
PROJS = ("gate_proj", "up_proj", "down_proj")
PARTS = ("weight", "scales", "biases")
_NP = {"uint32": np.uint32, "bfloat16": np.uint16, "float16": np.float16, "float32": np.float32}
_TORCH = {"uint32": torch.int32, "bfloat16": torch.bfloat16, "float16": torch.float16,
          "float32": torch.float32}


def _dtype_name(t):
    return {torch.int32: "uint32", torch.uint32: "uint32", torch.bfloat16: "bfloat16",
            torch.float16: "float16", torch.float32: "float32"}[t.dtype]


def _to_bytes(t):
    """Raw little-endian bytes of a tensor (bf16 as its 16-bit patterns)."""
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    elif t.dtype == torch.uint32:
        t = t.view(torch.int32)
    return t.numpy().tobytes()


def expert_from_bytes(buf, layout):
    """One expert's arrays from its packed bytes: {"gate_proj.weight": tensor, ...} (uint32
    words as int32 tensors holding the same bits)."""
    out = {}
    for name, a in layout["arrays"].items():
        count = int(np.prod(a["shape"]))
        arr = np.frombuffer(buf, dtype=_NP[a["dtype"]], count=count, offset=a["offset"])
        t = torch.from_numpy(arr.copy().reshape(a["shape"]))
        if a["dtype"] == "bfloat16":
            t = t.view(torch.int16).view(torch.bfloat16)
        elif a["dtype"] == "uint32":
            t = t.view(torch.int32)
        out[name] = t
    return out


def read_expert(pack_dir, layout, layer, e):
    with open(Path(pack_dir) / "experts" / f"layer_{layer:02d}.bin", "rb") as f:
        f.seek(e * layout["stride"])
        return expert_from_bytes(f.read(layout["stride"]), layout)


def read_layer(pack_dir, layout, layer):
    """Every expert of one layer stacked: {"gate_proj.weight": [E, ...], ...} (host tensors)."""
    E, stride = layout["num_experts"], layout["stride"]
    raw = (Path(pack_dir) / "experts" / f"layer_{layer:02d}.bin").read_bytes()
    if len(raw) < E * stride:
        raise ValueError(f"layer {layer}: {len(raw)} bytes, expected {E} experts x {stride}")
    out = {}
    for name, a in layout["arrays"].items():
        rows = np.frombuffer(raw, dtype=np.uint8).reshape(E, stride)
        nbytes = int(np.prod(a["shape"])) * np.dtype(_NP[a["dtype"]]).itemsize
        blk = np.ascontiguousarray(rows[:, a["offset"]:a["offset"] + nbytes])
        arr = blk.view(_NP[a["dtype"]]).reshape(E, *a["shape"])
        t = torch.from_numpy(arr.copy())
        if a["dtype"] == "bfloat16":
            t = t.view(torch.int16).view(torch.bfloat16)
        elif a["dtype"] == "uint32":
            t = t.view(torch.int32)
        out[name] = t
    return out


def model_weights(model):
    """An in-memory ``laguna.Model`` as a dict of MLX parameter names -> host tensors."""
    from . import laguna
    w = {}

    def put(prefix, mod):
        if isinstance(mod, laguna.QuantizedLinear):
            w[f"{prefix}.weight"], w[f"{prefix}.scales"], w[f"{prefix}.biases"] = mod.mat
        elif isinstance(mod, laguna.RMSNorm):
            w[f"{prefix}.weight"] = mod.weight
        elif isinstance(mod, torch.Tensor):
            w[f"{prefix}.weight"] = mod
        else:
            raise TypeError(f"{prefix}: {type(mod).__name__}")

    m = model.model
    put("model.embed_tokens", m.embed_tokens)
    put("model.norm", m.norm)
    put("lm_head", model.lm_head)
    for l, layer in enumerate(m.layers):
        p = f"model.layers.{l}"
        put(f"{p}.input_layernorm", layer.input_layernorm)
        put(f"{p}.post_attention_layernorm", layer.post_attention_layernorm)
        at = layer.self_attn
        for n in ("q_proj", "k_proj", "v_proj", "o_proj", "g_proj", "q_norm", "k_norm"):
            put(f"{p}.self_attn.{n}", getattr(at, n))
        mlp = layer.mlp
        if isinstance(mlp, laguna.SparseMoeBlock):
            put(f"{p}.mlp.gate", mlp.gate)
            w[f"{p}.mlp.e_score_correction_bias"] = mlp.e_score_correction_bias
            sw = laguna._fused_experts(mlp.switch_mlp)
            for n in PROJS:
                put(f"{p}.mlp.switch_mlp.{n}", getattr(sw, n))
            if mlp.shared_expert is not None:
                for n in PROJS:
                    put(f"{p}.mlp.shared_expert.{n}", getattr(mlp.shared_expert, n))
        else:
            for n in PROJS:
                put(f"{p}.mlp.{n}", getattr(mlp, n))
    return {k: v.detach().cpu().contiguous() for k, v in w.items()}


def model_config(args, group_size=64, bits=4):
    """config.json content for a model: its arguments plus the quantization (the router of
    every MoE layer 8-bit, laguna.py:236-238)."""
    import dataclasses
    c = dataclasses.asdict(args)
    q = {"group_size": group_size, "bits": bits}
    for l in range(args.num_hidden_layers):
        if l not in args.mlp_only_layers:
            q[f"model.layers.{l}.mlp.gate"] = {"group_size": 64, "bits": 8}
    c["quantization"] = q
    return c


def save_checkpoint(model, out_dir, group_size=64, bits=4):
    """Write ``model`` as an MLX-format checkpoint directory (``config.json`` +
    ``model.safetensors``, packed words as uint32), the layout ``laguna.load`` reads."""
    from safetensors.torch import save_file
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    w = {k: (t.view(torch.uint32) if t.dtype == torch.int32 else t)
         for k, t in model_weights(model).items()}
    save_file(w, str(out / "model.safetensors"))
    (out / "config.json").write_text(json.dumps(model_config(model.args, group_size, bits),
                                                indent=1))


def pack_model(model, out_dir, group_size=64, bits=4):
    """Write ``model`` in the pack format (same byte layout as scripts/pack_experts.py)."""
    from safetensors.torch import save_file
    out = Path(out_dir)
    (out / "experts").mkdir(parents=True, exist_ok=True)
    w = model_weights(model)
    key = lambda l, n: f"model.layers.{l}.mlp.switch_mlp.{n}"
    layers = sorted({int(k.split(".")[2]) for k in w if ".mlp.switch_mlp." in k})
    first = layers[0]
    E = w[key(first, "gate_proj.weight")].shape[0]
    arrays, offset = {}, 0
    for proj in PROJS:
        for part in PARTS:
            t = w[key(first, f"{proj}.{part}")][0]
            arrays[f"{proj}.{part}"] = {"offset": offset, "shape": list(t.shape),
                                        "dtype": _dtype_name(t)}
            offset += t.numel() * t.element_size()
    stride = -(-offset // PAGE) * PAGE
    for l in layers:
        stacked = {n: w.pop(key(l, n)) for n in arrays}
        with open(out / "experts" / f"layer_{l:02d}.bin", "wb") as f:
            for e in range(E):
                blob = b"".join(_to_bytes(stacked[n][e]) for n in arrays)
                f.write(blob + b"\0" * (stride - len(blob)))
    res = {}
    for k, t in w.items():
        res[k] = t.view(torch.uint32) if t.dtype == torch.int32 else t
    save_file(res, str(out / "resident.safetensors"))
    layout = {"num_experts": E, "stride": stride, "layers": layers, "arrays": arrays}
    (out / "layout.json").write_text(json.dumps(layout, indent=1))
    (out / "config.json").write_text(json.dumps(model_config(model.args, group_size, bits),
                                                indent=1))
    return layout
