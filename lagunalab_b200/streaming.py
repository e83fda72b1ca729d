"""The expert-streaming surface of lagunaLab (laguna_mlx/streaming.py:23-145) on B200.

The reference keeps a few expert "slots" per layer in memory and refills them from the pack's
per-layer files as the router asks for experts (an LFU slot cache over parallel preads). A
B200 holds every expert of the model in HBM, so here the same objects load each layer's
experts from the pack once, at construction, and serve every request from HBM:

* ``ExpertStore(pack_dir, layout, layer, slots, group_size, bits, hidden, inter)`` with
  ``load(experts) -> {expert: slot}``: the identity mapping (every expert has its own slot);
  ``hits`` counts the experts requested, ``misses`` and ``bytes_read`` (bytes read from the
  pack after construction) stay 0. ``slots`` is accepted for the same call surface; the
  resident slot count is the layer's expert count.
* ``StreamingSwitchGLU(store)(x, indices)``: the SwitchGLU call surface over the store; the
  decoder's fused expert kernels read the store's resident weights directly
  (``resident_glu``) and count their picks as hits.
* ``load_streaming(pack_dir, slots, cache_limit_gb=None) -> (model, tokenizer)`` and
  ``stream_stats(model) -> {hits, misses, hit_rate, bytes_read}``.
"""
import json
from pathlib import Path

import torch

from . import laguna, pack


class ExpertStore:
    """All experts of one MoE layer, read from the pack once and kept in HBM."""

    def __init__(self, pack_dir, layout, layer, slots, group_size, bits, hidden, inter,
                 device="cuda"):
        self.layout, self.layer = layout, layer
        E = layout["num_experts"]
        self.requested_slots = slots
        self.slots = E
        arrays = pack.read_layer(pack_dir, layout, layer)
        dev = torch.device(device)

        def mat(proj):
            q = arrays[f"{proj}.weight"].to(dev)
            s = arrays[f"{proj}.scales"].to(dev).to(torch.bfloat16)
            b = arrays[f"{proj}.biases"].to(dev).to(torch.bfloat16)
            return laguna.SwitchLinear(q, s, b, group_size, bits)

        self.glu = laguna.SwitchGLU(hidden, inter, E, mat("gate_proj"), mat("up_proj"),
                                    mat("down_proj"))
        self.bytes_loaded = E * layout["stride"]
        self.hits = self.misses = self.bytes_read = 0

    def load(self, experts):
        """Every expert is resident: {expert: expert}."""
        experts = [int(e) for e in experts]
        self.hits += len(experts)
        return {e: e for e in experts}

    def note_picks(self, n):
        self.hits += int(n)


class StreamingSwitchGLU:
    """SwitchGLU(x, indices) over an ExpertStore."""

    def __init__(self, store):
        self._store = [store]  # a list, as in the reference (kept out of parameter walks)

    @property
    def store(self):
        return self._store[0]

    def resident_glu(self):
        return self.store.glu

    def note_picks(self, n):
        self.store.note_picks(n)

    def __call__(self, x, indices):
        store = self.store
        experts = torch.unique(indices).tolist()
        store.load([e for e in experts if 0 <= e < store.slots])
        return store.glu(x, indices)

    @property
    def gate_proj(self):
        return self.store.glu.gate_proj

    @property
    def up_proj(self):
        return self.store.glu.up_proj

    @property
    def down_proj(self):
        return self.store.glu.down_proj


def _load_safetensors(path):
    from safetensors.torch import load_file
    return load_file(str(path))


def load_streaming(pack_dir, slots, cache_limit_gb=None, device="cuda"):
    """Model + tokenizer from an expert pack (resident.safetensors, experts/, layout.json,
    config.json). ``cache_limit_gb`` caps MLX's buffer pool in the reference; torch's caching
    allocator has no such pool limit on this path, so it is accepted and ignored."""
    pack_dir = Path(pack_dir)
    config = json.loads((pack_dir / "config.json").read_text())
    layout = json.loads((pack_dir / "layout.json").read_text())
    q = config["quantization"]
    args = laguna.ModelArgs.from_dict(config)
    stores = {
        l: StreamingSwitchGLU(ExpertStore(pack_dir, layout, l, slots, q["group_size"], q["bits"],
                                          args.hidden_size, args.moe_intermediate_size, device))
        for l in layout["layers"]
    }
    weights = _load_safetensors(pack_dir / "resident.safetensors")
    model = laguna.model_from_weights(args, weights, q, device, switch_mlps=stores)
    tok = None
    if (pack_dir / "tokenizer.json").exists():
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(str(pack_dir))
    return model, tok


def stream_stats(model):
    stores = [l.mlp.switch_mlp.store for l in model.layers
              if isinstance(getattr(l.mlp, "switch_mlp", None), StreamingSwitchGLU)]
    hits = sum(s.hits for s in stores)
    misses = sum(s.misses for s in stores)
    return {"hits": hits, "misses": misses, "hit_rate": hits / max(1, hits + misses),
            "bytes_read": sum(s.bytes_read for s in stores)}
