"""The full-decoder oracle (oracle/model_ref.py) pinned to Poolside's PyTorch model.

tests/golden/model_tiny.npz holds LagunaForCausalLM (tests/reference/modeling_laguna.py in
lagunaLab, the model its MLX port is tested against in tests/test_laguna.py:12-19) with
random fp32 weights and its logits for 12 tokens; the oracle's unrounded form must
reproduce them. The MLX-rounded form on quantized weights must then stay close to the
unrounded form on the same (dequantized) weights, and greedy decoding must agree with a
full-sequence forward (the KV cache path equals the no-cache path).
"""
from pathlib import Path

import numpy as np
import torch

from oracle import model_ref, moe_ref
from tests._util import cos, quant_np, rel_err

GOLDEN = Path(__file__).resolve().parent / "golden" / "model_tiny.npz"


def _golden():
    d = np.load(GOLDEN)
    t = lambda k: torch.from_numpy(d["w." + k]).float()
    W = {"embed": t("model.embed_tokens.weight"), "norm": t("model.norm.weight"),
         "lm_head": t("lm_head.weight"), "layers": []}
    for i in range(3):
        p = f"model.layers.{i}."
        L = {"in_norm": t(p + "input_layernorm.weight"),
             "post_norm": t(p + "post_attention_layernorm.weight"),
             "q_norm": t(p + "self_attn.q_norm.weight"), "k_norm": t(p + "self_attn.k_norm.weight")}
        for n in "qkvog":
            L[n] = t(p + f"self_attn.{n}_proj.weight")
        if "w." + p + "mlp.gate_proj.weight" in d:
            L["mlp"] = ("dense", tuple(t(p + f"mlp.{n}_proj.weight") for n in ("gate", "up", "down")))
        else:
            gu = t(p + "mlp.experts.gate_up_proj")
            I = gu.shape[1] // 2
            L["mlp"] = ("moe", {
                "gate": t(p + "mlp.gate.weight"), "bias": t(p + "mlp.gate.e_score_correction_bias"),
                "experts": (gu[:, :I], gu[:, I:], t(p + "mlp.experts.down_proj")),
                "shared": tuple(t(p + f"mlp.shared_expert.{n}_proj.weight")
                                for n in ("gate", "up", "down"))})
        W["layers"].append(L)
    args = dict(head_dim=32, heads=[4, 4, 4], kv_heads=2, eps=1e-6, rope_theta=1e4,
                gating="per-head", k=2, routed_scale=2.5, norm_topk_prob=True)
    return W, args, torch.from_numpy(d["ids"]), torch.from_numpy(d["ref_logits"])


def test_fp32_form_matches_the_pytorch_model():
    W, args, ids, ref = _golden()
    got = model_ref.forward_fp32(W, args, ids)
    assert got.shape == ref.shape
    assert (got - ref).abs().max() <= 1e-4 * ref.abs().max() + 1e-5


GOLDEN_SWA = Path(__file__).resolve().parent / "golden" / "model_swa.npz"
SWA_YARN = {"rope_theta": 500000.0, "rope_type": "yarn", "factor": 32.0,
            "original_max_position_embeddings": 8192, "beta_slow": 1.0, "beta_fast": 64.0,
            "attention_factor": 1.3465735902799727, "partial_rotary_factor": 0.5}
SWA_DEFAULT = {"rope_type": "default", "rope_theta": 10000.0, "partial_rotary_factor": 1.0}


def _golden_swa():
    d = np.load(GOLDEN_SWA)
    t = lambda k: torch.from_numpy(d["w." + k]).float()
    heads = [4, 4, 8, 4]
    W = {"embed": t("model.embed_tokens.weight"), "norm": t("model.norm.weight"),
         "lm_head": t("lm_head.weight"), "layers": []}
    for i in range(4):
        p = f"model.layers.{i}."
        L = {"in_norm": t(p + "input_layernorm.weight"),
             "post_norm": t(p + "post_attention_layernorm.weight"),
             "q_norm": t(p + "self_attn.q_norm.weight"), "k_norm": t(p + "self_attn.k_norm.weight")}
        for n in "qkvog":
            L[n] = t(p + f"self_attn.{n}_proj.weight")
        if "w." + p + "mlp.gate_proj.weight" in d:
            L["mlp"] = ("dense", tuple(t(p + f"mlp.{n}_proj.weight") for n in ("gate", "up", "down")))
        else:
            gu = t(p + "mlp.experts.gate_up_proj")
            I = gu.shape[1] // 2
            L["mlp"] = ("moe", {
                "gate": t(p + "mlp.gate.weight"), "bias": t(p + "mlp.gate.e_score_correction_bias"),
                "experts": (gu[:, :I], gu[:, I:], t(p + "mlp.experts.down_proj")),
                "shared": tuple(t(p + f"mlp.shared_expert.{n}_proj.weight")
                                for n in ("gate", "up", "down"))})
        W["layers"].append(L)
    full = model_ref.rope_params(SWA_YARN, 32)
    swa = model_ref.rope_params(SWA_DEFAULT, 32)
    args = dict(head_dim=32, heads=heads, kv_heads=2, eps=1e-6, rope_theta=1e4,
                gating="per-head", k=2, routed_scale=2.5, norm_topk_prob=True,
                rope=[full, swa, swa, full], window=[None, 5, 5, None])
    return W, args, torch.from_numpy(d["ids"]), int(d["pos0"]), torch.from_numpy(d["ref_logits"])


def test_sliding_window_and_yarn_partial_rotary_match_the_pytorch_model():
    """The real checkpoint's layer mix (laguna.py:62-72, :183-186, :209-214): sliding-window
    layers with default RoPE and full layers with YaRN on half the head dims, at positions
    3000.. (past the window, inside YaRN's frequency ramp)."""
    W, args, ids, pos0, ref = _golden_swa()
    got = model_ref.forward_fp32(W, args, ids, pos0)
    assert (got - ref).abs().max() <= 1e-4 * ref.abs().max() + 1e-5
    R, inv, ms = args["rope"][0]
    assert R == 16 and inv.shape == (8,) and abs(ms - 1.3465735902799727) < 1e-12


def _tiny_quantized(seed=0, V=160, H=128, D=64, Hq=4, Hkv=2, E=8, k=2, I=64, I_sh=64, I_d=128):
    """A 3-layer model with every inner dimension a multiple of 64 (quantizable at g64):
    fp32 weights, and the same weights in MLX 4-bit layout (router 8-bit)."""
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g) * 0.08
    nw = lambda n: 1.0 + 0.1 * torch.randn(n, generator=g)
    Wf = {"embed": r(V, H), "norm": nw(H), "lm_head": r(V, H), "layers": []}
    for i in range(3):
        L = {"in_norm": nw(H), "post_norm": nw(H), "q_norm": nw(D), "k_norm": nw(D),
             "q": r(Hq * D, H), "k": r(Hkv * D, H), "v": r(Hkv * D, H), "o": r(H, Hq * D),
             "g": r(Hq, H)}
        if i == 0:
            L["mlp"] = ("dense", (r(I_d, H), r(I_d, H), r(H, I_d)))
        else:
            L["mlp"] = ("moe", {"gate": r(E, H), "bias": 0.3 * torch.randn(E, generator=g),
                                "experts": (r(E, I, H), r(E, I, H), r(E, H, I)),
                                "shared": (r(I_sh, H), r(I_sh, H), r(H, I_sh))})
        Wf["layers"].append(L)
    # round weight values to what the quantized form holds, so both forms use the same weights
    q4 = lambda w: quant_np(w, 4)
    deq = lambda m, bits=4: moe_ref.dequantize(*m, 64, bits)
    Wq = {"embed": q4(Wf["embed"]), "norm": Wf["norm"].to(torch.bfloat16).float(),
          "lm_head": q4(Wf["lm_head"]), "layers": []}
    Wd = {"embed": deq(Wq["embed"]), "norm": Wq["norm"], "lm_head": deq(Wq["lm_head"]), "layers": []}
    for L in Wf["layers"]:
        Lq = {n: L[n].to(torch.bfloat16).float() for n in ("in_norm", "post_norm", "q_norm", "k_norm")}
        Ld = dict(Lq)
        for n in "qkvog":
            Lq[n] = q4(L[n])
            Ld[n] = deq(Lq[n])
        kind, m = L["mlp"]
        if kind == "dense":
            mq = tuple(q4(w) for w in m)
            Lq["mlp"], Ld["mlp"] = ("dense", mq), ("dense", tuple(deq(w) for w in mq))
        else:
            gq = quant_np(m["gate"], 8)
            eq = tuple(q4(w) for w in m["experts"])
            sq = tuple(q4(w) for w in m["shared"])
            Lq["mlp"] = ("moe", {"gate": gq, "bias": m["bias"], "experts": eq, "shared": sq})
            Ld["mlp"] = ("moe", {"gate": deq(gq, 8), "bias": m["bias"],
                                 "experts": tuple(deq(w) for w in eq),
                                 "shared": tuple(deq(w) for w in sq)})
        Wq["layers"].append(Lq)
        Wd["layers"].append(Ld)
    args = dict(head_dim=D, heads=[Hq] * 3, kv_heads=Hkv, eps=1e-6, rope_theta=1e4,
                gating="per-head", k=k, routed_scale=2.5, norm_topk_prob=True)
    return Wq, Wd, args


def test_rounded_quantized_form_tracks_the_fp32_form():
    Wq, Wd, args = _tiny_quantized()
    ids = torch.randint(0, 160, (10,), generator=torch.Generator().manual_seed(5))
    got = model_ref.forward(Wq, args, ids)
    want = model_ref.forward_fp32(Wd, args, ids)
    assert cos(got, want) >= 0.99 and rel_err(got, want) <= 0.1


def test_kv_cache_decode_equals_full_sequence_forward():
    Wq, _, args = _tiny_quantized(seed=1)
    prompt = torch.randint(0, 160, (6,), generator=torch.Generator().manual_seed(7))
    toks, gaps = model_ref.greedy(Wq, args, prompt, 4)
    seq = torch.cat([prompt, torch.tensor(toks[:-1])])
    full = model_ref.forward(Wq, args, seq)
    # the logits that chose each generated token, recomputed without a cache
    for i, t in enumerate(toks):
        row = full[len(prompt) - 1 + i]
        assert int(torch.argmax(row)) == t or gaps[i] < 0.05
