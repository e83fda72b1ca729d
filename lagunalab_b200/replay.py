"""Teacher-forced replay scoring on the B200 engine: compare a model with a stored reference
on captured sessions.

Follows lagunaLab ``replay/replay.py:1-168``. A reference ``.npz`` holds the session's token
ids, its assistant mask, and for every position whose next token is the assistant's the
reference model's top-64 log-probabilities (KL is truncated to those 64 tokens). ``score``
runs the model being tested over the same ids and reports the truncated KL and the top-1
agreement; ``build_ref`` writes such a reference from a model. The file format and the
``forward=`` contract are kept, so references built by the MLX harness score here and the
other way round.

    python -m lagunalab_b200.replay build-ref --model PACK --traces traces --refs refs
    python -m lagunalab_b200.replay score --model PACK --refs refs --out results/x.json

Host orchestration in torch: the model's forward and head run the sm_100a kernels; the
log-softmax, top-64 and KL over the resulting logits are small torch reductions.
"""
import argparse
import json
import time
from pathlib import Path

import numpy as np
import torch

from .session import load_session, tokenize

TOPK = 64
SUB = 256  # positions per log-softmax batch: 256 x 100k vocab x 4 B = 100 MB


def _device(model):
    if model is None:
        return torch.device("cpu")
    return model.model.embed_tokens.weight.device


def assistant_logprobs(model, ids, mask, chunk=2048, make_cache=None, forward=None):
    """Yield (positions int64 [n], log-probs fp32 [n, V]) for the positions whose next token
    is the assistant's (replay.py:23-50), prefilling ``ids`` in ``chunk``-token pieces
    through one cache.

    ``forward(ids [1, L], cache) -> logits [1, L, V]`` scores an engine that is not a model
    of this package; pass ``make_cache`` with it (``model`` may then be None, and ids are
    handed over as a CPU int32 tensor). It materialises a whole chunk's logits, where the
    default runs the head only on the assistant positions."""
    ids = np.asarray(ids)
    mask = np.asarray(mask, dtype=bool)
    target = np.zeros_like(mask)
    target[:-1] = mask[1:]
    cache = (make_cache or model.make_cache)()
    dev = _device(model) if forward is None else torch.device("cpu")
    for a in range(0, len(ids), chunk):
        b = min(a + chunk, len(ids))
        x = torch.from_numpy(np.ascontiguousarray(ids[None, a:b], dtype=np.int32)).to(dev)
        h = model.model(x, cache=cache)[0] if forward is None else forward(x, cache)[0]
        sel = np.nonzero(target[a:b])[0]
        for s in range(0, len(sel), SUB):
            part = sel[s:s + SUB]
            rows = h[torch.from_numpy(part).to(h.device)]
            lp = (model.lm_head(rows) if forward is None else rows).float()
            lp = lp - torch.logsumexp(lp, dim=-1, keepdim=True)
            yield part + a, lp


def _action(text):
    """The tool call if the reply has one, else the whole reply: what an agent would run."""
    i, j = text.find("<tool_call>"), text.find("</tool_call>")
    return text[i:j + len("</tool_call>")] if 0 <= i < j else text.strip()


def _eos_ids(tokenizer):
    ids = getattr(tokenizer, "eos_token_ids", None)
    if ids is None:
        e = getattr(tokenizer, "eos_token_id", None)
        ids = [] if e is None else ([e] if isinstance(e, int) else list(e))
    return {int(i) for i in ids}


def _greedy_text(model, tokenizer, prompt, max_new):
    """Greedy continuation of ``prompt`` (ids) up to ``max_new`` tokens or an end-of-sequence
    token (not included), detokenized; mlx-lm's ``generate`` as the reference calls it."""
    stop = _eos_ids(tokenizer)
    cache = model.make_cache()
    dev = _device(model)
    x = torch.as_tensor(np.asarray(prompt, dtype=np.int32), device=dev).reshape(1, -1)
    out = []
    for _ in range(max_new):
        logits = model.last_logits(x, cache)
        t = int(torch.argmax(logits.reshape(-1).float()))
        if t in stop:
            break
        out.append(t)
        x = torch.tensor([[t]], dtype=torch.int32, device=dev)
    return tokenizer.decode(out)


def greedy_actions(model, tokenizer, ids, starts, max_new):
    """Greedy action (tool call, else whole reply) at each assistant-turn start in ``starts``
    (replay.py:53-62); each re-prefills its whole prefix."""
    return [_action(_greedy_text(model, tokenizer, np.asarray(ids)[:s], max_new))
            for s in starts]


_greedy_actions = greedy_actions  # the reference's older name


def build_ref(model, tokenizer, session_path, out_path, max_tokens=65536, n_actions=2,
              max_new=1024, chunk=2048, seed=0, model_id=None):
    """Write the reference ``.npz`` of one captured session (replay.py:68-90): ids, mask,
    the top-64 log-probs (descending) of every assistant position, and the greedy actions
    at ``n_actions`` seeded assistant-turn starts. ``model_id`` is stored as ``model``."""
    msgs, tools = load_session(session_path)
    ids, mask, truncated = tokenize(tokenizer, msgs, tools, max_tokens)
    pos, top_ids, top_lp = [], [], []
    for p, lp in assistant_logprobs(model, ids, mask, chunk):
        vals, idx = torch.topk(lp, TOPK, dim=-1, largest=True, sorted=True)
        pos.append(p)
        top_ids.append(idx.to(torch.int32).cpu().numpy())
        top_lp.append(vals.cpu().numpy())
    if not pos:
        raise ValueError(f"{session_path}: no assistant tokens")
    starts = np.nonzero(mask & ~np.r_[False, mask[:-1]])[0]
    rng = np.random.default_rng(seed)
    starts = np.sort(rng.choice(starts, min(n_actions, len(starts)), replace=False))
    actions = greedy_actions(model, tokenizer, ids, starts, max_new)
    np.savez_compressed(out_path, ids=ids, mask=mask, truncated=truncated,
                        pos=np.concatenate(pos), top_ids=np.concatenate(top_ids),
                        top_lp=np.concatenate(top_lp), action_starts=starts,
                        actions=json.dumps(actions), max_new=max_new, model=model_id or "")


def score(model, ref_path, chunk=2048, make_cache=None, forward=None):
    """Truncated KL (reference top-64) and top-1 agreement of ``model`` (or ``forward``)
    against a reference ``.npz`` (replay.py:93-114). ``peak_mem_gb`` is torch's peak
    allocation on the current CUDA device (0 without one)."""
    ref = np.load(ref_path)
    ids, mask = ref["ids"], ref["mask"]
    kls, agree, i = [], [], 0
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.reset_peak_memory_stats()
    t0 = time.perf_counter()
    for p, lp in assistant_logprobs(model, ids, mask, chunk, make_cache, forward):
        n = len(p)
        if not (p == ref["pos"][i:i + n]).all():
            raise AssertionError("position mismatch vs reference")
        tid = torch.from_numpy(ref["top_ids"][i:i + n].astype(np.int64)).to(lp.device)
        rlp = torch.from_numpy(ref["top_lp"][i:i + n].astype(np.float32)).to(lp.device)
        i += n
        mlp_ = torch.gather(lp, -1, tid)
        kls.append((torch.exp(rlp) * (rlp - mlp_)).sum(dim=-1).cpu().numpy())
        agree.append((torch.argmax(lp, dim=-1) == tid[:, 0]).cpu().numpy())
    dt = time.perf_counter() - t0
    kl, ag = np.concatenate(kls), np.concatenate(agree)
    return {"tokens": int(len(ids)), "assistant_tokens": int(len(kl)),
            "truncated": bool(ref["truncated"]), "kl_top64_mean": float(kl.mean()),
            "kl_top64_p99": float(np.percentile(kl, 99)), "top1_agree": float(ag.mean()),
            "peak_mem_gb": (torch.cuda.max_memory_allocated() / 1e9) if cuda else 0.0,
            "tok_per_s": len(ids) / dt,
            "ref_model": (str(ref["model"]) or None) if "model" in ref.files else None}


def score_actions(model, tokenizer, ref_path, max_new=None):
    """Fraction of the reference's greedy actions the model reproduces exactly (replay.py:
    117-124); NaN when the reference stored none."""
    ref = np.load(ref_path)
    want = json.loads(str(ref["actions"]))
    if not want:
        return float("nan")
    got = greedy_actions(model, tokenizer, ref["ids"], ref["action_starts"],
                         max_new or int(ref["max_new"]))
    return float(np.mean([a == b for a, b in zip(got, want)]))


def main(argv=None):
    """CLI of replay.py:127-164; ``--model`` is an MLX-format checkpoint directory
    (``laguna.load``) or an expert pack directory (``load_streaming``, every expert
    resident)."""
    from .laguna import load
    from .streaming import load_streaming

    p = argparse.ArgumentParser()
    p.add_argument("cmd", choices=["build-ref", "score"])
    p.add_argument("--model", required=True)
    p.add_argument("--traces", default="traces")
    p.add_argument("--refs", default="refs")
    p.add_argument("--out")
    p.add_argument("--max-tokens", type=int, default=65536)
    p.add_argument("--actions", action="store_true")
    a = p.parse_args(argv)
    if (Path(a.model) / "layout.json").exists():
        model, tok = load_streaming(a.model, slots=0)
    else:
        model, tok = load(a.model)
    refs = Path(a.refs)
    if a.cmd == "build-ref":
        refs.mkdir(exist_ok=True)
        for f in sorted(Path(a.traces).glob("*.jsonl")):
            out = refs / f"{f.stem}.npz"
            if not out.exists():
                build_ref(model, tok, f, out, a.max_tokens, model_id=a.model)
                print("ref", f.stem, flush=True)
        return
    rows = []
    for r in sorted(refs.glob("*.npz")):
        row = {"session": r.stem, **score(model, r)}
        if a.actions:
            row["action_match"] = score_actions(model, tok, r)
        rows.append(row)
        print(row, flush=True)
    w = np.array([x["assistant_tokens"] for x in rows])
    summary = {k: float(np.average([x[k] for x in rows], weights=w))
               for k in ("kl_top64_mean", "top1_agree")}
    summary["peak_mem_gb"] = max(x["peak_mem_gb"] for x in rows)
    if a.actions:
        summary["action_match"] = float(np.nanmean([x["action_match"] for x in rows]))
    Path(a.out).write_text(json.dumps({"summary": summary, "sessions": rows}, indent=1))
    print(summary)


if __name__ == "__main__":
    main()
