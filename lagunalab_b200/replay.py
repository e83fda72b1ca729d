"""Teacher-forced replay scoring on the B200 engine: compare a model with a stored reference
on captured sessions.

Contract of lagunaLab ``replay/replay.py:23-164`` (kept so references move between the two
harnesses): a reference ``.npz`` holds a session's token ids, its assistant mask and, for each
position whose next token is the assistant's, the reference model's 64 largest
log-probabilities with their token ids (KL is truncated to those 64); ``score`` reports the
truncated KL and the top-1 agreement of another model over the same ids; ``build_ref`` writes
a reference; an engine outside this package plugs in through ``forward(ids [1, L], cache) ->
logits [1, L, V]`` with ``make_cache``.

    python -m lagunalab_b200.replay build-ref --model PACK --traces traces --refs refs
    python -m lagunalab_b200.replay score --model PACK --refs refs --out results/x.json

Everything per position stays on the device: the session's assistant positions are one index
tensor, each prefill chunk's hidden rows at those positions go through the head in
sub-batches, and the log-softmax, the top-64 (``build_ref``) or the gathered KL and the
argmax agreement (``score``) are batched reductions written into preallocated per-session
tensors. The host sees one copy per session, not one per sub-batch.
"""
import argparse
import json
import time
from pathlib import Path

import numpy as np
import torch

from .session import load_session, tokenize

TOPK = 64
HEAD_ROWS = 256  # positions per head + log-softmax batch: 256 x 100k vocab x 4 B = 100 MB


def _device(model, forward):
    if forward is not None or model is None:
        return torch.device("cpu")
    return model.model.embed_tokens.weight.device


def _targets(mask):
    """Positions whose next token is the assistant's (the positions a reference scores)."""
    mask = np.asarray(mask, dtype=bool)
    return np.nonzero(np.r_[mask[1:], False])[0]


def _chunks(model, ids, mask, chunk, make_cache, forward):
    """Per prefill chunk: (index range into the session's target list, log-probs fp32
    [n, V] of those targets), on the engine's device, HEAD_ROWS rows at a time."""
    ids = np.asarray(ids)
    tgt = _targets(mask)
    dev = _device(model, forward)
    cache = (make_cache or model.make_cache)()
    lo = 0
    for a in range(0, len(ids), chunk):
        b = min(a + chunk, len(ids))
        hi = int(np.searchsorted(tgt, b))
        x = torch.from_numpy(np.ascontiguousarray(ids[None, a:b], dtype=np.int32)).to(dev)
        out = forward(x, cache)[0] if forward is not None else model.model(x, cache=cache)[0]
        if hi > lo:
            rows = torch.from_numpy(tgt[lo:hi] - a).to(out.device)
            for s in range(0, hi - lo, HEAD_ROWS):
                r = rows[s:s + HEAD_ROWS]
                z = out[r] if forward is not None else model.lm_head(out[r])
                yield lo + s, torch.log_softmax(z.float(), dim=-1)
        lo = hi


def assistant_logprobs(model, ids, mask, chunk=2048, make_cache=None, forward=None):
    """Yield (positions int64 [n], log-probs fp32 [n, V]) for the positions whose next token
    is the assistant's, in order, prefilling ``ids`` in ``chunk``-token pieces through one
    cache (replay.py:23-50). With ``forward`` the ids go over as a CPU int32 tensor and
    ``model`` may be None; the default path runs the head only on those positions."""
    tgt = _targets(mask)
    for i, lp in _chunks(model, ids, mask, chunk, make_cache, forward):
        yield tgt[i:i + lp.shape[0]], lp


def _action(reply):
    """What an agent would execute from a reply: the span from the first opening tool-call tag
    through the first closing tag when the opening one comes first, otherwise the reply without
    surrounding whitespace (the rule the reference's stored actions were made with)."""
    open_tag, close_tag = "<tool_call>", "</tool_call>"
    a, b = reply.find(open_tag), reply.find(close_tag)
    return reply[a:b + len(close_tag)] if 0 <= a < b else reply.strip()


def _stop_ids(tokenizer):
    ids = getattr(tokenizer, "eos_token_ids", None)
    if ids is None:
        ids = getattr(tokenizer, "eos_token_id", None)
    if ids is None:
        return set()
    return {int(ids)} if isinstance(ids, int) else {int(i) for i in ids}


def _greedy_ids(model, prompt, max_new, stop):
    """Greedy continuation ids of ``prompt`` (mlx-lm ``generate`` at temperature 0), stopping
    at an end-of-sequence id (not returned) or after ``max_new`` ids. A model of this package
    on the GPU decodes one graph replay per token (``laguna.DecodeGraph``: token and position
    stay on the device); any other model steps ``last_logits`` eagerly."""
    from . import laguna
    dev = _device(model, None)
    x = torch.as_tensor(np.asarray(prompt, dtype=np.int32), device=dev).reshape(1, -1)
    out = []
    if max_new <= 0:
        return out
    if isinstance(model, laguna.Model) and dev.type == "cuda":
        from . import ops
        cap = (x.shape[1] + max_new + 2 + 255) // 256 * 256
        cache = model.make_cache(capacity=cap)
        tok = ops.argmax(model.last_logits(x, cache).reshape(1, -1))
        if int(tok) in stop:
            return out
        out.append(int(tok))
        if max_new == 1:
            return out
        dg = laguna.DecodeGraph(model, cache, tok)  # its first (eager) step already ran
        while int(dg.tok) not in stop:
            out.append(int(dg.tok))
            if len(out) >= max_new:
                break
            dg.step()
        return out
    cache = model.make_cache()
    while len(out) < max_new:
        t = int(torch.argmax(model.last_logits(x, cache).reshape(-1).float()))
        if t in stop:
            break
        out.append(t)
        x = torch.tensor([[t]], dtype=torch.int32, device=dev)
    return out


def greedy_actions(model, tokenizer, ids, starts, max_new):
    """The greedy action (tool call, else the whole reply) after each assistant-turn start in
    ``starts``, each from a fresh prefill of its prefix (replay.py:53-62)."""
    stop = _stop_ids(tokenizer)
    ids = np.asarray(ids)
    return [_action(tokenizer.decode(_greedy_ids(model, ids[:s], max_new, stop)))
            for s in starts]


_greedy_actions = greedy_actions  # the name the reference's older scripts import


def build_ref(model, tokenizer, session_path, out_path, max_tokens=65536, n_actions=2,
              max_new=1024, chunk=2048, seed=0, model_id=None):
    """Write the reference ``.npz`` of one captured session (replay.py:68-90): ids, mask,
    the 64 largest log-probs (descending) with their ids at every assistant position, and
    the greedy actions at ``n_actions`` seeded assistant-turn starts; ``model_id`` is stored
    as ``model``."""
    msgs, tools = load_session(session_path)
    ids, mask, truncated = tokenize(tokenizer, msgs, tools, max_tokens)
    tgt = _targets(mask)
    if not len(tgt):
        raise ValueError(f"{session_path}: no assistant tokens")
    dev = _device(model, None)
    top_lp = torch.empty(len(tgt), TOPK, dtype=torch.float32, device=dev)
    top_ids = torch.empty(len(tgt), TOPK, dtype=torch.int32, device=dev)
    for i, lp in _chunks(model, ids, mask, chunk, None, None):
        v, j = torch.topk(lp, TOPK, dim=-1, largest=True, sorted=True)
        top_lp[i:i + len(v)] = v
        top_ids[i:i + len(v)] = j.to(torch.int32)
    first = np.nonzero(np.asarray(mask, bool) & ~np.r_[False, np.asarray(mask, bool)[:-1]])[0]
    rng = np.random.default_rng(seed)
    starts = np.sort(rng.choice(first, min(n_actions, len(first)), replace=False))
    actions = greedy_actions(model, tokenizer, ids, starts, max_new)
    np.savez_compressed(out_path, ids=ids, mask=mask, truncated=truncated, pos=tgt,
                        top_ids=top_ids.cpu().numpy(), top_lp=top_lp.cpu().numpy(),
                        action_starts=starts, actions=json.dumps(actions), max_new=max_new,
                        model=model_id or "")


def score(model, ref_path, chunk=2048, make_cache=None, forward=None):
    """Truncated KL (over the reference's top-64) and top-1 agreement of ``model`` (or
    ``forward``) against a reference ``.npz`` (replay.py:93-114); ``peak_mem_gb`` is torch's
    peak allocation on the current CUDA device (0 without one)."""
    ref = np.load(ref_path)
    ids, mask = ref["ids"], ref["mask"]
    tgt = _targets(mask)
    if len(tgt) != len(ref["pos"]) or not (tgt == ref["pos"]).all():
        raise AssertionError("position mismatch vs reference")
    dev = _device(model, forward)
    r_ids = torch.from_numpy(ref["top_ids"].astype(np.int64)).to(dev)
    r_lp = torch.from_numpy(ref["top_lp"].astype(np.float32)).to(dev)
    kl = torch.empty(len(tgt), dtype=torch.float32, device=dev)
    agree = torch.empty(len(tgt), dtype=torch.bool, device=dev)
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.reset_peak_memory_stats()
    t0 = time.perf_counter()
    for i, lp in _chunks(model, ids, mask, chunk, make_cache, forward):
        n = lp.shape[0]
        rid, rlp = r_ids[i:i + n].to(lp.device), r_lp[i:i + n].to(lp.device)
        kl[i:i + n] = (rlp.exp() * (rlp - lp.gather(-1, rid))).sum(-1).to(dev)
        agree[i:i + n] = (lp.argmax(-1) == rid[:, 0]).to(dev)
    kl_h = kl.cpu().numpy()
    dt = time.perf_counter() - t0
    return {"tokens": int(len(ids)), "assistant_tokens": int(len(kl_h)),
            "truncated": bool(ref["truncated"]), "kl_top64_mean": float(kl_h.mean()),
            "kl_top64_p99": float(np.percentile(kl_h, 99)),
            "top1_agree": float(agree.float().mean()),
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
    return sum(a == b for a, b in zip(got, want)) / len(want)


def main(argv=None):
    """Command line of replay.py:127-164. ``--model`` is an MLX-format checkpoint directory
    (``laguna.load``) or an expert pack directory (``load_streaming`` with every expert
    resident)."""
    from .laguna import load
    from .streaming import load_streaming

    ap = argparse.ArgumentParser()
    ap.add_argument("cmd", choices=["build-ref", "score"])
    ap.add_argument("--model", required=True)
    ap.add_argument("--traces", default="traces")
    ap.add_argument("--refs", default="refs")
    ap.add_argument("--out")
    ap.add_argument("--max-tokens", type=int, default=65536)
    ap.add_argument("--actions", action="store_true")
    a = ap.parse_args(argv)
    pack = (Path(a.model) / "layout.json").exists()
    model, tok = load_streaming(a.model, slots=0) if pack else load(a.model)
    refs = Path(a.refs)
    if a.cmd == "build-ref":
        refs.mkdir(exist_ok=True)
        for trace in sorted(Path(a.traces).glob("*.jsonl")):
            dst = refs / f"{trace.stem}.npz"
            if not dst.exists():
                build_ref(model, tok, trace, dst, a.max_tokens, model_id=a.model)
                print("ref", trace.stem, flush=True)
        return
    rows = []
    for r in sorted(refs.glob("*.npz")):
        row = {"session": r.stem, **score(model, r)}
        if a.actions:
            row["action_match"] = score_actions(model, tok, r)
        rows.append(row)
        print(row, flush=True)
    weights = [x["assistant_tokens"] for x in rows]
    summary = {key: float(np.average([x[key] for x in rows], weights=weights))
               for key in ("kl_top64_mean", "top1_agree")}
    summary["peak_mem_gb"] = max(x["peak_mem_gb"] for x in rows)
    if a.actions:
        summary["action_match"] = float(np.nanmean([x["action_match"] for x in rows]))
    Path(a.out).write_text(json.dumps({"summary": summary, "sessions": rows}, indent=1))
    print(summary)


if __name__ == "__main__":
    main()
