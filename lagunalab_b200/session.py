"""Captured chat sessions (proxy JSONL) -> chat-template token ids + assistant mask.

Follows lagunaLab ``replay/session.py:1-62``: the last ``/chat/completions`` request of a
capture holds the whole conversation so far; its messages are normalised from the OpenAI
wire format to what the Laguna chat template expects, then tokenized with the assistant
mask the template marks. Host-side text handling only; nothing here touches the GPU.
"""
import json
from pathlib import Path

import numpy as np


def normalize(m):
    """One OpenAI-format message -> the chat template's form (session.py:8-31): list content
    is joined from its text parts, ``None`` content becomes "", and each tool call's JSON
    ``arguments`` string is parsed to a dict (malformed JSON, or JSON that is not an object,
    is kept as ``{"_raw": <the original text>}``)."""
    m = dict(m)
    c = m.get("content")
    if isinstance(c, list):
        m["content"] = "".join(p.get("text", "") for p in c if isinstance(p, dict))
    elif c is None:
        m["content"] = ""
    if m.get("tool_calls"):
        calls = []
        for tc in m["tool_calls"]:
            fn = tc["function"]
            args = fn.get("arguments", {})
            if isinstance(args, str):
                try:
                    parsed = json.loads(args)
                except ValueError:
                    parsed = None
                args = parsed if isinstance(parsed, dict) else {"_raw": args}
            calls.append({**tc, "function": {**fn, "arguments": args}})
        m["tool_calls"] = calls
    return m


def load_session(path):
    """(messages, tools) of the capture's last chat request (session.py:34-41); ValueError
    when the file holds none."""
    reqs = []
    for line in Path(path).read_text().splitlines():
        if not line.strip():
            continue
        r = json.loads(line)
        if r["path"].endswith("/chat/completions") and isinstance(r["request"], dict):
            reqs.append(r)
    if not reqs:
        raise ValueError(f"{path}: no chat requests")
    last = reqs[-1]["request"]
    return [normalize(m) for m in last["messages"]], last.get("tools")


def tokenize(tokenizer, messages, tools, max_tokens=None):
    """(ids int32 [L], assistant mask bool [L], truncated) (session.py:44-62), thinking
    enabled. A wrapper object that hides its Hugging Face tokenizer behind ``_tokenizer``
    and forces ``return_dict=False`` (mlx-lm's ``TokenizerWrapper``) is unwrapped first; a
    plain fast tokenizer keeps its own ``_tokenizer`` (the Rust backend) and is left alone."""
    if type(tokenizer).__name__ == "TokenizerWrapper":
        tokenizer = tokenizer._tokenizer
    enc = tokenizer.apply_chat_template(
        messages, tools=tools, tokenize=True, return_dict=True,
        return_assistant_tokens_mask=True, enable_thinking=True,
    )
    ids = np.asarray(enc["input_ids"], dtype=np.int32)
    mask = np.asarray(enc["assistant_masks"], dtype=bool)
    truncated = max_tokens is not None and len(ids) > max_tokens
    if truncated:
        ids, mask = ids[:max_tokens], mask[:max_tokens]
    return ids, mask, truncated
