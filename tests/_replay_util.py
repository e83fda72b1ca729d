"""Helpers for the replay tests: a character-level stand-in tokenizer with an assistant mask
(the real Laguna tokenizer is not available offline) and a synthetic proxy capture."""
import json

import numpy as np


class CharTokenizer:
    """Chat template stand-in: per message a role id, then one id per character (offset so
    ids stay in [4, vocab)); the assistant mask covers the assistant messages' characters.
    ``decode`` maps ids back to characters."""

    ROLE = {"system": 1, "user": 2, "assistant": 3, "tool": 2}
    eos_token_id = 0

    def __init__(self, vocab=512):
        self.vocab = vocab

    def _id(self, ch):
        return 4 + (ord(ch) % (self.vocab - 4))

    def apply_chat_template(self, messages, tools=None, tokenize=True, return_dict=True,
                            return_assistant_tokens_mask=True, enable_thinking=True):
        ids, mask = [], []
        text = lambda m: m["content"] + "".join(json.dumps(c["function"]["arguments"])
                                                for c in m.get("tool_calls") or [])
        for m in messages:
            ids.append(self.ROLE[m["role"]])
            mask.append(False)
            body = [self._id(c) for c in text(m)]
            ids += body
            mask += [m["role"] == "assistant"] * len(body)
        return {"input_ids": ids, "assistant_masks": mask}

    def decode(self, ids):
        return "".join(chr(i) for i in ids)


class TokenizerWrapper:
    """Shape of mlx-lm's wrapper: the real tokenizer sits behind ``_tokenizer`` and the
    wrapper itself cannot return the assistant mask."""

    def __init__(self, tok):
        self._tokenizer = tok

    def apply_chat_template(self, *a, **k):
        raise TypeError("return_dict is forced off by the wrapper")


MESSAGES = [
    {"role": "system", "content": "You are a coding agent."},
    {"role": "user", "content": [{"type": "text", "text": "List the files."}]},
    {"role": "assistant", "content": None, "tool_calls": [
        {"id": "c1", "type": "function",
         "function": {"name": "ls", "arguments": "{\"path\": \".\"}"}}]},
    {"role": "tool", "content": "a.py b.py"},
    {"role": "assistant", "content": "Two files: a.py and b.py."},
]


def write_capture(path, messages=MESSAGES):
    """A proxy capture: a non-chat request, an earlier chat request, then the last one."""
    rows = [
        {"path": "/v1/models", "request": None},
        {"path": "/v1/chat/completions", "request": {"messages": messages[:2]}},
        {"path": "/v1/chat/completions", "request": {"messages": messages, "tools": []}},
    ]
    path.write_text("\n".join(json.dumps(r) for r in rows) + "\n")
    return path


def target_positions(mask):
    t = np.zeros_like(mask)
    t[:-1] = mask[1:]
    return np.nonzero(t)[0]
