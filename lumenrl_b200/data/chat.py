"""Chat formatting and assistant-only loss masks for distillation / SFT data
(reference ``lumenrl/data/kimi_k25_parser.py:14-319``).

* ``normalize_conversation`` maps ShareGPT ``from/value`` turns to
  ``role/content`` and keeps a reasoning field as ``reasoning_content``.
* ``KimiK25Format`` renders a conversation with the Kimi-K2.5 special-token
  strings (these strings are the model's format, so they are fixed), drops
  ``<think>`` blocks from every assistant turn but the last, prepends an empty
  ``<think></think>`` where an assistant turn has none, and renders tool calls
  and tool results.
* ``assistant_loss_mask`` marks the tokens of every assistant turn's content
  (or only the last turn's).  With a fast tokenizer it tokenises the text ONCE
  and uses the character offsets of each token; otherwise it falls back to
  encoding text prefixes (one encode per turn boundary).
* ``pack_loss_mask``/``unpack_loss_mask`` run-length encode a 0/1 mask as
  alternating ``[zeros, ones, zeros, ...]`` run lengths (always starting with
  a zero run), serialised as a comma-separated string.
"""

from __future__ import annotations

import json
import re
from typing import Any, Sequence, Union

import torch
from torch import Tensor

ROLE_MAPPING = {"human": "user", "gpt": "assistant", "system": "system"}
_REASONING_FIELDS = ("thinking", "thinking_content", "reasoning_content", "reasoning")
_REAL_THINK = re.compile(r"<think>(?!\s*</think>)")
_THINK_BLOCK = re.compile(r"<think>[\s\S]*?</think>")


def has_thinking_content(conversation: Sequence[dict]) -> bool:
    """True if an assistant turn carries non-empty reasoning (an open
    ``<think>`` not immediately closed, or a reasoning field).  Call it before
    formatting: formatting injects empty ``<think></think>`` tags."""
    for m in conversation:
        if not isinstance(m, dict) or m.get("role") != "assistant":
            continue
        c = m.get("content", "")
        if isinstance(c, str) and _REAL_THINK.search(c):
            return True
        if any(m.get(f) for f in _REASONING_FIELDS):
            return True
    return False


def normalize_conversation(conversation: list[dict]) -> list[dict]:
    if not conversation:
        return conversation
    head = conversation[0]
    if "role" in head and "content" in head:
        return conversation
    if not ("from" in head and "value" in head):
        return conversation
    out = []
    for m in conversation:
        e = {"role": ROLE_MAPPING.get(m["from"], m["from"]), "content": m["value"]}
        for f in _REASONING_FIELDS:
            if m.get(f):
                e["reasoning_content"] = m[f]
                break
        out.append(e)
    return out


class KimiK25Format:
    MEDIA = "<|media_begin|>image<|media_content|><|media_pad|><|media_end|>"
    USER = "<|im_user|>user<|im_middle|>"
    ASSISTANT = "<|im_assistant|>assistant<|im_middle|>"
    SYSTEM = "<|im_system|>system<|im_middle|>"
    TOOL = "<|im_system|>tool<|im_middle|>"
    END = "<|im_end|>"
    IMAGE = "<|image|>"
    TC_SECTION = ("<|tool_calls_section_begin|>", "<|tool_calls_section_end|>")
    TC_CALL = ("<|tool_call_begin|>", "<|tool_call_argument_begin|>", "<|tool_call_end|>")

    def _flatten(self, items: list) -> str:
        parts = []
        for it in items:
            kind = it.get("type")
            if kind == "text":
                parts.append(it.get("text", ""))
            elif kind in ("image", "image_url"):
                parts.append(self.MEDIA + "\n")
        return "".join(parts)

    def _content(self, content: Any, role: str) -> str:
        if isinstance(content, list):
            return self._flatten(content)
        if not isinstance(content, str):
            return str(content)
        if content.startswith("["):
            try:
                parsed = json.loads(content)
            except (ValueError, TypeError):
                parsed = None
            if isinstance(parsed, list) and parsed and isinstance(parsed[0], dict) and "type" in parsed[0]:
                return self._flatten(parsed)
        return content.replace(self.IMAGE, self.MEDIA + "\n") if role == "user" else content

    def _tool_calls(self, calls: list) -> str:
        b, a, e = self.TC_CALL
        body = "".join(f"{b}{c.get('id', '')}{a}{c.get('function', {}).get('arguments', '')}{e}" for c in calls)
        return self.TC_SECTION[0] + body + self.TC_SECTION[1]

    def render(self, conversation: Sequence[dict], add_generation_prompt: bool = False) -> tuple[str, list]:
        """Returns (text, character spans of each assistant turn's content)."""
        last_asst = max((i for i, m in enumerate(conversation) if m["role"] == "assistant"), default=-1)
        text, spans = [], []
        pos = 0

        def emit(s: str) -> None:
            nonlocal pos
            text.append(s)
            pos += len(s)

        for i, m in enumerate(conversation):
            role = m["role"]
            c = self._content(m.get("content", ""), role)
            if role == "assistant":
                if i != last_asst:
                    c = _THINK_BLOCK.sub("", c)
                if m.get("tool_calls"):
                    c += self._tool_calls(m["tool_calls"])
                if not c.startswith("<think>"):
                    c = "<think></think>" + c
                emit(self.ASSISTANT)
                spans.append((pos, pos + len(c)))
                emit(c)
                emit(self.END)
            elif role == "system":
                emit(self.SYSTEM + c + self.END)
            elif role == "user":
                emit(self.USER + c + self.END)
            elif role == "tool":
                tid = m.get("tool_call_id", "")
                emit(self.TOOL + (f"## Return of {tid}\n{c}" if tid else c) + self.END)
        if add_generation_prompt:
            emit(self.ASSISTANT)
        return "".join(text), spans

    def format(self, conversation: Sequence[dict], add_generation_prompt: bool = False) -> str:
        return self.render(conversation, add_generation_prompt)[0]


def assistant_loss_mask(tokenizer, text: str, spans: list, max_length: int,
                        last_turn_only: bool = False) -> tuple[Tensor, Tensor]:
    """Token ids of ``text`` (truncated to ``max_length``) and a 0/1 mask over
    the tokens that start inside one of the assistant content ``spans``."""
    if last_turn_only and spans:
        spans = spans[-1:]
    try:
        enc = tokenizer(text, add_special_tokens=False, return_offsets_mapping=True, truncation=True,
                        max_length=max_length)
        ids = list(enc["input_ids"])
        offs = list(enc["offset_mapping"])
    except (NotImplementedError, TypeError, ValueError, KeyError):
        offs = None
        ids = tokenizer.encode(text, add_special_tokens=False)[:max_length]
    mask = torch.zeros(len(ids), dtype=torch.long)
    if offs is not None:
        starts = torch.tensor([o[0] for o in offs], dtype=torch.long)
        ends = torch.tensor([o[1] for o in offs], dtype=torch.long)
        for a, b in spans:
            mask |= ((starts >= a) & (starts < b) & (ends > starts)).long()
    else:
        for a, b in spans:
            lo = len(tokenizer.encode(text[:a], add_special_tokens=False))
            hi = len(tokenizer.encode(text[:b], add_special_tokens=False))
            lo, hi = min(lo, len(ids)), min(hi, len(ids))
            if lo < hi:
                mask[lo:hi] = 1
    return torch.tensor(ids, dtype=torch.long), mask


class KimiK25Parser:
    """Format + tokenise + mask (the reference's ``KimiK25Parser.parse``)."""

    def __init__(self, tokenizer) -> None:
        self.tokenizer = tokenizer
        self.fmt = KimiK25Format()

    def format(self, conversation, add_generation_prompt: bool = False) -> str:
        return self.fmt.format(conversation, add_generation_prompt)

    def parse(self, conversation, max_length: int, last_turn_only: bool = False) -> tuple[Tensor, Tensor]:
        text, spans = self.fmt.render(conversation)
        return assistant_loss_mask(self.tokenizer, text, spans, max_length, last_turn_only)


def pack_loss_mask(mask: Tensor) -> list[int]:
    m = mask.reshape(-1).to(torch.long)
    if m.numel() == 0:
        return []
    change = torch.nonzero(m[1:] != m[:-1]).reshape(-1) + 1
    bounds = torch.cat([torch.tensor([0]), change, torch.tensor([m.numel()])])
    runs = (bounds[1:] - bounds[:-1]).tolist()
    return ([0] + runs) if int(m[0]) == 1 else runs


def unpack_loss_mask(packed: Union[list[int], str]) -> Tensor:
    if isinstance(packed, str):
        packed = deserialize_packed_loss_mask(packed)
    if not packed:
        return torch.zeros(0, dtype=torch.long)
    vals = torch.arange(len(packed)) % 2
    return torch.repeat_interleave(vals, torch.tensor(packed, dtype=torch.long))


def serialize_packed_loss_mask(packed: list[int]) -> str:
    return ",".join(map(str, packed))


def deserialize_packed_loss_mask(s: str) -> list[int]:
    return [int(x) for x in s.split(",")] if s else []
