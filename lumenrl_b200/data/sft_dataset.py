"""Model-agnostic SFT dataset: the tokenizer's own chat template per turn,
loss on assistant tokens only (reference ``lumenrl/data/sft_dataset.py:18-244``).

Each turn is rendered on its own with ``apply_chat_template``.  The template's
system-prompt prefix (what a one-turn render has in front of the turn) is cut
from every turn after the first, and the assistant generation header is
excluded from the loss.  Both are found once by rendering probe
conversations and diffing them.  Output rows: ``input_ids``,
``attention_mask``, ``loss_mask``, ``position_ids`` (right-padded to
``max_length`` or unpadded, with right/left/error truncation).
"""

from __future__ import annotations

import json
import logging
from typing import Union

import torch

logger = logging.getLogger(__name__)


def as_id_list(out) -> list[int]:
    """Flatten whatever ``apply_chat_template(tokenize=True)`` returned
    (list, nested list, tensor, dict/BatchEncoding) to ``list[int]``."""
    if isinstance(out, dict) or hasattr(out, "input_ids"):
        out = out["input_ids"] if isinstance(out, dict) else out.input_ids
    if hasattr(out, "tolist"):
        out = out.tolist()
    out = list(out)
    if len(out) == 1 and isinstance(out[0], (list, tuple)):
        out = list(out[0])
    return [int(t) for t in out]


def template_prefixes(tokenizer, **kw) -> tuple[list[int], list[int]]:
    """(system-prompt prefix ids, assistant generation-prompt ids)."""
    one = as_id_list(tokenizer.apply_chat_template([{"role": "user", "content": ""}], tokenize=True, **kw))
    two = as_id_list(tokenizer.apply_chat_template([{"role": "user", "content": ""}] * 2, tokenize=True, **kw))
    per_turn = len(two) - len(one)
    system = one[: len(one) - per_turn]
    gen = as_id_list(tokenizer.apply_chat_template([{"role": "user", "content": ""}], tokenize=True,
                                                   add_generation_prompt=True, **kw))[len(one):]
    return system, gen


_ROLE = {"human": "user", "gpt": "assistant", "system": "system"}


class SFTDataset(torch.utils.data.Dataset):
    def __init__(self, data_files: Union[str, list[str]], tokenizer, max_length: int = 2048,
                 messages_key: str = "messages", pad_mode: str = "right", truncation: str = "right",
                 shuffle: bool = False, seed: int = 42, max_samples: int = -1) -> None:
        if isinstance(tokenizer, str):
            from transformers import AutoTokenizer
            tokenizer = AutoTokenizer.from_pretrained(tokenizer, trust_remote_code=True)
        if pad_mode not in ("right", "no_padding"):
            raise ValueError(f"unknown pad_mode {pad_mode!r}")
        if truncation not in ("right", "left", "error"):
            raise ValueError(f"unknown truncation {truncation!r}")
        self.tokenizer, self.max_length = tokenizer, max_length
        self.pad_mode, self.truncation = pad_mode, truncation
        self.system_prompt, self.gen_prompt = template_prefixes(tokenizer)
        self.messages_list = self._load([data_files] if isinstance(data_files, str) else data_files,
                                        messages_key, shuffle, seed, max_samples)

    @staticmethod
    def _load(files, key, shuffle, seed, max_samples) -> list:
        import numpy as np
        import pandas as pd
        frames = [pd.read_json(f, lines=f.endswith(".jsonl")) if f.endswith((".json", ".jsonl")) else pd.read_parquet(f)
                  for f in files]
        df = pd.concat(frames, ignore_index=True)
        n = len(df)
        if 0 < max_samples < n:
            idx = np.random.default_rng(seed).choice(n, max_samples, replace=False) if shuffle else np.arange(max_samples)
            df = df.iloc[list(idx)]
        elif shuffle:
            df = df.sample(frac=1, random_state=seed).reset_index(drop=True)
        return df[key].tolist()

    def __len__(self) -> int:
        return len(self.messages_list)

    def _turn(self, i: int, msg: dict) -> tuple[list[int], list[int]]:
        ids = as_id_list(self.tokenizer.apply_chat_template([msg], tokenize=True, add_generation_prompt=False))
        if i and msg.get("role") != "system":
            ids = ids[len(self.system_prompt):]
        if msg.get("role") == "assistant":
            head = min(len(self.gen_prompt), len(ids))
            mask = [0] * head + [1] * (len(ids) - head)
        else:
            mask = [0] * len(ids)
        return ids, mask

    def __getitem__(self, item: int) -> dict:
        msgs = self.messages_list[item]
        if isinstance(msgs, str):
            msgs = json.loads(msgs)
        if hasattr(msgs, "tolist"):
            msgs = msgs.tolist()
        msgs = [dict(m) for m in msgs]
        if msgs and "from" in msgs[0]:
            msgs = [{"role": _ROLE.get(m["from"], m["from"]), "content": m["value"]} for m in msgs]
        ids, mask = [], []
        for i, m in enumerate(msgs):
            a, b = self._turn(i, m)
            ids += a
            mask += b
        n, L = len(ids), self.max_length
        pos = list(range(n))
        if n > L:
            if self.truncation == "error":
                raise ValueError(f"sequence length {n} exceeds max_length {L}")
            # left truncation keeps the tail (padded mode only, as in the reference)
            sl = slice(n - L, n) if (self.truncation == "left" and self.pad_mode == "right") else slice(0, L)
            ids, mask, pos = ids[sl], mask[sl], pos[sl]
        attn = [1] * len(ids)
        if self.pad_mode == "right" and len(ids) < L:
            pad = L - len(ids)
            pid = self.tokenizer.pad_token_id or 0
            ids, attn, mask, pos = ids + [pid] * pad, attn + [0] * pad, mask + [0] * pad, pos + [0] * pad

        def t(v):
            return torch.tensor(v, dtype=torch.long)
        return {"input_ids": t(ids), "attention_mask": t(attn), "loss_mask": t(mask), "position_ids": t(pos)}
