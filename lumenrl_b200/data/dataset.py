"""Conversation dataset preprocessing with a worker pool and an on-disk cache
(reference ``lumenrl/data/dataset.py:28-169``).

``load_and_preprocess_dataset`` reads ShareGPT-style rows (a
``conversations`` list per row) from JSON/JSONL/Parquet, shuffles by seed,
tokenises each conversation with the Kimi-K2.5 format and an assistant-only
loss mask (optionally only the last assistant turn, or ``"auto"``: only when
the conversation has real reasoning), drops rows with fewer than
``min_loss_tokens`` supervised tokens, and caches the result keyed by the
file identity and every preprocessing knob.  Each sample is
``{"input_ids": list[int], "packed_loss_mask": "z,o,z,..."}``.
"""

from __future__ import annotations

import hashlib
import json
import logging
import multiprocessing as mp
import os
from typing import Any, Optional

import torch

from lumenrl_b200.data.chat import (KimiK25Parser, has_thinking_content, normalize_conversation, pack_loss_mask,
                                    serialize_packed_loss_mask)

logger = logging.getLogger(__name__)

_STATE: dict[str, Any] = {}


def _init(tokenizer, max_length: int, last_turn: str, min_loss_tokens: int) -> None:
    if isinstance(tokenizer, str):
        from transformers import AutoTokenizer
        tokenizer = AutoTokenizer.from_pretrained(tokenizer, trust_remote_code=True)
    _STATE.update(parser=KimiK25Parser(tokenizer), max_length=max_length, last_turn=last_turn,
                  min_loss_tokens=min_loss_tokens)


def _last_turn_only(messages) -> bool:
    mode = _STATE["last_turn"]
    return has_thinking_content(messages) if mode == "auto" else mode == "true"


def tokenize_conversation(messages) -> Optional[dict]:
    messages = normalize_conversation(messages)
    ids, mask = _STATE["parser"].parse(messages, _STATE["max_length"], last_turn_only=_last_turn_only(messages))
    if int(mask.sum()) < max(1, _STATE["min_loss_tokens"]):
        return None
    return {"input_ids": ids.tolist(), "packed_loss_mask": serialize_packed_loss_mask(pack_loss_mask(mask))}


def read_conversations(path: str, seed: int, key: str = "conversations") -> list:
    """Rows of ``key`` from a JSON/JSONL/Parquet file (or a directory of
    them), shuffled by ``seed``."""
    import numpy as np
    import pandas as pd
    files = [os.path.join(path, f) for f in sorted(os.listdir(path))] if os.path.isdir(path) else [path]
    frames = []
    for f in files:
        if f.endswith(".parquet"):
            frames.append(pd.read_parquet(f))
        elif f.endswith(".jsonl"):
            frames.append(pd.read_json(f, lines=True))
        elif f.endswith(".json"):
            with open(f) as fh:
                frames.append(pd.DataFrame(json.load(fh)))
    if not frames:
        raise FileNotFoundError(f"no .json/.jsonl/.parquet data under {path}")
    df = pd.concat(frames, ignore_index=True)
    if key not in df.columns:
        return []
    rows = []
    for i in np.random.default_rng(seed).permutation(len(df)):
        conv = df[key].iloc[int(i)]
        if isinstance(conv, str):
            conv = json.loads(conv)
        if conv is not None and hasattr(conv, "tolist"):
            conv = conv.tolist()
        if isinstance(conv, list) and conv:
            rows.append([dict(m) for m in conv])
    return rows


def load_and_preprocess_dataset(dataset_path: str, tokenizer, max_length: int, chat_template: str = "kimi-k25",
                                seed: int = 42, last_turn_loss_only: Any = "false", min_loss_tokens: int = 0,
                                num_workers: int = 16, cache_dir: str = "/dev/shm/lumenrl_cache") -> list:
    """``tokenizer`` is a path (each worker loads it) or a tokenizer object
    (tokenised in this process)."""
    if chat_template not in ("kimi-k25", "kimi_k25"):
        raise ValueError(f"unsupported chat_template {chat_template!r}")
    last_turn = str(last_turn_loss_only).lower()
    if last_turn not in ("true", "false", "auto"):
        raise ValueError("last_turn_loss_only must be true/false/auto")
    ident = dataset_path
    if os.path.isfile(dataset_path):
        st = os.stat(dataset_path)
        ident += f"-{st.st_size}-{st.st_mtime}"
    tok_id = tokenizer if isinstance(tokenizer, str) else getattr(tokenizer, "name_or_path", type(tokenizer).__name__)
    key = hashlib.sha256(f"{ident}|{tok_id}|{max_length}|{chat_template}|{last_turn}|{min_loss_tokens}|{seed}"
                         .encode()).hexdigest()[:32]
    cache = os.path.join(cache_dir, "tokenized_dataset", f"{key}.pt")
    if os.path.exists(cache):
        data = torch.load(cache, weights_only=False)
        logger.info("loaded %d cached samples from %s", len(data), cache)
        return data
    convs = read_conversations(dataset_path, seed)
    args = (tokenizer, max_length, last_turn, min_loss_tokens)
    if num_workers <= 1 or not isinstance(tokenizer, str):
        _init(*args)
        results = [tokenize_conversation(c) for c in convs]
    else:
        with mp.get_context("spawn").Pool(num_workers, initializer=_init, initargs=args) as pool:
            results = list(pool.imap(tokenize_conversation, convs, chunksize=64))
    data = [r for r in results if r is not None]
    if len(data) < len(results):
        logger.warning("skipped %d samples with too few supervised tokens", len(results) - len(data))
    os.makedirs(os.path.dirname(cache), exist_ok=True)
    torch.save(data, cache)
    return data
