"""Data pipeline on CPU: Kimi-K2.5 formatting, assistant loss masks (offset
and prefix-encode paths agree), RLE mask packing, cached preprocessing, and
the chat-template SFT dataset (behaviour of the reference's
``lumenrl/data/kimi_k25_parser.py`` and ``sft_dataset.py``)."""

import json

import torch

from lumenrl_b200.data.chat import (KimiK25Format, KimiK25Parser, has_thinking_content, normalize_conversation,
                                    pack_loss_mask, serialize_packed_loss_mask, unpack_loss_mask)
from lumenrl_b200.data.dataset import load_and_preprocess_dataset
from lumenrl_b200.data.sft_dataset import SFTDataset


class CharTok:
    """Character-level tokenizer: one token per character (id = ord)."""
    name_or_path = "char"
    pad_token_id = 0

    def __init__(self, offsets=True):
        self.offsets = offsets

    def encode(self, text, add_special_tokens=False):
        return [ord(c) for c in text]

    def __call__(self, text, add_special_tokens=False, return_offsets_mapping=False, truncation=False,
                 max_length=None):
        if return_offsets_mapping and not self.offsets:
            raise NotImplementedError
        ids = self.encode(text)[:max_length]
        return {"input_ids": ids, "offset_mapping": [(i, i + 1) for i in range(len(ids))]}

    def apply_chat_template(self, msgs, tokenize=True, add_generation_prompt=False, **kw):
        s = "<s>" + "".join(f"[{m['role']}]{m['content']}|" for m in msgs)
        if add_generation_prompt:
            s += "[assistant]"
        return self.encode(s)


CONV = [{"from": "system", "value": "sys"}, {"from": "human", "value": "hi <|image|>"},
        {"from": "gpt", "value": "<think>a</think>ok"}, {"from": "human", "value": "more"},
        {"from": "gpt", "value": "<think>b</think>done", "reasoning": "r"}]


def test_format_and_masks():
    conv = normalize_conversation(CONV)
    assert conv[1]["role"] == "user" and conv[4]["reasoning_content"] == "r"
    assert has_thinking_content(conv)
    assert not has_thinking_content([{"role": "assistant", "content": "<think></think>x"}])
    f = KimiK25Format()
    text = f.format(conv)
    assert text.startswith(f.SYSTEM + "sys" + f.END + f.USER + "hi " + f.MEDIA + "\n" + f.END)
    # thinking stripped from the earlier assistant turn, kept in the last; empty think injected
    assert f.ASSISTANT + "<think></think>ok" + f.END in text
    assert f.ASSISTANT + "<think>b</think>done" + f.END in text
    ids, mask = KimiK25Parser(CharTok()).parse(conv, 10_000)
    sel = "".join(chr(int(i)) for i, m in zip(ids, mask) if m)
    assert sel == "<think></think>ok<think>b</think>done"
    ids2, mask2 = KimiK25Parser(CharTok(offsets=False)).parse(conv, 10_000)
    assert torch.equal(ids, ids2) and torch.equal(mask, mask2)
    _, last = KimiK25Parser(CharTok()).parse(conv, 10_000, last_turn_only=True)
    assert int(last.sum()) == len("<think>b</think>done")
    tc = [{"role": "assistant", "content": "x", "tool_calls": [{"id": "c1", "function": {"arguments": "{}"}}]},
          {"role": "tool", "content": "42", "tool_call_id": "c1"}]
    t = f.format(tc, add_generation_prompt=True)
    assert "<|tool_call_begin|>c1<|tool_call_argument_begin|>{}<|tool_call_end|>" in t
    assert "## Return of c1\n42" in t and t.endswith(f.ASSISTANT)


def test_pack_loss_mask_roundtrip():
    assert pack_loss_mask(torch.tensor([0, 0, 1, 1, 1, 0, 0, 1, 1, 0])) == [2, 3, 2, 2, 1]
    assert pack_loss_mask(torch.tensor([1, 1, 0])) == [0, 2, 1]
    g = torch.Generator().manual_seed(0)
    for _ in range(20):
        r = (torch.rand(37, generator=g) > 0.5).long()
        assert torch.equal(unpack_loss_mask(serialize_packed_loss_mask(pack_loss_mask(r))), r)


def test_preprocess_cache(tmp_path):
    p = tmp_path / "d.jsonl"
    rows = [{"conversations": CONV}, {"conversations": [{"from": "human", "value": "q"}]}]
    p.write_text("\n".join(json.dumps(r) for r in rows))
    kw = dict(num_workers=1, cache_dir=str(tmp_path / "c"), last_turn_loss_only="auto")
    data = load_and_preprocess_dataset(str(p), CharTok(), 4096, **kw)
    assert len(data) == 1   # the second row has no assistant tokens
    m = unpack_loss_mask(data[0]["packed_loss_mask"])
    assert int(m.sum()) == len("<think>b</think>done")   # auto + real thinking -> last turn only
    assert load_and_preprocess_dataset(str(p), CharTok(), 4096, **kw) == data


def test_sft_dataset(tmp_path):
    p = tmp_path / "s.jsonl"
    msgs = [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo"}]
    p.write_text(json.dumps({"messages": msgs}) + "\n")
    ds = SFTDataset(str(p), CharTok(), max_length=40)
    assert ds.system_prompt == [ord(c) for c in "<s>"] and ds.gen_prompt == [ord(c) for c in "[assistant]"]
    row = ds[0]
    text = "".join(chr(int(i)) for i in row["input_ids"][row["attention_mask"].bool()])
    assert text == "<s>[user]hi|[assistant]yo|"
    sup = "".join(chr(int(i)) for i, m in zip(row["input_ids"], row["loss_mask"]) if m)
    assert sup == "yo|"
    assert row["input_ids"].shape == (40,)
    short = SFTDataset(str(p), CharTok(), max_length=10, truncation="left")[0]
    assert "".join(chr(int(i)) for i in short["input_ids"]) == "[assistant]yo|"[-10:]
