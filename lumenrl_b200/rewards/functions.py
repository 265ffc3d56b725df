"""Programmatic rewards (token-level synthetic tasks and the math scorer)."""

from __future__ import annotations

import re
from typing import Callable, Optional, Sequence

import torch
from torch import Tensor

from lumenrl_b200.core.registry import REWARD_REGISTRY

RewardFn = Callable[..., Tensor]


def _to_rows(responses) -> list[list[int]]:
    if isinstance(responses, Tensor):
        return [r.tolist() for r in responses]
    return [list(r) for r in responses]


def contains_token_reward(responses, prompts=None, token_id: int = 7, lengths: Optional[Tensor] = None, **_) -> Tensor:
    if isinstance(responses, Tensor) and lengths is not None:
        ar = torch.arange(responses.shape[1], device=responses.device).unsqueeze(0)
        valid = ar < lengths.to(responses.device).unsqueeze(1)
        return ((responses == token_id) & valid).any(1).float()
    return torch.tensor([1.0 if token_id in r else 0.0 for r in _to_rows(responses)])


def parity_reward(responses, prompts=None, lengths: Optional[Tensor] = None, **_) -> Tensor:
    """1.0 when the count of even token ids exceeds half the response length."""
    if isinstance(responses, Tensor) and lengths is not None:
        ar = torch.arange(responses.shape[1], device=responses.device).unsqueeze(0)
        L = lengths.to(responses.device)
        valid = ar < L.unsqueeze(1)
        even = ((responses % 2 == 0) & valid).sum(1)
        return (even * 2 > L).float()
    out = []
    for r in _to_rows(responses):
        even = sum(1 for t in r if t % 2 == 0)
        out.append(1.0 if 2 * even > len(r) else 0.0)
    return torch.tensor(out)


# ---------------------------------------------------------------------------
# math_dapo-style scorer: take the last "Answer:" in the tail of the response,
# normalise and compare with the ground truth; +1 correct, -1 wrong.
# ---------------------------------------------------------------------------

_SUBS = [("an ", ""), ("a ", ""), (".$", "$"), ("\\$", ""), ("\\ ", ""), (" ", ""), ("mbox", "text"),
         (",\\text{and}", ","), ("\\text{and}", ","), ("\\text{m}", "\\text{}")]
_REMOVE = ["square", "ways", "integers", "dollars", "mph", "inches", "hours", "km", "units", "\\ldots", "sue",
           "points", "feet", "minutes", "digits", "cents", "degrees", "cm", "gm", "pounds", "meters", "meals",
           "edges", "students", "childrentickets", "multiples", "\\text{s}", "\\text{.}", "\\text{\ns}",
           "\\text{}^2", "\\text{}^3", "\\text{\n}", "\\text{}", r"\mathrm{th}", r"^\circ", r"^{\circ}", r"\;",
           r",\!", "{,}", '"', "\\dots"]


def normalize_final_answer(ans: str) -> str:
    ans = ans.split("=")[-1]
    for a, b in _SUBS:
        ans = ans.replace(a, b)
    for r in _REMOVE:
        ans = ans.replace(r, "")
    ans = re.sub(r"(.*?)(\$)(.*?)(\$)(.*)", "$\\3$", ans)
    ans = re.sub(r"(\\text\{)(.*?)(\})", "\\2", ans)
    ans = re.sub(r"(\\textbf\{)(.*?)(\})", "\\2", ans)
    ans = re.sub(r"(\\overline\{)(.*?)(\})", "\\2", ans)
    ans = re.sub(r"(\\boxed\{)(.*)(\})", "\\2", ans)
    ans = re.sub(r"(frac)([^{])(.)", "frac{\\2}{\\3}", ans)
    ans = re.sub(r"(sqrt)([^{])", "sqrt{\\2}", ans)
    ans = ans.replace("$", "")
    if ans.replace(",", "").isdigit():
        ans = ans.replace(",", "")
    return ans.strip()


def math_score(text: str, ground_truth: str, tail_chars: int = 300) -> dict:
    tail = text[-tail_chars:]
    found = re.findall(r"(?i)Answer\s*:\s*([^\n]+)", tail)
    pred = normalize_final_answer(found[-1]) if found else "[INVALID]"
    ok = pred == normalize_final_answer(str(ground_truth))
    return {"score": 1.0 if ok else -1.0, "acc": ok, "pred": pred}


def math_reward(responses=None, prompts=None, texts: Optional[Sequence[str]] = None,
                ground_truths: Optional[Sequence[str]] = None, **_) -> Tensor:
    if texts is None or ground_truths is None:
        raise ValueError("math_reward needs decoded `texts` and `ground_truths`")
    return torch.tensor([math_score(t, g)["score"] for t, g in zip(texts, ground_truths)])


REWARD_REGISTRY.register("contains_token", contains_token_reward)
REWARD_REGISTRY.register("parity", parity_reward)
REWARD_REGISTRY.register("math_reward", math_reward)
REWARD_REGISTRY.register("math_dapo", math_reward)


def get_reward_fn(name: str) -> RewardFn:
    if name in REWARD_REGISTRY:
        return REWARD_REGISTRY.get(name)
    if ":" in name or "." in name:   # "module.path:function"
        import importlib
        mod, _, fn = name.replace(":", ".").rpartition(".")
        return getattr(importlib.import_module(mod), fn)
    return REWARD_REGISTRY.get(name)
