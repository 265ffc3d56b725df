"""Reward functions and their registry.

A reward function maps a batch of responses to one scalar per row:
``fn(responses: list[list[int]], prompts: list[list[int]], **ctx) -> Tensor[B]``.
Text-level scorers (math) receive decoded strings through ``ctx['texts']``.

Registered:
* ``contains_token``  -- 1.0 if the response contains ``token_id`` (default 7);
* ``parity``          -- 1.0 if more than half the response tokens are even ids;
* ``math_reward`` / ``math_dapo`` -- verl math_dapo-style answer check
  (reference ``lumenrl/rewards/math_reward.py:39-157``).
"""

from lumenrl_b200.rewards.functions import (  # noqa: F401
    contains_token_reward, parity_reward, math_reward, get_reward_fn, RewardFn,
)
