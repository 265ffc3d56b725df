"""RL algorithms: advantage estimators, losses, KL control, rollout correction.

Importing this package registers GRPO, DAPO, PPO and OPD in
``ALGORITHM_REGISTRY``.
"""

from lumenrl_b200.algorithms import advantage, losses, kl_controller, rollout_correction  # noqa: F401
from lumenrl_b200.algorithms.advantage import ADV_ESTIMATOR_REGISTRY, register_adv_est  # noqa: F401
from lumenrl_b200.algorithms.base import BaseAlgorithm  # noqa: F401
from lumenrl_b200.algorithms.dapo import DAPOAlgorithm  # noqa: F401
from lumenrl_b200.algorithms.grpo import GRPOAlgorithm  # noqa: F401
from lumenrl_b200.algorithms.opd import OPDAlgorithm  # noqa: F401
from lumenrl_b200.algorithms.ppo import PPOAlgorithm  # noqa: F401
