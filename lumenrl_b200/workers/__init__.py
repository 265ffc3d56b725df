"""Worker roles (actor, ref, rollout, reward, critic, teacher, hybrid)."""

from lumenrl_b200.workers.roles import (  # noqa: F401
    ActorWorker, BaseWorker, CriticWorker, HybridWorker, RefWorker, RewardWorker, RolloutWorker, TeacherWorker,
)
