"""``state_spectre._rollout``: the rollout client module under its
StateSpectre import path (everything resolves to statespectre_b200._rollout)."""

from statespectre_b200._rollout import *  # noqa: F401,F403
from statespectre_b200._rollout import RolloutWeightClient  # noqa: F401
