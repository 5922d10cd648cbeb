"""``state_spectre._wire``: the wire-format module under its StateSpectre
import path (everything resolves to statespectre_b200._wire)."""

from statespectre_b200._wire import *  # noqa: F401,F403
