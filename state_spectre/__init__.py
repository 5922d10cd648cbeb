"""Import-compatible entry point: ``import state_spectre as ss`` keeps working
for code written against StateSpectre's Python package; everything resolves to
statespectre_b200."""

from statespectre_b200 import *  # noqa: F401,F403
from statespectre_b200 import __all__, __version__  # noqa: F401
from statespectre_b200 import _wire  # noqa: F401
