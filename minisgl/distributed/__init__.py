"""Alias of ``minisgl.parallel`` under the reference's module name."""

from minisgl.parallel import *  # noqa: F401,F403
from minisgl.parallel import __all__  # noqa: F401
