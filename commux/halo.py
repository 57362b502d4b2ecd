"""``import commux.halo``: the 26-direction halo exchange helper of
``commux_b200`` under the reference's package name."""

from commux_b200.halo import *  # noqa: F401,F403
from commux_b200.halo import __all__  # noqa: F401
