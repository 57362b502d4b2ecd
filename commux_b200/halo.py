"""``commux_b200.halo`` (also ``commux.halo``): the 26-direction halo exchange
of a 3-D field over tagged p2p (tags 1000 + direction). Re-exports
:mod:`commux_b200.parallel.halo`."""

from .parallel.halo import (DIRECTIONS, TAG_BASE, CartGrid, HaloExchange, dir_index,  # noqa: F401
                            factor3, reference_exchange)

__all__ = ["DIRECTIONS", "TAG_BASE", "CartGrid", "HaloExchange", "dir_index", "factor3",
           "reference_exchange"]
