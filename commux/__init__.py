"""``import commux`` -- the public package name of the reference.

Re-exports commux_b200 so code written for the reference (``import commux;
commux.register()``) runs unchanged.
"""

from commux_b200 import *  # noqa: F401,F403
from commux_b200 import (IOContext, TAG_MASK_ANY_SOURCE, batch_p2p, create_backend,  # noqa: F401
                         is_commux, library_paths, make_tcp_io_context, make_ucp_tag,
                         p2p_plan, preferred_backend, register, reset_stats, stats, transports)
