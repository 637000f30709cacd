"""Mirror of the reference's tv.runtime graph/session API for the PTQ path."""
from .session import *  # noqa: F401,F403
