"""Same module as ``telescope_cache_b200.range_spec`` under the reference's
split-module path (``telescoping_attn/range_spec.py``)."""

from ..range_spec import *  # noqa: F401,F403
from ..range_spec import __all__  # noqa: F401
