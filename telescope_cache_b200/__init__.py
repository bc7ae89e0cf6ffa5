"""B200-native (sm_100a) telescoping multiresolution attention.

``telescope_cache_b200.reference`` mirrors the reference's ``reference.py``
API; ``telescope_cache_b200.range_spec`` its integer schedule; and
``telescope_cache_b200.telescoping_attn.*`` its split modules.  All compute
runs in ``_lib/libtelescope_b200.so`` (CUDA, sm_100a) through a C ABI
(``include/telescope_cache.h``).
"""

from . import range_spec  # noqa: F401
from .reference import *  # noqa: F401,F403
from .reference import __all__  # noqa: F401
