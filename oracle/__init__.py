"""CPU oracle of tropnn's routed-layer hot path — test infrastructure only.

Imported by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs,
never by the ``tropnn_b200`` package.
"""

from .tropnn_oracle import *  # noqa: F401,F403
from .tropnn_oracle import __all__  # noqa: F401
