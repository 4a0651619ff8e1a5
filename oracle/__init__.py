"""CPU oracle for the routed-MoE hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``locali_b200`` imports this package:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may use it, and only as the checker
(or as the timed CPU stand-in for the reference's MLX CPU path, which cannot be
imported here).  The product path fails loudly when its CUDA library is
missing; it never falls back to this code.

Every function restates the reference's algorithm and cites the reference
file:line it follows (paths within gabrielekarra/locali).
"""

from .moe_oracle import *  # noqa: F401,F403
