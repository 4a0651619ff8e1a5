"""locali_b200 - B200-native routed-MoE hot path for Locali-style expert arenas.

The package keeps the reference's module interfaces (``V4ArenaMoE`` and the
``ArenaStore`` slot API) while the arena lives in HBM and every expert
product runs in hand-written sm_100a kernels reached through the C ABI in
``include/lmoe.h``.
"""

__version__ = "0.1.0"
