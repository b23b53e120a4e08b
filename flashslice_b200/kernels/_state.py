"""Module-global modes shared by the op surface (not thread-safe, as in the
reference, ``slice_ops.py:346-352``)."""

import os

STATS_MODES = ("online", "two-pass")
stats_mode = os.environ.get("FLASHSLICE_STATS_MODE", "").lower() or "online"
if stats_mode not in STATS_MODES:
    raise ValueError("FLASHSLICE_STATS_MODE must be one of %s, got %r"
                     % (STATS_MODES, stats_mode))
block_g = None

# Which kernels serve the ops: "auto" (tensor-core kernels where they apply,
# the exact-fp32 FMA kernels elsewhere) or "fma" (always the FMA kernels).
ENGINES = ("auto", "fma")
engine = os.environ.get("FLASHSLICE_B200_ENGINE", "").lower() or "auto"
if engine not in ENGINES:
    raise ValueError("FLASHSLICE_B200_ENGINE must be one of %s, got %r" % (ENGINES, engine))


def set_engine(name):
    """Select the kernels: "auto" or "fma" (see ``ENGINES``)."""
    global engine
    if name not in ENGINES:
        raise ValueError("engine must be one of %s, got %r" % (ENGINES, name))
    engine = name
