"""Module-global modes shared by the op surface (not thread-safe, as in the
reference, ``slice_ops.py:346-352``)."""

import os

STATS_MODES = ("online", "two-pass")
stats_mode = os.environ.get("FLASHSLICE_STATS_MODE", "").lower() or "online"
if stats_mode not in STATS_MODES:
    raise ValueError("FLASHSLICE_STATS_MODE must be one of %s, got %r"
                     % (STATS_MODES, stats_mode))
block_g = None
