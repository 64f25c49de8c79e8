"""Drop-in for the reference module's SSD dispatcher (``modules/mamba2.py:53-74``).

The reference tries the Pallas path and, on any exception, falls back to the naive
XLA path with a sticky global flag.  Here there is one implementation and no
fallback: ``_ssd_combined_fwd`` always runs the B200 kernels and lets errors raise.
``use_pallas`` is accepted for signature compatibility and ignored.
"""

from __future__ import annotations

from .kernels.ssd_combined import mamba_chunk_scan_combined_fwd
from .ops.selective_state_update import selective_state_update


def _ssd_combined_fwd(use_pallas: bool = True, **kwargs):
    return mamba_chunk_scan_combined_fwd(**kwargs)


__all__ = ["_ssd_combined_fwd", "selective_state_update"]
