"""SSD forward kernels (B200 replacements of ``src/mamba2_jax/kernels/__init__.py``)."""
from .ssd_combined import mamba_chunk_scan_combined_fwd, workspace_bytes
from .stages import (bmm_chunk_fwd, chunk_cumsum_fwd, chunk_scan_fwd, chunk_state_fwd,
                     chunk_state_varlen_mosaic, state_passing_fwd)

__all__ = ["mamba_chunk_scan_combined_fwd", "workspace_bytes", "chunk_cumsum_fwd",
           "chunk_state_fwd", "state_passing_fwd", "bmm_chunk_fwd", "chunk_scan_fwd",
           "chunk_state_varlen_mosaic"]
