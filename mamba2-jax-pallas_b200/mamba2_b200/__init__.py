"""B200 (sm_100a) Mamba2 SSD forward + decode step behind the reference's Python API.

Functions mirror AlexG1105/mamba2-jax-pallas (``mamba2_jax.kernels`` / ``mamba2_jax.ops``)
with torch CUDA tensors in place of JAX arrays; all compute runs in libssd_b200.so.
"""
from .kernels import (bmm_chunk_fwd, chunk_cumsum_fwd, chunk_scan_fwd, chunk_state_fwd,
                      chunk_state_varlen_mosaic, mamba_chunk_scan_combined_fwd,
                      state_passing_fwd)
from .ops import causal_conv1d, causal_conv1d_update, rms_norm_gated, selective_state_update

__all__ = ["mamba_chunk_scan_combined_fwd", "chunk_cumsum_fwd", "chunk_state_fwd",
           "state_passing_fwd", "bmm_chunk_fwd", "chunk_scan_fwd", "chunk_state_varlen_mosaic",
           "selective_state_update", "causal_conv1d", "causal_conv1d_update", "rms_norm_gated"]
