"""Ops around the SSD (B200 replacements of ``src/mamba2_jax/ops``)."""
from .causal_conv1d import causal_conv1d, causal_conv1d_update
from .rms_norm import rms_norm_gated
from .selective_state_update import selective_state_update

__all__ = ["selective_state_update", "causal_conv1d", "causal_conv1d_update", "rms_norm_gated"]
