"""Decode-step op (B200 replacement of ``src/mamba2_jax/ops/selective_state_update.py``)."""
from .selective_state_update import selective_state_update

__all__ = ["selective_state_update"]
