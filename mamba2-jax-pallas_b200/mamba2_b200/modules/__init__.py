"""Layer wiring of the B200 kernels (the reference's ``mamba2_jax.modules``)."""
from .mamba2 import Mamba2, allocate_inference_cache

__all__ = ["Mamba2", "allocate_inference_cache"]
