"""``jax.nn`` subset on NumPy: softplus and silu (see the package docstring)."""
import numpy as _np


def softplus(x):
    # jax.nn.softplus(x) = log(1 + exp(x)), evaluated as logaddexp(x, 0)
    return _np.logaddexp(x, _np.zeros((), dtype=x.dtype))


def sigmoid(x):
    one = _np.ones((), dtype=x.dtype)
    return one / (one + _np.exp(-x))


def silu(x):
    return x * sigmoid(x)
