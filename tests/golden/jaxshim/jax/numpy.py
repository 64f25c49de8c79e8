"""``jax.numpy`` subset on NumPy (see the package docstring)."""
import os as _os

import numpy as _np

F64 = _os.environ.get("JAXSHIM_F64", "0") == "1"
float32 = _np.float64 if F64 else _np.float32
float64 = _np.float64
int32 = _np.int32
bool_ = _np.bool_
inf = _np.inf
ndarray = _np.ndarray


def _default(dtype):
    return float32 if dtype is None else dtype


def asarray(a, dtype=None):
    return _np.asarray(a, dtype=dtype)


def zeros(shape, dtype=None):
    return _np.zeros(shape, dtype=_default(dtype))


def ones(shape, dtype=None):
    return _np.ones(shape, dtype=_default(dtype))


def pad(a, pad_width, mode="constant", constant_values=0):
    return _np.pad(a, pad_width, mode=mode, constant_values=constant_values)


def clip(a, a_min=None, a_max=None):
    out = a
    if a_min is not None:
        out = _np.maximum(out, _np.asarray(a_min, dtype=a.dtype))
    if a_max is not None:
        out = _np.minimum(out, _np.asarray(a_max, dtype=a.dtype))
    return out


def einsum(spec, *ops, **kw):
    # one contraction at a time, in the result dtype of the operands (float32 stays float32)
    return _np.einsum(spec, *ops, optimize=True)


transpose = _np.transpose
repeat = _np.repeat
concatenate = _np.concatenate
cumsum = _np.cumsum
exp = _np.exp
where = _np.where
tril = _np.tril
sqrt = _np.sqrt
sum = _np.sum  # noqa: A001
mean = _np.mean
log = _np.log
log1p = _np.log1p
maximum = _np.maximum
minimum = _np.minimum
logaddexp = _np.logaddexp
