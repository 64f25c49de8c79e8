"""``jax.lax`` subset on NumPy: the depthwise 1-D case of conv_general_dilated
(see the package docstring)."""
import numpy as _np


def conv_general_dilated(lhs, rhs, window_strides, padding, dimension_numbers=None,
                         feature_group_count=1, **kw):
    """XLA convolution restricted to what ops/causal_conv1d.py uses: NCH input, OIH kernel with
    one input channel per group (depthwise, feature_group_count == channels), stride 1,
    VALID padding.  XLA convolutions are cross-correlations (the kernel is not flipped):
    out[b, c, t] = sum_j lhs[b, c, t + j] * rhs[c, 0, j]."""
    if tuple(dimension_numbers) != ("NCH", "OIH", "NCH") or padding != "VALID" or tuple(window_strides) != (1,):
        raise NotImplementedError("only the depthwise NCH/OIH/NCH, stride 1, VALID case is restated")
    b, c, t = lhs.shape
    o, i, k = rhs.shape
    if feature_group_count != c or o != c or i != 1:
        raise NotImplementedError("only depthwise convolution is restated")
    n = t - k + 1
    out = _np.zeros((b, c, n), dtype=_np.result_type(lhs.dtype, rhs.dtype))
    for j in range(k):
        out += lhs[:, :, j:j + n] * rhs[None, :, 0, j, None]
    return out
