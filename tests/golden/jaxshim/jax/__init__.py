"""NumPy-backed stand-in for the handful of ``jax`` names the reference's pure-JAX ops use.

Test infrastructure only: ``tests/golden/make_fixtures.py`` puts this directory on
``sys.path`` so that the reference's own ``ops/ssd_naive.py``, ``ops/selective_state_update.py``,
``ops/rms_norm.py`` and ``ops/causal_conv1d.py`` run unmodified (loaded by file path) and
produce golden outputs.  JAX itself is not installable in this image.

Each function restates the published semantics of the JAX function of the same name
(jax.numpy follows NumPy's definitions; the differences that matter here are handled
explicitly: JAX's default float dtype is float32, ``jnp.clip`` takes ``a_min``/``a_max``,
``jax.nn.softplus(x) = logaddexp(x, 0)``, ``jax.nn.silu(x) = x * sigmoid(x)``, and
``lax.conv_general_dilated`` is a cross-correlation).

Precision: ``JAXSHIM_F64=1`` (read at import) maps ``jnp.float32`` to float64, so the
reference's computation runs end to end in float64 (a tight pin for the float64 oracle);
otherwise it runs in float32 as JAX on CPU would.
"""
import numpy as _np

from . import numpy  # noqa: F401
from . import nn  # noqa: F401
from . import lax  # noqa: F401

Array = _np.ndarray
