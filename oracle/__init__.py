"""CPU oracle for the tattn hot path: test infrastructure only (see ``oracle/tiled.py``).

Nothing in the product package imports this; tests, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` use it as the checker / the timed reference CPU path.
"""

from oracle.tiled import (  # noqa: F401
    LOG2E,
    flops,
    naive_attention,
    naive_gradients,
    preprocess_delta,
    tiled_backward,
    tiled_forward,
)
