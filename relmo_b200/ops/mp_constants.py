"""Constants shared by the runtime loader, dispatch and facade.

Same values as relmo's ``src/relmo/ops/mp_constants.py:9-26``.
"""

from __future__ import annotations

from typing import Final

MODE_SUM: Final[int] = 0
MODE_LOGSUMEXP: Final[int] = 1
MODE_MEAN: Final[int] = 2

# Ops the loaded library must register for the loader to accept it
# (reference mp_constants.py:19-26).
REQUIRED_NAMESPACE_OPS: Final[tuple[str, ...]] = (
    "fanout_scatter",
    "fanout_scatter_backward",
    "fanin_reduce",
    "fanin_reduce_sum_backward",
    "fanin_reduce_logsumexp_backward",
    "build_info",
)
