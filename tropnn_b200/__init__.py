"""tropnn_b200: backend="b200" for tropnn's TropLinear, TropFanLinear and PairwiseLinear on
NVIDIA B200.

Public surface:
  * ``TropLinear``, ``TropFanLinear``, ``PairwiseLinear``, ``RoutedLinearBase`` — drop-in
    layers with the reference's constructor arguments, parameters and ``state_dict``.
  * ``trop_route_hidden_b200``, ``pairwise_b200`` — the operator-level entry points
    (mirroring ``trop_route_hidden_tilelang`` / ``pairwise_tilelang``).
  * ``register(tropnn)`` — lets the reference package's own classes accept
    ``backend="b200"``.
  * ``tropnn_b200.distributed`` — batch-row sharding and gradient all-reduce for
    one-process-per-GPU data parallelism.
"""

from __future__ import annotations

from typing import Any

from .layers import (
    PairwiseLinear,
    RoutedLinearBase,
    TropFanLinear,
    TropLinear,
    fan_forward_b200,
    pairwise_forward_b200,
    trop_forward_b200,
)
from .ops import (
    packed_route_index_dtype,
    pairwise_anchor_index,
    pairwise_b200,
    trop_route_hidden_b200,
    trop_route_hidden_packed,
)

__all__ = [
    "PairwiseLinear",
    "RoutedLinearBase",
    "TropFanLinear",
    "TropLinear",
    "packed_route_index_dtype",
    "pairwise_anchor_index",
    "pairwise_b200",
    "register",
    "trop_route_hidden_b200",
    "trop_route_hidden_packed",
]


def register(tropnn: Any) -> None:
    """Adds backend="b200" to the reference package's TropLinear, TropFanLinear and
    PairwiseLinear.

    After ``register(tropnn)``, ``tropnn.TropLinear(..., backend="b200")`` builds the
    reference module itself (same init, same parameters; the constructor runs with the
    torch backend and then switches) and routes its forward through the b200 kernels.
    Every other backend string keeps its reference behaviour. Idempotent.
    """
    trop_cls = tropnn.TropLinear
    pair_cls = tropnn.PairwiseLinear
    if getattr(trop_cls, "_tropnn_b200_registered", False):
        return

    def _wrap_init(cls: Any) -> None:
        original = cls.__init__

        def __init__(self: Any, *args: Any, backend: str = "torch", **kwargs: Any) -> None:
            if backend == "b200":
                original(self, *args, backend="torch", **kwargs)
                self.backend = "b200"
            else:
                original(self, *args, backend=backend, **kwargs)

        __init__.__doc__ = original.__doc__
        cls.__init__ = __init__

    _wrap_init(trop_cls)
    _wrap_init(pair_cls)
    fan_cls = getattr(tropnn, "TropFanLinear", None)
    if fan_cls is not None:
        _wrap_init(fan_cls)
        fan_forward = fan_cls.forward

        def _fan_forward(self: Any, x: Any) -> Any:
            if self.backend == "b200":
                return fan_forward_b200(self, x)
            return fan_forward(self, x)

        fan_cls.forward = _fan_forward

    trop_forward = trop_cls.forward

    def _trop_forward(self: Any, x: Any) -> Any:
        if self.backend == "b200":
            return trop_forward_b200(self, x)
        return trop_forward(self, x)

    pair_forward = pair_cls.forward

    def _pair_forward(self: Any, x: Any) -> Any:
        if self.backend == "b200":
            return pairwise_forward_b200(self, x)
        return pair_forward(self, x)

    trop_cls.forward = _trop_forward
    pair_cls.forward = _pair_forward
    trop_cls._tropnn_b200_registered = True
